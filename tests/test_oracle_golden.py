"""Pin the CPU oracle (``oracle/``) to golden vectors made by the reference itself."""

import hashlib

import numpy as np
import pytest
import torch

import oracle
from tests import golden_io as gio
from torch2iron_b200 import synth
from torch2iron_b200.config import QuantizedQwenConfig


def test_autogptq_gemv_matches_reference():
    d = gio.load("gemv_autogptq.npz")
    lin = gio.linear(d, "p")
    x = torch.from_numpy(d["x"])
    y = oracle.autogptq_gemv(x, lin.qweight, lin.qzeros, lin.scales)
    assert torch.equal(y, torch.from_numpy(d["y"]))  # same arithmetic -> bit-exact
    # the runtime (per-group) form agrees within fp32 rounding
    y2 = oracle.GroupedW4A16Linear(lin.qweight, lin.qzeros, lin.scales)(x)
    torch.testing.assert_close(y2, y, rtol=1e-5, atol=1e-5)


def test_config0_generator_and_gemv_pinned():
    d = gio.load("config0.npz")
    g = torch.Generator().manual_seed(0)
    w = torch.randn(3072, 1024, generator=g) * 0.02
    x = torch.randn(1, 1024, generator=g).to(torch.float16)
    lin = synth.quantize_rtn_autogptq(w)
    digest = hashlib.sha256(lin.qweight.numpy().tobytes() + lin.qzeros.numpy().tobytes()
                            + lin.scales.numpy().tobytes()).hexdigest()
    assert digest == str(d["weights_sha256"])
    assert torch.equal(x, torch.from_numpy(d["x"]))
    y = oracle.autogptq_gemv(x, lin.qweight, lin.qzeros, lin.scales)
    assert torch.equal(y, torch.from_numpy(d["y"]))


def test_unpack_roundtrip_and_zero_range():
    g = torch.Generator().manual_seed(3)
    w = torch.randn(64, 256, generator=g) * 0.02
    lin = synth.quantize_rtn_autogptq(w)
    z = oracle.unpack_autogptq_qzeros(lin.qzeros, 64)
    assert int(z.min()) >= 1 and int(z.max()) <= 15
    dense = oracle.autogptq_linear_to_dense(lin.qweight, lin.qzeros, lin.scales)
    err = (dense - w).abs().max().item()
    assert err <= lin.scales.float().max().item() * 0.5 + 1e-6


def test_qparam_linear_matches_reference_runtime():
    d = gio.load("qparam_linear.npz")
    qparam = torch.from_numpy(d["qparam"])
    packed, scales = oracle.split_qparam(qparam, 512)
    x = gio.bf16(d["x"]).to(torch.float32)
    y = oracle.packed_w4a16_linear(x, packed, scales, 512, 256)
    assert torch.equal(y, torch.from_numpy(d["y"]))


def test_rms_norm_rope_matches_reference():
    d = gio.load("rope_norm.npz")
    ang = oracle.compute_rope_angles(128, 64, 1e6)
    assert torch.equal(ang, torch.from_numpy(d["angles"]))
    x = torch.from_numpy(d["x"])
    w = torch.from_numpy(d["w"])
    y = oracle.apply_rope(oracle.rms_norm(x, w, 1e-6), ang[5:6])
    assert torch.equal(y, torch.from_numpy(d["y"]))
    y_rows = oracle.apply_rope_rows(oracle.rms_norm(x[:, 0], w, 1e-6), ang[[5, 5]])
    assert torch.equal(y_rows, y[:, 0])


def _layer_from(d, prefix=""):
    names = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
    lins = {}
    for n in names:
        lin = gio.linear(d, prefix + n)
        lins[n] = oracle.GroupedW4A16Linear(lin.qweight, lin.qzeros, lin.scales)
    return oracle.OracleLayer(
        **lins,
        input_layernorm=gio.bf16(d[prefix + "input_layernorm"]),
        post_attention_layernorm=gio.bf16(d[prefix + "post_attention_layernorm"]),
        q_norm=gio.bf16(d[prefix + "q_norm"]), k_norm=gio.bf16(d[prefix + "k_norm"]))


def test_decoder_layer_matches_reference():
    d = gio.load("layer_small.npz")
    shape = oracle.OracleShape(vocab_size=512, emb_dim=256, n_layers=1, n_heads=4, n_kv_groups=2, head_dim=64,
                               hidden_dim=512, rms_norm_eps=1e-6, rope_base=1e6)
    layer = _layer_from(d)
    dec = oracle.OracleDecoder(shape, [layer], embed=torch.zeros(512, 256), final_norm=torch.ones(256),
                               lm_head=torch.zeros(512, 256), max_ctx=64, batch=2, kv_dtype=torch.float32)
    pos = int(d["pos"])
    dec.k_cache[0][:, :, :pos] = torch.from_numpy(d["past_k"])
    dec.v_cache[0][:, :, :pos] = torch.from_numpy(d["past_v"])
    x = torch.from_numpy(d["x"])[:, 0]
    out = dec.layer_step(0, x, torch.tensor([pos, pos]))
    torch.testing.assert_close(out, torch.from_numpy(d["out"])[:, 0], rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(dec.k_cache[0][:, :, :pos + 1], torch.from_numpy(d["present_k"]), rtol=2e-5,
                               atol=2e-5)
    torch.testing.assert_close(dec.v_cache[0][:, :, :pos + 1], torch.from_numpy(d["present_v"]), rtol=2e-5,
                               atol=2e-5)


def test_tiny_model_generate_matches_reference():
    d = gio.load("model_tiny.npz")
    shape = oracle.OracleShape(vocab_size=512, emb_dim=256, n_layers=2, n_heads=4, n_kv_groups=2, head_dim=64,
                               hidden_dim=512, rms_norm_eps=1e-6, rope_base=1e6)
    layers = [_layer_from(d, f"l{i}.") for i in range(2)]
    emb = gio.bf16(d["embed"])
    dec = oracle.OracleDecoder(shape, layers, embed=emb, final_norm=gio.bf16(d["final_norm"]), lm_head=emb,
                               max_ctx=64, batch=1, kv_dtype=torch.float32)
    prompt = torch.from_numpy(d["prompt"])
    logits = dec.prefill(prompt)
    torch.testing.assert_close(logits[0], torch.from_numpy(d["logits_last"]), rtol=1e-4, atol=1e-4)
    dec2 = oracle.OracleDecoder(shape, layers, embed=emb, final_norm=gio.bf16(d["final_norm"]), lm_head=emb,
                                max_ctx=64, batch=1, kv_dtype=torch.float32)
    gen = dec2.generate(prompt, 8)
    assert torch.equal(gen[0], torch.from_numpy(d["generated"]))


def test_packet_attention_matches_reference():
    d = gio.load("attention_packet.npz")
    out = oracle.chunked_attention_packet(gio.bf16(d["q"]), gio.bf16(d["packet_after"]), int(d["seq"]),
                                          int(d["chunk"]))
    ref = gio.bf16(d["out"])
    assert torch.equal(out, ref)


@pytest.mark.parametrize("case", [0, 1])
def test_gqa_attention_matches_kv_plane_reference(case):
    """The oracle's attention core against the reference's KV-plane attention
    (``kv_plane_reference.py:122-187``), read through this library's cache layout."""
    d = gio.load("kv_plane_attention.npz")
    q, k, v, attend, out, qpg, hd = gio.kv_plane_case(d, case, max_ctx=80)
    y = oracle.gqa_attention(q.view(8 * qpg, hd), k[0, :, :attend], v[0, :, :attend]).reshape(-1)
    assert (y - out).abs().max().item() <= 8e-3        # the reference output is rounded to bf16


def test_q4nx_layout_matches_reference():
    """The Q4NX group-32 restatement against the reference's own packing of a
    96 x 512 weight (rows padded to a 64-row patch): dequantisation bit-exact,
    the linear within the reference's final bf16 rounding."""
    d = gio.load("q4nx_linear.npz")
    out_f, in_f, padded = (int(v) for v in d["shape"])
    assert (out_f, in_f, padded) == (96, 512, 128)
    data = d["data"].tobytes()
    assert len(data) == padded // oracle.Q4NX_OUT_CHUNK * (in_f // oracle.Q4NX_IN_CHUNK) * oracle.Q4NX_CHUNK_BYTES
    dense = oracle.q4nx_dequantize_linear(data, in_f, out_f)
    assert torch.equal(dense, torch.from_numpy(d["dense"]))
    x = gio.bf16(d["x"])
    y = oracle.q4nx_linear(x, data, in_f, out_f)
    assert torch.equal(y.to(torch.bfloat16), gio.bf16(d["y"]))
    with pytest.raises(ValueError):
        oracle.q4nx_dequantize_linear(data[:-1], in_f, out_f)


def test_oracle_dense_cache_and_last_only_prefill_agree_with_the_plain_forms():
    """The two shortcuts the full-size checks use: a linear contracting its
    cached dequantised matrix in one matmul equals the per-group loop of
    model.py:133-146 up to fp32 association, and the last-token prefill
    logits are the last row of the all-token ones."""
    from tests.gpu_util import oracle_decoder
    from torch2iron_b200 import synth
    from torch2iron_b200.config import QuantizedQwenConfig

    cfg = QuantizedQwenConfig(vocab_size=300, emb_dim=256, n_layers=2, n_heads=4, n_kv_groups=2, head_dim=64,
                              hidden_dim=512, rms_norm_eps=1e-6, rope_base=1e6)
    model = synth.random_model(cfg, seed=8)
    prompts = torch.randint(0, cfg.vocab_size, (3, 10), generator=torch.Generator().manual_seed(9))
    full = oracle_decoder(cfg, model, 3, 64).prefill_chunked(prompts, chunk=4)
    fast = oracle_decoder(cfg, model, 3, 64, dense=True).prefill_chunked(prompts, chunk=4, last_only=True)
    assert full.shape == (3, 10, 300) and fast.shape == (3, 300)
    assert torch.allclose(fast, full[:, -1], atol=1e-5, rtol=0)

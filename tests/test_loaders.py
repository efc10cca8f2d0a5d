"""Artifact loaders on the CPU: the reference's packed artifact and the AutoGPTQ
checkpoint it was packed from (``tests/golden/packed_tiny``, written by the
reference's own packer; ``make_packed_artifact.py`` beside it), checked
against the reference model's logits and greedy tokens, against each other,
and for the reference's error behaviour."""

import json
import shutil
from pathlib import Path

import numpy as np
import pytest
import torch
from safetensors.torch import load_file, save_file

import oracle
from tests.gpu_util import oracle_layer, oracle_shape
from torch2iron_b200 import loaders as LD
from torch2iron_b200 import synth
from torch2iron_b200.synth import LINEAR_NAMES, AutoGPTQLinear

GOLD = Path(__file__).resolve().parent / "golden"
MODEL_DIR = GOLD / "packed_tiny"
PACKED_DIR = MODEL_DIR / LD.PACKED_DIRNAME


def _dense(lin: AutoGPTQLinear) -> torch.Tensor:
    return oracle.autogptq_linear_to_dense(lin.qweight, lin.qzeros, lin.scales)


def _golden():
    return np.load(GOLD / "packed_tiny.npz")


def _oracle_decoder(cfg, model, kv_dtype):
    lm = model["lm_head"]
    lm = _dense(lm) if isinstance(lm, AutoGPTQLinear) else (model["embed"] if lm is None else lm)
    return oracle.OracleDecoder(oracle_shape(cfg), [oracle_layer(l, cfg) for l in model["layers"]],
                                embed=model["embed"], final_norm=model["final_norm"], lm_head=lm, max_ctx=64,
                                batch=1, kv_dtype=kv_dtype)


def test_find_packed_dir_from_model_or_artifact_dir(tmp_path):
    assert LD.find_packed_dir(MODEL_DIR) == PACKED_DIR
    assert LD.find_packed_dir(PACKED_DIR) == PACKED_DIR
    assert LD.find_packed_dir(GOLD) == PACKED_DIR              # found below, newest manifest
    assert LD.find_packed_dir(tmp_path) is None


def test_packed_artifact_config_and_heads():
    cfg, model = LD.load_packed_artifact(MODEL_DIR)
    assert (cfg.vocab_size, cfg.emb_dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_groups, cfg.head_dim,
            cfg.hidden_dim) == (512, 256, 2, 4, 2, 64, 512)
    assert cfg.qk_norm and cfg.rope_base == 1e6 and cfg.rms_norm_eps == 1e-6
    cfg.validate()
    # the packer quantized the dense head into a synthetic W4A16 head (packed_format.py:583-648)
    assert isinstance(model["lm_head"], AutoGPTQLinear)
    assert model["lm_head"].scales.dtype == torch.float16
    assert model["embed"].dtype == torch.bfloat16 and model["embed"].shape == (512, 256)


def test_qparam_conversion_is_the_reference_dequant():
    """Each loaded linear dequantizes bit-exactly to the reference runtime's
    ``(nibble - 8) * bf16 scale`` of the raw qparam segment."""
    art = LD.PackedArtifact(PACKED_DIR)
    _, model = LD.load_packed_artifact(MODEL_DIR)
    for li in range(2):
        for name in LINEAR_NAMES:
            prefix = f"model.layers.{li}.{'self_attn' if name.endswith(('q_proj', 'k_proj', 'v_proj', 'o_proj')) else 'mlp'}.{name}"
            spec, qp = art.qparam(prefix)
            k, n = int(spec["in_features"]), int(spec["out_features"])
            packed, scales = oracle.split_qparam(qp, k)
            signed = oracle.unpack_biased_int4(packed, k).to(torch.float32)
            ref = (signed.view(n, -1, 128) * scales.to(torch.float32)[..., None]).view(n, k)
            assert torch.equal(_dense(model["layers"][li][name]), ref), prefix


def test_packed_artifact_matches_reference_logits():
    """The oracle decoder over the loaded weights reproduces the reference
    model's logits (fp32 KV: 1e-4; the GPU's bf16 KV cache: 2e-2), its greedy
    tokens and the logits along them."""
    cfg, model = LD.load_packed_artifact(MODEL_DIR)
    g = _golden()
    prompt, ref = torch.from_numpy(g["prompt"]), torch.from_numpy(g["logits"])
    P = prompt.shape[1]
    for kv, tol in ((torch.float32, 1e-4), (torch.bfloat16, 2e-2)):
        dec = _oracle_decoder(cfg, model, kv)
        lg = torch.stack([dec.step(prompt[:, p], torch.tensor([p]))[0] for p in range(P)])
        assert (lg - ref).abs().max().item() <= tol
        for i, tok in enumerate(g["greedy"][:-1]):           # teacher-forced along the reference's tokens
            lg = dec.step(torch.tensor([int(tok)]), torch.tensor([P + i]))[0]
            assert (lg - torch.from_numpy(g["gen_logits"][i + 1])).abs().max().item() <= tol
    toks = _oracle_decoder(cfg, model, torch.float32).generate(prompt, len(g["greedy"]))
    assert toks[0].tolist() == g["greedy"].tolist()


def test_checkpoint_with_reference_numerics_equals_packed():
    """Loading the AutoGPTQ checkpoint with the packer's numerics gives the
    artifact's weights bit for bit (bf16-rounded scales, quantized head)."""
    _, packed = LD.load_packed_artifact(MODEL_DIR)
    cfg, ckpt = LD.load_autogptq_checkpoint(MODEL_DIR, numerics="reference")
    for li in range(cfg.n_layers):
        for name in LINEAR_NAMES:
            assert torch.equal(_dense(ckpt["layers"][li][name]), _dense(packed["layers"][li][name])), (li, name)
        for nrm in ("input_layernorm", "post_attention_layernorm", "q_norm", "k_norm"):
            assert torch.equal(ckpt["layers"][li][nrm], packed["layers"][li][nrm])
    a, b = ckpt["lm_head"], packed["lm_head"]
    assert torch.equal(a.qweight, b.qweight) and torch.equal(a.scales, b.scales) and torch.equal(a.qzeros, b.qzeros)
    assert torch.equal(ckpt["embed"], packed["embed"]) and torch.equal(ckpt["final_norm"], packed["final_norm"])


def test_checkpoint_numerics_keeps_fp16_scales_and_dense_head(tmp_path):
    cfg, model = LD.load_autogptq_checkpoint(MODEL_DIR, numerics="checkpoint")
    t = load_file(str(MODEL_DIR / "model.safetensors"))
    lin = model["layers"][1]["down_proj"]
    assert torch.equal(lin.scales, t["model.layers.1.mlp.down_proj.scales"])
    assert torch.equal(lin.qweight, t["model.layers.1.mlp.down_proj.qweight"])
    assert torch.equal(model["lm_head"], t["lm_head.weight"]) and not cfg.tie_word_embeddings
    # without a head tensor: tied to the embedding (checkpoint numerics) or the
    # embedding quantized, as the packer does (reference numerics)
    del t["lm_head.weight"]
    save_file(t, str(tmp_path / "model.safetensors"))
    shutil.copy(MODEL_DIR / "config.json", tmp_path)
    cfg, model = LD.load_autogptq_checkpoint(tmp_path, numerics="checkpoint")
    assert model["lm_head"] is None and cfg.tie_word_embeddings
    _, model = LD.load_autogptq_checkpoint(tmp_path)
    q = LD.quantize_head_w4(t["model.embed_tokens.weight"])
    assert torch.equal(model["lm_head"].qweight, q.qweight) and torch.equal(model["lm_head"].scales, q.scales)
    with pytest.raises(ValueError, match="numerics"):
        LD.load_autogptq_checkpoint(MODEL_DIR, numerics="fp8")


def test_sharded_checkpoint_loads_like_single_file(tmp_path):
    t = load_file(str(MODEL_DIR / "model.safetensors"))
    names = sorted(t)
    half = len(names) // 2
    shards = {"model-00001-of-00002.safetensors": names[:half], "model-00002-of-00002.safetensors": names[half:]}
    for fname, keys in shards.items():
        save_file({k: t[k] for k in keys}, str(tmp_path / fname))
    weight_map = {k: f for f, keys in shards.items() for k in keys}
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    shutil.copy(MODEL_DIR / "config.json", tmp_path)
    _, a = LD.load_autogptq_checkpoint(tmp_path)
    _, b = LD.load_autogptq_checkpoint(MODEL_DIR)
    assert torch.equal(_dense(a["layers"][0]["gate_proj"]), _dense(b["layers"][0]["gate_proj"]))
    assert torch.equal(a["lm_head"].qweight, b["lm_head"].qweight)


def test_load_model_prefers_the_artifact(tmp_path):
    cfg, m = LD.load_model(MODEL_DIR)
    assert isinstance(m["lm_head"], AutoGPTQLinear)
    # a checkpoint that was never packed: the reference raises there; this loads it
    shutil.copy(MODEL_DIR / "config.json", tmp_path)
    shutil.copy(MODEL_DIR / "model.safetensors", tmp_path)
    cfg2, m2 = LD.load_model(tmp_path)
    assert torch.equal(_dense(m2["layers"][0]["q_proj"]), _dense(m["layers"][0]["q_proj"]))


# ---- reference error behaviour ---------------------------------------------
def _copy_model(tmp_path) -> Path:
    d = tmp_path / "m"
    shutil.copytree(MODEL_DIR, d)
    return d


def test_rejects_wrong_format_and_quantization(tmp_path):
    d = _copy_model(tmp_path)
    mpath = d / LD.PACKED_DIRNAME / "manifest.json"
    man = json.loads(mpath.read_text())
    man["format"] = "quantized_qwen3_w4a16_inference_v12"
    mpath.write_text(json.dumps(man))
    with pytest.raises(RuntimeError, match="unsupported packed format"):
        LD.PackedArtifact(d / LD.PACKED_DIRNAME)
    assert LD.find_packed_dir(d) is None                      # an unsupported manifest is not found
    cfgj = json.loads((d / "config.json").read_text())
    for bad, msg in (({"bits": 8}, "bits=8"), ({"bits": 4, "sym": False}, "symmetric")):
        cfgj["quantization_config"] = bad
        (d / "config.json").write_text(json.dumps(cfgj))
        with pytest.raises(ValueError, match=msg):
            LD.load_autogptq_checkpoint(d)


def test_rejects_out_of_range_segment_and_config_mismatch(tmp_path):
    d = _copy_model(tmp_path)
    mpath = d / LD.PACKED_DIRNAME / "manifest.json"
    man = json.loads(mpath.read_text())
    man["linears"]["model.layers.1.mlp.down_proj"]["qparam"]["byte_offset"] = man["total_bytes"]
    mpath.write_text(json.dumps(man))
    with pytest.raises(ValueError, match="outside"):
        LD.load_packed_artifact(d)
    man["linears"]["model.layers.1.mlp.down_proj"]["qparam"]["byte_offset"] = 0
    man["model_config"]["hidden_size"] = 512
    mpath.write_text(json.dumps(man))
    with pytest.raises(ValueError, match="hidden_size"):
        LD.load_packed_artifact(d)


def test_rejects_act_order_g_idx(tmp_path):
    d = tmp_path / "c"
    d.mkdir()
    shutil.copy(MODEL_DIR / "config.json", d)
    t = load_file(str(MODEL_DIR / "model.safetensors"))
    k = 256
    t["model.layers.0.self_attn.q_proj.g_idx"] = torch.arange(k, dtype=torch.int32) // 128
    save_file(t, str(d / "model.safetensors"))
    LD.load_autogptq_checkpoint(d)                            # trivial g_idx: accepted
    t["model.layers.0.self_attn.q_proj.g_idx"] = (torch.arange(k, dtype=torch.int32) % 2)
    save_file(t, str(d / "model.safetensors"))
    with pytest.raises(ValueError, match="g_idx"):
        LD.load_autogptq_checkpoint(d)


def test_bf16_scales_outside_fp16_are_rejected_unless_the_group_is_zero():
    n, k = 8, 128
    nib = torch.full((n, k), 9, dtype=torch.uint8)            # q - 8 = 1 everywhere
    packed = nib[:, 0::2] | (nib[:, 1::2] << 4)
    scales = torch.full((n, 1), 0.01, dtype=torch.bfloat16)
    lin = LD.qparam_to_autogptq(torch.cat([packed, scales.view(torch.uint8)], 1), k, n)
    assert torch.equal(_dense(lin), torch.full((n, k), float(scales[0, 0])))
    tiny = scales.clone()
    tiny[3, 0] = 1e-7                                         # below fp16's exact range for bf16 values
    with pytest.raises(ValueError, match="no exact fp16"):
        LD.qparam_to_autogptq(torch.cat([packed, tiny.view(torch.uint8)], 1), k, n)
    packed[3] = 0x88                                          # that row's group is all zero-point: any scale
    lin = LD.qparam_to_autogptq(torch.cat([packed, tiny.view(torch.uint8)], 1), k, n)
    assert torch.equal(_dense(lin)[3], torch.zeros(k))


def test_head_quantizer_is_the_packer_rtn():
    """``quantize_head_w4`` on the fixture's dense head gives the artifact's synthetic head."""
    art = LD.PackedArtifact(PACKED_DIR)
    _, qp = art.qparam("lm_head")
    assert art.manifest["linears"]["lm_head"]["qparam"]["source"] == "lm_head.weight"
    mine = LD.quantize_head_w4(art.dense("lm_head.weight"))
    ref = LD.qparam_to_autogptq(qp, 256, 512)
    assert torch.equal(mine.qweight, ref.qweight) and torch.equal(mine.scales, ref.scales)


@pytest.mark.parametrize("chunk", [12, 5, 1])
def test_oracle_chunked_prefill_matches_reference_forward(chunk):
    """The chunked-prefill restatement (the semantics the GPU prefill implements)
    gives the reference model's full-prompt logits at every position."""
    cfg, model = LD.load_packed_artifact(MODEL_DIR)
    g = _golden()
    prompt, ref = torch.from_numpy(g["prompt"]), torch.from_numpy(g["logits"])
    dec = _oracle_decoder(cfg, model, torch.float32)
    lg = dec.prefill_chunked(prompt, chunk)[0]
    assert lg.shape == ref.shape
    assert (lg - ref).abs().max().item() <= 1e-4


# ---- fast Qwen3 artifact (Q4NX group-32) ------------------------------------
FAST_DIR = MODEL_DIR / LD.FAST_DIRNAME


def test_fast_artifact_linears_match_reference():
    """Every Q4NX linear read by the loader dequantises to the reference's dense
    weight (sha256 of its fp32 bytes) and gives the reference's output on a
    seeded input, through the oracle's Q4NX restatement."""
    import hashlib
    cfg, model = LD.load_fast_qwen3_artifact(MODEL_DIR)
    g = np.load(GOLD / "fast_tiny.npz")
    assert LD.find_fast_dir(MODEL_DIR) == FAST_DIR
    for li in range(cfg.n_layers):
        for name in LINEAR_NAMES:
            prefix = f"model.layers.{li}.{'self_attn' if name in ('q_proj', 'k_proj', 'v_proj', 'o_proj') else 'mlp'}.{name}"
            lin = model["layers"][li][name]
            assert isinstance(lin, LD.Q4NXLinear)
            raw = lin.data.numpy().tobytes()
            dense = oracle.q4nx_dequantize_linear(raw, lin.in_features, lin.out_features)
            assert hashlib.sha256(dense.numpy().tobytes()).hexdigest() == str(g[f"{prefix}.sha256"]), prefix
            x = torch.from_numpy(g[f"{prefix}.x"].view(np.int16)).view(torch.bfloat16)
            y = oracle.q4nx_linear(x, raw, lin.in_features, lin.out_features).to(torch.bfloat16)
            assert torch.equal(y, torch.from_numpy(g[f"{prefix}.y"].view(np.int16)).view(torch.bfloat16)), prefix


def test_fast_artifact_dense_tensors_and_config():
    cfg, fast = LD.load_fast_qwen3_artifact(MODEL_DIR)
    _, packed = LD.load_packed_artifact(MODEL_DIR)
    assert torch.equal(fast["embed"], packed["embed"]) and torch.equal(fast["final_norm"], packed["final_norm"])
    for nrm in ("input_layernorm", "post_attention_layernorm", "q_norm", "k_norm"):
        assert torch.equal(fast["layers"][1][nrm], packed["layers"][1][nrm])
    assert fast["lm_head"].dtype == torch.bfloat16 and not cfg.tie_word_embeddings   # the dense head stays dense
    assert (cfg.emb_dim, cfg.n_layers, cfg.head_dim) == (256, 2, 64)


def test_fast_artifact_errors_and_engine_refusal(tmp_path):
    d = tmp_path / "m"
    shutil.copytree(MODEL_DIR, d)
    mpath = d / LD.FAST_DIRNAME / "manifest.json"
    man = json.loads(mpath.read_text())
    bad = dict(man, format="fast_qwen3_q4nx_layer_v0")
    mpath.write_text(json.dumps(bad))
    with pytest.raises(RuntimeError, match="unsupported fast Qwen3 format"):
        LD.FastArtifact(d / LD.FAST_DIRNAME)
    man["linears"]["model.layers.0.mlp.down_proj"]["byte_length"] -= 16
    mpath.write_text(json.dumps(man))
    with pytest.raises(ValueError, match="layout needs"):
        LD.load_fast_qwen3_artifact(d)
    from torch2iron_b200.engine import DecodeEngine
    cfg, model = LD.load_fast_qwen3_artifact(MODEL_DIR)
    # one weight format per layer: a Q4NX layer with one AutoGPTQ linear is refused before any device work
    mixed = dict(model, layers=[dict(model["layers"][0], o_proj=synth.random_linear(
        cfg.emb_dim, cfg.q_dim, torch.Generator().manual_seed(0)))] + model["layers"][1:])
    with pytest.raises(NotImplementedError, match="one format per layer"):
        DecodeEngine(cfg, mixed, batch=1, max_ctx=64)
    # the tensor-parallel engine refuses before sharding (which reads AutoGPTQ tensors)
    from torch2iron_b200.tp import TPDecodeEngine
    with pytest.raises(NotImplementedError, match="AutoGPTQ"):
        TPDecodeEngine(cfg, model, batch=1, max_ctx=64, tp=1, rank=0)

"""Chunked prefill: the causal prefill attention kernel against an fp32 torch
reference, and the engine's chunked prefill (every linear over all B x chunk
prompt tokens at once) against the one-token-per-step prefill, the oracle and
the reference model's golden logits."""

from pathlib import Path

import numpy as np
import pytest
import torch

from tests.gpu_util import max_abs, oracle_decoder
from torch2iron_b200 import _lib, synth
from torch2iron_b200 import loaders as LD
from torch2iron_b200.config import QuantizedQwenConfig
from torch2iron_b200.engine import DecodeEngine

pytestmark = pytest.mark.gpu

SMALL = QuantizedQwenConfig(vocab_size=512, emb_dim=256, n_layers=2, n_heads=4, n_kv_groups=2, head_dim=64,
                            hidden_dim=512, rms_norm_eps=1e-6, rope_base=1e6)


def _ref_prefill_attention(q, kc, vc, C, p0, nq, nkv, hd):
    B = kc.shape[0]
    qpg = nq // nkv
    q = q.float().view(B, C, nq, hd)
    out = torch.empty(B, C, nq, hd)
    for b in range(B):
        for i in range(C):
            n = p0 + i + 1
            k = kc[b, :, :n].float().repeat_interleave(qpg, 0)          # [nq, n, hd]
            v = vc[b, :, :n].float().repeat_interleave(qpg, 0)
            w = torch.softmax(torch.einsum("hd,hnd->hn", q[b, i], k) / hd ** 0.5, -1)
            out[b, i] = torch.einsum("hn,hnd->hd", w, v)
    return out.view(B * C, nq * hd)


# attention operands N(0, 1): P is rounded to bf16 for the PV product (as in
# flash attention), so the bar is 2e-2 max-abs on outputs of magnitude ~1
@pytest.mark.parametrize("B,C,p0,nq,nkv,hd,max_ctx", [
    (2, 40, 0, 4, 2, 64, 128),       # one chunk from position 0, partial CTA
    (1, 37, 70, 4, 1, 128, 128),     # a later chunk: keys before and inside it
    (3, 64, 64, 16, 8, 128, 192),    # Qwen3-0.6B heads
    (2, 16, 5, 32, 8, 64, 64),       # Llama-3.2-1B heads (qpg 4)
    (1, 1, 0, 2, 1, 128, 64),        # a single token
])
def test_prefill_attention_vs_torch(B, C, p0, nq, nkv, hd, max_ctx):
    g = torch.Generator().manual_seed(B * 1000 + C + p0)
    q = torch.randn(B * C, nq * hd, generator=g).to(torch.bfloat16)
    kc = torch.randn(B, nkv, max_ctx, hd, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, nkv, max_ctx, hd, generator=g).to(torch.bfloat16)
    qd, kd, vd = q.cuda(), kc.cuda(), vc.cuda()
    ref = _ref_prefill_attention(q, kc, vc, C, p0, nq, nkv, hd)
    for dt in (torch.bfloat16, torch.float16):      # reference-style bf16, and the fused layer's fp16
        out = torch.full((B * C, nq * hd), float("nan"), dtype=dt, device="cuda")
        _lib.call("t2b_prefill_attention", _lib.ptr(qd), _lib.ptr(kd), _lib.ptr(vd), _lib.ptr(out), _lib.DTYPE[dt], B,
                  C, p0, nq, nkv, hd, max_ctx, _lib.stream())
        torch.cuda.synchronize()
        assert not torch.isnan(out.float()).any()
        assert max_abs(out, ref) <= 2e-2


def test_prefill_attention_rejects_bad_shapes():
    t = torch.zeros(64, dtype=torch.bfloat16, device="cuda")
    L = _lib.lib()
    p = _lib.ptr(t)
    assert L.t2b_prefill_attention(p, p, p, p, 0, 1, 8, 60, 4, 2, 64, 64, None) != 0     # p0 + C > max_ctx
    assert L.t2b_prefill_attention(p, p, p, p, 0, 1, 8, 0, 4, 2, 96, 64, None) != 0      # head_dim
    assert L.t2b_prefill_attention(p, p, p, p, 0, 1, 8, 0, 6, 4, 64, 64, None) != 0      # heads not a multiple
    assert L.t2b_prefill_attention(p, p, p, p, 2, 1, 8, 0, 4, 2, 64, 64, None) == 6      # fp32 output


@pytest.mark.parametrize("chunk", [None, 16])
def test_chunked_prefill_matches_stepwise_and_oracle(chunk):
    cfg = SMALL
    model = synth.random_model(cfg, seed=41)
    B, P = 3, 37
    prompts = torch.randint(0, cfg.vocab_size, (B, P), generator=torch.Generator().manual_seed(42))
    a = DecodeEngine(cfg, model, batch=B, max_ctx=64, use_graph=False)
    a.prefill(prompts, chunk=chunk)
    b = DecodeEngine(cfg, model, batch=B, max_ctx=64, use_graph=False)
    b.prefill(prompts, stepwise=True)
    torch.cuda.synchronize()
    assert int(a.err.item()) == 0
    for li in range(cfg.n_layers):
        assert max_abs(a.k_cache[li][:, :, :P], b.k_cache[li][:, :, :P]) <= 5e-2
        assert max_abs(a.v_cache[li][:, :, :P], b.v_cache[li][:, :, :P]) <= 5e-2
        assert a.k_cache[li][:, :, P:].abs().max().item() == 0          # nothing written past the prompt
    assert max_abs(a.logits, b.logits) <= 2e-2
    ref = oracle_decoder(cfg, model, B, 64).prefill(prompts)
    assert max_abs(a.logits, ref) <= 2e-2
    top = torch.topk(ref, 2, dim=-1).values
    sure = (top[:, 0] - top[:, 1]) > 4e-2
    assert torch.equal(a.next_tokens.cpu().long()[sure], ref.argmax(-1)[sure])
    # decoding continues from the chunked prefill as from the stepwise one (same next token fed)
    a.tokens.copy_(b.tokens)
    a.advance()
    b.advance()
    assert max_abs(a.logits, b.logits) <= 2e-2


@pytest.mark.parametrize("B,P,force", [(8, 40, False), (3, 37, True)])
def test_chunked_prefill_large_m_kernel(monkeypatch, B, P, force):
    """Chunks of >= 257 prompt tokens (or any, forced) run every fused linear on
    the large-M tcgen05 kernel: same caches and logits as the stepwise prefill."""
    cfg = SMALL
    model = synth.random_model(cfg, seed=43)
    prompts = torch.randint(0, cfg.vocab_size, (B, P), generator=torch.Generator().manual_seed(44))
    b = DecodeEngine(cfg, model, batch=B, max_ctx=64, use_graph=False)
    b.prefill(prompts, stepwise=True)
    if force:
        monkeypatch.setenv("T2B_PREFILL_MIN_M", "1")
    a = DecodeEngine(cfg, model, batch=B, max_ctx=64, use_graph=False)
    a.prefill(prompts)
    torch.cuda.synchronize()
    assert int(a.err.item()) == 0
    for li in range(cfg.n_layers):
        assert max_abs(a.k_cache[li][:, :, :P], b.k_cache[li][:, :, :P]) <= 5e-2
        assert max_abs(a.v_cache[li][:, :, :P], b.v_cache[li][:, :, :P]) <= 5e-2
    assert max_abs(a.logits, b.logits) <= 2e-2
    assert max_abs(a.x, b.x) <= 2e-2 * b.x.abs().max().item()


def test_chunked_prefill_on_reference_artifact():
    """The packed artifact's model: logits after the prompt against the reference model's."""
    model_dir = Path(__file__).resolve().parent / "golden" / "packed_tiny"
    cfg, model = LD.load_packed_artifact(model_dir)
    g = np.load(model_dir.parent / "packed_tiny.npz")
    prompt = torch.from_numpy(g["prompt"])
    eng = DecodeEngine(cfg, model, batch=1, max_ctx=64, use_graph=True)
    eng.prefill(prompt, chunk=5)
    torch.cuda.synchronize()
    assert max_abs(eng.logits[0], torch.from_numpy(g["logits"][-1])) <= 2e-2
    eng.check_device_errors()


@pytest.mark.parametrize("force_large_m,reuse", [(False, False), (True, False), (False, True)])
def test_ragged_prompts_match_per_sequence_oracle(monkeypatch, force_large_m, reuse):
    """Right-padded prompts of lengths 5, 13 and 9: each row's greedy head and
    its continued decode match the oracle run on that sequence alone (chunk
    linears on the decode tcgen05 kernel, or forced onto the large-M kernel).
    ``reuse``: the engine first generates from other, full-length prompts, so
    the cache slots past each ragged length hold that run's keys and values
    (the padded positions read them, masked, and must not disturb the rows)."""
    if force_large_m:
        monkeypatch.setenv("T2B_PREFILL_MIN_M", "12")   # the 12-row chunks, not the 3-row decode step
    cfg = SMALL
    model = synth.random_model(cfg, seed=45)
    lens = [5, 13, 9]
    B, P = len(lens), max(lens)
    prompts = torch.randint(0, cfg.vocab_size, (B, P), generator=torch.Generator().manual_seed(46))
    eng = DecodeEngine(cfg, model, batch=B, max_ctx=64, use_graph=False)
    if reuse:
        other = torch.randint(0, cfg.vocab_size, (B, P), generator=torch.Generator().manual_seed(47))
        eng.generate(other, 8)
        torch.cuda.synchronize()
    eng.prefill(prompts, chunk=4, lengths=lens)
    torch.cuda.synchronize()
    assert eng.pos.cpu().tolist() == lens
    first = eng.logits.cpu().clone()
    eng.tokens.copy_(torch.tensor([7, 8, 9], dtype=torch.int32))   # fixed next inputs for a decode step
    eng.run_step()
    second = eng.logits.cpu().clone()
    eng.check_device_errors()
    for b, n in enumerate(lens):
        dec = oracle_decoder(cfg, model, 1, 64)
        ref = dec.prefill(prompts[b:b + 1, :n])
        assert max_abs(first[b], ref[0]) <= 2e-2, b
        ref2 = dec.step(torch.tensor([7 + b]), torch.tensor([n]))
        assert max_abs(second[b], ref2[0]) <= 2e-2, b
    with pytest.raises(ValueError):
        eng.prefill(prompts, lengths=[0, 13, 9])
    with pytest.raises(ValueError):
        eng.prefill(prompts, stepwise=True, lengths=lens)

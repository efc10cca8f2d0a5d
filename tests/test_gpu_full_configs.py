"""The decode criteria at the benchmark configurations' full size.

Bars: decoder logits within 2e-2 max-abs of the reference path and greedy
tokens agreeing on >= 99 % of the steps, checked teacher-forced (every step
of the engine is fed the oracle's previous greedy token, so one disagreement
cannot derail the steps after it).  The oracle restates the reference's
``QuantizedQwenForCausalLM.forward`` / ``generate`` (``model.py:453-498``) in
fp32 on the host, over the same seeded synthetic weights.

* configuration 2: Qwen3-0.6B (28 layers, vocab 151936, tied bf16 head),
  128-token prompts, 8 rows x 128 generated tokens and 64 rows x 16;
* configuration 3: Llama-3.2-1B (16 layers, vocab 128256, head_dim 64, no
  QK-norm), 32 rows over a KV cache pre-filled to a 2048-token context
  (N(0,1) bf16, the same values in both), 16 steps.

Each case prints its worst logit error and the agreement.
"""

import pytest
import torch

from tests.gpu_util import oracle_decoder
from torch2iron_b200 import synth
from torch2iron_b200.config import LLAMA_3_2_1B, QWEN3_0_6B
from torch2iron_b200.engine import DecodeEngine

pytestmark = pytest.mark.gpu

LOGIT_BAR = 2e-2
AGREE_BAR = 0.99


def _cpu_model(model: dict) -> dict:
    out = {"layers": [], "embed": model["embed"].cpu(), "final_norm": model["final_norm"].cpu(),
           "lm_head": None if model.get("lm_head") is None else model["lm_head"].cpu()}
    for layer in model["layers"]:
        out["layers"].append({k: (v.to("cpu") if hasattr(v, "to") else v) for k, v in layer.items()})
    return out


def _teacher_forced(eng, dec, first_logits_ref, first_logits, pos0: int, steps: int, checks: set):
    """Steps 1..steps-1 fed the oracle's previous greedy token; returns
    (agreement, worst logit error at the checked steps)."""
    B = eng.B
    ref_tok = torch.argmax(first_logits_ref, -1)
    hits = int((eng.next_tokens.cpu().long() == ref_tok).sum())
    worst = float((first_logits - first_logits_ref).abs().max()) if 0 in checks else 0.0
    for t in range(1, steps):
        pos = torch.full((B,), pos0 + t - 1, dtype=torch.long)
        ref_logits = dec.step(ref_tok, pos)
        eng.tokens.copy_(ref_tok.to(torch.int32))
        eng.pos.copy_(pos.to(torch.int32))
        eng.run_step()
        got = eng.next_tokens.cpu().long()
        ref_tok = torch.argmax(ref_logits, -1)
        hits += int((got == ref_tok).sum())
        if t in checks:
            worst = max(worst, float((eng.logits.cpu() - ref_logits).abs().max()))
    eng.check_device_errors()
    return hits / (B * steps), worst


@pytest.mark.parametrize("batch,steps", [(8, 128), (64, 16)])
def test_config2_qwen3_0_6b_full_model(batch, steps):
    cfg, P = QWEN3_0_6B, 128
    model = synth.random_model(cfg, seed=2024, device="cuda")
    prompts = torch.randint(0, cfg.vocab_size, (batch, P), generator=torch.Generator().manual_seed(2025))
    max_ctx = ((P + steps + 63) // 64) * 64
    eng = DecodeEngine(cfg, model, batch=batch, max_ctx=max_ctx, use_graph=True, keep_logits=True)
    eng.prefill(prompts)
    torch.cuda.synchronize()
    first = eng.logits.cpu().clone()
    dec = oracle_decoder(cfg, _cpu_model(model), batch, max_ctx, dense=True)
    del model
    first_ref = dec.prefill_chunked(prompts, chunk=P, last_only=True)
    checks = {0, steps // 4, steps // 2, steps - 1}
    agree, worst = _teacher_forced(eng, dec, first_ref, first, P, steps, checks)
    print(f"\nconfig2 B={batch} steps={steps}: agreement {agree:.4f}, worst logit error {worst:.2e} "
          f"(steps {sorted(checks)}), logit range {float(first_ref.abs().max()):.3f}")
    assert worst <= LOGIT_BAR
    assert agree >= AGREE_BAR


def test_config3_llama_3_2_1b_full_model():
    cfg, B, ctx, steps = LLAMA_3_2_1B, 32, 2048, 16
    model = synth.random_model(cfg, seed=3031, device="cuda")
    max_ctx = ((ctx + steps + 63) // 64) * 64
    eng = DecodeEngine(cfg, model, batch=B, max_ctx=max_ctx, use_graph=True, keep_logits=True)
    dec = oracle_decoder(cfg, _cpu_model(model), B, max_ctx, dense=True)
    del model
    g = torch.Generator(device="cuda").manual_seed(3032)
    for li in range(cfg.n_layers):            # the same N(0,1) bf16 context in both caches
        for cache, ref in ((eng.k_cache[li], dec.k_cache[li]), (eng.v_cache[li], dec.v_cache[li])):
            cache[:, :, :ctx].normal_(generator=g)
            ref[:, :, :ctx].copy_(cache[:, :, :ctx].cpu())
    tok = torch.randint(0, cfg.vocab_size, (B,), generator=torch.Generator().manual_seed(3033))
    eng.tokens.copy_(tok.to(torch.int32))
    eng.pos.fill_(ctx)
    eng.run_step()
    torch.cuda.synchronize()
    first = eng.logits.cpu().clone()
    first_ref = dec.step(tok, torch.full((B,), ctx, dtype=torch.long))
    checks = {0, steps // 2, steps - 1}
    agree, worst = _teacher_forced(eng, dec, first_ref, first, ctx + 1, steps, checks)
    print(f"\nconfig3 B={B} ctx={ctx} steps={steps}: agreement {agree:.4f}, worst logit error {worst:.2e} "
          f"(steps {sorted(checks)}), logit range {float(first_ref.abs().max()):.3f}")
    assert worst <= LOGIT_BAR
    assert agree >= AGREE_BAR

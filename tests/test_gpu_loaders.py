"""The decode engine on weights loaded from the reference's own artifacts
(``tests/golden/packed_tiny``): logits against the reference model's over the
prompt and teacher-forced along its greedy tokens (2e-2 max-abs, the
decoder-logit bar), and its greedy picks wherever the reference's top-2
margin exceeds twice that bar, through the W4A16 lm_head path (the
artifact's quantized head); and the checkpoint's own numerics (bf16 head)
against the oracle."""

from pathlib import Path

import numpy as np
import pytest
import torch

from tests.gpu_util import max_abs, oracle_decoder
from torch2iron_b200 import loaders as LD

pytestmark = pytest.mark.gpu

MODEL_DIR = Path(__file__).resolve().parent / "golden" / "packed_tiny"
LOGIT_TOL = 2e-2


def _golden():
    return np.load(MODEL_DIR.parent / "packed_tiny.npz")


def _teacher_forced(eng, tokens, positions):
    """Run one step per (token, position) on every row; returns the fp32 logits per step."""
    out = []
    for tok, p in zip(tokens, positions):
        eng.tokens.fill_(int(tok))
        eng.pos.fill_(int(p))
        eng.run_step()
        out.append((eng.logits.cpu().clone(), eng.next_tokens.cpu().clone()))
    return out


@pytest.mark.parametrize("use_graph", [False, True])
def test_engine_on_packed_artifact_matches_reference(use_graph):
    from torch2iron_b200.engine import DecodeEngine
    cfg, model = LD.load_packed_artifact(MODEL_DIR)
    g = _golden()
    prompt, greedy = g["prompt"][0], g["greedy"]
    P = len(prompt)
    B = 3                                                   # the same sequence on every row
    eng = DecodeEngine(cfg, model, batch=B, max_ctx=64, use_graph=use_graph)
    assert eng.lm_w4 is not None and eng.kernels_per_step() == 1 + 5 * cfg.n_layers + 1 + 2
    toks = list(prompt) + list(greedy[:-1])
    ref = [torch.from_numpy(r) for r in g["logits"]] + [torch.from_numpy(r) for r in g["gen_logits"][1:]]
    steps = _teacher_forced(eng, toks, range(len(toks)))
    eng.check_device_errors()
    picks = 0
    for i, ((lg, nxt), r) in enumerate(zip(steps, ref)):
        for row in range(B):
            assert max_abs(lg[row], r) <= LOGIT_TOL, (i, row)
        top = torch.topk(r, 2).values
        if i >= P - 1 and float(top[0] - top[1]) > 2 * LOGIT_TOL:
            assert (nxt.long() == int(greedy[i - P + 1])).all(), i
            picks += 1
    assert picks >= 3
    eng.release()


def test_engine_on_checkpoint_numerics_matches_oracle():
    from torch2iron_b200.engine import DecodeEngine
    cfg, model = LD.load_autogptq_checkpoint(MODEL_DIR, numerics="checkpoint")
    prompt = torch.from_numpy(_golden()["prompt"])
    eng = DecodeEngine(cfg, model, batch=1, max_ctx=64, use_graph=True)
    assert eng.lm_w4 is None
    ora = oracle_decoder(cfg, model, batch=1, max_ctx=64)
    for p in range(prompt.shape[1]):
        eng.tokens.fill_(int(prompt[0, p]))
        eng.pos.fill_(p)
        eng.run_step()
        ref = ora.step(prompt[:, p], torch.tensor([p]))
        assert max_abs(eng.logits.cpu()[0], ref[0]) <= LOGIT_TOL, p
    eng.check_device_errors()
    eng.release()

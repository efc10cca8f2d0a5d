"""The decode engine on weights loaded from the reference's own artifacts
(``tests/golden/packed_tiny``): per-position logits against the reference
model's (2e-2 max-abs, the decoder-logit bar) and its greedy tokens, through
the W4A16 lm_head path (the artifact's quantized head) and through the bf16
tied head (the checkpoint's numerics, against the oracle)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from tests.gpu_util import max_abs, oracle_decoder
from torch2iron_b200 import loaders as LD

pytestmark = pytest.mark.gpu

MODEL_DIR = Path(__file__).resolve().parent / "golden" / "packed_tiny"


def _golden():
    g = np.load(MODEL_DIR.parent / "packed_tiny.npz")
    return torch.from_numpy(g["prompt"]), torch.from_numpy(g["logits"]), g["greedy"].tolist()


@pytest.mark.parametrize("use_graph", [False, True])
def test_engine_on_packed_artifact_matches_reference(use_graph):
    from torch2iron_b200.engine import DecodeEngine
    cfg, model = LD.load_packed_artifact(MODEL_DIR)
    prompt, ref, greedy = _golden()
    B = 3                                                   # the same prompt on every row
    eng = DecodeEngine(cfg, model, batch=B, max_ctx=64, use_graph=use_graph)
    assert eng.lm_w4 is not None and eng.kernels_per_step() == 1 + 5 * cfg.n_layers + 1 + 2
    for p in range(prompt.shape[1]):
        eng.tokens.fill_(int(prompt[0, p]))
        eng.pos.fill_(p)
        eng.run_step()
        lg = eng.logits.cpu()
        for r in range(B):
            assert max_abs(lg[r], ref[p]) <= 2e-2, (p, r)
    eng.tokens.copy_(eng.next_tokens)
    eng.pos.fill_(prompt.shape[1])
    toks = [eng.next_tokens.cpu().clone()]
    for _ in range(len(greedy) - 1):
        eng.advance()
        toks.append(eng.next_tokens.cpu().clone())
    eng.check_device_errors()
    got = torch.stack(toks, 1)
    for r in range(B):
        assert got[r].tolist() == greedy
    eng.release()


def test_engine_on_checkpoint_numerics_matches_oracle():
    from torch2iron_b200.engine import DecodeEngine
    cfg, model = LD.load_autogptq_checkpoint(MODEL_DIR, numerics="checkpoint")
    prompt, _, _ = _golden()
    eng = DecodeEngine(cfg, model, batch=1, max_ctx=64, use_graph=True)
    assert eng.lm_w4 is None
    ora = oracle_decoder(cfg, model, batch=1, max_ctx=64)
    for p in range(prompt.shape[1]):
        eng.tokens.fill_(int(prompt[0, p]))
        eng.pos.fill_(p)
        eng.run_step()
        ref = ora.step(prompt[:, p], torch.tensor([p]))
        assert max_abs(eng.logits.cpu()[0], ref[0]) <= 2e-2, p
    eng.check_device_errors()
    eng.release()

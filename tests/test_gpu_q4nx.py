"""Q4NX group-32 weights (the fast Qwen3 artifact, ``fast_qwen3/q4nx_layout.py``)
on the three linear kernels and through the decode engine.

* every linear of the reference-written fixture
  (``tests/golden/packed_tiny/fast_qwen3_q4nx``) against the reference's own
  output (``FastQwen3Store.linear_reference``, recorded in ``fast_tiny.npz``;
  bf16 there, hence 1e-2) and against the oracle's fp32 dequantisation: the
  CUDA-core path computes (q - zero) * scale in fp32 as the reference does
  (1e-4), the tcgen05 and large-M paths round the weight to bf16 once (1e-2);
* Qwen3-0.6B shapes with seeded random nibbles, scales and fractional zero
  points, on each path;
* the decode engine on the fixture model, teacher-forced, logits within 2e-2
  of the oracle decoder over the same Q4NX weights.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from tests.gpu_util import max_abs, oracle_decoder, rel_err
from tests import golden_io as gio
from torch2iron_b200 import _lib
from torch2iron_b200 import loaders as LD
from torch2iron_b200 import weights as W

pytestmark = pytest.mark.gpu

MODEL_DIR = Path(__file__).resolve().parent / "golden" / "packed_tiny"
PATHS = {"cuda_core": ({"T2B_TC_MIN_M": "1000000", "T2B_PREFILL_MIN_M": "1000000"}, 1e-4),
         "tcgen05": ({}, 1e-2),
         "large_m": ({"T2B_PREFILL_MIN_M": "1"}, 1e-2)}


def _gemm(w: W.W4Weight, x: torch.Tensor) -> torch.Tensor:
    M, K = x.shape
    N = w.out_features
    y = torch.empty(M, N, dtype=torch.float32, device="cuda")
    L = _lib.lib()
    n = max(L.t2b_w4a16_gemm_workspace_bytes(M, N, K), 256)
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    _lib.call("t2b_w4a16_gemm", _lib.ptr(w.qw), _lib.ptr(w.meta), _lib.WFMT_Q4NX, _lib.ptr(x), _lib.DTYPE[x.dtype],
              _lib.ptr(y), _lib.DTYPE[y.dtype], M, N, K, 32, _lib.ptr(ws), n, _lib.stream())
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("path", sorted(PATHS))
def test_fixture_linears_match_reference(monkeypatch, path):
    env, bar = PATHS[path]
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    art = LD.FastArtifact(LD.find_fast_dir(MODEL_DIR))
    g = np.load(MODEL_DIR.parent / "fast_tiny.npz")
    names = sorted({k.rsplit(".", 1)[0] for k in g.files})
    assert len(names) == 14
    for name in names:
        lin = art.linear(name)
        w = W.from_q4nx(lin)
        x = gio.bf16(g[f"{name}.x"])
        y = _gemm(w, x.cuda())
        dense = W.dequantize(w).cpu()
        assert torch.equal(dense, __import__("oracle").q4nx_dequantize_linear(lin.data.numpy().tobytes(),
                                                                              lin.in_features, lin.out_features))
        assert rel_err(y, x.float() @ dense.t()) <= bar, name
        assert rel_err(y, gio.bf16(g[f"{name}.y"]).float()) <= 1e-2, name


@pytest.mark.parametrize("path", sorted(PATHS))
@pytest.mark.parametrize("M,N,K", [(1, 4096, 1024), (4, 1024, 3072), (64, 6144, 1024), (300, 1024, 2048)])
def test_synthetic_q4nx_shapes(monkeypatch, path, M, N, K):
    env, bar = PATHS[path]
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    gen = torch.Generator().manual_seed(M * 31 + N + K)
    q = torch.randint(0, 16, (N, K), generator=gen, dtype=torch.int64).to(torch.uint8)
    scale = (torch.rand(N, K // 32, generator=gen) * 0.004 + 0.001).to(torch.bfloat16)
    zero = (torch.rand(N, K // 32, generator=gen) * 15).to(torch.bfloat16)       # fractional zero points
    w = W.from_q4nx_parts(q.cuda(), scale.cuda(), zero.cuda())
    dense = (q.float() - zero.float().repeat_interleave(32, 1)) * scale.float().repeat_interleave(32, 1)
    x = torch.randn(M, K, generator=gen).to(torch.bfloat16)
    y = _gemm(w, x.cuda())
    assert rel_err(y, x.float() @ dense.t()) <= bar


def test_engine_on_fast_artifact_matches_oracle():
    from torch2iron_b200.engine import DecodeEngine
    cfg, model = LD.load_fast_qwen3_artifact(MODEL_DIR)
    prompt = torch.from_numpy(np.load(MODEL_DIR.parent / "packed_tiny.npz")["prompt"])
    B = 2
    for use_graph in (False, True):
        eng = DecodeEngine(cfg, model, batch=B, max_ctx=64, use_graph=use_graph)
        assert eng.layers[0].qkv.fmt == W.WFMT_Q4NX
        ora = oracle_decoder(cfg, model, batch=B, max_ctx=64)
        for p in range(prompt.shape[1]):
            tok = torch.full((B,), int(prompt[0, p]))
            eng.tokens.copy_(tok.to(torch.int32))
            eng.pos.fill_(p)
            eng.run_step()
            ref = ora.step(tok, torch.full((B,), p))
            assert max_abs(eng.logits.cpu(), ref) <= 2e-2, (use_graph, p)
        eng.check_device_errors()
        eng.release()
    # the chunked prefill over the same weights (large-M and tcgen05 kernels on Q4NX)
    eng = DecodeEngine(cfg, model, batch=B, max_ctx=64, use_graph=True)
    eng.prefill(prompt.expand(B, -1).contiguous(), chunk=5)
    torch.cuda.synchronize()
    assert max_abs(eng.logits.cpu(), ref) <= 2e-2
    eng.check_device_errors()

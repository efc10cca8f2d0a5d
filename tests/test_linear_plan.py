"""Launch plans of every W4A16 linear the decode paths run (CPU: the planner
is host code behind ``t2b_linear_plan``).  On the tcgen05 path each CTA of a
split-K cluster finishes ``Bp / KS`` batch rows and expects the other
``(KS - 1) * Bp / KS`` rows from its peers, so KS must divide Bp; a plan
that broke this (KS = 3 for K = 1536, the Qwen3-8B down projection at TP8)
left a receive barrier one row short of its expected bytes."""

import ctypes as C

import pytest

from torch2iron_b200 import _lib
from torch2iron_b200 import tp as TP
from torch2iron_b200.config import LLAMA_3_2_1B, QWEN3_0_6B, QWEN3_8B

BATCHES = [1, 2, 3, 4, 5, 7, 8, 9, 12, 16, 17, 24, 31, 32, 33, 48, 63, 64, 65, 96, 128, 129, 192, 200, 256,
           257, 1000, 8192]   # the last three: prefill chunks (large-M kernel)


def _plan(M, N, K, qkv=False):
    out = [C.c_int() for _ in range(4)]
    f = _lib.load().t2b_linear_plan_qkv if qkv else _lib.load().t2b_linear_plan
    st = f(M, N, K, *[C.byref(v) for v in out])
    return st, tuple(v.value for v in out)


def _linears(cfg, tp):
    lc = TP.local_config(cfg, tp) if tp > 1 else cfg
    h = cfg.emb_dim
    return {"qkv": ((lc.n_heads + 2 * lc.n_kv_groups) * lc.head_dim, h), "o": (h, lc.n_heads * lc.head_dim),
            "gate_up": (2 * lc.hidden_dim, h), "down": (h, lc.hidden_dim)}


CASES = [(c, t) for c, tps in ((QWEN3_0_6B, (1, 2)), (LLAMA_3_2_1B, (1, 2, 4, 8)), (QWEN3_8B, (1, 2, 4, 8)))
         for t in tps]


@pytest.mark.parametrize("cfg,tp", CASES, ids=[f"{c.emb_dim}-{c.n_layers}-tp{t}" for c, t in CASES])
def test_plans_cover_k_and_split_the_batch_tile_evenly(cfg, tp):
    plans = [(name, n, k, False) for name, (n, k) in _linears(cfg, tp).items()]
    plans.append(("qkv (fused)",) + _linears(cfg, tp)["qkv"] + (True,))
    for name, n, k, qkv in plans:
        for m in BATCHES:
            st, (path, rows, groups, ks) = _plan(m, n, k, qkv)
            assert st == _lib.T2B_OK, (name, m, n, k)
            assert groups * ks * 128 == k, (name, m, n, k, rows, groups, ks)
            if path == 2:   # prefill chunks, or decode batches on linears too wide for one tcgen05 wave
                assert rows == 128 and ks == 1 and (m >= 257 or (m >= 16 and not qkv))
            elif path == 1:
                assert rows in (16, 32, 64, 128, 256) and 1 <= ks <= 8 and rows % ks == 0, (name, m, n, k, rows, ks)
            else:
                assert path == 0 and rows in (1, 2, 4, 8) and rows >= min(m, 8)


def test_qwen3_8b_tp8_down_projection_plan():
    """K = 1536 (12 groups): 3 groups per CTA in clusters of 4, not 4 groups in clusters of 3."""
    assert _plan(64, 4096, 1536) == (_lib.T2B_OK, (1, 64, 3, 4))


def test_qkv_plan_caps_rows_per_cta():
    """The fused qkv launch of Qwen3-0.6B at 64 rows: 32-row tiles, 2 groups per CTA in
    clusters of 4 (8 rows per CTA); the generic plan keeps 64-row tiles in clusters of 2."""
    assert _plan(64, 4096, 1024, qkv=True) == (_lib.T2B_OK, (1, 32, 2, 4))
    assert _plan(64, 4096, 1024) == (_lib.T2B_OK, (1, 64, 4, 2))
    for m in (1, 8):   # the CUDA-core path is the same plan
        assert _plan(m, 4096, 1024, qkv=True) == _plan(m, 4096, 1024)


def test_wide_decode_linears_take_the_large_m_kernel():
    """Qwen3-8B gate/up (N 24576) and down (K 12288) at 64 rows: the tcgen05 decode grid
    would run 1536 / 1024 CTAs of one weight-tile slice each; the persistent large-M kernel
    streams whole tiles instead.  o_proj (256 CTAs) stays on the decode kernel, and the fused
    qkv (fp32 q) never moves."""
    assert _plan(64, 24576, 4096)[1][0] == 2
    assert _plan(64, 4096, 12288)[1][0] == 2
    assert _plan(64, 4096, 4096)[1][0] == 1
    assert _plan(64, 24576, 4096, qkv=True)[1][0] == 1
    assert _plan(8, 24576, 4096)[1][0] == 1    # fewer than 16 rows stay on the decode kernel


def test_plan_rejects_bad_shapes():
    assert _plan(1, 100, 1024)[0] != _lib.T2B_OK
    assert _plan(1, 128, 1000)[0] != _lib.T2B_OK
    assert _plan(0, 128, 1024)[0] != _lib.T2B_OK

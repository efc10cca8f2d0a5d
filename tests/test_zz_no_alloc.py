"""The no-allocation GEMM entry point against the allocating one.

``t2b_w4a16_gemm_noalloc`` serves callers that cannot allocate device memory
(a host runtime that owns the device heap, or a thread where cudaMalloc could
block): its split-K scratch is a fixed array inside the library.  These tests
call it through the C ABI on shapes whose CUDA-core path splits K (so the
scratch is really used), twice in a row (the array keeps the previous
call's contents), and compare with ``t2b_w4a16_gemm`` given a workspace the
caller allocated.  The file is named to be collected last.
"""

import pytest
import torch

import oracle
from tests.gpu_util import rel_err
from torch2iron_b200 import _lib, synth
from torch2iron_b200 import weights as W

pytestmark = pytest.mark.gpu


def _allocating(w, x):
    M, K = x.shape
    N = w.out_features
    y = torch.empty(M, N, dtype=torch.float32, device="cuda")
    L = _lib.lib()
    n = max(L.t2b_w4a16_gemm_workspace_bytes(M, N, K), 256)
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    _lib.call("t2b_w4a16_gemm", _lib.ptr(w.qw), _lib.ptr(w.meta), _lib.WFMT_T2B, _lib.ptr(x), _lib.DTYPE[x.dtype],
              _lib.ptr(y), _lib.DTYPE[y.dtype], M, N, K, 128, _lib.ptr(ws), n, _lib.stream())
    torch.cuda.synchronize()
    return y


def _noalloc(w, x):
    M, K = x.shape
    N = w.out_features
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    _lib.call("t2b_w4a16_gemm_noalloc", _lib.ptr(w.qw), _lib.ptr(w.meta), _lib.WFMT_T2B, _lib.ptr(x),
              _lib.DTYPE[x.dtype], _lib.ptr(y), _lib.DTYPE[y.dtype], M, N, K, 128, _lib.stream())
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("M,N,K,needs_ws", [
    (1, 1024, 3072, False), (4, 4096, 1024, False), (8, 1024, 2048, False), (3, 6144, 1024, False),  # cluster split-K
    (1, 1024, 12288, True), (2, 512, 16384, True),     # more k-slices than a cluster holds: workspace split-K
])
def test_noalloc_matches_allocating_entry_point(monkeypatch, M, N, K, needs_ws):
    monkeypatch.setenv("T2B_TC_MIN_M", "16")   # keep these row counts on the split-K CUDA-core path
    L = _lib.lib()
    n = L.t2b_w4a16_gemm_workspace_bytes(M, N, K)
    assert n <= L.t2b_w4a16_gemm_noalloc_max_workspace()
    assert (n > 0) == needs_ws
    g = torch.Generator().manual_seed(M * 131 + N + K)
    lin = synth.random_linear(N, K, g)
    w = W.from_autogptq(lin)
    torch.cuda.synchronize()
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    ref = _allocating(w, x)
    assert rel_err(ref, oracle.GroupedW4A16Linear(lin.qweight, lin.qzeros, lin.scales)(x.float().cpu())) <= 1e-4
    for _ in range(2):
        y = _noalloc(w, x)
        assert not torch.isnan(y).any()
        assert rel_err(y, ref) <= 1e-4


def test_noalloc_takes_the_tcgen05_path_without_scratch():
    """Batch rows on the tcgen05 path need no scratch at any K: a Qwen3-8B down
    projection at 64 rows (K = 12288, more than the CUDA-core path could hold)
    runs and matches the allocating entry point."""
    M, N, K = 64, 1024, 12288
    L = _lib.lib()
    import ctypes as C
    path, rows, groups, ks = C.c_int(), C.c_int(), C.c_int(), C.c_int()
    assert L.t2b_linear_plan(M, N, K, C.byref(path), C.byref(rows), C.byref(groups), C.byref(ks)) == 0
    assert path.value == 1
    g = torch.Generator().manual_seed(77)
    lin = synth.random_linear(N, K, g)
    w = W.from_autogptq(lin)
    torch.cuda.synchronize()
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    ref = _allocating(w, x)
    for _ in range(2):
        assert rel_err(_noalloc(w, x), ref) <= 1e-4


def test_noalloc_rejects_sizes_beyond_its_scratch(monkeypatch):
    import ctypes as C
    monkeypatch.setenv("T2B_TC_MIN_M", "16")   # 8 rows on the CUDA-core split-K path
    L = _lib.lib()
    cap = L.t2b_w4a16_gemm_noalloc_max_workspace()
    M, N, K = 8, 65536, 16384         # needs more scratch than the library holds
    path, rows, groups, ks = C.c_int(), C.c_int(), C.c_int(), C.c_int()
    assert L.t2b_linear_plan(M, N, K, C.byref(path), C.byref(rows), C.byref(groups), C.byref(ks)) == 0
    assert path.value == 0
    assert L.t2b_w4a16_gemm_workspace_bytes(M, N, K) > cap
    # aligned stand-in pointers: the call must return before touching them
    status = L.t2b_w4a16_gemm_noalloc(256, 256, 0, 256, 0, 256, 0, M, N, K, 128, None)
    assert status == 5   # T2B_ERR_WORKSPACE, returned before anything is enqueued
    # argument errors come first, also before anything is enqueued
    assert L.t2b_w4a16_gemm_noalloc(None, None, 0, None, 0, None, 0, M, N, K, 128, None) == 6
    assert L.t2b_w4a16_gemm_noalloc(256, 256, 0, 256, 0, 256, 0, M, N, K, 64, None) == 1

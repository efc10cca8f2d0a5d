"""W4A16 GEMV/GEMM parity through the C-ABI against the oracle and reference goldens.

Bar (the parity target of the decode path): each GEMV/GEMM within 1e-2 relative error
(max-abs error / max |ref|) of fp32-accumulated dequantized math.  The
CUDA-core path (1 row, fp16/fp32 activations, reference qparam rows)
dequantizes exactly in fp32, so its fp32 outputs are held to 1e-4; the
tensor-core path (2+ bf16 rows) dequantizes to bf16 like the reference's NPU
kernels and is held to the 1e-2 bar.
"""

import pytest
import torch

import oracle
from tests import golden_io as gio
from tests.gpu_util import rel_err
from torch2iron_b200 import _lib, synth
from torch2iron_b200 import weights as W
from torch2iron_b200.operators import W4A16GEMM, W4A16GEMV

pytestmark = pytest.mark.gpu


def gemm(w: W.W4Weight, x: torch.Tensor, out_dtype=torch.float32) -> torch.Tensor:
    M, K = x.shape
    N = w.out_features
    y = torch.empty(M, N, dtype=out_dtype, device="cuda")
    L = _lib.lib()
    n = max(L.t2b_w4a16_gemm_workspace_bytes(M, N, K), 256)
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    _lib.call("t2b_w4a16_gemm", _lib.ptr(w.qw), _lib.ptr(w.meta), _lib.WFMT_T2B, _lib.ptr(x), _lib.DTYPE[x.dtype],
              _lib.ptr(y), _lib.DTYPE[out_dtype], M, N, K, 128, _lib.ptr(ws), n, _lib.stream())
    torch.cuda.synchronize()
    return y


def test_config0_gemv_fp16():
    d = gio.load("config0.npz")
    g = torch.Generator().manual_seed(0)
    w = torch.randn(3072, 1024, generator=g) * 0.02
    x = torch.randn(1, 1024, generator=g).to(torch.float16)
    lin = synth.quantize_rtn_autogptq(w)
    dw = W.from_autogptq(lin)
    torch.cuda.synchronize()
    y = gemm(dw, x.cuda(), torch.float16)
    assert rel_err(y, torch.from_numpy(d["y"])) <= 1e-2
    y32 = gemm(dw, x.cuda(), torch.float32)
    assert rel_err(y32, torch.from_numpy(d["y"])) <= 1e-5


def test_repack_matches_reference_dequant():
    d = gio.load("gemv_autogptq.npz")
    lin = gio.linear(d, "p")
    dw = W.from_autogptq(lin)
    torch.cuda.synchronize()
    dense = oracle.autogptq_linear_to_dense(lin.qweight, lin.qzeros, lin.scales)
    assert torch.equal(W.dequantize(dw).cpu(), dense)


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8])
def test_golden_gemv_batches(monkeypatch, M):
    """fp16 activations at 1-8 rows on the exact CUDA-core path (fp32 dequant);
    the tensor-core path, which rounds the weights to fp16, is held to 1e-3."""
    d = gio.load("gemv_autogptq.npz")
    lin = gio.linear(d, "p")
    dw = W.from_autogptq(lin)
    torch.cuda.synchronize()
    x = torch.from_numpy(d["x"])[:M].cuda()
    ref = torch.from_numpy(d["y"])[:M]
    if M > 1:
        assert rel_err(gemm(dw, x, torch.float32), ref) <= 1e-3      # tcgen05, fp16 weights
    monkeypatch.setenv("T2B_TC_MIN_M", "16")
    y = gemm(dw, x, torch.float32)
    assert rel_err(y, ref) <= 1e-5


@pytest.mark.parametrize("N,K", [(4096, 1024), (1024, 3072), (6144, 1024), (1024, 2048), (256, 512), (128, 256),
                                 (512, 1536)])   # K = 12 groups: cluster split 4 x 3 groups (Qwen3-8B down at TP8)
@pytest.mark.parametrize("M", [1, 2, 4, 8, 13, 16, 17, 33, 64, 100, 128, 200, 257, 513])
def test_gemm_shapes_vs_oracle(N, K, M):
    g = torch.Generator().manual_seed(N * 7 + K + M)
    lin = synth.random_linear(N, K, g)
    dw = W.from_autogptq(lin)
    torch.cuda.synchronize()
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    ref = oracle.GroupedW4A16Linear(lin.qweight, lin.qzeros, lin.scales)(x.float())
    y = gemm(dw, x.cuda(), torch.float32)
    assert rel_err(y, ref) <= (1e-4 if M == 1 else 1e-2)
    yb = gemm(dw, x.cuda(), torch.bfloat16)
    assert rel_err(yb, ref) <= 1e-2


def test_gemm_operator_and_repeat_calls_reuse_workspace():
    """Counters re-arm: the same workspace serves consecutive calls."""
    g = torch.Generator().manual_seed(11)
    lin = synth.random_linear(1024, 3072, g)
    dw = W.from_autogptq(lin)
    torch.cuda.synchronize()
    x = torch.randn(4, 3072, generator=g).to(torch.bfloat16)
    ref = oracle.GroupedW4A16Linear(lin.qweight, lin.qzeros, lin.scales)(x.float())
    op = W4A16GEMM(M=4, K=3072, N=1024)
    for _ in range(3):
        c = torch.empty(4, 1024, dtype=torch.bfloat16, device="cuda")
        op(x.cuda(), dw, c)
        torch.cuda.synchronize()
        assert rel_err(c, ref) <= 1e-2


def test_qparam_gemv_operator_matches_reference_runtime():
    d = gio.load("qparam_linear.npz")
    qparam = torch.from_numpy(d["qparam"]).cuda()
    x = gio.bf16(d["x"]).cuda()
    op = W4A16GEMV(M=256, K=512, num_batches=3, shared_qparam=True)
    y = torch.empty(3, 256, dtype=torch.bfloat16, device="cuda")
    op(qparam, x, y)
    torch.cuda.synchronize()
    assert rel_err(y, torch.from_numpy(d["y"])) <= 1e-2


@pytest.mark.parametrize("M,batches,shared", [(256, 3, False), (200, 1, False), (72, 2, True), (300, 2, False)])
def test_qparam_gemv_per_batch_and_ragged_rows(M, batches, shared):
    """Per-batch qparam (``w4a16_gemv/op.py:115-126``: ``qparam_dim = (batch,)``
    unless shared) and row counts that are not a multiple of the 128-row tile,
    against the reference runtime linear restated by the oracle (fp32)."""
    K = 512
    g = torch.Generator().manual_seed(M * 7 + batches)
    nq = 1 if shared else batches
    qps, refs = [], []
    x = torch.randn(batches, K, generator=g).to(torch.bfloat16)
    for b in range(nq):
        packed = torch.randint(0, 256, (M, K // 2), generator=g, dtype=torch.int64).to(torch.uint8)
        scales = (torch.rand(M, K // 128, generator=g) * 0.01 + 1e-3).to(torch.bfloat16)
        qps.append(torch.cat([packed, scales.view(torch.uint8)], dim=1))
        refs.append((packed, scales))
    qparam = torch.stack(qps) if not shared and batches > 1 else qps[0]
    op = W4A16GEMV(M=M, K=K, num_batches=batches, shared_qparam=shared)
    assert tuple(op.get_arg_spec()[0].shape) == tuple(qparam.shape)
    y = torch.empty(batches, M, dtype=torch.bfloat16, device="cuda") if batches > 1 else \
        torch.empty(M, dtype=torch.bfloat16, device="cuda")
    op(qparam.cuda(), (x if batches > 1 else x[0]).cuda(), y)
    torch.cuda.synchronize()
    y = y.view(batches, M).float().cpu()
    for b in range(batches):
        packed, scales = refs[0 if shared else b]
        ref = oracle.packed_w4a16_linear(x[b:b + 1].float(), packed, scales, K, M, 128)
        assert rel_err(y[b:b + 1], ref) <= 1e-2


def test_shape_errors_raise():
    with pytest.raises(_lib.T2BError):
        dw = W.W4Weight(torch.zeros(100, 128, dtype=torch.uint8, device="cuda"),
                        torch.zeros(100, 2, dtype=torch.int32, device="cuda"), 100, 256)
        gemm(dw, torch.zeros(1, 256, dtype=torch.bfloat16, device="cuda"))


@pytest.mark.parametrize("M", [16, 64])
def test_wide_decode_linear_takes_the_large_m_kernel(M):
    """A decode batch on a linear whose tcgen05 grid would run more than two waves (the
    Qwen3-8B gate/up shape of a TP2 rank) goes to the persistent large-M kernel by
    default, and matches the oracle there."""
    import ctypes as C
    N, K = 12288, 4096
    plan = [C.c_int() for _ in range(4)]
    _lib.load().t2b_linear_plan(M, N, K, *[C.byref(v) for v in plan])
    assert plan[0].value == 2
    g = torch.Generator().manual_seed(M + 12288)
    lin = synth.random_linear(N, K, g)
    dw = W.from_autogptq(lin)
    torch.cuda.synchronize()
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    ref = oracle.GroupedW4A16Linear(lin.qweight, lin.qzeros, lin.scales)(x.float())
    assert rel_err(gemm(dw, x.cuda(), torch.float32), ref) <= 1e-2
    assert rel_err(gemm(dw, x.cuda(), torch.bfloat16), ref) <= 1e-2


@pytest.mark.parametrize("M", [1, 5, 128, 130])
@pytest.mark.parametrize("N,K", [(1024, 3072), (384, 256), (256, 12288)])
def test_large_m_kernel_forced(monkeypatch, M, N, K):
    """The large-M (prefill) tcgen05 kernel at any row count matches the oracle."""
    monkeypatch.setenv("T2B_PREFILL_MIN_M", "1")
    g = torch.Generator().manual_seed(M * 3 + N + K)
    lin = synth.random_linear(N, K, g)
    dw = W.from_autogptq(lin)
    torch.cuda.synchronize()
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    ref = oracle.GroupedW4A16Linear(lin.qweight, lin.qzeros, lin.scales)(x.float())
    assert rel_err(gemm(dw, x.cuda(), torch.float32), ref) <= 1e-2
    assert rel_err(gemm(dw, x.cuda(), torch.bfloat16), ref) <= 1e-2


@pytest.mark.parametrize("M", [1, 3, 8, 16])
@pytest.mark.parametrize("N,K", [(1024, 3072), (4096, 1024), (256, 12288)])
def test_tcgen05_forced_small_batch(monkeypatch, M, N, K):
    """The tensor-core path at any row count (padded to 16) matches the oracle."""
    monkeypatch.setenv("T2B_TC_MIN_M", "1")
    g = torch.Generator().manual_seed(M + N + K)
    lin = synth.random_linear(N, K, g)
    dw = W.from_autogptq(lin)
    torch.cuda.synchronize()
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    ref = oracle.GroupedW4A16Linear(lin.qweight, lin.qzeros, lin.scales)(x.float())
    y = gemm(dw, x.cuda(), torch.float32)
    assert rel_err(y, ref) <= 1e-2

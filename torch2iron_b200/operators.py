"""The reference's decode operators, by name, backed by the sm_100a kernels.

Each class keeps the constructor fields of the torch2iron operator it
replaces (NPU-only tiling fields are accepted and validated the same way, so
existing call sites construct them unchanged), raises ``ValueError`` from
``__post_init__`` on bad shapes as the reference does, reports an
``get_arg_spec()`` list of ``ArgSpec(direction, shape, dtype)``, and runs on
``__call__(*buffers)`` with CUDA tensors in arg-spec order.

Replaced operators (reference file:line):

* ``W4A16GEMV``        src/models/quantized_qwen3/operators/w4a16_gemv/op.py:21-126
* ``W4A16GEMM``, ``W4A16KGroupGEMM``, ``W4A16PairedKGroupGEMM``, ``W4A16NShardGEMM``
                       src/models/quantized_qwen3/operators/w4a16_gemm/op.py:22-399
* ``RMSNormRoPE``      src/torch2iron/operators/rms_norm_rope/op.py:19-90
* ``LlamaChunkedAttention``  src/torch2iron/operators/llama_chunked_attention/op.py:20-165
* ``ResidualAddRMSNorm``     src/torch2iron/operators/residual_add_rms_norm/op.py:19-85
* ``SiLUMul``          src/torch2iron/operators/silu_mul/op.py:20-80
* ``CopyPresentPacketKV``    src/torch2iron/operators/copy_present_packet_kv/op.py:18-80

The GEMM family's weight argument is the T2B layout (``W4Weight``) instead
of the AIE ``aie::mmul<4,8,8>`` tile stream, which has no meaning off the
NPU; ``W4A16GEMV`` consumes the reference's own ``qparam`` rows unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import NamedTuple

import torch

from . import _lib
from .weights import W4Weight


class ArgSpec(NamedTuple):
    direction: str
    shape: tuple
    dtype: torch.dtype


def _ws(nbytes: int, device) -> tuple[torch.Tensor, int]:
    n = max(int(nbytes), 256)
    t = torch.zeros(n, dtype=torch.uint8, device=device)
    return t, n


def _check_shape(t: torch.Tensor, shape, name: str):
    if tuple(t.shape) != tuple(shape) and t.numel() != int(torch.tensor(shape).prod()):
        raise ValueError(f"{name}: expected shape {tuple(shape)}, got {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: must be contiguous")


@dataclass
class W4A16GEMV:
    """``y = x . W^T`` over the reference ``qparam`` rows: a batch-1 GEMV, or
    ``num_batches`` rows, sharing one ``qparam`` (``shared_qparam``, one
    launch over all rows) or each with its own (one launch per row, as the
    reference's per-batch arg spec lays them out).  ``M`` not a multiple of
    the kernel's 128-row tile runs on a zero-padded copy of the rows."""

    M: int
    K: int
    num_aie_columns: int = 1
    tile_size_input: int = 2
    tile_size_output: int | None = None
    num_batches: int = 1
    shared_qparam: bool = False
    group_size: int = 128
    kernel_vector_size: int = field(default=32, repr=False)
    context: object = field(default=None, repr=False)

    def __post_init__(self):
        if self.tile_size_output is None:
            self.tile_size_output = self.tile_size_input
        if self.K % 2 != 0:
            raise ValueError("K must be even for packed int4 weights")
        if self.K % self.group_size != 0:
            raise ValueError("K must be a multiple of group_size")
        if self.kernel_vector_size != 32:
            raise ValueError("W4A16GEMV currently supports kernel_vector_size=32 only")
        if self.group_size % self.kernel_vector_size != 0:
            raise ValueError("group_size must be a multiple of kernel_vector_size")
        if not (self.tile_size_output % self.tile_size_input == 0 and self.tile_size_output >= self.tile_size_input):
            raise ValueError("tile_size_output must be a multiple of tile_size_input")
        # B200 kernel constraints
        if self.group_size != 128:
            raise ValueError("the B200 kernel supports group_size=128")
        if self.K % 256:
            raise ValueError("the B200 kernel needs K % 256 == 0")

    @property
    def num_groups(self) -> int:
        return self.K // self.group_size

    @property
    def qparam_row_bytes(self) -> int:
        return self.K // 2 + self.num_groups * 2

    def get_arg_spec(self):
        batch_dim = (self.num_batches,) if self.num_batches > 1 else ()
        qparam_dim = () if self.shared_qparam else batch_dim
        return [ArgSpec("in", qparam_dim + (self.M, self.qparam_row_bytes), torch.uint8),
                ArgSpec("in", batch_dim + (self.K,), torch.bfloat16),
                ArgSpec("out", batch_dim + (self.M,), torch.bfloat16)]

    def __call__(self, qparam: torch.Tensor, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        for t, spec, nm in zip((qparam, x, y), self.get_arg_spec(), ("qparam", "x", "y")):
            _check_shape(t, spec.shape, nm)
        L = _lib.lib()
        rows = self.num_batches
        n_pad = -(-self.M // 128) * 128
        per_batch = rows > 1 and not self.shared_qparam
        qp = qparam.reshape(rows if per_batch else 1, self.M, self.qparam_row_bytes)
        if n_pad != self.M:                                   # rows past M: zero weights and scales
            padded = torch.zeros(qp.shape[0], n_pad, self.qparam_row_bytes, dtype=torch.uint8, device=qp.device)
            padded[:, :self.M].copy_(qp)
            qp = padded
            out = torch.empty(rows, n_pad, dtype=y.dtype, device=y.device)
        else:
            out = y.reshape(rows, self.M)
        xr = x.reshape(rows, self.K)
        ws, n = _ws(L.t2b_w4a16_gemm_workspace_bytes(1 if per_batch else rows, n_pad, self.K), qparam.device)
        calls = [(qp[b], xr[b:b + 1], out[b:b + 1], 1) for b in range(rows)] if per_batch else \
            [(qp[0], xr, out, rows)]
        for w, xb, yb, m in calls:
            _lib.call("t2b_w4a16_gemm", _lib.ptr(w), None, _lib.WFMT_QPARAM, _lib.ptr(xb), _lib.DTYPE[x.dtype],
                      _lib.ptr(yb), _lib.DTYPE[y.dtype], m, n_pad, self.K, self.group_size, _lib.ptr(ws), n,
                      _lib.stream())
        if n_pad != self.M:
            y.reshape(rows, self.M).copy_(out[:, :self.M])
        return y


@dataclass
class W4A16GEMM:
    """``C[M,N] = A[M,K] . W^T`` with ``W`` a T2B ``W4Weight`` ``[N, K]``."""

    M: int
    K: int
    N: int
    num_aie_columns: int = 8
    num_aie_rows: int = 4
    tile_m: int = 8
    tile_k: int = 128
    tile_n: int = 64
    group_size: int = 128
    context: object = field(default=None, repr=False)

    def __post_init__(self):
        self._reference_checks()
        if self.group_size != 128 or self.K % 256 or self.N % 128:
            raise ValueError("the B200 kernel needs group_size=128, K % 256 == 0, N % 128 == 0")

    def _reference_checks(self):
        if self.tile_k != self.group_size:
            raise ValueError("W4A16GEMM currently requires tile_k == group_size")
        if self.K % self.tile_k != 0:
            raise ValueError("K must be a multiple of tile_k")

    def get_arg_spec(self):
        return [ArgSpec("in", (self.M, self.K), torch.bfloat16),
                ArgSpec("in", (self.N, self.K // 2), torch.uint8),
                ArgSpec("out", (self.M, self.N), torch.bfloat16)]

    def __call__(self, a: torch.Tensor, w: W4Weight, c: torch.Tensor) -> torch.Tensor:
        if (w.out_features, w.in_features) != (self.N, self.K):
            raise ValueError("weight shape does not match the operator")
        _check_shape(a, (self.M, self.K), "A")
        _check_shape(c, (self.M, self.N), "C")
        L = _lib.lib()
        ws, n = _ws(L.t2b_w4a16_gemm_workspace_bytes(self.M, self.N, self.K), a.device)
        _lib.call("t2b_w4a16_gemm", _lib.ptr(w.qw), _lib.ptr(w.meta), _lib.WFMT_T2B, _lib.ptr(a), _lib.DTYPE[a.dtype],
                  _lib.ptr(c), _lib.DTYPE[c.dtype], self.M, self.N, self.K, self.group_size, _lib.ptr(ws), n,
                  _lib.stream())
        return c


@dataclass
class W4A16KGroupGEMM(W4A16GEMM):
    """Same contraction; ``k_group`` (K tiles per AIE call) is a scheduling hint with no B200 meaning."""

    k_group: int = 2

    def _reference_checks(self):
        super()._reference_checks()
        if (self.K // self.tile_k) % self.k_group != 0:
            raise ValueError("k_tiles must be divisible by k_group")


@dataclass
class W4A16NShardGEMM(W4A16GEMM):
    pass


@dataclass
class W4A16PairedKGroupGEMM(W4A16KGroupGEMM):
    """One activation stream, two weights (K/V or gate/up), two outputs."""

    def get_arg_spec(self):
        return [ArgSpec("in", (self.M, self.K), torch.bfloat16),
                ArgSpec("in", (2, self.N, self.K // 2), torch.uint8),
                ArgSpec("out", (self.M, self.N), torch.bfloat16),
                ArgSpec("out", (self.M, self.N), torch.bfloat16)]

    def __call__(self, a: torch.Tensor, w_pair: W4Weight, c0: torch.Tensor, c1: torch.Tensor):
        """``w_pair`` holds the two weights row-concatenated (``weights.concat_rows``)."""
        if (w_pair.out_features, w_pair.in_features) != (2 * self.N, self.K):
            raise ValueError("paired weight must be [2N, K]")
        tmp = torch.empty(self.M, 2 * self.N, dtype=c0.dtype, device=a.device)
        W4A16GEMM(self.M, self.K, 2 * self.N)(a, w_pair, tmp)
        c0.copy_(tmp[:, :self.N])
        c1.copy_(tmp[:, self.N:])
        return c0, c1


@dataclass
class RMSNormRoPE:
    """Weighted RMSNorm then RoPE per row; ``rope_mode`` "interleaved" follows
    ``model.py:184-196`` (the CPU reference), "two_halves" follows the NPU
    kernel ``rms_norm_rope/kernel.cc:39-67``."""

    rows: int
    cols: int
    angle_rows: int
    num_aie_columns: int = 8
    epsilon: float = 1e-5
    rope_mode: str = "interleaved"
    context: object = field(default=None, repr=False)

    def __post_init__(self):
        if self.cols % 32 != 0:
            raise ValueError("cols must be divisible by 32")
        if self.rows % self.num_aie_columns != 0:
            raise ValueError("rows must be divisible by num_aie_columns")
        if self.angle_rows > self.rows or self.rows % self.angle_rows != 0:
            raise ValueError("angle_rows must divide rows")
        if self.angle_rows < self.num_aie_columns or self.angle_rows % self.num_aie_columns != 0:
            raise ValueError("angle_rows must be divisible by num_aie_columns")
        if self.epsilon <= 0:
            raise ValueError("epsilon must be positive")
        if self.rope_mode not in ("interleaved", "two_halves"):
            raise ValueError("rope_mode must be 'interleaved' or 'two_halves'")

    def get_arg_spec(self):
        bf = torch.bfloat16
        return [ArgSpec("in", (self.rows, self.cols), bf), ArgSpec("in", (self.cols,), bf),
                ArgSpec("in", (self.angle_rows, self.cols), bf), ArgSpec("out", (self.rows, self.cols), bf)]

    def __call__(self, inp, w, angles, out):
        for t, spec, nm in zip((inp, w, angles, out), self.get_arg_spec(), ("in", "w", "angles", "out")):
            _check_shape(t, spec.shape, nm)
        _lib.call("t2b_rms_norm_rope", _lib.ptr(inp), _lib.ptr(w), _lib.ptr(angles), _lib.ptr(out), self.rows,
                  self.cols, self.angle_rows, self.epsilon, 0 if self.rope_mode == "interleaved" else 1,
                  _lib.stream())
        return out


@dataclass
class LlamaChunkedAttention:
    """GQA decode attention over the packet cache (mask-skipped slots)."""

    max_seq_len: int
    num_kv_groups: int = 8
    q_heads_per_group: int = 4
    head_dim: int = 64
    chunk_size: int = 64
    packed_fifo_depth: int | None = None
    kernel_vector_size: int = field(default=32, repr=False)
    context: object = field(default=None, repr=False)

    def __post_init__(self):
        if self.max_seq_len <= 0:
            raise ValueError("max_seq_len must be positive")
        if self.chunk_size <= 0:
            raise ValueError("chunk_size must be positive")
        if self.max_seq_len % self.chunk_size != 0:
            raise ValueError("max_seq_len must be divisible by chunk_size")
        if self.num_kv_groups <= 0:
            raise ValueError("num_kv_groups must be positive")
        if self.q_heads_per_group <= 0:
            raise ValueError("q_heads_per_group must be positive")
        if self.head_dim <= 0:
            raise ValueError("head_dim must be positive")
        if self.head_dim % self.kernel_vector_size != 0:
            raise ValueError("head_dim must be divisible by kernel_vector_size")
        if self.chunk_size != 64 or self.head_dim not in (64, 128) or self.q_heads_per_group not in (1, 2, 4, 8):
            raise ValueError("the B200 kernel needs chunk_size=64, head_dim in (64,128), q_heads_per_group in 1/2/4/8")

    @property
    def packed_chunk_elements(self):
        return 2 * self.chunk_size * self.head_dim + self.chunk_size

    @property
    def packed_elements(self):
        return self.num_kv_groups * (self.max_seq_len // self.chunk_size) * self.packed_chunk_elements

    def get_arg_spec(self):
        bf = torch.bfloat16
        q = (self.num_kv_groups, self.q_heads_per_group, self.head_dim)
        return [ArgSpec("in", q, bf), ArgSpec("in", (self.packed_elements,), bf), ArgSpec("out", q, bf)]

    def __call__(self, q, packet, out):
        for t, spec, nm in zip((q, packet, out), self.get_arg_spec(), ("Q", "packet", "out")):
            _check_shape(t, spec.shape, nm)
        L = _lib.lib()
        ws, n = _ws(L.t2b_decode_attention_workspace_bytes(1, self.num_kv_groups * self.q_heads_per_group,
                                                           self.num_kv_groups, self.head_dim, self.max_seq_len),
                    q.device)
        _lib.call("t2b_packet_attention", _lib.ptr(q), _lib.ptr(packet), _lib.ptr(out), self.num_kv_groups,
                  self.q_heads_per_group, self.head_dim, self.max_seq_len, self.chunk_size, _lib.ptr(ws), n,
                  _lib.stream())
        return out


@dataclass
class ResidualAddRMSNorm:
    size: int
    num_aie_columns: int
    tile_size: int
    epsilon: float = 1e-5
    context: object = field(default=None, repr=False)

    def __post_init__(self):
        if self.epsilon <= 0:
            raise ValueError("epsilon must be positive")
        if self.size % (self.num_aie_columns * self.tile_size) != 0:
            raise ValueError("size must be divisible by num_aie_columns * tile_size")

    def get_arg_spec(self):
        bf = torch.bfloat16
        return [ArgSpec("in", (self.size,), bf), ArgSpec("in", (self.size,), bf), ArgSpec("in", (self.tile_size,), bf),
                ArgSpec("out", (self.size,), bf), ArgSpec("out", (self.size,), bf)]

    def __call__(self, x, update, w, x_out, norm_out):
        for t, spec, nm in zip((x, update, w, x_out, norm_out), self.get_arg_spec(),
                               ("x", "update", "w", "x_out", "norm_out")):
            _check_shape(t, spec.shape, nm)
        _lib.call("t2b_residual_add_rms_norm", _lib.ptr(x), _lib.ptr(update), _lib.ptr(w), _lib.ptr(x_out),
                  _lib.ptr(norm_out), self.size, self.tile_size, self.epsilon, _lib.stream())
        return x_out, norm_out


@dataclass
class SiLUMul:
    size: int
    tile_size: int
    num_aie_columns: int = 8
    context: object = field(default=None, repr=False)

    def __post_init__(self):
        if self.size % (self.num_aie_columns * self.tile_size) != 0:
            raise ValueError(f"size ({self.size}) must be a multiple of "
                             f"num_aie_columns * tile_size ({self.num_aie_columns * self.tile_size})")

    def get_arg_spec(self):
        bf = torch.bfloat16
        return [ArgSpec("in", (self.size,), bf), ArgSpec("in", (self.size,), bf), ArgSpec("out", (self.size,), bf)]

    def __call__(self, a, b, out):
        for t, spec, nm in zip((a, b, out), self.get_arg_spec(), ("left", "right", "out")):
            _check_shape(t, spec.shape, nm)
        _lib.call("t2b_silu_mul", _lib.ptr(a), _lib.ptr(b), _lib.ptr(out), self.size, _lib.stream())
        return out


@dataclass
class CopyPresentPacketKV:
    kv_dim: int
    num_kv_groups: int
    head_dim: int
    packet_elements: int
    packet_elements_per_group: int
    key_packet_offset: int
    value_packet_offset: int
    dtype: object = field(default=torch.bfloat16, repr=False)
    transfer_size: int | None = None
    mask_packet_offset: int | None = None
    context: object = field(default=None, repr=False)

    def __post_init__(self):
        if self.kv_dim != self.num_kv_groups * self.head_dim:
            raise ValueError("kv_dim must equal num_kv_groups * head_dim")

    def get_arg_spec(self):
        bf = torch.bfloat16
        return [ArgSpec("in", (self.kv_dim,), bf), ArgSpec("in", (self.kv_dim,), bf),
                ArgSpec("out", (self.kv_dim,), bf), ArgSpec("out", (self.kv_dim,), bf),
                ArgSpec("out", (self.packet_elements,), bf)]

    def __call__(self, k, v, present_k, present_v, packet):
        for t, spec, nm in zip((k, v, present_k, present_v, packet), self.get_arg_spec(),
                               ("key", "value", "present_key", "present_value", "packet")):
            _check_shape(t, spec.shape, nm)
        moff = -1 if self.mask_packet_offset is None else self.mask_packet_offset
        _lib.call("t2b_copy_present_packet_kv", _lib.ptr(k), _lib.ptr(v), _lib.ptr(present_k), _lib.ptr(present_v),
                  _lib.ptr(packet), self.num_kv_groups, self.head_dim, self.packet_elements_per_group,
                  self.key_packet_offset, self.value_packet_offset, moff, _lib.stream())
        return present_k, present_v, packet

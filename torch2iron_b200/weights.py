"""Device-resident W4A16 weights in the T2B layout (see ``include/t2b.h``).

Conversion from AutoGPTQ tensors runs once at load through the CUDA repack
kernel (``t2b_repack_autogptq``); nothing here is on the per-token path.
Q4NX group-32 weights (the fast Qwen3 artifact, ``fast_qwen3/q4nx_layout.py``)
use the same 8 KB nibble blocks with a meta word per 32-k piece instead of
per 128-k group (format ``WFMT_Q4NX``): bits 0-15 the bf16 scale, bits 16-31
the bf16 zero point, ``W = (q - zero) * scale``; a block's 512 words are
ordered ``[piece 4][row 128]``.  They are rearranged with torch ops on the
device at load (``from_q4nx``).

Fused matrices:

* ``qkv``      -- ``[q; k; v]`` rows concatenated (one launch, heads aligned
                  to the 128-row tiles of the GEMV);
* ``gate_up``  -- gate and up interleaved in 64-row blocks so each 128-row
                  tile holds ``gate[64b:64b+64]`` then ``up[64b:64b+64]``
                  (the SwiGLU epilogue pairs them in-CTA; the reference pairs
                  the same two matrices in one GEMM stream,
                  ``w4a16_gemm/op.py:177-263``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .synth import AutoGPTQLinear

PAIR_BLOCK = 64
WFMT_T2B = 0        # T2B_WFMT_T2B: group 128, fp16 scale + integer zero per (row, group)
WFMT_Q4NX = 2       # T2B_WFMT_Q4NX: group 32, bf16 scale + bf16 zero per (row, 32-k piece)
_SLOT_K = (0, 2, 4, 6, 1, 3, 5, 7)   # k (within a word's 8) held by nibble slot 0..7: even k first


@dataclass
class W4Weight:
    qw: torch.Tensor      # uint8, N*K/2 bytes in 8 KB (128-row x 128-k) blocks; shape [N, K/2]
    meta: torch.Tensor    # int32 [N, K/128] (T2B) or [N, K/32] (Q4NX) storage, block-ordered
    out_features: int
    in_features: int
    fmt: int = WFMT_T2B

    @property
    def nbytes_algorithmic(self) -> int:
        """int4 + the per-group scale and zero point (the bytes the layout must move):
        g128 fp16 scale + 4-bit zero, or g32 bf16 scale + bf16 zero."""
        n, k = self.out_features, self.in_features
        if self.fmt == WFMT_Q4NX:
            return n * k // 2 + n * (k // 32) * 4
        return n * k // 2 + n * (k // 128) * 2 + n * (k // 128) // 2

    @property
    def nbytes_stored(self) -> int:
        return self.qw.numel() + self.meta.numel() * 4


def _empty(n: int, k: int, device) -> W4Weight:
    if n % 128 or k % 256:
        raise ValueError(f"T2B weights need out_features % 128 == 0 and in_features % 256 == 0, got [{n}, {k}]")
    return W4Weight(torch.empty(n, k // 2, dtype=torch.uint8, device=device),
                    torch.empty(n, k // 128, dtype=torch.int32, device=device), n, k)


def _repack_into(dst: W4Weight, lin: AutoGPTQLinear, row0: int, block_rows: int, block_stride: int) -> None:
    dev = dst.qw.device
    qweight = lin.qweight.to(dev, torch.int32).contiguous()
    qzeros = lin.qzeros.to(dev, torch.int32).contiguous()
    scales = lin.scales.to(dev, torch.float16).contiguous().view(torch.int16)
    _lib.call("t2b_repack_autogptq", _lib.ptr(qweight), _lib.ptr(qzeros), _lib.ptr(scales), lin.in_features,
              lin.out_features, lin.group_size, _lib.ptr(dst.qw), _lib.ptr(dst.meta), row0, block_rows, block_stride,
              _lib.stream())


def from_autogptq(lin: AutoGPTQLinear, device="cuda") -> W4Weight:
    w = _empty(lin.out_features, lin.in_features, device)
    _repack_into(w, lin, 0, lin.out_features, 0)
    return w


def concat_rows(lins: list[AutoGPTQLinear], device="cuda") -> W4Weight:
    k = lins[0].in_features
    if any(l.in_features != k for l in lins):
        raise ValueError("all parts of a fused weight need the same in_features")
    w = _empty(sum(l.out_features for l in lins), k, device)
    row = 0
    for l in lins:
        _repack_into(w, l, row, l.out_features, 0)
        row += l.out_features
    return w


def pair_blocks(gate: AutoGPTQLinear, up: AutoGPTQLinear, device="cuda") -> W4Weight:
    if gate.out_features != up.out_features or gate.out_features % PAIR_BLOCK:
        raise ValueError("gate/up must have equal out_features, a multiple of 64")
    w = _empty(2 * gate.out_features, gate.in_features, device)
    _repack_into(w, gate, 0, PAIR_BLOCK, 2 * PAIR_BLOCK)
    _repack_into(w, up, PAIR_BLOCK, PAIR_BLOCK, 2 * PAIR_BLOCK)
    return w


# ---------------------------------------------------------------------------
# Q4NX group-32
# ---------------------------------------------------------------------------
def q4nx_unpack(lin, device="cuda") -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """A stored Q4NX linear (``loaders.Q4NXLinear``) -> (q uint8 ``[N, K]``,
    scale bf16 ``[N, K/32]``, zero bf16 ``[N, K/32]``), the padding rows
    dropped.  Chunk order: 64-row patches, K-chunk-major, two 32-row chunks per
    (patch, 256-k chunk); a chunk is scales ``[32][8]``, zero points ``[32][8]``
    (bf16) and ``[32][128]`` bytes of nibbles, low nibble = even k
    (``q4nx_layout.py:92-113,132-174``)."""
    K, Np, N = lin.in_features, lin.padded_out_features, lin.out_features
    if K % 256 or Np % 64:
        raise ValueError(f"Q4NX linear [{N}, {K}] padded to {Np} rows is not a whole number of chunks")
    c = lin.data.to(device).view(Np // 64, K // 256, 2, 5120)
    scale = c[..., :512].contiguous().view(torch.bfloat16).view(Np // 64, K // 256, 2, 32, 8)
    zero = c[..., 512:1024].contiguous().view(torch.bfloat16).view(Np // 64, K // 256, 2, 32, 8)
    packed = c[..., 1024:].view(Np // 64, K // 256, 2, 32, 128)
    q = torch.stack((packed & 0xF, packed >> 4), dim=-1).view(Np // 64, K // 256, 2, 32, 256)

    def rows(t):   # (patch, kchunk, half, row, cols) -> [Np, K-ish]
        return t.permute(0, 2, 3, 1, 4).reshape(Np, -1)[:N].contiguous()

    return rows(q), rows(scale), rows(zero)


def pack_nibbles(q: torch.Tensor) -> torch.Tensor:
    """Dense nibbles ``[N, K]`` (0..15) -> the block-ordered T2B bytes ``[N, K/2]``."""
    n, k = q.shape
    if n % 128 or k % 128:
        raise ValueError(f"T2B blocks need [N, K] multiples of 128, got [{n}, {k}]")
    t = q.to(torch.uint8).view(n // 128, 128, k // 128, 4, 4, 8)[..., list(_SLOT_K)]   # [nb, r, g, p, w, slot]
    b = t[..., 0::2] | (t[..., 1::2] << 4)                                            # [nb, r, g, p, w, byte]
    return b.permute(0, 2, 3, 1, 4, 5).contiguous().view(n, k // 2)


def from_q4nx_parts(q: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor) -> W4Weight:
    """Device weight from unpacked Q4NX parts (q ``[N, K]``, bf16 scale/zero ``[N, K/32]``)."""
    n, k = q.shape
    if n % 128 or k % 256:
        raise ValueError(f"the kernels need out_features % 128 == 0 and in_features % 256 == 0, got [{n}, {k}]")
    word = (scale.contiguous().view(torch.int16).to(torch.int32) & 0xFFFF) | \
        (zero.contiguous().view(torch.int16).to(torch.int32) << 16)
    meta = word.view(n // 128, 128, k // 128, 4).permute(0, 2, 3, 1).contiguous().view(n, k // 32)
    return W4Weight(pack_nibbles(q), meta, n, k, WFMT_Q4NX)


def from_q4nx(lin, device="cuda") -> W4Weight:
    return from_q4nx_parts(*q4nx_unpack(lin, device))


def q4nx_concat_rows(lins: list, device="cuda") -> W4Weight:
    parts = [q4nx_unpack(l, device) for l in lins]
    return from_q4nx_parts(*(torch.cat([p[i] for p in parts], dim=0) for i in range(3)))


def q4nx_pair_blocks(gate, up, device="cuda") -> W4Weight:
    """gate/up interleaved in 64-row blocks, as ``pair_blocks``."""
    g, u = q4nx_unpack(gate, device), q4nx_unpack(up, device)
    n = g[0].shape[0]
    if u[0].shape[0] != n or n % PAIR_BLOCK:
        raise ValueError("gate/up must have equal out_features, a multiple of 64")

    def inter(a, b):
        return torch.stack((a.view(n // PAIR_BLOCK, PAIR_BLOCK, -1), b.view(n // PAIR_BLOCK, PAIR_BLOCK, -1)),
                           dim=1).reshape(2 * n, -1)

    return from_q4nx_parts(*(inter(g[i], u[i]) for i in range(3)))


def dequantize(w: W4Weight) -> torch.Tensor:
    """Dense fp32 ``[N, K]`` view of a T2B weight (host-side check helper).

    Undoes the tiled block order (block (nt, g) = [piece 4][row 128][16 B])
    and the even-k-first nibble order inside each 32-bit word.
    """
    n, k = w.out_features, w.in_features
    g = k // 128
    qb = w.qw.reshape(n // 128, g, 4, 128, 16).permute(0, 3, 1, 2, 4).reshape(n, k // 8, 4).to(torch.int32)
    nib = torch.stack((qb & 0xF, qb >> 4), dim=-1).reshape(n, k // 8, 8)   # nibble slots 0..7 of each word
    order = torch.tensor([0, 4, 1, 5, 2, 6, 3, 7], device=nib.device)      # slot holding k = 0..7
    q = nib[:, :, order].reshape(n, k).float()
    if w.fmt == WFMT_Q4NX:
        meta = w.meta.reshape(n // 128, g, 4, 128).permute(0, 3, 1, 2).reshape(n, k // 32).to(torch.int64)
        scale = (meta & 0xFFFF).to(torch.int16).view(torch.bfloat16).float()
        zero = ((meta >> 16) & 0xFFFF).to(torch.int16).view(torch.bfloat16).float()
        return (q - zero.repeat_interleave(32, dim=1)) * scale.repeat_interleave(32, dim=1)
    meta = w.meta.reshape(n // 128, g, 128).permute(0, 2, 1).reshape(n, g).to(torch.int64) & 0xFFFFFFFF
    scale = (meta & 0xFFFF).to(torch.int16).view(torch.float16).float()
    zero = ((meta >> 16) & 0x1F).float()
    return (q - zero.repeat_interleave(128, dim=1)) * scale.repeat_interleave(128, dim=1)

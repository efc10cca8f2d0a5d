"""Device-resident W4A16 weights in the T2B layout (see ``include/t2b.h``).

Conversion from AutoGPTQ tensors runs once at load through the CUDA repack
kernel (``t2b_repack_autogptq``); nothing here is on the per-token path.
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


@dataclass
class W4Weight:
    qw: torch.Tensor      # uint8, N*K/2 bytes in 8 KB (128-row x 128-k) blocks; shape [N, K/2]
    meta: torch.Tensor    # int32 [N, K/128] storage, 128-entry blocks (uint32: fp16 scale | zero << 16)
    out_features: int
    in_features: int

    @property
    def nbytes_algorithmic(self) -> int:
        """int4 + fp16 scale + 4-bit zero per group (the bytes a W4A16 g128 layout must move)."""
        n, k = self.out_features, self.in_features
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
    meta = w.meta.reshape(n // 128, g, 128).permute(0, 2, 1).reshape(n, g).to(torch.int64) & 0xFFFFFFFF
    scale = (meta & 0xFFFF).to(torch.int16).view(torch.float16).float()
    zero = ((meta >> 16) & 0x1F).float()
    return (q - zero.repeat_interleave(128, dim=1)) * scale.repeat_interleave(128, dim=1)

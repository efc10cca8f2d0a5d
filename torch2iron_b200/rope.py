"""RoPE angle table in the reference's layout.

``[ctx, head_dim]`` fp32 with cos at even and sin at odd slots, computed on
the host in fp32 exactly as ``compute_rope_angles``
(``src/models/quantized_qwen3/model.py:351-358``) so the device kernels see
the same angles the CPU reference uses.  Built once per engine; the decode
kernels read row ``pos`` of it.
"""

from __future__ import annotations

import torch


def rope_angles(head_dim: int, context_length: int, rope_base: float) -> torch.Tensor:
    inv_freq = 1.0 / (rope_base ** (torch.arange(0, head_dim, 2).float() / head_dim))
    freqs = torch.outer(torch.arange(context_length).float(), inv_freq)
    angles = torch.empty(context_length, head_dim)
    angles[:, 0::2] = torch.cos(freqs)
    angles[:, 1::2] = torch.sin(freqs)
    return angles

"""Helpers to read the golden ``.npz`` fixtures into torch tensors."""

import os

import numpy as np
import torch

from torch2iron_b200.synth import AutoGPTQLinear

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name: str) -> dict:
    return dict(np.load(os.path.join(GOLDEN, name)))


def bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.uint16).view(np.int16).copy()).view(torch.bfloat16)


def linear(d: dict, prefix: str) -> AutoGPTQLinear:
    qw = torch.from_numpy(d[f"{prefix}.qweight"])
    qz = torch.from_numpy(d[f"{prefix}.qzeros"])
    sc = torch.from_numpy(d[f"{prefix}.scales"])
    return AutoGPTQLinear(qw, qz, sc, qw.shape[0] * 8, qw.shape[1], 128)


def kv_plane_case(d, case: int, max_ctx: int):
    """One case of ``kv_plane_attention.npz`` in this library's layouts:
    q ``[1, n_heads*hd]`` bf16, K/V caches ``[1, 8, max_ctx, hd]`` bf16 (plane
    slot s -> cache position s), the attended length and the reference output
    ``[n_heads*hd]`` (fp32 of its bf16 values).  Plane layout of
    ``kv_plane_reference.py:15-55``: 4 planes (K of kv heads 0-3, V of 0-3, K of
    4-7, V of 4-7), token stride 4*hd, kv head g at (g % 4)*hd in its plane."""
    import torch
    cur, attend, seq, qpg, hd = (int(v) for v in d[f"c{case}.meta"])
    plane = bf16(d[f"c{case}.plane"])
    qc = bf16(d[f"c{case}.q_current"]).view(8, (qpg + 2) * hd)
    pe = seq * 4 * hd
    k = torch.zeros(1, 8, max_ctx, hd, dtype=torch.bfloat16)
    v = torch.zeros(1, 8, max_ctx, hd, dtype=torch.bfloat16)
    for g in range(8):
        kp, vp = (0, 1) if g < 4 else (2, 3)
        for slot in range(seq):
            off = slot * 4 * hd + (g % 4) * hd
            k[0, g, slot] = plane[kp * pe + off: kp * pe + off + hd]
            v[0, g, slot] = plane[vp * pe + off: vp * pe + off + hd]
    q = qc[:, :qpg * hd].reshape(1, 8 * qpg * hd)
    out = bf16(d[f"c{case}.out"]).float().reshape(-1)
    return q, k, v, attend, out, qpg, hd

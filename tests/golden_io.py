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

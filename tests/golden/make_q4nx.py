"""Golden vectors for the Q4NX group-32 layout of the fast Qwen3 path.

Runs the reference's own ``pack_linear_weight``, ``dequantize_linear`` and
``q4nx_linear_reference`` (``src/models/fast_qwen3/q4nx_layout.py:115-303``)
on a seeded fp32 weight of 96 x 512 (output rows padded to the 64-row patch)
and a bf16 input, and writes ``tests/golden/q4nx_linear.npz``: the packed
bytes, the reference dequantisation and the reference output.

Run once, in a container where the reference is mounted:
    python tests/golden/make_q4nx.py <reference root>
"""

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    from models.fast_qwen3.q4nx_layout import dequantize_linear, pack_linear_weight, q4nx_linear_reference

    g = torch.Generator().manual_seed(77)
    w = torch.randn(96, 512, generator=g) * 0.02
    x = torch.randn(3, 512, generator=g).to(torch.bfloat16)
    data, spec = pack_linear_weight(w)
    dense = dequantize_linear(data, spec)
    y = q4nx_linear_reference(x, data, spec)
    np.savez_compressed(HERE / "q4nx_linear.npz", data=np.frombuffer(data, dtype=np.uint8),
                        shape=np.array([spec.out_features, spec.in_features, spec.padded_out_features]),
                        dense=dense.numpy(), x=x.view(torch.int16).numpy().view(np.uint16),
                        y=y.view(torch.int16).numpy().view(np.uint16))
    print("wrote", HERE / "q4nx_linear.npz", len(data), "bytes packed")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_q4nx.py <reference root>")
    main(sys.argv[1])

"""Golden vectors for decode attention over the reference's KV plane layout.

Runs the reference's own ``update_q_current_in_kv_plane`` and
``plane_attention_current_reference``
(``src/models/fast_qwen3/kv_plane_reference.py:77-187``) on seeded bf16
inputs and writes ``tests/golden/kv_plane_attention.npz``: for each case the
flat plane (past keys / values), the current q/k/v rows, the current slot, the
attended length and the reference output.  Case 0 (head_dim 128, 2 q heads per
kv group) puts the current token at the last attended slot -- the decode
step's layout, keys 0..pos with the new key at pos; case 1 (head_dim 64, 4 q
heads per group) puts it in the middle of a shorter attended range.

Run once, in a container where the reference is mounted:
    python tests/golden/make_kv_plane.py <reference root>
"""

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    from models.fast_qwen3.kv_plane_reference import (kv_plane_total_elements, plane_attention_current_reference,
                                                      update_q_current_in_kv_plane)

    g = torch.Generator().manual_seed(2024)
    out = {}
    # (current slot, attended length, plane length, q heads per kv group, head_dim)
    for case, (cur, attend, seq, qpg, hd) in enumerate(((71, 72, 72, 2, 128), (20, 40, 48, 4, 64))):
        plane = torch.randn(kv_plane_total_elements(seq, hd), generator=g).to(torch.bfloat16)
        q_current = torch.randn(8, (qpg + 2) * hd, generator=g).to(torch.bfloat16)
        update_q_current_in_kv_plane(q_current, plane, cur, seq, qpg)
        y = plane_attention_current_reference(q_current, plane, cur, attend, seq, qpg)
        out.update({f"c{case}.plane": bits(plane), f"c{case}.q_current": bits(q_current),
                    f"c{case}.out": bits(y), f"c{case}.meta": np.array([cur, attend, seq, qpg, hd])})
    np.savez_compressed(HERE / "kv_plane_attention.npz", **out)
    print("wrote", HERE / "kv_plane_attention.npz")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_kv_plane.py <reference root>")
    main(sys.argv[1])

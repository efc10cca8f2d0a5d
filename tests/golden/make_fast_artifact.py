"""Golden fixture for the fast Qwen3 (Q4NX) artifact loader, made by the reference.

Packs the AutoGPTQ checkpoint of ``tests/golden/packed_tiny`` with the
reference's own ``write_fast_qwen3_artifact``
(src/models/fast_qwen3/fast_packed_format.py:178-262) into
``tests/golden/packed_tiny/fast_qwen3_q4nx/`` and records in
``tests/golden/fast_tiny.npz``, per Q4NX linear, the sha256 of the
reference's dense dequantisation (``dequantize_linear``, q4nx_layout.py:217-237)
and the reference's output on a seeded input (``FastQwen3Store.linear_reference``,
fast_packed_format.py:299-300).

Run once, in a container where the reference is mounted:
    python tests/golden/make_fast_artifact.py <reference root>
"""

import hashlib
import json
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
MODEL = HERE / "packed_tiny"
OUT = MODEL / "fast_qwen3_q4nx"


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    from models.fast_qwen3.fast_packed_format import FastQwen3Store, write_fast_qwen3_artifact
    from models.fast_qwen3.q4nx_layout import dequantize_linear

    if OUT.exists():
        shutil.rmtree(OUT)
    with tempfile.TemporaryDirectory() as tmp:   # the writer reads only config.json + model.safetensors
        shutil.copy(MODEL / "config.json", tmp)
        shutil.copy(MODEL / "model.safetensors", tmp)
        write_fast_qwen3_artifact(tmp, OUT)
    manifest = json.loads((OUT / "manifest.json").read_text())
    manifest["source_model_dir"] = "packed_tiny"          # the temp dir name is not reproducible
    (OUT / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n")

    store = FastQwen3Store(OUT)
    g = torch.Generator().manual_seed(99)
    out = {}
    for prefix in sorted(manifest["linears"]):
        spec = store.linear_spec(prefix)
        dense = dequantize_linear(store.linear_bytes(prefix), spec)
        x = torch.randn(2, spec.in_features, generator=g).to(torch.bfloat16)
        y = store.linear_reference(prefix, x)
        out[f"{prefix}.sha256"] = np.array(hashlib.sha256(dense.numpy().tobytes()).hexdigest())
        out[f"{prefix}.x"] = x.view(torch.int16).numpy().view(np.uint16)
        out[f"{prefix}.y"] = y.view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(HERE / "fast_tiny.npz", **out)
    print("wrote", OUT, "and fast_tiny.npz;", len(manifest["linears"]), "Q4NX linears")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_fast_artifact.py <reference root>")
    main(sys.argv[1])

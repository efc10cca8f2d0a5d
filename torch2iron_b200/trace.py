"""Device-side diagnostics with the trace build of the library.

    python -m torch2iron_b200.build --trace          # builds libt2b_trace.so
    python -m torch2iron_b200.trace prefill [B P]    # role waits of the large-M GEMM

``prefill`` runs the chunked prefill of Qwen3-0.6B (random weights, B
sequences of P tokens) twice on the trace library and prints, per fused
linear kind, the median share of each CTA's run that its roles spent
waiting: the MMA warp on a dequantised A stage, on an activation stage and
on a free accumulator; the producers on raw weights and on a free A stage;
the epilogue warps on a finished accumulator.  The role that never waits
bounds the kernel.  The trace library must not be loaded together with the
product library; this module sets ``T2B_LIBRARY`` before the first load.
"""

from __future__ import annotations

import ctypes as C
import os
import sys
from pathlib import Path

TRACE_LIB = Path(__file__).resolve().parent.parent / "_build" / "libt2b_trace.so"
_KINDS = {30: "store", 31: "residual (o, down)", 32: "swiglu (gate/up)", 33: "qkv"}
_COLUMNS = [(1, "mma<-A"), (2, "mma<-X"), (3, "mma<-acc"), (4, "prod<-W"), (5, "prod<-Afree"), (6, "epi<-acc")]


def prefill_role_waits(batch: int = 64, prompt: int = 128) -> dict:
    """kind -> {'ctas': n, 'run_cycles': median, column: median share of the run}."""
    os.environ["T2B_LIBRARY"] = str(TRACE_LIB)
    import numpy as np
    import torch

    from . import _lib, synth
    from .config import QWEN3_0_6B
    from .engine import DecodeEngine

    if _lib._lib is not None and _lib.LIB_PATH != TRACE_LIB:
        raise RuntimeError("the product library is already loaded in this process; run this module on its own")
    _lib.LIB_PATH = TRACE_LIB
    cfg = QWEN3_0_6B
    model = synth.random_model(cfg, seed=0, device="cuda")
    max_ctx = ((prompt + 63) // 64) * 64
    eng = DecodeEngine(cfg, model, batch=batch, max_ctx=max_ctx, use_graph=False, keep_logits=False)
    prompts = torch.randint(0, cfg.vocab_size, (batch, prompt), generator=torch.Generator().manual_seed(1))
    dump = _lib.load().t2b_trace_dump_prefill
    dump.argtypes = [C.c_void_p, C.c_int, C.c_int]
    dump.restype = C.c_int
    buf = np.zeros((1 << 15, 12), dtype=np.uint64)
    eng.prefill(prompts)                       # warm-up; its records are discarded
    torch.cuda.synchronize()
    dump(buf.ctypes.data, 1 << 15, 1)
    eng.prefill(prompts)
    torch.cuda.synchronize()
    eng.check_device_errors()
    m = dump(buf.ctypes.data, 1 << 15, 1)
    recs = buf[:m].copy()
    tags = recs[:, 8:].view(np.int32).reshape(m, 8)[:, 0]
    out = {}
    for tag in sorted(set(tags.tolist())):
        t = recs[tags == tag, :8].astype(np.float64)
        run = t[:, 7]
        row = {"ctas": int((tags == tag).sum()), "run_cycles": float(np.median(run))}
        for k, name in _COLUMNS:
            row[name] = float(np.median(t[:, k] / run))
        out[_KINDS.get(tag, str(tag))] = row
    return out


def main(argv: list[str]) -> None:
    if not argv or argv[0] != "prefill":
        raise SystemExit("usage: python -m torch2iron_b200.trace prefill [batch prompt]")
    batch = int(argv[1]) if len(argv) > 1 else 64
    prompt = int(argv[2]) if len(argv) > 2 else 128
    for kind, row in prefill_role_waits(batch, prompt).items():
        cols = " ".join(f"{name}={row[name] * 100:5.1f}%" for _, name in _COLUMNS)
        print(f"{kind:20s} ctas={row['ctas']:5d} run={row['run_cycles']:9.0f} cycles | {cols}")


if __name__ == "__main__":
    main(sys.argv[1:])

"""Device-side diagnostics with the trace build of the library.

    python -m torch2iron_b200.build --trace          # builds _build/libt2b_trace.so
    python -m torch2iron_b200.trace prefill [B P]    # role waits of the large-M GEMM
    python -m torch2iron_b200.trace decode [B C]     # phase timeline of the decode-step kernels

``prefill`` runs the chunked prefill of Qwen3-0.6B (random weights, B
sequences of P tokens) twice on the trace library and prints, per fused
linear kind, the median share of each CTA's run that its roles spent
waiting: the MMA warp on a dequantised A stage, on an activation stage and
on a free accumulator; the producers on raw weights and on a free A stage;
the epilogue warps on a finished accumulator.  The role that never waits
bounds the kernel.

``decode`` runs Qwen3-0.6B greedy decode steps (B rows, context C) on the
trace library and prints, per kernel kind, the median over launches of each
phase stamp relative to the launch's first CTA start, for the median CTA and
the last CTA, and the spacing from one launch's end to the next one's (the
time each kernel adds to the step).  Phase stamps of the tcgen05 linear: 1
TMEM held, 2 weights dequantised (before the dependency wait), 3 wait
returned, 4 accumulator complete, 5 drained, 6 cluster reduction done, 7
epilogue done, 8 activations arrived, 9 MMAs issued, 10 row scales, 11
epilogue inputs staged; of decode attention: 1 wait returned, 2 first tile,
3 last tile arrived, 4 last tile consumed, 5 last unit written, 6 end; of the
CUDA-core GEMV: 1 wait returned, 2 activations staged, 3 products done, 4-5
reduction and epilogue.

The trace library must not be loaded together with the product library;
this module sets ``T2B_LIBRARY`` before the first load.
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
    buf = np.zeros((1 << 15, 16), dtype=np.uint64)   # 128-byte records: t[12] + 8 ints
    eng.prefill(prompts)                       # warm-up; its records are discarded
    torch.cuda.synchronize()
    dump(buf.ctypes.data, 1 << 15, 1)
    eng.prefill(prompts)
    torch.cuda.synchronize()
    eng.check_device_errors()
    m = dump(buf.ctypes.data, 1 << 15, 1)
    recs = buf[:m].copy()
    tags = recs[:, 12:].view(np.int32).reshape(m, 8)[:, 0]
    out = {}
    for tag in sorted(set(tags.tolist())):
        t = recs[tags == tag, :8].astype(np.float64)
        run = t[:, 7]
        row = {"ctas": int((tags == tag).sum()), "run_cycles": float(np.median(run))}
        for k, name in _COLUMNS:
            row[name] = float(np.median(t[:, k] / run))
        out[_KINDS.get(tag, str(tag))] = row
    return out


_DECODE_KINDS = {10: "attention", 1: "tc.store", 2: "tc.residual", 3: "tc.swiglu", 4: "tc.qkv",
                 20: "gemv.store", 21: "gemv.residual", 22: "gemv.swiglu", 23: "gemv.qkv"}


def decode_timeline(batch: int = 64, ctx: int = 190, steps: int = 2) -> dict:
    """kind -> {'launches', 'ctas', 'marks': {phase: (median CTA us, last CTA us)},
    'end_us', 'spacing_us'} over ``steps`` decode steps (CUDA graph replays)."""
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
    eng = DecodeEngine(cfg, model, batch=batch, max_ctx=((ctx + 64 + 63) // 64) * 64, keep_logits=False)
    prompts = torch.randint(0, cfg.vocab_size, (batch, min(128, ctx - 1)), generator=torch.Generator().manual_seed(1))
    eng.prefill(prompts)
    for _ in range(max(0, ctx - 1 - int(eng.pos[0].item()))):
        eng.advance()
    torch.cuda.synchronize()
    L = _lib.load()
    dumps = []
    for unit in ("attn", "tc", "gemv"):
        f = getattr(L, f"t2b_trace_dump_{unit}")
        f.argtypes = [C.c_void_p, C.c_int, C.c_int]
        f.restype = C.c_int
        dumps.append(f)
    cap = 1 << 15
    buf = np.zeros((cap, 16), dtype=np.uint64)
    for f in dumps:
        f(buf.ctypes.data, cap, 1)                # drop the warm-up records
    for _ in range(steps):
        eng.advance()
    torch.cuda.synchronize()
    eng.check_device_errors()
    parts = []
    for f in dumps:
        m = f(buf.ctypes.data, cap, 1)
        if m >= cap:
            raise RuntimeError("trace buffer full: take fewer steps")
        parts.append(buf[:m].copy())
    recs = np.concatenate(parts)
    t = recs[:, :12].astype(np.int64)
    ints = recs[:, 12:].view(np.int32).reshape(-1, 8)
    tag, nblocks = ints[:, 0], ints[:, 4]
    # launches: per kind, consecutive groups of `nblocks` records in arrival order
    launches = []
    for tg in sorted(set(tag.tolist())):
        idx = np.nonzero(tag == tg)[0]
        idx = idx[np.argsort(t[idx, 0], kind="stable")]
        k = 0
        while k < len(idx):
            grp = idx[k:k + int(nblocks[idx[k]])]
            launches.append((int(t[grp, 0].min()), int(t[grp, 1:].max()), tg, grp))
            k += len(grp)
    launches.sort()
    out = {}
    for i, (t0, end, tg, grp) in enumerate(launches):
        row = out.setdefault(_DECODE_KINDS.get(tg, str(tg)), {"launches": 0, "ctas": len(grp), "marks": {},
                                                              "end": [], "spacing": []})
        row["launches"] += 1
        tt = t[grp].astype(np.float64)
        for ph in range(1, 12):
            v = tt[:, ph][tt[:, ph] > 0]
            if len(v):
                row["marks"].setdefault(ph, []).append(((np.median(v) - t0) / 1e3, (v.max() - t0) / 1e3))
        row["end"].append((end - t0) / 1e3)
        if i > 0:
            row["spacing"].append((end - launches[i - 1][1]) / 1e3)
    for row in out.values():
        row["marks"] = {ph: (float(np.median([a for a, _ in v])), float(np.median([b for _, b in v])))
                        for ph, v in row["marks"].items()}
        row["end_us"] = float(np.median(row.pop("end")))
        sp = row.pop("spacing")
        row["spacing_us"] = float(np.median(sp)) if sp else None
    return out


def main(argv: list[str]) -> None:
    usage = "usage: python -m torch2iron_b200.trace prefill [batch prompt] | decode [batch ctx]"
    if not argv or argv[0] not in ("prefill", "decode"):
        raise SystemExit(usage)
    if argv[0] == "decode":
        batch = int(argv[1]) if len(argv) > 1 else 64
        ctx = int(argv[2]) if len(argv) > 2 else 190
        for kind, row in decode_timeline(batch, ctx).items():
            print(f"{kind}: {row['launches']} launches, {row['ctas']} CTAs, last CTA ends at {row['end_us']:.2f} us, "
                  f"adds {row['spacing_us']:.2f} us to the step" if row["spacing_us"] is not None else "")
            for ph, (med, last) in sorted(row["marks"].items()):
                print(f"    stamp {ph:2d}: median CTA {med:6.2f} us, last CTA {last:6.2f} us")
        return
    batch = int(argv[1]) if len(argv) > 1 else 64
    prompt = int(argv[2]) if len(argv) > 2 else 128
    for kind, row in prefill_role_waits(batch, prompt).items():
        cols = " ".join(f"{name}={row[name] * 100:5.1f}%" for _, name in _COLUMNS)
        print(f"{kind:20s} ctas={row['ctas']:5d} run={row['run_cycles']:9.0f} cycles | {cols}")


if __name__ == "__main__":
    main(sys.argv[1:])

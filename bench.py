"""Decode throughput benchmark (decode tokens/s of Qwen3 W4A16 greedy decode).

Workload (benchmark configuration 2 at bs 64): Qwen3-0.6B shapes, 28 layers, tied
bf16 embedding/lm_head, random N(0,0.02) weights quantized int4 g128
(AutoGPTQ-v1 asymmetric RTN), 64 prompts of 128 uniform-random token ids
per GPU, greedy decode.  The prompt is prefilled (untimed), ``--warmup``
decode steps run untimed, then ``--steps`` decode steps are timed.  One step
= one new token for every row.  Multi-GPU (torchrun): data parallel, every
rank decodes its own 64 rows (weak scaling, no collective on the data path);
the N>1 line also carries configuration 4 (Qwen3-8B, 64 rows, ctx 4096)
tensor parallel over the same ranks under ``tp``.

Prints one JSON line on rank 0.  ``--impl reference`` times the reference
algorithm on the host CPU instead (the oracle restatement of
``src/models/quantized_qwen3/model.py``; the reference itself is Python and
has no compiled path to run).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from torch2iron_b200 import _lib, synth  # noqa: E402
from torch2iron_b200.config import PRESETS  # noqa: E402

METRIC = "decode tokens/s (Qwen3 W4A16, bs 1-64, 1/2/4/8 GPU)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=120)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="t2b", choices=["t2b", "reference"])
    ap.add_argument("--batch", type=int, default=64, help="rows per GPU")
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--gen", type=int, default=128,
                    help="tokens the configuration generates per sequence: the timed window is centred on "
                         "the mean decode context prompt + gen/2")
    ap.add_argument("--model", default="qwen3-0.6b", choices=sorted(PRESETS))
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-sample-steps", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemv", action="store_true")
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip the batch sweep (config 2 at 1/8/32 rows) and the config 3 line (N=1 only)")
    ap.add_argument("--no-tp", action="store_true",
                    help="skip the config 4 tensor-parallel run that N>1 bench lines carry under 'tp'")
    ap.add_argument("--tp", type=int, default=0,
                    help="tensor-parallel ranks (config 4: --model qwen3-8b --tp 8 under torchrun); "
                         "the batch is then the global batch")
    ap.add_argument("--ctx", type=int, default=4096, help="--tp: KV cache pre-filled to this many positions")
    ap.add_argument("--tp-eager", action="store_true", help="--tp: launch every step eagerly (no CUDA graph)")
    ap.add_argument("--tp-collective", default="auto", choices=["auto", "nccl", "p2p", "push"],
                    help="tensor parallel: sum the row-parallel partials by NCCL all-reduce, or by the "
                         "peer-memory kernel fused with the residual step (p2p: it loads the peers' partials; "
                         "push: each GEMM epilogue stores its partial into every rank's memory; auto: push "
                         "up to 4 ranks, p2p above)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="one GPU: time the chunked prefill of --batch x --prompt tokens only (profiling case)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock and clock-event reasons of this rank's GPU, sampled every 10 ms
    through NVML (read-only queries) while the timed region runs; nvidia-smi
    (200 ms) when NVML is unavailable."""
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.samples, self._stop = index, [], threading.Event()
        self._nvml = None
        try:
            import pynvml
            self._h = torch.cuda._get_pynvml_handler(index)
            self._nvml = pynvml
            self._bits = (pynvml.nvmlClocksEventReasonHwSlowdown, pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                          pynvml.nvmlClocksEventReasonSwThermalSlowdown, pynvml.nvmlClocksEventReasonSwPowerCap)
            self._max = float(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
        except Exception:
            self._nvml = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _sample(self):
        if self._nvml is not None:
            nv = self._nvml
            sm = float(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
            mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            return [sm, self._max] + [bool(mask & b) for b in self._bits]
        out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                              "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
        parts = [p.strip() for p in out.stdout.strip().split(",")]
        if len(parts) != 6 or not parts[0].replace(".", "").isdigit():
            return None
        return [float(parts[0]), float(parts[1])] + [x.lower() == "active" for x in parts[2:]]

    def _run(self):
        while not self._stop.is_set():
            try:
                smp = self._sample()
                if smp is not None:
                    self.samples.append(smp)
            except Exception:
                pass
            self._stop.wait(0.01 if self._nvml is not None else 0.2)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = sorted({self.NAMES[i] for s in self.samples for i in range(4) if s[2 + i]})
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples), "reasons": reasons, "samples": len(self.samples),
                "source": "nvml" if self._nvml is not None else "nvidia-smi"}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# CPU side (oracle = the reference algorithm restated; checker / baseline only)
# ---------------------------------------------------------------------------
def cpu_decode_rate(cfg, model_cpu, batch, first_ctx, steps, seed, warmup=1):
    """Time ``steps`` oracle decode steps for ``batch`` rows on the host cores,
    step s attending ``first_ctx + s`` keys (positions before ``first_ctx - 1``
    pre-filled with N(0,1) bf16); ``warmup`` untimed steps first."""
    import oracle
    from tests.gpu_util import oracle_decoder

    torch.set_num_threads(os.cpu_count() or 1)
    fill = first_ctx - 1
    dec = oracle_decoder(cfg, model_cpu, batch, first_ctx + steps)
    g = torch.Generator().manual_seed(seed)
    for li in range(cfg.n_layers):
        dec.k_cache[li][:, :, :fill] = torch.randn(batch, cfg.n_kv_groups, fill, cfg.head_dim,
                                                   generator=g).to(torch.bfloat16)
        dec.v_cache[li][:, :, :fill] = torch.randn(batch, cfg.n_kv_groups, fill, cfg.head_dim,
                                                   generator=g).to(torch.bfloat16)
    tok = torch.randint(0, cfg.vocab_size, (batch,), generator=g)
    for _ in range(max(1, warmup)):                                        # page-in; rewrites slot fill
        dec.step(tok, torch.full((batch,), fill, dtype=torch.long))
    t0 = time.perf_counter()
    for s in range(steps):
        logits = dec.step(tok, torch.full((batch,), fill + s, dtype=torch.long))
        tok = torch.argmax(logits, -1)
    dt = time.perf_counter() - t0
    del oracle
    return batch * steps / dt, dt, torch.get_num_threads()


def model_to_cpu(model):
    out = {"layers": [], "embed": model["embed"].cpu(), "final_norm": model["final_norm"].cpu(),
           "lm_head": None if model.get("lm_head") is None else model["lm_head"].cpu()}
    for l in model["layers"]:
        out["layers"].append({k: (v.to("cpu") if hasattr(v, "to") else v) for k, v in l.items()})
    return out


def timed_window(args) -> tuple[int, int]:
    """Keys attended by the first and the last timed step.  The window of
    ``--steps`` steps is centred on the configuration's mean decode context
    (prompt + gen/2: 192 for 128 prompt + 128 generated tokens), and starts
    after the prompt and the warm-up steps."""
    first = max(args.prompt + args.warmup + 1, args.prompt + args.gen // 2 - args.steps // 2)
    return first, first + args.steps - 1


L2_NOTE = "inputs larger than L2 (126 MB): every step reads all weights, the lm_head and the KV cache once"


def arm_config(args, world):
    """The workload description both arms report (identical for the reference arm)."""
    c0, c1 = timed_window(args)
    cfg_no = {"qwen3-0.6b": 2, "llama-3.2-1b": 3, "qwen3-8b": 4}.get(args.model, 2)   # benchmark configuration number
    return {"workload": f"config{cfg_no} {args.model} greedy decode, {args.batch} rows/GPU, prompt {args.prompt}, "
                        f"timed ctx {c0}..{c1}",
            "model": args.model, "global_batch": world * args.batch, "seq_len": c1, "parallelism": f"dp{world}",
            "l2": L2_NOTE}


def run_reference(args, cfg):
    """The reference arm: the reference's CPU decode path (the oracle
    restatement of ``model.py``) on the host cores, rank 0 only, every one of
    the ``--steps`` timed steps run (``--warmup`` untimed steps first) on the
    GPU arm's workload and timed window."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    model = synth.random_model(cfg, seed=args.seed, device="cpu")
    c0, c1 = timed_window(args)
    rate, dt, cores = cpu_decode_rate(cfg, model, args.batch, c0, args.steps, args.seed, warmup=args.warmup)
    line = {"metric": METRIC, "value": round(rate, 3), "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1000 * args.batch / rate, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4-weights/fp32-compute", "data": "synthetic",
            "impl": "reference",
            "config": arm_config(args, args.gpus),
            "cpu_baseline": {"value": round(rate, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"all {args.steps} timed decode steps x {args.batch} rows, ctx {c0}..{c1} "
                                       f"({dt:.1f} s), after {args.warmup} untimed steps; one host process "
                                       "whatever the GPU count"},
            "e2e": {"value": round(rate, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------
# dram__bytes_read.sum + dram__bytes_write.sum of one decode_attention_kernel<128, 2, 3> launch
# captured with ncu on this workload (64 rows x 8 kv heads, ctx 182: 192 keys loaded per unit).
NCU_ATTN = {"dram_bytes": 50_922_496 + 78_336, "units": 64 * 8, "keys_loaded": 192, "head_dim": 128,
            "cold_us": 20.80, "cold_ctx": 182,
            "source": "ncu capture, profiles/decode_attention_qwen3_0.6b_bs64_ctx182.md, scaled by keys loaded"}


def gemv_batch1(eng, peak, n_streams: int = 1):
    """Batch-1 GEMV sweep over every linear of the model (qkv, o, gate_up, down per
    layer) captured in one CUDA graph; the working set (~229 MB) exceeds L2.

    n_streams = 1: one stream, so each GEMV waits for the previous one (the
    dependent-chain cost).  n_streams > 1: the GEMVs are dealt round-robin to
    that many streams forked inside the graph, each with its own output and
    workspace, so independent projections overlap (the streaming cost)."""
    L = _lib.lib()
    cfg = eng.cfg
    ws_n = 1 << 20
    wss = [torch.zeros(ws_n, dtype=torch.uint8, device="cuda") for _ in range(n_streams)]
    x = torch.randn(1, max(cfg.emb_dim, cfg.hidden_dim, cfg.q_dim), device="cuda").to(torch.bfloat16)
    ys = [torch.empty(1, 2 * cfg.hidden_dim + cfg.q_dim + 2 * cfg.kv_dim, dtype=torch.bfloat16, device="cuda")
          for _ in range(n_streams)]
    ws_used = max(L.t2b_w4a16_gemm_workspace_bytes(1, w.out_features, w.in_features)
                  for l in eng.layers for w in (l.qkv, l.o_proj, l.gate_up, l.down))
    assert ws_used <= ws_n
    linears = [w for l in eng.layers for w in (l.qkv, l.o_proj, l.gate_up, l.down)]
    streams = [torch.cuda.Stream() for _ in range(n_streams)]

    def launch(w, i):
        _lib.check("t2b_w4a16_gemm", L.t2b_w4a16_gemm(
            _lib.ptr(w.qw), _lib.ptr(w.meta), 0, _lib.ptr(x), 0, _lib.ptr(ys[i]), 0, 1, w.out_features,
            w.in_features, 128, _lib.ptr(wss[i]), ws_n, _lib.stream()))

    def seq():
        if n_streams == 1:
            for w in linears:
                launch(w, 0)
            return
        main = torch.cuda.current_stream()
        for st in streams:
            st.wait_stream(main)
        for j, w in enumerate(linears):
            with torch.cuda.stream(streams[j % n_streams]):
                launch(w, j % n_streams)
        for st in streams:
            main.wait_stream(st)

    nbytes = sum(w.nbytes_algorithmic + 2 * w.in_features + 2 * w.out_features for w in linears)
    seq()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        seq()
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g):
        seq()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 50
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000 / reps
    gbs = nbytes / (us * 1e-6) / 1e9
    how = "one stream (each waits for the previous)" if n_streams == 1 else \
        f"{n_streams} streams forked in the graph (independent GEMVs overlap)"
    return {"workload": f"{len(linears)} batch-1 GEMVs (all linears of {cfg.n_layers} layers) in one CUDA graph, {how}",
            "bytes": nbytes, "us": round(us, 2), "achieved_gbs": round(gbs, 1), "peak_gbs": peak,
            "frac": round(gbs / peak, 4), "launches": len(linears)}


def kernel_profile(eng, steps):
    """Per-kernel device time over `steps` eager steps (CUDA events on the launch stream)."""
    import collections

    L = _lib.lib()
    cfg, B = eng.cfg, eng.B
    p = _lib.ptr
    times = collections.defaultdict(float)
    counts = collections.defaultdict(int)
    st_obj = torch.cuda.current_stream()
    st = st_obj.cuda_stream
    evs = []

    def rec(name, fn):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st_obj)
        fn()
        b.record(st_obj)
        evs.append((name, a, b))

    for _ in range(steps):
        for li in range(cfg.n_layers):
            lw = eng.layers[li]
            H, hd, nq, nkv = cfg.emb_dim, cfg.head_dim, cfg.n_heads, cfg.n_kv_groups
            rec("qkv_norm_rope_kvwrite", lambda: L.t2b_qkv_norm_rope_kvwrite(
                p(lw.qkv.qw), p(lw.qkv.meta), lw.qkv.fmt, p(eng.xw), p(eng.ssq_a), cfg.rms_norm_eps,
                p(lw.q_norm), p(lw.k_norm), p(eng.angles), p(eng.pos), p(eng.q), _lib.DTYPE[eng.q.dtype],
                p(eng.k_cache[li]),
                p(eng.v_cache[li]), p(eng.ssq_b), B, H, nq, nkv, hd, eng.max_ctx, *eng._ws("qkv"), st))
            rec("decode_attention", lambda: L.t2b_decode_attention_after_kvwrite(
                p(eng.q), _lib.DTYPE[eng.q.dtype], p(eng.k_cache[li]), p(eng.v_cache[li]), p(eng.pos), p(eng.attn),
                _lib.DTYPE[_lib.ACT], B,
                nq, nkv, hd,
                eng.max_ctx, *eng._ws("attn"), st))
            rec("oproj_residual", lambda: L.t2b_oproj_residual(
                p(lw.o_proj.qw), p(lw.o_proj.meta), lw.o_proj.fmt, p(eng.attn), p(eng.x), p(eng.ssq_b), p(lw.post_attention_layernorm), p(eng.xw), B, H, cfg.q_dim,
                *eng._ws("o"), st))
            rec("upgate_swiglu", lambda: L.t2b_upgate_swiglu(
                p(lw.gate_up.qw), p(lw.gate_up.meta), lw.gate_up.fmt, p(eng.xw), p(eng.ssq_b),
                cfg.rms_norm_eps, p(eng.h), p(eng.ssq_a), B, H, cfg.hidden_dim, *eng._ws("ug"), st))
            rec("down_residual", lambda: L.t2b_down_residual(
                p(lw.down.qw), p(lw.down.meta), lw.down.fmt, p(eng.h), p(eng.x), p(eng.ssq_a), p(eng.next_norm_weight(li)), p(eng.xw), B, H, cfg.hidden_dim,
                *eng._ws("down"), st))
        rec("lm_head_argmax", lambda: L.t2b_lm_head_argmax(
            p(eng.xn), p(eng.lm_head), _lib.DTYPE[eng.lm_head.dtype], B, cfg.emb_dim, cfg.vocab_size,
            p(eng.next_tokens), None, None, *eng._ws("lm"), st))
    torch.cuda.synchronize()
    for name, a, b in evs:
        times[name] += a.elapsed_time(b)
        counts[name] += 1
    return {k: (times[k] / counts[k], counts[k]) for k in times}


def kernel_profile_graph(eng, rounds=5):
    """Per-launch device time of each fused op: the op of every layer in turn
    (layer 0, 1, ..., n_layers-1, so consecutive launches read different
    weights and KV caches: at bs 64 the 28 KV caches of the attention launches
    are ~1.4 GB, far above L2) captured as one CUDA graph of back-to-back
    launches -- chained by programmatic dependent launch as in the decode
    step, so a launch's constant-data prologue overlaps its predecessor --
    replayed ``rounds`` times between CUDA events on the capture stream; the
    lm_head 20 times (its 311 MB table exceeds L2).  Returns name -> (ms per
    launch, launches per decode step)."""
    L = _lib.lib()
    cfg, B = eng.cfg, eng.B
    p = _lib.ptr
    H, hd, nq, nkv = cfg.emb_dim, cfg.head_dim, cfg.n_heads, cfg.n_kv_groups
    nl = cfg.n_layers
    lw = eng.layers
    ops = {
        "qkv_norm_rope_kvwrite": (nl, lambda st, i: L.t2b_qkv_norm_rope_kvwrite(
            p(lw[i].qkv.qw), p(lw[i].qkv.meta), lw[i].qkv.fmt, p(eng.xw), p(eng.ssq_a), cfg.rms_norm_eps, p(lw[i].q_norm),
            p(lw[i].k_norm), p(eng.angles), p(eng.pos), p(eng.q), _lib.DTYPE[eng.q.dtype], p(eng.k_cache[i]),
            p(eng.v_cache[i]), p(eng.ssq_b),
            B, H, nq, nkv, hd, eng.max_ctx, *eng._ws("qkv"), st)),
        "decode_attention": (nl, lambda st, i: L.t2b_decode_attention_after_kvwrite(
            p(eng.q), _lib.DTYPE[eng.q.dtype], p(eng.k_cache[i]), p(eng.v_cache[i]), p(eng.pos), p(eng.attn),
            _lib.DTYPE[_lib.ACT], B, nq, nkv,
            hd, eng.max_ctx, *eng._ws("attn"), st)),
        "oproj_residual": (nl, lambda st, i: L.t2b_oproj_residual(
            p(lw[i].o_proj.qw), p(lw[i].o_proj.meta), lw[i].o_proj.fmt, p(eng.attn), p(eng.x), p(eng.ssq_b),
            p(lw[i].post_attention_layernorm), p(eng.xw), B, H, cfg.q_dim, *eng._ws("o"), st)),
        "upgate_swiglu": (nl, lambda st, i: L.t2b_upgate_swiglu(
            p(lw[i].gate_up.qw), p(lw[i].gate_up.meta), lw[i].gate_up.fmt, p(eng.xw), p(eng.ssq_b), cfg.rms_norm_eps, p(eng.h),
            p(eng.ssq_a), B, H, cfg.hidden_dim, *eng._ws("ug"), st)),
        "down_residual": (nl, lambda st, i: L.t2b_down_residual(
            p(lw[i].down.qw), p(lw[i].down.meta), lw[i].down.fmt, p(eng.h), p(eng.x), p(eng.ssq_a), p(eng.next_norm_weight(i)),
            p(eng.xw), B, H, cfg.hidden_dim, *eng._ws("down"), st)),
    }
    if eng.lm_w4 is None:
        ops["lm_head_argmax"] = (1, lambda st, i: L.t2b_lm_head_argmax(
            p(eng.xn), p(eng.lm_head), _lib.DTYPE[eng.lm_head.dtype], B, cfg.emb_dim, cfg.vocab_size,
            p(eng.next_tokens), None, None, *eng._ws("lm"), st))
    out = {}
    side = torch.cuda.Stream()
    for name, (per_step, fn) in ops.items():
        reps = nl if per_step == nl else 20
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(2):
                _lib.check(name, fn(side.cuda_stream, i % nl))
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            st = torch.cuda.current_stream()
            for i in range(reps):
                fn(st.cuda_stream, i % nl)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(rounds):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        out[name] = (e0.elapsed_time(e1) / (rounds * reps), per_step)
        del g
    return out


def advance_to(eng, first_ctx: int) -> None:
    """Untimed greedy steps until the next step attends ``first_ctx`` keys."""
    n = first_ctx - 1 - int(eng.pos[0].item())
    if n < 0:
        raise ValueError(f"the engine is already past context {first_ctx}")
    for _ in range(n):
        eng.advance()
    torch.cuda.synchronize()


def time_steps(eng, steps: int) -> float:
    """Device time (ms, CUDA events on the replay stream) of ``steps`` greedy steps."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        eng.advance()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def decode_point(cfg, model, B, args, first_ctx, peak, seed, prefill=True) -> dict:
    """tokens/s and byte-roofline fraction of B rows decoding from context
    ``first_ctx`` (one GPU): the prompt prefilled (``prefill``) or the KV cache
    filled with N(0,1) bf16 up to ``first_ctx - 1`` positions."""
    from torch2iron_b200.engine import DecodeEngine

    last = first_ctx + args.steps - 1
    max_ctx = ((last + 63) // 64) * 64
    eng = DecodeEngine(cfg, model, batch=B, max_ctx=max_ctx, use_graph=True, keep_logits=False)
    g = torch.Generator().manual_seed(seed)
    if prefill:
        eng.prefill(torch.randint(0, cfg.vocab_size, (B, args.prompt), generator=g))
    else:
        gd = torch.Generator(device="cuda").manual_seed(seed)
        for kc, vc in zip(eng.k_cache, eng.v_cache):
            kc[:, :, :first_ctx - 1].normal_(generator=gd)
            vc[:, :, :first_ctx - 1].normal_(generator=gd)
        eng.tokens.copy_(torch.randint(0, cfg.vocab_size, (B,), generator=g))
        eng.pos.fill_(first_ctx - 1)
        for _ in range(args.warmup):          # warm-up steps rewrite slot first_ctx - 1
            eng.advance()
            eng.pos.fill_(first_ctx - 1)
    advance_to(eng, first_ctx)
    ms = time_steps(eng, args.steps)
    eng.check_device_errors()
    avg = sum(eng.step_bytes([c] * B) for c in range(first_ctx, last + 1)) / args.steps
    gbs = avg / (ms / args.steps * 1e-3) / 1e9
    out = {"batch": B, "value": round(B * args.steps / (ms / 1000), 1), "unit": "tokens/s",
           "ms_per_step": round(ms / args.steps, 4), "ctx": f"{first_ctx}..{last}",
           "algorithmic_bytes_per_step": int(avg), "achieved_gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4)}
    eng.release()
    del eng
    torch.cuda.empty_cache()
    return out


def run_t2b(args, cfg):
    import torch.distributed as dist

    from torch2iron_b200.engine import DecodeEngine

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    B, P = args.batch, args.prompt
    first, last = timed_window(args)
    max_ctx = ((last + 63) // 64) * 64
    model = synth.random_model(cfg, seed=args.seed, device="cuda")
    eng = DecodeEngine(cfg, model, batch=B, max_ctx=max_ctx, use_graph=True, keep_logits=False)
    g = torch.Generator().manual_seed(args.seed * 1000 + rank)
    prompts = torch.randint(0, cfg.vocab_size, (B, P), generator=g)
    eng.prefill(prompts)                     # chunked prefill; the first call sizes its buffers
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    q0.record()
    eng.prefill(prompts)                     # timed: the same prompts again (rewrites the same cache rows)
    q1.record()
    torch.cuda.synchronize()
    prefill_ms = q0.elapsed_time(q1)
    if world > 1:
        t = torch.tensor([prefill_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        prefill_ms = float(t.item())
    advance_to(eng, first)                   # the warm-up steps and the way to the window
    start_tokens = eng.tokens.clone()
    start_pos = eng.pos.clone()
    step_bytes = [eng.step_bytes([c] * B) for c in range(first, last + 1)]

    # ---- device-resident timed region -------------------------------------
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        torch.cuda.nvtx.range_push("timed")   # profiler filter: ncu --nvtx --nvtx-include "timed/"
        e0.record()
        for _ in range(args.steps):
            eng.advance()
        e1.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()

    # ---- end to end through the host API: DecodeEngine.decode_step ---------
    # (pinned host tokens and positions in, next tokens and the status word out,
    # one synchronisation per step)
    eng.tokens.copy_(start_tokens)
    eng.pos.copy_(start_pos)
    tok_h = torch.empty(B, dtype=torch.int32).pin_memory()
    pos_h = torch.empty(B, dtype=torch.int32).pin_memory()
    tok_h.copy_(start_tokens.cpu())
    pos_h.copy_(start_pos.cpu())
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        out = eng.decode_step(tok_h, pos_h)
        tok_h.copy_(out)
        pos_h.add_(1)
    f1.record()
    torch.cuda.synchronize()
    ms_e2e = f0.elapsed_time(f1)
    if world > 1:
        t = torch.tensor([ms_e2e], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    fail_on_device_status(eng, world)

    peak, peak_kind = peaks()
    result = None
    if rank == 0:
        tokens = world * B * args.steps
        value = tokens / (ms / 1000)
        e2e = tokens / (ms_e2e / 1000)
        avg_bytes = sum(step_bytes) / len(step_bytes)
        # roofline of the dominant kernel, from a live per-kernel event profile
        eng.tokens.copy_(start_tokens)
        eng.pos.copy_(start_pos)
        eager = kernel_profile(eng, 2)
        prof = kernel_profile_graph(eng)
        dom = max(prof, key=lambda k: prof[k][0] * prof[k][1])   # device time per decode step
        ctx0 = int(start_pos[0].item()) + 1                      # keys the profiled launches attend
        kv_tok = 2 * cfg.n_kv_groups * cfg.head_dim * 2
        l0 = eng.layers[0]
        kernel_bytes = {
            # K+V of the attended keys, fp32 q in, fp16 output
            "decode_attention": B * ctx0 * kv_tok + B * cfg.q_dim * (4 + 2),
            # weights, fp16 norm input in, fp32 q and bf16 k / v out
            "qkv_norm_rope_kvwrite": l0.qkv.nbytes_algorithmic + B * cfg.emb_dim * 2
                                     + B * (cfg.q_dim * 4 + 2 * cfg.kv_dim * 2),
            # weights, fp16 input, fp32 residual read and written, fp16 next-norm input out
            "oproj_residual": l0.o_proj.nbytes_algorithmic + B * cfg.q_dim * 2 + 2 * B * cfg.emb_dim * 4
                              + B * cfg.emb_dim * 2,
            "upgate_swiglu": l0.gate_up.nbytes_algorithmic + B * cfg.emb_dim * 2 + B * cfg.hidden_dim * 2,
            "down_residual": l0.down.nbytes_algorithmic + B * cfg.hidden_dim * 2 + 2 * B * cfg.emb_dim * 4
                             + B * cfg.emb_dim * 2,
            "lm_head_argmax": eng.lm_head.numel() * 2 + B * cfg.emb_dim * 2 + B * 4,
        }
        dur_ms = prof[dom][0]
        achieved = kernel_bytes[dom] / (dur_ms * 1e-3) / 1e9
        traffic, traffic_src = None, None
        if dom == "decode_attention" and cfg.head_dim == NCU_ATTN["head_dim"]:
            # ncu DRAM bytes of one capture, scaled by the keys this launch loads
            # (tiles load whole 16-key boxes at the end of each unit)
            loaded = 64 * (ctx0 // 64) + 16 * -(-(ctx0 % 64) // 16)
            per_key = NCU_ATTN["dram_bytes"] / (NCU_ATTN["units"] * NCU_ATTN["keys_loaded"])
            traffic = int(per_key * B * cfg.n_kv_groups * loaded)
            traffic_src = NCU_ATTN["source"]
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4-weights/fp16-activations/fp32-accumulate",
            "data": "synthetic (seeded N(0,0.02) weights, uniform-random prompt ids)",
            "config": arm_config(args, world),
            "hbm": {"algorithmic_bytes_per_step": int(avg_bytes),
                    "achieved_gbs": round(avg_bytes / (ms / args.steps * 1e-3) / 1e9, 1),
                    "frac_of_peak": round(avg_bytes / (ms / args.steps * 1e-3) / 1e9 / peak, 4),
                    "peak_gbs": peak, "peak_source": peak_kind},
            "roofline": {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                         "traffic_source": traffic_src,
                         "bytes_per_launch": kernel_bytes[dom], "avg_launch_us": round(dur_ms * 1000, 2),
                         "ctx": ctx0, "peak_source": peak_kind,
                         "timing": "per launch in a CUDA graph of the op over all layers in turn (different "
                                   "weights and KV caches each launch; PDL-chained as in the step), 5 replays, "
                                   "CUDA events on the capture stream",
                         "ncu_cold_launch": ({"us": NCU_ATTN["cold_us"], "ctx": NCU_ATTN["cold_ctx"],
                                              "frac": round(kernel_bytes[dom] / (NCU_ATTN["cold_us"] * 1e-6) / 1e9 / peak, 4),
                                              "note": "the same launch in the decode step under ncu: cold cache, "
                                                      "serialised, no overlap with the qkv kernel"}
                                             if traffic is not None else None),
                         "kernel_avg_us": {k: round(v[0] * 1000, 2) for k, v in prof.items()},
                         "kernel_eager_us": {k: round(v[0] * 1000, 2) for k, v in eager.items()}},
            "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": 2 * B * 4,
                    "d2h_bytes_per_step": B * 4 + 4,
                    "how": "DecodeEngine.decode_step per step: pinned host tokens and positions in, next tokens "
                           "and the status word out (one synchronisation)"},
            "gpu_launches": eng.kernels_per_step() * args.steps,
            "clocks": clocks.summary(),
            "prefill": {"value": round(world * B * P / (prefill_ms / 1000), 1), "unit": "prompt tokens/s",
                        "ms": round(prefill_ms, 3), "prompt_tokens_per_gpu": B * P,
                        "chunk_tokens_per_sequence": min(P, max(1, eng.PREFILL_ROWS // B)),
                        "note": "chunked prefill (all prompt tokens of a chunk per launch), device-resident "
                                "prompts, CUDA events, max over ranks; not part of value"},
        }
        if not args.no_gemv:
            line["gemv_b1"] = gemv_batch1(eng, peak)
            line["gemv_b1_streams"] = gemv_batch1(eng, peak, n_streams=4)
        result = line
    eng.release()
    del eng
    torch.cuda.empty_cache()
    if result is not None and world == 1:
        if not args.no_cpu_baseline:            # host-core baseline: rank 0 at N=1 only
            mcpu = model_to_cpu(model)
            rate, dt, cores = cpu_decode_rate(cfg, mcpu, B, first, args.cpu_sample_steps, args.seed)
            del mcpu
            result["cpu_baseline"] = {"value": round(rate, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                                      "sample": f"{args.cpu_sample_steps} oracle decode steps x {B} rows at ctx "
                                                f"{first}..{first + args.cpu_sample_steps - 1} ({dt:.1f} s)"}
        if not args.no_sweep and args.model == "qwen3-0.6b":
            # the other batch sizes of configuration 2 (same weights, same timed window)
            result["sweep"] = [decode_point(cfg, model, b, args, first, peak, seed=args.seed + b)
                               for b in (1, 8, 32) if b != B]
            # configuration 3: Llama-3.2-1B, 32 rows, KV cache pre-filled to a 2048-token context
            del model
            torch.cuda.empty_cache()
            from torch2iron_b200.config import LLAMA_3_2_1B
            m3 = synth.random_model(LLAMA_3_2_1B, seed=args.seed, device="cuda")
            f3 = 2048 + args.gen // 2 - args.steps // 2
            result["config3"] = dict(decode_point(LLAMA_3_2_1B, m3, 32, args, f3, peak, seed=args.seed + 3,
                                                  prefill=False),
                                     workload="config3 llama-3.2-1b greedy decode, 32 rows, KV cache "
                                              "pre-filled N(0,1) bf16 to a 2048-token context")
            del m3
            torch.cuda.empty_cache()
    if world > 1 and not args.no_tp and args.model == "qwen3-0.6b":
        # configuration 4 on the same ranks: Qwen3-8B tensor parallel over all N GPUs
        del model
        torch.cuda.empty_cache()
        tp_line = tp_measure(args, PRESETS["qwen3-8b"], world, rank, local, batch=64, ctx=4096)
        if result is not None:
            result["tp"] = tp_line
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)


def device_status(eng, world: int) -> int:
    """The largest device status word over the ranks (0: no kernel timed out a
    wait); every rank takes this collective at the same point."""
    code = eng.err.to(torch.int32).clone()
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(code, op=dist.ReduceOp.MAX)
    return int(code.item())


def fail_on_device_status(eng, world: int) -> None:
    """Exit non-zero (after releasing graphs and the process group) when a kernel
    recorded a timed-out wait: its outputs, and so this run's numbers, are void."""
    code = device_status(eng, world)
    if code == 0:
        return
    eng.release()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    raise SystemExit(f"a decode kernel recorded status {code} "
                     f"({_lib.load().t2b_status_string(code).decode()}): measurement void")


def tp_measure(args, cfg, world, rank, local, batch, ctx) -> dict | None:
    """Config 4 on the initialised process group: one model split over the
    ``world`` ranks (tensor parallel), ``batch`` rows in total, the KV cache
    pre-filled with N(0,1) bf16 to ``ctx`` positions; ``--steps`` timed decode
    steps (one CUDA graph per step, the two NCCL all-reduces per layer
    captured between the fused kernels).  Returns rank 0's description (None
    on the other ranks); every rank takes the same collective steps."""
    import torch.distributed as dist

    from torch2iron_b200.tp import TPDecodeEngine

    B, C = batch, ctx
    max_ctx = ((C + args.warmup + args.steps + 1 + 63) // 64) * 64
    model = synth.random_model(cfg, seed=args.seed, device="cuda")
    eng = TPDecodeEngine(cfg, model, batch=B, max_ctx=max_ctx, tp=world, rank=rank, use_graph=not args.tp_eager,
                         collective=args.tp_collective)
    del model
    torch.cuda.empty_cache()
    g = torch.Generator(device="cuda").manual_seed(args.seed * 1000 + 7 + rank)
    for kc, vc in zip(eng.k_cache, eng.v_cache):
        kc[:, :, :C].normal_(generator=g)
        vc[:, :, :C].normal_(generator=g)
    tok = torch.randint(0, cfg.vocab_size, (B,), generator=torch.Generator().manual_seed(args.seed + 3))
    eng.tokens.copy_(tok)
    eng.pos.fill_(C)
    for _ in range(args.warmup):
        eng.advance()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # a step far slower than the byte floor (e.g. a collective stalling) would make
    # the timed loop run for minutes on every GPU: time one step first and cut
    # the loop to ~10 s (every rank takes the same decision: max over ranks)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    eng.advance()
    p1.record()
    torch.cuda.synchronize()
    probe = torch.tensor([p0.elapsed_time(p1)], device="cuda")
    if world > 1:
        dist.all_reduce(probe, op=dist.ReduceOp.MAX)
    steps = max(1, min(args.steps, int(10_000 / max(float(probe.item()), 1e-3))))
    c_first = int(eng.pos[0].item()) + 1
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record()
        for _ in range(steps):
            eng.advance()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    status = device_status(eng, world)
    # bytes one GPU must move per step: its weight shard, lm_head slice, KV of its kv heads
    lc = eng.lcfg
    c_mid = c_first + steps // 2
    kv_tok = 2 * lc.n_kv_groups * cfg.head_dim * 2
    w_bytes = sum(l.algorithmic_bytes for l in eng.layers) + eng.lm_head.numel() * 2
    gpu_bytes = w_bytes + B * c_mid * kv_tok * cfg.n_layers
    peak, peak_kind = peaks()
    line = None
    if rank == 0:
        per_gpu_gbs = gpu_bytes / (ms / steps * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(B * steps / (ms / 1000), 1) if status == 0 else None,
            "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
            "ms_per_step": round(ms / steps, 4), "scaling": "strong",
            "config": {"workload": f"config4 {cfg_name(cfg)} greedy decode, {B} rows, tensor parallel over {world} "
                                   f"GPUs, KV cache pre-filled N(0,1) bf16, ctx {c_first}..{c_first + steps - 1}",
                       "model": cfg_name(cfg), "global_batch": B, "seq_len": c_first + steps - 1,
                       "parallelism": f"tp{world}", "l2": L2_NOTE},
            "hbm": {"algorithmic_bytes_per_step_per_gpu": int(gpu_bytes), "achieved_gbs_per_gpu": round(per_gpu_gbs, 1),
                    "frac_of_peak": round(per_gpu_gbs / peak, 4), "peak_gbs": peak, "peak_source": peak_kind},
            "gpu_launches": eng.kernels_per_step() * steps,
            "collectives_per_step": ({"peer_memory_allreduce_residual": 2 * cfg.n_layers, "head_argmax_merge": 1,
                                      "nccl": 0} if eng.collective in ("p2p", "push") else
                                     {"nccl_allreduce": 2 * cfg.n_layers, "nccl_allgather": 2}),
            "allreduce_dtype": str(eng.partial_dtype).replace("torch.", ""),
            "allreduce": {"nccl": "NCCL all-reduce + t2b_residual_norm_input",
                          "p2p": "t2b_tp_allreduce_residual_norm_input (peer-memory loads over NVLink)",
                          "push": "t2b_w4a16_gemm_push (epilogue stores over NVLink) + "
                                  "t2b_tp_allreduce_residual_norm_input (local loads)"}[eng.collective],
            "device_status": status,
            "clocks": clocks.summary(),
        }
    eng.release()   # graphs holding NCCL calls go before the process group
    del eng
    torch.cuda.empty_cache()
    return line


def cfg_name(cfg) -> str:
    return next((k for k, v in PRESETS.items() if v == cfg), "custom")


def run_tp(args, cfg):
    """``--tp N`` under torchrun: config 4 alone (see tp_measure), one JSON line."""
    import torch.distributed as dist
    from datetime import timedelta

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.tp:
        raise SystemExit(f"--tp {args.tp} needs {args.tp} ranks (torchrun --nproc-per-node {args.tp}), got {world}")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    line = tp_measure(args, cfg, world, rank, local, batch=args.batch, ctx=args.ctx)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        line.update(higher_is_better=True, vs_baseline=None, dtype="int4-weights/fp16-activations/fp32-accumulate",
                    data="synthetic (seeded N(0,0.02) weights, N(0,1) bf16 KV pre-fill, uniform-random token ids)")
        print(json.dumps(line), flush=True)
        if line["device_status"]:
            raise SystemExit(f"a decode kernel recorded status {line['device_status']}: measurement void")


def main():
    args = parse()
    cfg = PRESETS[args.model]
    if args.impl == "reference":
        run_reference(args, cfg)
        return
    if args.tp:
        run_tp(args, cfg)
        return
    if args.prefill_only:
        run_prefill_only(args, cfg)
        return
    run_t2b(args, cfg)


def run_prefill_only(args, cfg):
    """The chunked prefill alone (no decode, no CPU baseline): one untimed call,
    then --steps timed calls; prints one JSON line."""
    from torch2iron_b200.engine import DecodeEngine

    B, P = args.batch, args.prompt
    max_ctx = ((P + 63) // 64) * 64
    model = synth.random_model(cfg, seed=args.seed, device="cuda")
    eng = DecodeEngine(cfg, model, batch=B, max_ctx=max_ctx, use_graph=False, keep_logits=False)
    prompts = torch.randint(0, cfg.vocab_size, (B, P), generator=torch.Generator().manual_seed(args.seed))
    eng.prefill(prompts)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        eng.prefill(prompts)
    e1.record()
    torch.cuda.synchronize()
    eng.check_device_errors()
    ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"metric": "prefill prompt tokens/s", "value": round(B * P / (ms / 1000), 1),
                      "unit": "prompt tokens/s", "ms": round(ms, 3), "model": args.model, "batch": B, "prompt": P,
                      "steps": args.steps}), flush=True)


if __name__ == "__main__":
    main()

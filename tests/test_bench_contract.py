"""bench.py's JSON contract on the host (no GPU): the reference arm prints one
line with every key the driver reads, and both arms describe the workload with
the same `config`."""

import argparse
import io
import json
from contextlib import redirect_stdout

import bench
from torch2iron_b200.config import QuantizedQwenConfig

TINY = QuantizedQwenConfig(vocab_size=512, emb_dim=256, n_layers=1, n_heads=4, n_kv_groups=2, head_dim=64,
                           hidden_dim=512, rms_norm_eps=1e-6, rope_base=1e6)


def _args(**kw):
    a = dict(gpus=1, steps=2, warmup=3, impl="reference", batch=2, prompt=8, gen=16, model="qwen3-0.6b", seed=0,
             cpu_sample_steps=1, no_cpu_baseline=False, no_gemv=True, no_sweep=True, no_tp=True, tp=0, ctx=4096,
             tp_eager=False)
    a.update(kw)
    return argparse.Namespace(**a)


def test_reference_arm_line_has_the_contract_keys():
    out = io.StringIO()
    with redirect_stdout(out):
        bench.run_reference(_args(), TINY)
    line = json.loads(out.getvalue().strip().splitlines()[-1])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["impl"] == "reference" and line["value"] > 0 and line["higher_is_better"] is True
    assert line["metric"] == bench.METRIC and line["unit"] == "tokens/s"
    assert {"value", "unit", "cores", "kind", "sample"} <= set(line["cpu_baseline"])
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    # the reference arm runs every timed step, and reports the GPU arm's workload exactly
    assert line["steps"] == 2 and line["cpu_baseline"]["sample"].startswith("all 2 timed decode steps")
    assert line["config"] == bench.arm_config(_args(), 1)


def test_both_arms_share_the_workload_description():
    a = _args()
    ref_cfg = bench.arm_config(a, a.gpus)
    assert ref_cfg["workload"].startswith("config2 qwen3-0.6b greedy decode")
    assert ref_cfg["global_batch"] == a.batch and ref_cfg["parallelism"] == "dp1"
    first, last = bench.timed_window(a)
    assert (first, last) == (a.prompt + a.gen // 2 - a.steps // 2, a.prompt + a.gen // 2 - a.steps // 2 + 1)
    assert ref_cfg["seq_len"] == last and ref_cfg["l2"] == bench.L2_NOTE
    # the window is centred on prompt + gen/2 (192 for configuration 2's 128 + 128 tokens, 20 steps)
    c2 = _args(prompt=128, gen=128, steps=20, warmup=5)
    assert bench.timed_window(c2) == (182, 201)
    # ... and never starts before the prompt and the warm-up steps
    assert bench.timed_window(_args(prompt=128, gen=128, steps=120, warmup=5)) == (134, 253)
    assert bench.arm_config(_args(model="llama-3.2-1b"), 1)["workload"].startswith("config3")
    assert bench.arm_config(_args(gpus=8), 8)["global_batch"] == 8 * a.batch

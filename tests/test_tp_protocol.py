"""Race check of the tensor-parallel peer-memory protocol, on the CPU.

A small model of what every rank's stream does in one decode step, written
from the kernels it abstracts:

* the row-parallel GEMM (``t2b_w4a16_gemm`` / ``t2b_w4a16_gemm_push``) writes
  its partial tile by tile: into this rank's own buffer (``collective="p2p"``)
  or into this rank's slot of every rank's receive buffer (``"push"``);
  o_proj and down alternate between two buffers (``torch2iron_b200/tp.py``);
* ``tp_allreduce_residual_kernel`` (``csrc/tp_collective.cu``): one CTA per
  row; the call number is the rank's counter + 1, read at entry; CTA 0 stores
  it into flag word ``rank`` of every rank; every CTA waits until all of its
  own flag words reach the call, then reads every rank's partial (peer
  buffers for p2p, its own slots for push); the last CTA stores the counter;
* ``lm_head_argmax_kernel<.., TP=true>`` (``csrc/lm_head.cu``): its last CTA
  writes this rank's keys into every rank's gather buffer, signals on the head
  flags, waits for every rank and reads the gathered keys.

Kernels of one rank run in stream order (every kernel waits for the one before
it); the CTAs of one kernel and the ranks interleave in any order the
scheduler picks.  Each memory operation is one atomic step and the fence
before a flag store makes every earlier write visible first, which is the
ordering the kernels' system-scope fences and acquire loads provide.  A read
that finds another call's data, or a run in which no rank can move, fails.

The mistakes the test plants live in this model only: one buffer for both
linears, and a flag stored while the GEMM's stores are still in flight.
"""

import random

import pytest

ROWS, TILES = 2, 2


def rank_program(rank, world, layers, steps, mode, single_buffer=False, early_signal=False):
    """The kernels one rank enqueues, each a list of CTAs, each a list of ops."""
    prog = []
    for s in range(steps):
        for li in range(layers):
            for which in (0, 1):
                buf = 0 if single_buffer else which
                tag = (s, li, which)
                if mode == "push":
                    dests = [("part", buf, q, rank) for q in range(world)]
                else:
                    dests = [("part", buf, rank)]
                gemm = [[("write", d, tag) for d in dests] for _ in range(TILES)]
                if mode == "push":
                    srcs = [("part", buf, rank, q) for q in range(world)]
                else:
                    srcs = [("part", buf, q) for q in range(world)]
                reads = [("read", k, tag) for k in srcs]
                ctas = [[("signal", "ar", q) for q in range(world)] + [("wait", "ar")] + reads]
                ctas += [[("wait", "ar")] + reads for _ in range(ROWS - 1)]
                if early_signal:
                    # planted: the flag goes out while the GEMM's tiles are still being stored
                    prog.append(("ar", ctas + gemm))
                else:
                    prog.append(("gemm", gemm))
                    prog.append(("ar", ctas))
        head = [("write", ("gather", q, rank), s) for q in range(world)]
        head += [("signal", "head", q) for q in range(world)] + [("wait", "head")]
        head += [("read", ("gather", rank, q), s) for q in range(world)]
        prog.append(("head", [head]))
    return prog


def simulate(world, layers, steps, mode, seed, **plant):
    """Runs every rank's program under one random interleaving; returns the
    list of bad reads (empty when the protocol held)."""
    rng = random.Random(seed)
    speed = [rng.uniform(0.05, 1.0) for _ in range(world)]    # some ranks run far ahead of others
    progs = [rank_program(r, world, layers, steps, mode, **plant) for r in range(world)]
    mem = {}
    flags = {k: [[0] * world for _ in range(world)] for k in ("ar", "head")}   # flags[k][owner][signaller]
    counter = {k: [0] * world for k in ("ar", "head")}
    kernel = [0] * world                       # index of the running kernel per rank
    ctas = [None] * world                      # its CTAs' remaining ops
    call = [0] * world
    bad = []

    def start(r):
        if kernel[r] >= len(progs[r]):
            ctas[r] = None
            return
        kind, body = progs[r][kernel[r]]
        ctas[r] = [list(c) for c in body]
        k = "head" if kind == "head" else "ar"
        call[r] = counter[k][r] + 1

    def enabled(r, ci):
        op = ctas[r][ci][0]
        if op[0] != "wait":
            return True
        return all(f >= call[r] for f in flags[op[1]][r])

    for r in range(world):
        start(r)
    while True:
        choices = [(r, ci) for r in range(world) if ctas[r] is not None
                   for ci, c in enumerate(ctas[r]) if c and enabled(r, ci)]
        if not choices:
            live = [r for r in range(world) if ctas[r] is not None]
            if live:
                raise AssertionError(f"no rank can move (ranks {live} wait): the protocol deadlocked")
            return bad
        weights = [speed[r] for r, _ in choices]
        r, ci = rng.choices(choices, weights)[0]
        op = ctas[r][ci].pop(0)
        if op[0] == "write":
            mem[op[1]] = op[2]
        elif op[0] == "signal":
            flags[op[1]][op[2]][r] = call[r]
        elif op[0] == "read":
            if mem.get(op[1]) != op[2]:
                bad.append((r, op[1], op[2], mem.get(op[1])))
        if not any(ctas[r]):                   # kernel done: the last CTA stores the call counter
            kind = progs[r][kernel[r]][0]
            if kind in ("ar", "head"):
                counter["head" if kind == "head" else "ar"][r] = call[r]
            kernel[r] += 1
            start(r)


@pytest.mark.parametrize("mode", ["p2p", "push"])
@pytest.mark.parametrize("world,seeds", [(2, 300), (3, 150), (4, 100), (8, 25)])
def test_protocol_has_no_race_or_deadlock(mode, world, seeds):
    """Every interleaving tried: each rank reads exactly the partials of the
    call it is in, and every run ends."""
    for seed in range(seeds):
        bad = simulate(world, layers=3, steps=2, mode=mode, seed=seed)
        assert not bad, f"seed {seed}: rank {bad[0][0]} read {bad[0][1]} expecting {bad[0][2]}, found {bad[0][3]}"


@pytest.mark.parametrize("mode", ["p2p", "push"])
def test_model_finds_a_shared_buffer_race(mode):
    """With one buffer for o_proj and down, a fast rank's down GEMM overwrites a
    partial a slower rank is still reading: the model must find it."""
    found = sum(bool(simulate(2, layers=3, steps=2, mode=mode, seed=s, single_buffer=True)) for s in range(200))
    assert found > 0


@pytest.mark.parametrize("mode", ["p2p", "push"])
def test_model_finds_a_flag_before_the_data(mode):
    """A flag stored before the GEMM's stores finished lets a peer read a stale
    partial: the model must find it."""
    found = sum(bool(simulate(2, layers=3, steps=2, mode=mode, seed=s, early_signal=True)) for s in range(200))
    assert found > 0

"""CPU oracle for the W4A16 decode hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch-CPU fp32 arithmetic, the reference
implementation of torch2iron's quantized Qwen3 decode path
(``src/models/quantized_qwen3/model.py``,
``src/models/fast_qwen3/fast_packed_format.py``, the attention references of
``src/models/fast_qwen3/`` and the Q4NX layout of
``src/models/fast_qwen3/q4nx_layout.py``).  Every function cites the
reference file:line it follows.

It is the checker, never the product:

* only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
  / ``--impl reference`` legs may import it;
* the ``torch2iron_b200`` package never imports it and has no CPU fallback.

Parity pin: ``tests/golden/make_golden.py`` imports the reference itself (in
the build container, where it is mounted) and writes golden input/output
vectors to ``tests/golden/*.npz`` (``make_packed_artifact.py``,
``make_kv_plane.py`` and ``make_q4nx.py`` beside it cover the packed artifact,
the KV-plane attention and the Q4NX layout); ``tests/test_oracle_golden.py``
and ``tests/test_loaders.py`` check this restatement against them.
"""

from .reference_port import *  # noqa: F401,F403

"""B200-native (sm_100a) W4A16 group-128 decode hot path of torch2iron.

Public surface:

* ``torch2iron_b200.operators`` -- the reference's operator names
  (``W4A16GEMV``, the ``W4A16GEMM`` family, ``RMSNormRoPE``,
  ``LlamaChunkedAttention``, ``ResidualAddRMSNorm``, ``SiLUMul``,
  ``CopyPresentPacketKV``) backed by
  CUDA kernels through the C-ABI library ``libt2b.so``;
* ``torch2iron_b200.engine`` -- ``DecodeEngine``: the fused decode step (five
  launches per layer, CUDA graph, programmatic dependent launch), chunked
  prefill and greedy generation;
* ``torch2iron_b200.tp`` -- ``TPDecodeEngine``: the same step tensor-parallel
  over NCCL ranks;
* ``torch2iron_b200.loaders`` -- the reference's packed artifact and AutoGPTQ
  checkpoints into the engine's model dict;
* ``torch2iron_b200.synth`` -- seeded synthetic AutoGPTQ weights;
* ``torch2iron_b200.trace`` -- role-wait diagnostics with the trace build.

Importing the package does not load CUDA code; the first kernel call does,
and it raises if ``libt2b.so`` is missing (there is no CPU fallback).
"""

__all__ = ["config", "synth"]

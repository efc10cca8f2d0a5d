"""B200-native (sm_100a) W4A16 group-128 decode hot path of torch2iron.

Public surface:

* ``torch2iron_b200.operators`` -- the reference's operator names
  (``W4A16GEMV``, ``W4A16GEMM``, ``RMSNormRoPE``, ``LlamaChunkedAttention``,
  ``ResidualAddRMSNorm``, ``SiLUMul``, ``CopyPresentPacketKV``) backed by
  CUDA kernels through the C-ABI library ``libt2b.so``;
* ``torch2iron_b200.modules`` -- ``PackedW4A16Linear`` / ``QuantizedQwenLayer``
  style modules and the CUDA-graph decode engine;
* ``torch2iron_b200.synth`` -- seeded synthetic AutoGPTQ weights.

Importing the package does not load CUDA code; the first kernel call does,
and it raises if ``libt2b.so`` is missing (there is no CPU fallback).
"""

__all__ = ["config", "synth"]

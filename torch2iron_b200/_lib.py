"""ctypes binding of ``libt2b.so`` (declarations mirror ``include/t2b.h``).

The library is loaded on first use.  There is no fallback: if the shared
object is missing or no CUDA device is present, ``lib()`` raises.
"""

from __future__ import annotations

import ctypes as C
import os
from contextlib import contextmanager
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("T2B_LIBRARY") or Path(__file__).resolve().parent / "libt2b.so")

T2B_OK = 0
DTYPE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}
ACT = torch.float16          # the fused decode layer's activations (linear inputs), see include/t2b.h
QDT = torch.float32          # its q between the qkv kernel and the decode attention (two-term score MMAs)
WFMT_T2B = 0
WFMT_QPARAM = 1
WFMT_Q4NX = 2

P = C.c_void_p
I = C.c_int
F = C.c_float
Z = C.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "t2b_version": (I, []),
    "t2b_status_string": (C.c_char_p, [I]),
    "t2b_workspace_init": (I, [P, Z, P]),
    "t2b_repack_autogptq": (I, [P, P, P, I, I, I, P, P, I, I, I, P]),
    "t2b_w4a16_gemm_workspace_bytes": (Z, [I, I, I]),
    "t2b_linear_plan": (I, [I, I, I, P, P, P, P]),
    "t2b_linear_plan_qkv": (I, [I, I, I, P, P, P, P]),
    "t2b_tp_allreduce_state_bytes": (Z, []),
    "t2b_w4a16_gemm_push": (I, [P, P, I, P, I, P, I, P, I, I, I, I, I, P, Z, P]),
    "t2b_lm_head_argmax_tp": (I, [P, P, I, I, I, I, I, P, P, P, I, I, P, P, Z, P]),
    "t2b_tp_allreduce_residual_norm_input": (I, [P, I, P, P, I, I, P, P, P, P, I, I, P]),
    "t2b_w4a16_gemm": (I, [P, P, I, P, I, P, I, I, I, I, I, P, Z, P]),
    "t2b_w4a16_gemm_noalloc_max_workspace": (Z, []),
    "t2b_w4a16_gemm_noalloc": (I, [P, P, I, P, I, P, I, I, I, I, I, P]),
    "t2b_qkv_workspace_bytes": (Z, [I, I, I, I, I]),
    "t2b_qkv_norm_rope_kvwrite": (I, [P, P, I, P, P, F, P, P, P, P, P, I, P, P, P, I, I, I, I, I, I, P, Z, P]),
    "t2b_qkv_norm_rope_kvwrite_seq": (I, [P, P, I, P, P, F, P, P, P, P, P, I, P, P, P, P, I, I, I, I, I, I, P, Z, P]),
    "t2b_prefill_attention": (I, [P, P, P, P, I, I, I, I, I, I, I, I, P]),
    "t2b_decode_attention_workspace_bytes": (Z, [I, I, I, I, I]),
    "t2b_decode_attention": (I, [P, I, P, P, P, P, I, I, I, I, I, I, P, Z, P]),
    "t2b_decode_attention_after_kvwrite": (I, [P, I, P, P, P, P, I, I, I, I, I, I, P, Z, P]),
    "t2b_packet_attention": (I, [P, P, P, I, I, I, I, I, P, Z, P]),
    "t2b_oproj_residual_workspace_bytes": (Z, [I, I, I]),
    "t2b_oproj_residual": (I, [P, P, I, P, P, P, P, P, I, I, I, P, Z, P]),
    "t2b_upgate_swiglu_workspace_bytes": (Z, [I, I, I]),
    "t2b_upgate_swiglu": (I, [P, P, I, P, P, F, P, P, I, I, I, P, Z, P]),
    "t2b_down_residual_workspace_bytes": (Z, [I, I, I]),
    "t2b_down_residual": (I, [P, P, I, P, P, P, P, P, I, I, I, P, Z, P]),
    "t2b_embed_rows": (I, [P, P, P, P, P, P, I, I, I, P]),
    "t2b_rms_norm_rows": (I, [P, P, P, F, P, I, I, I, P]),
    "t2b_set_error_word": (I, [P]),
    "t2b_bind_error_word": (I, [P, P]),
    "t2b_error_word_for_stream": (I, [P, P]),
    "t2b_selftest_bounded_wait": (I, [P, I, P]),
    "t2b_residual_norm_input": (I, [P, I, P, P, P, P, I, I, P]),
    "t2b_lm_head_argmax_workspace_bytes": (Z, [I]),
    "t2b_lm_head_argmax": (I, [P, P, I, I, I, I, P, P, P, P, Z, P]),
    "t2b_argmax_workspace_bytes": (Z, [I, I]),
    "t2b_argmax_rows": (I, [P, I, I, I, I, P, P, Z, P]),
    "t2b_rms_norm_rope": (I, [P, P, P, P, I, I, I, F, I, P]),
    "t2b_residual_add_rms_norm": (I, [P, P, P, P, P, I, I, F, P]),
    "t2b_silu_mul": (I, [P, P, P, I, P]),
    "t2b_copy_present_packet_kv": (I, [P, P, P, P, P, I, I, I, I, I, I, P]),
}

_lib = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Load the shared library and declare every entry point (no device needed)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p} is missing: build it with `python -m torch2iron_b200.build` "
                           "(the CUDA path has no CPU fallback)")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def lib() -> C.CDLL:
    """The loaded library, for calls that launch kernels (requires CUDA)."""
    if not torch.cuda.is_available():
        raise RuntimeError("torch2iron_b200 kernels need a CUDA device (sm_100a); there is no CPU fallback")
    return load()


class T2BError(RuntimeError):
    def __init__(self, fn: str, status: int):
        msg = load().t2b_status_string(status).decode()
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.status = status


def check(fn: str, status: int) -> None:
    if status != T2B_OK:
        raise T2BError(fn, status)


def call(fn: str, *args) -> None:
    check(fn, getattr(lib(), fn)(*args))


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    return t.data_ptr()


def stream(s: torch.cuda.Stream | None = None) -> int:
    return (s or torch.cuda.current_stream()).cuda_stream


@contextmanager
def status_word(word: torch.Tensor, st: int):
    """Launches on stream ``st`` inside this block record timed-out device waits
    in ``word`` (int32 device tensor): the stream is bound to it
    (``t2b_bind_error_word``) and unbound on exit.  A block nested in one
    that already bound the same word leaves the binding alone."""
    L = load()
    mine = ptr(word)
    cur = C.c_void_p()
    check("t2b_error_word_for_stream", L.t2b_error_word_for_stream(st, C.byref(cur)))
    if cur.value == mine:
        yield
        return
    check("t2b_bind_error_word", L.t2b_bind_error_word(st, mine))
    try:
        yield
    finally:
        L.t2b_bind_error_word(st, None)

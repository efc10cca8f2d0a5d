"""CPU checks of the C-ABI library: it loads and exports every symbol the header declares."""

import re
from pathlib import Path

import pytest

from torch2iron_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "t2b.h").read_text()
    return sorted(set(re.findall(r"T2B_API\s+[\w\s\*]+?\b(t2b_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = header_symbols()
    assert len(syms) >= 20
    assert "t2b_w4a16_gemm" in syms and "t2b_decode_attention" in syms


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    for s in header_symbols():
        assert hasattr(lib, s), s


def test_binding_covers_header():
    assert set(header_symbols()) == set(_lib.SIGNATURES)


def test_status_strings_and_host_side_errors():
    lib = _lib.load()
    assert lib.t2b_version() >= 1
    assert b"shape" in lib.t2b_status_string(1)
    # host-side validation happens before any launch: no device needed
    assert lib.t2b_w4a16_gemm(None, None, 0, None, 0, None, 0, 1, 128, 256, 128, None, 0, None) == 6
    assert lib.t2b_w4a16_gemm(1, 1, 0, 1, 0, 1, 0, 1, 128, 256, 64, None, 0, None) == 1   # group 64
    assert lib.t2b_decode_attention(16, 0, 16, 16, 16, 16, 0, 1, 16, 8, 128, 100, None, 0, None) == 1  # ctx % 8
    assert lib.t2b_decode_attention(16, 0, 16, 16, 16, 16, 2, 1, 16, 8, 128, 128, None, 0, None) == 6  # fp32 out
    assert lib.t2b_decode_attention(16, 1, 16, 16, 16, 16, 0, 1, 16, 8, 128, 128, None, 0, None) == 6  # fp16 q
    args = (1e-6, 16, 16, 16, 16, 16, 2, 16, 16, 16)       # eps, norms, angles, pos, q (fp32), caches, ssq_clear
    assert lib.t2b_qkv_norm_rope_kvwrite(16, 16, 0, 16, 16, *args, 1, 1024, 16, 8, 96, 64, None, 0,
                                         None) == 1   # head_dim 96
    assert lib.t2b_qkv_norm_rope_kvwrite(16, 16, 1, 16, 16, *args, 1, 1024, 16, 8, 128, 64, None, 0,
                                         None) == 6   # the fused ops take T2B or Q4NX weights, not qparam rows
    assert lib.t2b_w4a16_gemm(16, 16, 2, 16, 0, 16, 0, 1, 128, 256, 128, None, 0, None) == 1   # Q4NX is group 32


def test_workspace_queries():
    lib = _lib.load()
    assert lib.t2b_w4a16_gemm_workspace_bytes(1, 128, 256) >= 0
    assert lib.t2b_w4a16_gemm_workspace_bytes(8, 1024, 3072) == 0     # k-slices meet in a cluster
    assert lib.t2b_w4a16_gemm_workspace_bytes(1, 1024, 12288) > 0     # more than 8 k-slices: workspace
    assert lib.t2b_decode_attention_workspace_bytes(64, 16, 8, 128, 256) > 0   # tickets + partial records
    assert lib.t2b_decode_attention_workspace_bytes(1, 16, 8, 128, 4096) > 0


def _header_prototypes():
    """name -> (return type, [parameter types]) of every T2B_API declaration."""
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "t2b.h").read_text(), flags=re.S)
    protos = {}
    for m in re.finditer(r"T2B_API\s+([\w\s\*]+?)\s*\b(t2b_\w+)\s*\(([^)]*)\)\s*;", text):
        ret, name, params = m.group(1).strip(), m.group(2), m.group(3).strip()
        types = [] if params in ("", "void") else [p.strip().rsplit(" ", 1)[0] if not p.strip().endswith("*")
                                                     else p.strip() for p in params.split(",")]
        protos[name] = (ret, [p.replace(" ", "") if "*" in p else p for p in types])
    return protos


def _ctype(c_type):
    import ctypes as C
    t = " ".join(c_type.split())
    if "*" in t:
        return C.c_void_p
    if t.endswith("size_t"):
        return C.c_size_t
    if t.endswith("float"):
        return C.c_float
    if t.endswith("int") or t.endswith("int32_t"):
        return C.c_int
    raise AssertionError(f"unmapped C type {c_type!r}")


def test_binding_signatures_match_header_prototypes():
    """Every ctypes declaration has the header's parameter count and kinds
    (pointer / int / float / size_t) and return kind, so a changed C signature
    cannot be called with a stale argument list."""
    import ctypes as C
    protos = _header_prototypes()
    assert set(protos) == set(_lib.SIGNATURES)
    for name, (ret, params) in protos.items():
        res, args = _lib.SIGNATURES[name]
        assert len(args) == len(params), (name, params)
        for i, (a, p) in enumerate(zip(args, params)):
            assert a == _ctype(p), (name, i, p)
        want_ret = C.c_char_p if "char" in ret else _ctype(ret)
        assert res == want_ret, (name, ret)


def test_status_word_bindings_are_per_stream_and_per_thread():
    """Host-side table of the device status words (no device work): a stream's
    binding wins over the thread's default; defaults are per host thread."""
    import ctypes as C
    import threading

    lib = _lib.load()

    def word_for(stream):
        out = C.c_void_p()
        assert lib.t2b_error_word_for_stream(stream, C.byref(out)) == 0
        return out.value

    s1, s2, w1, w2, wd = 0x1000, 0x2000, 0x10, 0x20, 0x30     # stand-in handles, never dereferenced
    assert lib.t2b_set_error_word(wd) == 0
    assert lib.t2b_bind_error_word(s1, w1) == 0
    assert lib.t2b_bind_error_word(s2, w2) == 0
    assert word_for(s1) == w1 and word_for(s2) == w2 and word_for(0x3000) == wd
    assert lib.t2b_bind_error_word(s1, w2) == 0                # rebinding replaces
    assert word_for(s1) == w2
    seen = {}
    t = threading.Thread(target=lambda: seen.update(other=word_for(0x3000), bound=word_for(s2)))
    t.start()
    t.join()
    assert seen == {"other": None, "bound": w2}                # another thread: no default, same bindings
    for s in (s1, s2):
        assert lib.t2b_bind_error_word(s, None) == 0
    assert word_for(s1) == wd
    assert lib.t2b_set_error_word(None) == 0
    assert word_for(s1) is None


def test_tp_allreduce_rejects_bad_arguments_on_the_host():
    """The peer-memory all-reduce checks its arguments before anything touches a device."""
    import ctypes as C

    import torch
    L = _lib.load()
    buf = (C.c_uint8 * 4096)()
    base = (C.addressof(buf) + 255) & ~255           # 16-byte aligned host stand-ins (never dereferenced)
    parts = (C.c_void_p * 2)(base, base + 1024)
    flags = (C.c_void_p * 2)(base + 2048, base + 2048 + 16)
    st = base + 3072
    f = L.t2b_tp_allreduce_residual_norm_input
    BF16, F16 = _lib.DTYPE[torch.bfloat16], _lib.DTYPE[torch.float16]
    ERR_SHAPE, ERR_ALIGN, ERR_ARG = 1, 2, 6                  # t2b.h status codes

    def call(world=2, rank=0, dtype=BF16, M=4, H=64, parts_=parts, x=base + 512, w=None, xw=None):
        return f(C.addressof(parts_), dtype, C.addressof(flags), st, rank, world, x, None, w, xw, M, H, None)

    assert call(world=0) == ERR_ARG
    assert call(world=9) == ERR_ARG
    assert call(rank=2) == ERR_ARG
    assert call(dtype=F16) == ERR_ARG
    assert call(w=base + 16) == ERR_ARG            # norm weight without an output (or the reverse)
    assert call(H=60) == ERR_SHAPE
    assert call(M=0) == ERR_SHAPE
    assert call(parts_=(C.c_void_p * 2)(base + 4, base + 1024)) == ERR_ALIGN
    assert call(x=base + 4) == ERR_ALIGN
    assert L.t2b_tp_allreduce_state_bytes() >= 8


def test_tp_head_rejects_bad_arguments_on_the_host():
    """The tensor-parallel greedy head checks its arguments before anything touches a device."""
    import ctypes as C
    L = _lib.load()
    buf = (C.c_uint8 * 8192)()
    base = (C.addressof(buf) + 255) & ~255           # 16-byte aligned host stand-ins (never dereferenced)
    gather = (C.c_void_p * 2)(base, base + 1024)
    flags = (C.c_void_p * 2)(base + 2048, base + 2048 + 16)
    f = L.t2b_lm_head_argmax_tp
    ERR_SHAPE, ERR_ALIGN, ERR_ARG = 1, 2, 6                  # t2b.h status codes

    def call(world=2, rank=0, off=0, V=1024, xn=base + 4096, gather_=gather):
        return f(xn, base + 6144, 0, 4, 64, V, off, C.addressof(gather_), C.addressof(flags), base + 3072, rank, world,
                 base + 3584, base + 7168, 512, None)

    assert call(world=0) == ERR_ARG
    assert call(world=9) == ERR_ARG
    assert call(rank=2) == ERR_ARG
    assert call(off=-1) == ERR_ARG
    assert call(off=0x7FFFFFF0, V=1024) == ERR_SHAPE
    assert call(xn=base + 4100) == ERR_ALIGN
    assert call(gather_=(C.c_void_p * 2)(base + 4, base + 1024)) == ERR_ALIGN


def test_gemm_push_rejects_bad_arguments_on_the_host():
    """The row-parallel GEMM that pushes its partial into peer buffers checks the
    peers, the output type and the alignment before it launches anything."""
    import ctypes as C

    import torch
    L = _lib.load()
    buf = (C.c_uint8 * 8192)()
    base = (C.addressof(buf) + 255) & ~255           # 16-byte aligned host stand-ins (never dereferenced)
    f = L.t2b_w4a16_gemm_push
    BF16, F16, F32 = (_lib.DTYPE[t] for t in (torch.bfloat16, torch.float16, torch.float32))
    ERR_SHAPE, ERR_ALIGN, ERR_ARG = 1, 2, 6                  # t2b.h status codes
    good = (C.c_void_p * 7)(*[base + 4096 + 256 * i for i in range(7)])

    def call(peers=good, n=1, y=base + 2048, y_dtype=BF16, N=128, K=256):
        return f(base, base + 1024, _lib.WFMT_T2B, base + 1536, F16, y, y_dtype, C.addressof(peers) if peers else None,
                 n, 4, N, K, 128, None, 0, None)

    assert call(n=8) == ERR_ARG
    assert call(n=-1) == ERR_ARG
    assert call(peers=None) == ERR_ARG
    assert call(y_dtype=F16) == ERR_ARG
    assert call(N=96) == ERR_SHAPE
    assert call(y=base + 2052, y_dtype=F32) == ERR_ALIGN
    assert call(peers=(C.c_void_p * 2)(base + 4096, base + 4100), n=2) == ERR_ALIGN
    assert call(peers=(C.c_void_p * 2)(base + 4096, None), n=2) == ERR_ARG

"""Tensor-parallel decode for the largest config (Qwen3-8B on 8 GPUs, one rank per GPU).

The sharding follows the Megatron split the reference's own N-shard operator
describes for its projections (``W4A16NShardGEMM``,
``src/models/quantized_qwen3/operators/w4a16_gemm/op.py:336-399``), applied to a
decoder layer (``model.py:240-327``):

* q/k/v -- column-parallel by head: rank r owns q heads ``[r*nq/tp, (r+1)*nq/tp)``
  and kv heads ``[r*nkv/tp, ...)``, so QK-norm, RoPE, the KV cache and the
  attention over it stay on the rank (they are per head);
* o_proj -- row-parallel: rank r holds the input columns of its q heads and
  produces a partial ``[B, H]`` that is summed across ranks;
* gate / up -- column-parallel (``I/tp`` rows each, interleaved in 64-row
  blocks as on one GPU), SwiGLU local;
* down -- row-parallel over the ``I/tp`` columns of the rank's gate/up rows;
* lm_head -- vocab-parallel: each rank scores ``V/tp`` rows, takes its local
  argmax, and the (value, index) pairs of all ranks are gathered (greedy
  decoding needs no full logits row on any rank).

Every split falls on a 128-wide quantization group (``H/tp``, ``I/tp`` and
the head blocks are multiples of 128), so no scale or zero point is split.
The residual stream, embedding and norms are replicated.  The two row-parallel
partials per layer (bf16 by default, ``[B, H]`` = 512 KiB at 64 rows of
Qwen3-8B; fp32 on request) are summed across ranks and added into the fp32
residual stream by one of:

* ``collective="p2p"``: ``t2b_tp_allreduce_residual_norm_input``, one
  kernel that signals and reads the peers' partials over NVLink (peer-mapped
  buffers from ``torch.distributed._symmetric_memory``) and does the residual
  step; o_proj and down write alternate partial buffers;
* ``collective="push"``: o_proj and down run as ``t2b_w4a16_gemm_push``, whose
  epilogue stores each output tile into this rank's slot of every rank's
  receive buffer; the same all-reduce kernel then sums the slots from local
  memory;
* ``collective="nccl"``: an NCCL all-reduce on the decode stream followed by
  ``t2b_residual_norm_input``;
* ``collective="auto"`` (default): push up to ``AUTO_PUSH_MAX_RANKS`` ranks,
  p2p above.

With the peer-memory collectives the greedy head also merges its pick over the
ranks inside its kernel (``t2b_lm_head_argmax_tp``); with ``"nccl"`` the local
(max, index) pairs are all-gathered and merged by ``merge_argmax``.
"""

from __future__ import annotations

import torch

from .synth import AutoGPTQLinear


# ---------------------------------------------------------------------------
# shard helpers on AutoGPTQ-v1 tensors (qweight [K/8, N], qzeros [G, N/8], scales [G, N])
# ---------------------------------------------------------------------------
def shard_out(lin: AutoGPTQLinear, n0: int, n1: int) -> AutoGPTQLinear:
    """Output rows ``[n0, n1)`` of a linear (column-parallel shard)."""
    if n0 % 8 or n1 % 8 or not 0 <= n0 < n1 <= lin.out_features:
        raise ValueError(f"output split [{n0}, {n1}) must be 8-aligned inside [0, {lin.out_features})")
    return AutoGPTQLinear(lin.qweight[:, n0:n1].contiguous(), lin.qzeros[:, n0 // 8:n1 // 8].contiguous(),
                          lin.scales[:, n0:n1].contiguous(), lin.in_features, n1 - n0, lin.group_size)


def shard_in(lin: AutoGPTQLinear, k0: int, k1: int) -> AutoGPTQLinear:
    """Input columns ``[k0, k1)`` of a linear (row-parallel shard); group-aligned."""
    g = lin.group_size
    if k0 % g or k1 % g or not 0 <= k0 < k1 <= lin.in_features:
        raise ValueError(f"input split [{k0}, {k1}) must fall on {g}-wide groups inside [0, {lin.in_features})")
    return AutoGPTQLinear(lin.qweight[k0 // 8:k1 // 8].contiguous(), lin.qzeros[k0 // g:k1 // g].contiguous(),
                          lin.scales[k0 // g:k1 // g].contiguous(), k1 - k0, lin.out_features, g)


def check_tp(cfg, tp: int) -> None:
    if tp < 1 or cfg.n_kv_groups % tp or cfg.n_heads % tp:
        raise ValueError(f"tp={tp} must divide the {cfg.n_heads} q and {cfg.n_kv_groups} kv heads")
    if (cfg.hidden_dim // tp) % 256 or cfg.hidden_dim % tp:
        raise ValueError(f"intermediate {cfg.hidden_dim} / tp={tp} must be a multiple of 256")
    if (cfg.n_heads // tp * cfg.head_dim) % 256:
        raise ValueError("the q columns of a rank must be a multiple of 256 (o_proj K split)")
    if cfg.vocab_size % tp:
        raise ValueError(f"vocab {cfg.vocab_size} must divide by tp={tp}")


def shard_layer(layer: dict, cfg, tp: int, rank: int) -> dict:
    """The rank's share of one layer's AutoGPTQ linears; norms are shared."""
    check_tp(cfg, tp)
    hd = cfg.head_dim
    nq, nkv, ib = cfg.n_heads // tp, cfg.n_kv_groups // tp, cfg.hidden_dim // tp
    q0, kv0, i0 = rank * nq * hd, rank * nkv * hd, rank * ib
    out = {
        "q_proj": shard_out(layer["q_proj"], q0, q0 + nq * hd),
        "k_proj": shard_out(layer["k_proj"], kv0, kv0 + nkv * hd),
        "v_proj": shard_out(layer["v_proj"], kv0, kv0 + nkv * hd),
        "o_proj": shard_in(layer["o_proj"], q0, q0 + nq * hd),
        "gate_proj": shard_out(layer["gate_proj"], i0, i0 + ib),
        "up_proj": shard_out(layer["up_proj"], i0, i0 + ib),
        "down_proj": shard_in(layer["down_proj"], i0, i0 + ib),
    }
    for k in ("input_layernorm", "post_attention_layernorm", "q_norm", "k_norm"):
        if k in layer:
            out[k] = layer[k]
    return out


def local_config(cfg, tp: int):
    """Shapes one rank computes with (heads, intermediate divided by tp)."""
    check_tp(cfg, tp)
    return cfg.scaled(n_heads=cfg.n_heads // tp, n_kv_groups=cfg.n_kv_groups // tp, hidden_dim=cfg.hidden_dim // tp)


def vocab_slice(cfg, tp: int, rank: int) -> tuple[int, int]:
    v = cfg.vocab_size // tp
    return rank * v, (rank + 1) * v


def merge_argmax(vals: torch.Tensor, idx: torch.Tensor, v_per_rank: int) -> torch.Tensor:
    """Greedy token from per-rank (max, local index) pairs ``[tp, B]``: largest
    value, ties to the lowest global index (torch.argmax over the full row)."""
    glob = idx.to(torch.int64) + v_per_rank * torch.arange(vals.shape[0], device=vals.device)[:, None]
    best = vals.max(dim=0, keepdim=True).values
    cand = torch.where(vals == best, glob, torch.full_like(glob, torch.iinfo(torch.int64).max))
    return cand.min(dim=0).values.to(torch.int32)


# ---------------------------------------------------------------------------
# the engine (one rank)
# ---------------------------------------------------------------------------
AUTO_PUSH_MAX_RANKS = 4   # collective="auto": push up to this many ranks, p2p above


def push_slots(bases: list[int], rank: int, slot_bytes: int) -> tuple[list[int], list[int]]:
    """Addresses of the push collective's receive buffer, one [world][slot]
    buffer per rank (``bases``: its address as every rank maps it).

    Returns (reads, pushes): ``reads[q]`` is slot q of this rank's own buffer,
    where rank q's partial lands (read locally by the all-reduce kernel);
    ``pushes`` lists, for every other rank q in rank order, slot ``rank`` of
    rank q's buffer (written over NVLink by this rank's GEMM epilogue)."""
    world = len(bases)
    if not 0 <= rank < world or slot_bytes <= 0:
        raise ValueError("rank outside the group or empty slot")
    reads = [bases[rank] + q * slot_bytes for q in range(world)]
    pushes = [bases[q] + rank * slot_bytes for q in range(world) if q != rank]
    return reads, pushes


class TPDecodeEngine:
    """Greedy batch decoder for one tensor-parallel rank.

    ``model`` is the full synthetic model dict (``synth.random_model``); the
    rank keeps its shard.  ``group`` is an initialised NCCL process group of
    ``tp`` ranks (the default group when None).  All ``B`` rows run on every
    rank (replicated residual stream).  With ``use_graph`` the step -- NCCL
    all-reduces and gathers included -- is captured once in a CUDA graph
    (every rank captures the same sequence); ``release()`` drops the graphs,
    which must happen before the process group is destroyed.

    ``collective`` picks how the row-parallel partials are summed: "push"
    (the GEMM epilogue stores them into every rank's memory), "p2p" (the
    all-reduce kernel loads them from the peers), "nccl", or "auto": push up
    to 4 ranks and p2p above, the faster one measured on 8-GPU B200 boxes at
    each size where both were timed (Qwen3-8B, 64 rows: TP2 8.73k against
    8.54k tok/s, TP4 11.95k against 11.56k; at TP8 only p2p was timed).
    """

    def __init__(self, cfg, model: dict, batch: int, max_ctx: int, tp: int, rank: int, group=None,
                 device="cuda", use_graph: bool = False, partial_dtype: torch.dtype = torch.bfloat16,
                 collective: str = "auto"):
        import torch.distributed as dist
        from . import _lib
        from . import weights as W
        from .engine import load_layer
        from .rope import rope_angles

        self.dist, self.group, self.tp, self.rank = dist, group, tp, rank
        self.cfg, self.lcfg = cfg, local_config(cfg, tp)
        self.B, self.max_ctx, self.device = batch, max_ctx, torch.device(device)
        if partial_dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("the row-parallel partials are bf16 or fp32")
        self.partial_dtype = partial_dtype
        if collective not in ("auto", "push", "p2p", "nccl"):
            raise ValueError("collective is 'auto', 'push', 'p2p' or 'nccl'")
        if collective == "auto":
            collective = "push" if tp <= AUTO_PUSH_MAX_RANKS else "p2p"
        self.collective = collective
        if max_ctx % 64:
            raise ValueError("max_ctx must be a multiple of 64")
        dev, lc = self.device, self.lcfg
        for li, l in enumerate(model["layers"]):   # the sharding reads AutoGPTQ tensors (.qweight, ...)
            for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
                if not isinstance(l[name], AutoGPTQLinear):
                    raise NotImplementedError(
                        f"layer {li} {name} is a {type(l[name]).__name__}: tensor-parallel decode shards "
                        "group-128 AutoGPTQ-derived weights only")
        self.layers = [load_layer(shard_layer(l, cfg, tp, rank), lc, dev) for l in model["layers"]]
        self.embed = model["embed"].to(dev, torch.bfloat16).contiguous()
        lm = model.get("lm_head")
        if lm is not None and not isinstance(lm, torch.Tensor):
            raise NotImplementedError("tensor-parallel decode takes a bf16 lm_head (tied or untied); "
                                      "a W4A16 head runs on the single-GPU engine")
        full_lm = model["embed"] if lm is None else lm
        v0, v1 = vocab_slice(cfg, tp, rank)
        self.v_local = v1 - v0
        self.lm_head = full_lm[v0:v1].to(dev, torch.float16).contiguous()   # fp16 head (t2b_lm_head_argmax)
        self.final_norm = model["final_norm"].to(dev, torch.bfloat16).contiguous()
        self.angles = rope_angles(cfg.head_dim, max_ctx, cfg.rope_base).to(dev)
        B, H, hd = batch, cfg.emb_dim, cfg.head_dim
        f32, bf = torch.float32, torch.bfloat16
        self.x = torch.zeros(B, H, dtype=f32, device=dev)
        if collective in ("push", "p2p"):
            self._setup_p2p(B, H, partial_dtype)
        else:   # one partial, all-reduced in place
            self.y_bufs = [torch.zeros(B, H, dtype=partial_dtype, device=dev)] * 2
        act = _lib.ACT                                            # fp16 linear inputs (t2b.h)
        self.xw = torch.zeros(B, H, dtype=act, device=dev)
        self.ssq_a = torch.zeros(B, dtype=f32, device=dev)
        self.ssq_b = torch.zeros(B, dtype=f32, device=dev)
        self.q = torch.zeros(B, lc.q_dim, dtype=_lib.QDT, device=dev)
        self.attn = torch.zeros(B, lc.q_dim, dtype=act, device=dev)
        self.h = torch.zeros(B, lc.hidden_dim, dtype=act, device=dev)
        self.xn = torch.zeros(B, H, dtype=torch.float16, device=dev)
        self.local_max = torch.zeros(B, dtype=f32, device=dev)
        self.tokens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.local_idx = torch.zeros(B, dtype=torch.int32, device=dev)
        self.next_tokens = torch.zeros(B, dtype=torch.int32, device=dev)
        kv_shape = (B, lc.n_kv_groups, max_ctx, hd)
        self.k_cache = [torch.zeros(kv_shape, dtype=bf, device=dev) for _ in range(cfg.n_layers)]
        self.v_cache = [torch.zeros(kv_shape, dtype=bf, device=dev) for _ in range(cfg.n_layers)]
        L = _lib.load()
        nq, nkv = lc.n_heads, lc.n_kv_groups
        sizes = {
            "qkv": L.t2b_qkv_workspace_bytes(B, H, nq, nkv, hd),
            "attn": L.t2b_decode_attention_workspace_bytes(B, nq, nkv, hd, max_ctx),
            "o": L.t2b_w4a16_gemm_workspace_bytes(B, H, lc.q_dim),
            "ug": L.t2b_upgate_swiglu_workspace_bytes(B, H, lc.hidden_dim),
            "down": L.t2b_w4a16_gemm_workspace_bytes(B, H, lc.hidden_dim),
            "lm": L.t2b_lm_head_argmax_workspace_bytes(B),
        }
        self.ws = {k: (torch.zeros(max(v, 256), dtype=torch.uint8, device=dev), max(v, 256)) for k, v in sizes.items()}
        self._lib, self._W = _lib, W
        # this rank's status word; the launch stream is bound to it while the engine enqueues
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.use_graph, self.graph, self._step_graph = use_graph, None, None
        self.vals = [torch.zeros(B, dtype=f32, device=dev) for _ in range(tp)]
        self.idxs = [torch.zeros(B, dtype=torch.int32, device=dev) for _ in range(tp)]
        torch.cuda.synchronize(dev)

    def _ws(self, k):
        t, n = self.ws[k]
        return self._lib.ptr(t), n

    def next_norm_weight(self, li: int) -> torch.Tensor:
        return self.layers[li + 1].input_layernorm if li + 1 < len(self.layers) else self.final_norm

    def _setup_p2p(self, B, H, dtype) -> None:
        """Peer-mapped partial buffers (two: o_proj and down alternate) and flag words."""
        import ctypes as C

        import torch.distributed._symmetric_memory as symm_mem

        from . import _lib
        group = self.group if self.group is not None else self.dist.group.WORLD
        name = group.group_name
        if hasattr(symm_mem, "enable_symm_mem_for_group"):   # needed by older torch versions only
            import warnings
            with warnings.catch_warnings():
                warnings.simplefilter("ignore")
                try:
                    symm_mem.enable_symm_mem_for_group(name)
                except Exception:   # already enabled, or not needed by this torch version
                    pass
        dev, tp = self.device, self.tp
        esize = torch.tensor([], dtype=dtype).element_size()
        self.y_bufs, ptrs, self._push = [], [], []
        for _ in range(2):
            if self.collective == "push":
                # [tp][B][H]: slot q holds rank q's partial, written by rank q's GEMM epilogue
                t = symm_mem.empty((tp, B, H), dtype=dtype, device=dev)
                t.zero_()
                hdl = symm_mem.rendezvous(t, name)
                reads, pushes = push_slots([int(q) for q in hdl.buffer_ptrs], self.rank, B * H * esize)
                self.y_bufs.append(t[self.rank])                              # this rank's own slot
                ptrs.append((C.c_void_p * tp)(*reads))
                self._push.append((C.c_void_p * max(tp - 1, 1))(*pushes))
            else:
                t = symm_mem.empty((B, H), dtype=dtype, device=dev)
                t.zero_()
                hdl = symm_mem.rendezvous(t, name)
                self.y_bufs.append(t)
                ptrs.append((C.c_void_p * tp)(*[int(q) for q in hdl.buffer_ptrs]))
            self._p2p_keep = getattr(self, "_p2p_keep", []) + [hdl, t]
        flags = symm_mem.empty((tp,), dtype=torch.int32, device=dev)
        flags.zero_()
        fh = symm_mem.rendezvous(flags, name)
        flag_ptrs = (C.c_void_p * tp)(*[int(q) for q in fh.buffer_ptrs])
        # the greedy head: every rank's [tp][B] best-key buffer and its own flag words
        gather = symm_mem.empty((tp * B,), dtype=torch.int64, device=dev)
        gather.zero_()
        gh = symm_mem.rendezvous(gather, name)
        hflags = symm_mem.empty((tp,), dtype=torch.int32, device=dev)
        hflags.zero_()
        hh = symm_mem.rendezvous(hflags, name)
        gather_ptrs = (C.c_void_p * tp)(*[int(q) for q in gh.buffer_ptrs])
        hflag_ptrs = (C.c_void_p * tp)(*[int(q) for q in hh.buffer_ptrs])
        self._p2p = {"parts": [C.addressof(a) for a in ptrs], "flags": C.addressof(flag_ptrs),
                     "gather": C.addressof(gather_ptrs), "head_flags": C.addressof(hflag_ptrs),
                     "head_state": torch.zeros(4, dtype=torch.int32, device=dev),
                     "keep": [ptrs, flag_ptrs, flags, fh, gather, gh, hflags, hh, gather_ptrs, hflag_ptrs],
                     "state": torch.zeros(max(_lib.load().t2b_tp_allreduce_state_bytes(), 16) // 4,
                                          dtype=torch.int32, device=dev)}
        torch.cuda.synchronize(dev)
        self.dist.barrier(group=group)   # every rank's flags are zero before anyone signals

    def _row_parallel(self, which, lw_lin, x, K, st) -> None:
        """A row-parallel linear (o_proj / down) writing its partial into buffer ``which``."""
        lib, L, p = self._lib, self._lib.lib(), self._lib.ptr
        H = self.cfg.emb_dim
        ws = self._ws("o" if which == 0 else "down")
        if self.collective == "push":   # partial pushed into every rank's buffer from the GEMM epilogue
            import ctypes as C
            peers = self._push[which]
            lib.check("t2b_w4a16_gemm_push", L.t2b_w4a16_gemm_push(
                p(lw_lin.qw), p(lw_lin.meta), lib.WFMT_T2B, p(x), lib.DTYPE[lib.ACT], p(self.y_bufs[which]),
                lib.DTYPE[self.partial_dtype], C.addressof(peers), self.tp - 1, self.B, H, K, 128, *ws, st))
            return
        lib.check("t2b_w4a16_gemm", L.t2b_w4a16_gemm(
            p(lw_lin.qw), p(lw_lin.meta), lib.WFMT_T2B, p(x), lib.DTYPE[lib.ACT], p(self.y_bufs[which]),
            lib.DTYPE[self.partial_dtype], self.B, H, K, 128, *ws, st))

    def _allreduce_residual(self, which, ssq_out, next_w):
        lib, p = self._lib, self._lib.ptr
        if self.collective in ("push", "p2p"):
            q = self._p2p
            lib.check("t2b_tp_allreduce_residual_norm_input", lib.lib().t2b_tp_allreduce_residual_norm_input(
                q["parts"][which], lib.DTYPE[self.partial_dtype], q["flags"], p(q["state"]), self.rank, self.tp,
                p(self.x), p(ssq_out), p(next_w), p(self.xw), self.B, self.cfg.emb_dim, lib.stream()))
            return
        self.dist.all_reduce(self.y_bufs[which], group=self.group)
        lib.check("t2b_residual_norm_input", lib.lib().t2b_residual_norm_input(
            p(self.y_bufs[which]), lib.DTYPE[self.partial_dtype], p(self.x), p(ssq_out), p(next_w), p(self.xw),
            self.B, self.cfg.emb_dim, lib.stream()))

    def enqueue_layer(self, li: int) -> None:
        cfg, lc, B = self.cfg, self.lcfg, self.B
        H, hd, nq, nkv = cfg.emb_dim, cfg.head_dim, lc.n_heads, lc.n_kv_groups
        lib = self._lib
        L, p, st = lib.lib(), lib.ptr, lib.stream()
        lw = self.layers[li]
        lib.check("t2b_qkv_norm_rope_kvwrite", L.t2b_qkv_norm_rope_kvwrite(
            p(lw.qkv.qw), p(lw.qkv.meta), lw.qkv.fmt, p(self.xw), p(self.ssq_a), cfg.rms_norm_eps,
            p(lw.q_norm), p(lw.k_norm), p(self.angles), p(self.pos), p(self.q), lib.DTYPE[lib.QDT], p(self.k_cache[li]),
            p(self.v_cache[li]), p(self.ssq_b), B, H, nq, nkv, hd, self.max_ctx, *self._ws("qkv"), st))
        lib.check("t2b_decode_attention_after_kvwrite", L.t2b_decode_attention_after_kvwrite(
            p(self.q), lib.DTYPE[lib.QDT], p(self.k_cache[li]), p(self.v_cache[li]), p(self.pos), p(self.attn),
            lib.DTYPE[lib.ACT], B,
            nq, nkv, hd, self.max_ctx, *self._ws("attn"), st))
        self._row_parallel(0, lw.o_proj, self.attn, lc.q_dim, st)
        self._allreduce_residual(0, self.ssq_b, lw.post_attention_layernorm)
        lib.check("t2b_upgate_swiglu", L.t2b_upgate_swiglu(
            p(lw.gate_up.qw), p(lw.gate_up.meta), lw.gate_up.fmt, p(self.xw), p(self.ssq_b), cfg.rms_norm_eps, p(self.h),
            p(self.ssq_a), B, H, lc.hidden_dim, *self._ws("ug"), st))
        self._row_parallel(1, lw.down, self.h, lc.hidden_dim, st)
        self._allreduce_residual(1, self.ssq_a, self.next_norm_weight(li))

    def enqueue_step(self) -> None:
        with self._lib.status_word(self.err, self._lib.stream()):
            self._enqueue_step()

    def _enqueue_step(self) -> None:
        cfg, B = self.cfg, self.B
        lib = self._lib
        L, p, st = lib.lib(), lib.ptr, lib.stream()
        lib.check("t2b_embed_rows", L.t2b_embed_rows(p(self.embed), p(self.tokens), p(self.x), p(self.ssq_a),
                                                     p(self.layers[0].input_layernorm), p(self.xw), B, cfg.emb_dim,
                                                     cfg.vocab_size, st))
        for li in range(cfg.n_layers):
            self.enqueue_layer(li)
        f16 = lib.DTYPE[torch.float16]
        lib.check("t2b_rms_norm_rows", L.t2b_rms_norm_rows(p(self.x), p(self.ssq_a), p(self.final_norm),
                                                           cfg.rms_norm_eps, p(self.xn), f16, B, cfg.emb_dim, st))
        if self.collective in ("push", "p2p"):   # the pick merged over the ranks inside the head kernel
            q = self._p2p
            lib.check("t2b_lm_head_argmax_tp", L.t2b_lm_head_argmax_tp(
                p(self.xn), p(self.lm_head), f16, B, cfg.emb_dim, self.v_local, self.rank * self.v_local, q["gather"],
                q["head_flags"], p(q["head_state"]), self.rank, self.tp, p(self.next_tokens), *self._ws("lm"), st))
            return
        lib.check("t2b_lm_head_argmax", L.t2b_lm_head_argmax(
            p(self.xn), p(self.lm_head), f16, B, cfg.emb_dim, self.v_local, p(self.local_idx), p(self.local_max),
            None, *self._ws("lm"), st))
        self.dist.all_gather(self.vals, self.local_max, group=self.group)
        self.dist.all_gather(self.idxs, self.local_idx, group=self.group)
        self.next_tokens.copy_(merge_argmax(torch.stack(self.vals), torch.stack(self.idxs), self.v_local))

    def kernels_per_step(self) -> int:
        """Launches of this library's kernels per step (NCCL collectives and the final merge excluded)."""
        return 1 + 7 * self.cfg.n_layers + 2

    def capture(self) -> None:
        """Capture ``step`` and ``step + (tokens <- next, pos += 1)`` as CUDA graphs."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):   # NCCL communicators, cuBLAS and lazy init outside the capture
                self.enqueue_step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.enqueue_step()
        self._step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._step_graph):
            self.enqueue_step()
            self.tokens.copy_(self.next_tokens)
            self.pos.add_(1)
        torch.cuda.synchronize(self.device)

    def run_step(self) -> None:
        if self.use_graph:
            if self.graph is None:
                self.capture()
            self.graph.replay()
        else:
            self.enqueue_step()

    def advance(self) -> None:
        if self.use_graph:
            if self._step_graph is None:
                self.capture()
            self._step_graph.replay()
        else:
            self.enqueue_step()
            self.tokens.copy_(self.next_tokens)
            self.pos.add_(1)

    def prefill(self, prompts: torch.Tensor) -> None:
        P = prompts.shape[1]
        prompts = prompts.to(self.device, torch.int32)
        for t in range(P):
            self.tokens.copy_(prompts[:, t])
            self.pos.fill_(t)
            self.run_step()
        self.tokens.copy_(self.next_tokens)
        self.pos.fill_(P)

    def check_device_errors(self) -> None:
        """Raise (and clear) the status a kernel of this rank recorded for a timed-out device wait."""
        code = int(self.err.item())
        if code:
            self.err.zero_()
            raise self._lib.T2BError("a decode-step kernel (device status word)", code)

    def release(self) -> None:
        """Drop the captured graphs (before destroying the process group)."""
        torch.cuda.synchronize(self.device)
        self.graph = None
        self._step_graph = None

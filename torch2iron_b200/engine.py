"""Batch decode engine: the reference's per-step decode composition on B200.

One decode step for ``B`` rows (one new token each) follows the op order of
``build_batch_decode_fused_op`` (``src/models/quantized_qwen3/batch_decode_fused.py:426-539``)
and the math of ``QuantizedQwenForCausalLM.forward`` (``model.py:453-478``),
as 5 fused launches per layer:

    embed_rows                      x = E[tok]            (+ sum of squares)
    per layer:
      qkv_norm_rope_kvwrite         RMSNorm, [q;k;v] GEMV, QK-norm, RoPE, KV write
      decode_attention              split-K GQA attention over the bf16 cache
      oproj_residual                x += o_proj(ctx)      (+ sum of squares)
      upgate_swiglu                 RMSNorm, [gate|up] GEMV, silu(g)*u
      down_residual                 x += down(h)          (+ sum of squares)
    rms_norm_rows                   final norm -> bf16
    lm_head_argmax                  bf16 lm_head GEMM with the greedy argmax fused in
                                    (logits written only with keep_logits)
  or, for a W4A16 head (the packed artifact's quantized ``lm_head`` linear,
  ``model.py:410-414``):
    w4a16_gemm + argmax_rows        fp32 logits, then the greedy argmax

The whole step is captured once in a CUDA graph and replayed; the kernels
chain with programmatic dependent launch.  The residual stream is fp32; the
activations entering each linear are bf16 (A16).  KV caches are bf16
``[B][n_kv][max_ctx][head_dim]`` per layer -- the reference's host-synced
packet cache (``decode_packet_cache.py``) becomes a device-resident cache
written by the qkv epilogue, so no per-layer host copy remains.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from . import weights as W
from .config import QuantizedQwenConfig
from .rope import rope_angles
from .synth import AutoGPTQLinear


@dataclass
class LayerWeights:
    qkv: W.W4Weight
    o_proj: W.W4Weight
    gate_up: W.W4Weight
    down: W.W4Weight
    input_layernorm: torch.Tensor
    post_attention_layernorm: torch.Tensor
    q_norm: torch.Tensor | None
    k_norm: torch.Tensor | None

    @property
    def algorithmic_bytes(self) -> int:
        b = sum(w.nbytes_algorithmic for w in (self.qkv, self.o_proj, self.gate_up, self.down))
        b += 2 * (self.input_layernorm.numel() + self.post_attention_layernorm.numel())
        if self.q_norm is not None:
            b += 2 * (self.q_norm.numel() + self.k_norm.numel())
        return b


def load_layer(layer: dict, cfg: QuantizedQwenConfig, device="cuda") -> LayerWeights:
    """One layer's device weights: group-128 AutoGPTQ-derived linears (the
    packed artifact, checkpoints, synthetic models) into the T2B layout, or
    the fast artifact's Q4NX group-32 linears into its group-32 variant; the
    seven linears of a layer share one format."""
    names = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
    kinds = {type(layer[n]) for n in names}
    if kinds == {AutoGPTQLinear}:
        concat, single, pair = W.concat_rows, W.from_autogptq, W.pair_blocks
    elif len(kinds) == 1 and all(hasattr(layer[n], "padded_out_features") for n in names):
        concat, single, pair = W.q4nx_concat_rows, W.from_q4nx, W.q4nx_pair_blocks
    else:
        raise NotImplementedError(
            f"layer linears are {sorted(k.__name__ for k in kinds)}: the decode kernels take group-128 "
            "AutoGPTQ-derived weights or Q4NX group-32 weights, one format per layer")

    def bf(t):
        return None if t is None else t.to(device=device, dtype=torch.bfloat16).contiguous()

    return LayerWeights(
        qkv=concat([layer["q_proj"], layer["k_proj"], layer["v_proj"]], device),
        o_proj=single(layer["o_proj"], device),
        gate_up=pair(layer["gate_proj"], layer["up_proj"], device),
        down=single(layer["down_proj"], device),
        input_layernorm=bf(layer["input_layernorm"]),
        post_attention_layernorm=bf(layer["post_attention_layernorm"]),
        q_norm=bf(layer.get("q_norm")) if cfg.qk_norm else None,
        k_norm=bf(layer.get("k_norm")) if cfg.qk_norm else None,
    )


class DecodeEngine:
    """Greedy batch decoder over device-resident W4A16 weights.

    ``model`` is the dict produced by ``synth.random_model`` or ``loaders``
    (AutoGPTQ linears per layer, bf16 ``embed``, ``final_norm``, and
    ``lm_head``: ``None`` when tied, bf16 ``[V, H]``, or an ``AutoGPTQLinear``).
    """

    def __init__(self, cfg: QuantizedQwenConfig, model: dict, batch: int, max_ctx: int, device="cuda",
                 use_graph: bool = True, keep_logits: bool = True):
        cfg.validate()
        if max_ctx % 64:
            raise ValueError("max_ctx must be a multiple of 64")
        self.cfg, self.B, self.max_ctx, self.device = cfg, batch, max_ctx, torch.device(device)
        self.use_graph, self.keep_logits = use_graph, keep_logits
        dev = self.device
        self.layers = [load_layer(l, cfg, dev) for l in model["layers"]]
        if len(self.layers) != cfg.n_layers:
            raise ValueError("layer count does not match the config")
        self.embed = model["embed"].to(dev, torch.bfloat16).contiguous()
        lm = model.get("lm_head")
        self.lm_w4: W.W4Weight | None = None          # W4A16 head (a packed artifact's ``lm_head`` linear)
        if isinstance(lm, AutoGPTQLinear) or hasattr(lm, "padded_out_features"):
            if (lm.out_features, lm.in_features) != (cfg.vocab_size, cfg.emb_dim):
                raise ValueError("lm_head shape does not match the config")
            self.lm_w4 = W.from_autogptq(lm, dev) if isinstance(lm, AutoGPTQLinear) else W.from_q4nx(lm, dev)
            self.lm_head = None
        else:
            # the greedy head runs in fp16: an fp16 copy of the (bf16) table, exact for every value in fp16
            # range, so the normalised rows keep 11 significant bits (t2b_lm_head_argmax)
            self.lm_head = (self.embed if lm is None else lm).to(dev, torch.float16).contiguous()
        self.final_norm = model["final_norm"].to(dev, torch.bfloat16).contiguous()
        self.angles = rope_angles(cfg.head_dim, max_ctx, cfg.rope_base).to(dev)

        B, H, hd = batch, cfg.emb_dim, cfg.head_dim
        f32, bf = torch.float32, torch.bfloat16
        self.x = torch.zeros(B, H, dtype=f32, device=dev)
        act = _lib.ACT                                            # fp16 linear inputs (t2b.h)
        self.xw = torch.zeros(B, H, dtype=act, device=dev)       # fp16(x * next norm weight)
        self.ssq_a = torch.zeros(B, dtype=f32, device=dev)
        self.ssq_b = torch.zeros(B, dtype=f32, device=dev)
        self.q = torch.zeros(B, cfg.q_dim, dtype=_lib.QDT, device=dev)
        self.attn = torch.zeros(B, cfg.q_dim, dtype=act, device=dev)
        self.h = torch.zeros(B, cfg.hidden_dim, dtype=act, device=dev)
        self.xn = torch.zeros(B, H, dtype=torch.float16, device=dev)   # final norm output (fp16 head input)
        self.logits = torch.zeros(B, cfg.vocab_size, dtype=f32, device=dev)
        # host-facing int32 words in one device buffer, 16-byte aligned segments:
        # [tokens | pos | next_tokens | status word], so decode_step moves its
        # inputs with one host->device copy and its outputs with one copy back
        seg = (B + 3) // 4 * 4
        self._io = torch.zeros(3 * seg + 4, dtype=torch.int32, device=dev)
        self._io_seg = seg
        self.tokens = self._io[0:B]
        self.pos = self._io[seg:seg + B]
        self.next_tokens = self._io[2 * seg:2 * seg + B]
        kv_shape = (B, cfg.n_kv_groups, max_ctx, hd)
        self.k_cache = [torch.zeros(kv_shape, dtype=bf, device=dev) for _ in range(cfg.n_layers)]
        self.v_cache = [torch.zeros(kv_shape, dtype=bf, device=dev) for _ in range(cfg.n_layers)]

        L = _lib.load()
        nq, nkv = cfg.n_heads, cfg.n_kv_groups
        sizes = {
            "qkv": L.t2b_qkv_workspace_bytes(B, H, nq, nkv, hd),
            "attn": L.t2b_decode_attention_workspace_bytes(B, nq, nkv, hd, max_ctx),
            "o": L.t2b_oproj_residual_workspace_bytes(B, H, cfg.q_dim),
            "ug": L.t2b_upgate_swiglu_workspace_bytes(B, H, cfg.hidden_dim),
            "down": L.t2b_down_residual_workspace_bytes(B, H, cfg.hidden_dim),
        }
        if self.lm_w4 is None:
            sizes["lm"] = L.t2b_lm_head_argmax_workspace_bytes(B)
        else:
            sizes["lm"] = L.t2b_w4a16_gemm_workspace_bytes(B, cfg.vocab_size, H)
            sizes["am"] = L.t2b_argmax_workspace_bytes(B, cfg.vocab_size)
        # one workspace per op kind: consecutive ops never share counters
        self.ws = {k: (torch.zeros(max(v, 256), dtype=torch.uint8, device=dev), max(v, 256)) for k, v in sizes.items()}
        # device status word: this engine's kernels record a timed-out wait here (the
        # launch stream is bound to it while the engine enqueues, t2b_bind_error_word)
        self.err = self._io[3 * seg:3 * seg + 1]
        # pinned staging for decode_step: [tokens | pos] in, [next_tokens | status] out
        self._host_in = torch.zeros(2 * seg, dtype=torch.int32).pin_memory()
        self._host_in_np = self._host_in.numpy()
        self._host_out = torch.zeros(seg + 4, dtype=torch.int32).pin_memory()
        torch.cuda.synchronize(dev)   # repacked weights complete before any PDL launch reads them
        self.graph = None
        self._step_graph = None
        self._io_graph = None

    # -- byte accounting (algorithmic, for the roofline) ---------------------
    def weight_bytes(self) -> int:
        b = sum(l.algorithmic_bytes for l in self.layers)
        b += self.lm_head_bytes() + self.final_norm.numel() * 2
        return b

    def lm_head_bytes(self) -> int:
        return self.lm_w4.nbytes_algorithmic if self.lm_w4 is not None else self.lm_head.numel() * 2

    def step_bytes(self, ctx_lens: list[int] | None = None) -> int:
        """Algorithmic HBM bytes of one decode step with per-row context lengths (keys attended)."""
        cfg = self.cfg
        kv_tok = 2 * cfg.n_kv_groups * cfg.head_dim * 2
        if ctx_lens is None:
            ctx_lens = [int(p) + 1 for p in self.pos.tolist()]
        kv_read = sum(ctx_lens) * kv_tok * cfg.n_layers
        kv_write = self.B * kv_tok * cfg.n_layers
        emb = self.B * cfg.emb_dim * 2
        return self.weight_bytes() + kv_read + kv_write + emb

    # -- launch sequence -----------------------------------------------------
    def _ws(self, k):
        t, n = self.ws[k]
        return _lib.ptr(t), n

    def next_norm_weight(self, li: int) -> torch.Tensor:
        """Weight of the RMSNorm that follows layer li's MLP (next layer's input norm, or the final norm)."""
        return self.layers[li + 1].input_layernorm if li + 1 < len(self.layers) else self.final_norm

    def enqueue_layer(self, li: int, st: int) -> None:
        with _lib.status_word(self.err, st):
            self._enqueue_layer(li, st)

    def _enqueue_layer(self, li: int, st: int) -> None:
        cfg, B = self.cfg, self.B
        H, hd, nq, nkv = cfg.emb_dim, cfg.head_dim, cfg.n_heads, cfg.n_kv_groups
        L = _lib.lib()
        lw = self.layers[li]
        p = _lib.ptr
        _lib.check("t2b_qkv_norm_rope_kvwrite", L.t2b_qkv_norm_rope_kvwrite(
            p(lw.qkv.qw), p(lw.qkv.meta), lw.qkv.fmt, p(self.xw), p(self.ssq_a), cfg.rms_norm_eps,
            p(lw.q_norm), p(lw.k_norm), p(self.angles), p(self.pos), p(self.q), _lib.DTYPE[_lib.QDT], p(self.k_cache[li]),
            p(self.v_cache[li]), p(self.ssq_b), B, H, nq, nkv, hd, self.max_ctx, *self._ws("qkv"), st))
        _lib.check("t2b_decode_attention_after_kvwrite", L.t2b_decode_attention_after_kvwrite(
            p(self.q), _lib.DTYPE[_lib.QDT], p(self.k_cache[li]), p(self.v_cache[li]), p(self.pos), p(self.attn),
            _lib.DTYPE[_lib.ACT], B,
            nq, nkv, hd, self.max_ctx, *self._ws("attn"), st))
        _lib.check("t2b_oproj_residual", L.t2b_oproj_residual(
            p(lw.o_proj.qw), p(lw.o_proj.meta), lw.o_proj.fmt, p(self.attn), p(self.x), p(self.ssq_b),
            p(lw.post_attention_layernorm), p(self.xw), B, H, cfg.q_dim, *self._ws("o"), st))
        _lib.check("t2b_upgate_swiglu", L.t2b_upgate_swiglu(
            p(lw.gate_up.qw), p(lw.gate_up.meta), lw.gate_up.fmt, p(self.xw), p(self.ssq_b), cfg.rms_norm_eps, p(self.h),
            p(self.ssq_a), B, H, cfg.hidden_dim, *self._ws("ug"), st))
        _lib.check("t2b_down_residual", L.t2b_down_residual(
            p(lw.down.qw), p(lw.down.meta), lw.down.fmt, p(self.h), p(self.x), p(self.ssq_a), p(self.next_norm_weight(li)),
            p(self.xw), B, H, cfg.hidden_dim, *self._ws("down"), st))

    def enqueue_step(self) -> None:
        """Enqueue one full decode step on the current stream (tokens/pos already on device)."""
        cfg, B = self.cfg, self.B
        L = _lib.lib()
        st = _lib.stream()
        p = _lib.ptr
        with _lib.status_word(self.err, st):     # this engine's word for every launch below
            _lib.check("t2b_embed_rows", L.t2b_embed_rows(p(self.embed), p(self.tokens), p(self.x), p(self.ssq_a),
                                                          p(self.layers[0].input_layernorm), p(self.xw), B,
                                                          cfg.emb_dim, cfg.vocab_size, st))
            for li in range(cfg.n_layers):
                self._enqueue_layer(li, st)
            self._enqueue_head(st)

    def _enqueue_head(self, st) -> None:
        """Final RMSNorm of ``x`` (with ``ssq_a``) and the greedy lm_head into ``next_tokens``."""
        cfg, B = self.cfg, self.B
        L = _lib.lib()
        p = _lib.ptr
        f16 = _lib.DTYPE[torch.float16]
        _lib.check("t2b_rms_norm_rows", L.t2b_rms_norm_rows(p(self.x), p(self.ssq_a), p(self.final_norm),
                                                            cfg.rms_norm_eps, p(self.xn), f16, B, cfg.emb_dim, st))
        if self.lm_w4 is None:
            _lib.check("t2b_lm_head_argmax", L.t2b_lm_head_argmax(
                p(self.xn), p(self.lm_head), f16, B, cfg.emb_dim, cfg.vocab_size, p(self.next_tokens), None,
                p(self.logits) if self.keep_logits else None, *self._ws("lm"), st))
        else:
            _lib.check("t2b_w4a16_gemm", L.t2b_w4a16_gemm(
                p(self.lm_w4.qw), p(self.lm_w4.meta), self.lm_w4.fmt, p(self.xn), f16,
                p(self.logits), _lib.DTYPE[torch.float32], B, cfg.vocab_size, cfg.emb_dim,
                32 if self.lm_w4.fmt == W.WFMT_Q4NX else 128, *self._ws("lm"), st))
            _lib.check("t2b_argmax_rows", L.t2b_argmax_rows(
                p(self.logits), _lib.DTYPE[torch.float32], B, cfg.vocab_size, cfg.vocab_size, p(self.next_tokens),
                *self._ws("am"), st))

    def set_hidden(self, x: torch.Tensor) -> None:
        """Load a residual-stream state (fp32 [B, H]) and its split norm input for layer 0."""
        self.x.copy_(x.to(self.device, torch.float32))
        self.ssq_a.copy_((self.x.double() ** 2).sum(-1).float())
        self.xw.copy_((self.x * self.layers[0].input_layernorm.float()).to(_lib.ACT))

    def kernels_per_step(self) -> int:
        """Launches of this library's kernels per step (embed, 5 per layer, final norm, lm_head + argmax)."""
        return 1 + 5 * self.cfg.n_layers + 1 + (1 if self.lm_w4 is None else 2)

    # -- graph capture -------------------------------------------------------
    def capture(self) -> None:
        """Capture ``step + (tokens <- next, pos += 1)`` as one CUDA graph."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm up cuBLAS / lazy init outside the capture
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
        # decode_step's graph: the host->device copy of the pinned tokens and
        # positions, the step, and the device->host copy of the next tokens and
        # the status word, so one replay and one synchronisation serve a call
        seg = self._io_seg
        self._io_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._io_graph):
            self._io[:2 * seg].copy_(self._host_in, non_blocking=True)
            self.enqueue_step()
            self._host_out.copy_(self._io[2 * seg:], non_blocking=True)

    def run_step(self) -> None:
        """One step from the device-resident tokens / pos (outputs ``next_tokens``, ``logits``)."""
        if self.use_graph:
            if self.graph is None:
                self.capture()
            self.graph.replay()
        else:
            self.enqueue_step()

    def advance(self) -> None:
        """Greedy self-feeding step: run, then tokens <- next_tokens, pos += 1 (all on device)."""
        if self.use_graph:
            if self._step_graph is None:
                self.capture()
            self._step_graph.replay()
        else:
            self.enqueue_step()
            self.tokens.copy_(self.next_tokens)
            self.pos.add_(1)

    def check_device_errors(self) -> None:
        """Raise (and clear) the status a kernel recorded for a timed-out device wait."""
        code = int(self.err.item())
        if code:
            self.err.zero_()
            raise _lib.T2BError("a decode-step kernel (device status word)", code)

    # -- host-facing API (the reference runner's decode_step, qwen_npu.py:166-236) --
    def decode_step(self, tokens, positions) -> torch.Tensor:
        """tokens / positions: host sequences of length B -> next greedy tokens (host int32 [B])."""
        B, seg = self.B, self._io_seg
        hin = self._host_in_np                    # the pinned staging buffer, as numpy
        try:
            tok = np.asarray(tokens).reshape(-1)
            pos = np.asarray(positions).reshape(-1)
        except (TypeError, ValueError) as e:
            raise ValueError(f"decode_step takes {B} tokens and {B} positions") from e
        if tok.shape != (B,) or pos.shape != (B,):
            raise ValueError(f"decode_step takes {B} tokens and {B} positions")
        if tok.min() < 0 or tok.max() >= self.cfg.vocab_size:
            raise ValueError(f"token ids must be in [0, {self.cfg.vocab_size})")
        if pos.min() < 0 or pos.max() >= self.max_ctx:
            raise ValueError(f"positions must be in [0, {self.max_ctx}) (the KV cache length)")
        hin[:B] = tok
        hin[seg:seg + B] = pos
        if self.use_graph:
            if self.graph is None:
                self.capture()
            self._io_graph.replay()              # copy in, step, copy out
        else:
            self._io[:2 * seg].copy_(self._host_in, non_blocking=True)    # one host->device copy
            self.run_step()
            # one device->host read per step: the next tokens and the status word
            self._host_out.copy_(self._io[2 * seg:], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        if int(self._host_out[seg]):
            self.check_device_errors()
        return self._host_out[:B].clone()

    # -- chunked prefill (prefill_runtime.py:95-164, for B sequences at once) --
    PREFILL_ROWS = 8192      # prompt tokens (all sequences) per chunk by default

    def _prefill_buffers(self, rows: int) -> dict:
        """Activations and workspaces for a chunk of ``rows`` prompt tokens (kept for reuse)."""
        pf = getattr(self, "_pf", None)
        if pf is not None and pf["rows"] >= rows:
            return pf
        cfg, dev = self.cfg, self.device
        H, f32, bf, i32 = cfg.emb_dim, torch.float32, torch.bfloat16, torch.int32
        L = _lib.load()
        nq, nkv, hd = cfg.n_heads, cfg.n_kv_groups, cfg.head_dim
        sizes = {"qkv": L.t2b_qkv_workspace_bytes(rows, H, nq, nkv, hd),
                 "o": L.t2b_oproj_residual_workspace_bytes(rows, H, cfg.q_dim),
                 "ug": L.t2b_upgate_swiglu_workspace_bytes(rows, H, cfg.hidden_dim),
                 "down": L.t2b_down_residual_workspace_bytes(rows, H, cfg.hidden_dim)}
        pf = {"rows": rows,
              "x": torch.zeros(rows, H, dtype=f32, device=dev), "xw": torch.zeros(rows, H, dtype=_lib.ACT, device=dev),
              "ssq_a": torch.zeros(rows, dtype=f32, device=dev), "ssq_b": torch.zeros(rows, dtype=f32, device=dev),
              "q": torch.zeros(rows, cfg.q_dim, dtype=bf, device=dev),
              "attn": torch.zeros(rows, cfg.q_dim, dtype=_lib.ACT, device=dev),
              "h": torch.zeros(rows, cfg.hidden_dim, dtype=_lib.ACT, device=dev),
              "tokens": torch.zeros(rows, dtype=i32, device=dev), "pos": torch.zeros(rows, dtype=i32, device=dev),
              "seq": torch.zeros(rows, dtype=i32, device=dev),
              "ws": {k: (torch.zeros(max(v, 256), dtype=torch.uint8, device=dev), max(v, 256))
                     for k, v in sizes.items()}}
        self._pf = pf
        return pf

    def enqueue_prefill_chunk(self, pf: dict, n: int, c0: int, st) -> None:
        """One chunk: tokens ``c0 .. c0+n-1`` of every sequence (rows ``b*n + i``
        of ``pf``, already holding tokens / pos / seq) through all layers."""
        cfg, B = self.cfg, self.B
        M = B * n
        H, hd, nq, nkv = cfg.emb_dim, cfg.head_dim, cfg.n_heads, cfg.n_kv_groups
        L = _lib.lib()
        p = _lib.ptr

        def ws(k):
            t, nb = pf["ws"][k]
            return p(t), nb

        x, xw, sa, sb = pf["x"], pf["xw"], pf["ssq_a"], pf["ssq_b"]
        _lib.check("t2b_embed_rows", L.t2b_embed_rows(p(self.embed), p(pf["tokens"]), p(x), p(sa),
                                                      p(self.layers[0].input_layernorm), p(xw), M, H,
                                                      cfg.vocab_size, st))
        for li, lw in enumerate(self.layers):
            _lib.check("t2b_qkv_norm_rope_kvwrite_seq", L.t2b_qkv_norm_rope_kvwrite_seq(
                p(lw.qkv.qw), p(lw.qkv.meta), lw.qkv.fmt, p(xw), p(sa), cfg.rms_norm_eps, p(lw.q_norm), p(lw.k_norm),
                p(self.angles), p(pf["pos"]), p(pf["seq"]), B, p(pf["q"]), p(self.k_cache[li]), p(self.v_cache[li]),
                p(sb), M, H, nq, nkv, hd, self.max_ctx, *ws("qkv"), st))
            _lib.check("t2b_prefill_attention", L.t2b_prefill_attention(
                p(pf["q"]), p(self.k_cache[li]), p(self.v_cache[li]), p(pf["attn"]), _lib.DTYPE[_lib.ACT], B, n, c0,
                nq, nkv, hd,
                self.max_ctx, st))
            _lib.check("t2b_oproj_residual", L.t2b_oproj_residual(
                p(lw.o_proj.qw), p(lw.o_proj.meta), lw.o_proj.fmt, p(pf["attn"]), p(x), p(sb), p(lw.post_attention_layernorm),
                p(xw), M, H, cfg.q_dim, *ws("o"), st))
            _lib.check("t2b_upgate_swiglu", L.t2b_upgate_swiglu(
                p(lw.gate_up.qw), p(lw.gate_up.meta), lw.gate_up.fmt, p(xw), p(sb), cfg.rms_norm_eps, p(pf["h"]), p(sa), M, H,
                cfg.hidden_dim, *ws("ug"), st))
            _lib.check("t2b_down_residual", L.t2b_down_residual(
                p(lw.down.qw), p(lw.down.meta), lw.down.fmt, p(pf["h"]), p(x), p(sa), p(self.next_norm_weight(li)), p(xw), M,
                H, cfg.hidden_dim, *ws("down"), st))

    def prefill(self, prompts: torch.Tensor, chunk: int | None = None, stepwise: bool = False,
                lengths=None) -> None:
        """Fill the KV caches from ``prompts [B, P]`` in chunks of ``chunk`` tokens per
        sequence (default: up to ``PREFILL_ROWS`` prompt tokens per chunk): every
        linear runs over all ``B * chunk`` tokens at once and attention is causal
        within and before the chunk (``t2b_prefill_attention``).  ``lengths``
        (B ints in 1..P) gives ragged prompts, right-padded in ``prompts``: a
        padded position writes no cache entry and each row continues from its
        own length.  ``stepwise`` feeds the prompt one position per decode step
        instead (equal lengths only).

        Leaves ``next_tokens`` = the greedy token after each prompt (``logits``
        for it with ``keep_logits``), and ``tokens``/``pos`` ready for ``advance()``.

        With ragged prompts, a chunk's padded query rows attend cache slots
        this prefill does not write (whatever an earlier run left there).
        Their outputs are discarded, and valid rows mask those keys out, but a
        masked key still enters the P.V product with P = 0, so the caches
        must hold finite values: they start zeroed and every write is a
        kernel's finite bf16 output.
        """
        if stepwise:
            if lengths is not None:
                raise ValueError("stepwise prefill takes prompts of equal length")
            self._prefill_stepwise(prompts)
            return
        B, P = prompts.shape
        if B != self.B:
            raise ValueError(f"prompts hold {B} sequences, the engine {self.B}")
        if P < 1 or P > self.max_ctx:
            raise ValueError(f"prompt length {P} outside 1..{self.max_ctx}")
        lens = torch.full((B,), P, dtype=torch.int64) if lengths is None else \
            torch.as_tensor(lengths, dtype=torch.int64).cpu()
        if lens.shape != (B,) or int(lens.min()) < 1 or int(lens.max()) > P:
            raise ValueError(f"lengths must be {B} values in 1..{P}")
        Pmax = int(lens.max())
        C = chunk or max(1, min(Pmax, self.PREFILL_ROWS // B))
        pf = self._prefill_buffers(B * min(C, Pmax))
        dev = self.device
        valid = torch.arange(P)[None, :] < lens[:, None]                       # [B, P]
        prompts = torch.where(valid, prompts.cpu().to(torch.int64), 0).to(dev, torch.int32)   # padding -> token 0
        lens_d = lens.to(dev)
        st = _lib.stream()
        with _lib.status_word(self.err, st):
            self._prefill_chunks(prompts, lens_d, pf, B, C, Pmax, st)
        self.tokens.copy_(self.next_tokens)
        self.pos.copy_(lens_d.to(torch.int32))

    def _prefill_chunks(self, prompts, lens_d, pf, B, C, Pmax, st) -> None:
        dev = self.device
        seq_all = torch.arange(B, dtype=torch.int64, device=dev)
        for c0 in range(0, Pmax, C):
            n = min(C, Pmax - c0)
            M = B * n
            posm = torch.arange(c0, c0 + n, device=dev)[None, :].expand(B, n)
            pf["tokens"][:M].copy_(prompts[:, c0:c0 + n].reshape(-1))
            pf["pos"][:M].copy_(torch.where(posm < lens_d[:, None], posm, -1).reshape(-1))   # -1: no cache write
            pf["seq"][:M].copy_(seq_all.repeat_interleave(n))
            self.enqueue_prefill_chunk(pf, n, c0, st)
            # rows whose last prompt token is in this chunk: residual state for the head
            ends = (lens_d - 1 >= c0) & (lens_d - 1 < c0 + n)
            rows = seq_all[ends]
            if rows.numel():
                src = rows * n + (lens_d[ends] - 1 - c0)
                self.x.index_copy_(0, rows, pf["x"].index_select(0, src))
                self.ssq_a.index_copy_(0, rows, pf["ssq_a"].index_select(0, src))
        self._enqueue_head(st)

    def _prefill_stepwise(self, prompts: torch.Tensor) -> None:
        """The prompt one position per decode step (teacher forcing)."""
        P = prompts.shape[1]
        prompts = prompts.to(self.device, torch.int32)
        for t in range(P):
            self.tokens.copy_(prompts[:, t])
            self.pos.fill_(t)
            self.run_step()
        self.tokens.copy_(self.next_tokens)
        self.pos.fill_(P)

    def generate(self, prompts: torch.Tensor, new_tokens: int, stepwise_prefill: bool = False,
                 lengths=None) -> torch.Tensor:
        """Greedy decode ``new_tokens`` per row after ``prompts`` (right-padded to
        ``lengths`` when given) -> ``[B, new_tokens]``."""
        longest = prompts.shape[1] if lengths is None else max(int(n) for n in lengths)
        if new_tokens < 1 or longest + new_tokens - 1 > self.max_ctx:
            raise ValueError(f"{longest} prompt + {new_tokens} new tokens do not fit max_ctx {self.max_ctx}")
        self.prefill(prompts, stepwise=stepwise_prefill, lengths=lengths)
        out = [self.next_tokens.clone()]
        for _ in range(new_tokens - 1):
            self.advance()
            out.append(self.next_tokens.clone())
        self.check_device_errors()
        return torch.stack(out, dim=1)

    def release(self) -> None:
        """Drop the captured graphs (the engine's buffers stay usable for eager steps)."""
        self.graph = None
        self._step_graph = None
        self._io_graph = None

"""The reference's decode-layer ``nn.Module`` surface, backed by the sm_100a kernels.

Drop-ins for ``src/models/quantized_qwen3/model.py``:

* ``PackedW4A16Linear`` (``model.py:84-146``) -- same constructor
  (``packed_weight`` uint8 ``[N, K/2]``, low nibble = even k, zero point 8;
  ``scales`` bf16 ``[N, K/group]``; ``in_features``, ``out_features``,
  ``group_size``, ``compute_dtype``), same ``from_store(store, prefix,
  compute_dtype=)`` and the same ``forward(x) -> compute_dtype`` result,
  computed by ``t2b_w4a16_gemm`` on ``x``'s CUDA device.
* ``T2BTensorWeights`` -- the weights provider of ``PackedTensorWeights``
  (``model.py:149-169``): ``dense(name)``, ``has_linear(prefix)`` and
  ``linear(prefix, *, compute_dtype)``, the last returning the CUDA linear
  above.  The reference's own ``QuantizedQwenLayer`` /
  ``QuantizedQwenForCausalLM`` built over it run every linear on ``libt2b``.
  ``AutoGPTQWeights`` is the same provider over AutoGPTQ tensors (synthetic
  models, checkpoints; asymmetric zero points).
* ``QuantizedQwenLayer`` (``model.py:283-327``) -- same constructor
  ``(weights, layer_idx, config, *, compute_dtype)`` and
  ``forward(x, angles, past_key_value) -> (x, present)``, running the fused
  decode layer: qkv + QK-norm + RoPE + KV write, GQA attention, o_proj +
  residual, gate/up + SwiGLU, down + residual (five launches).  The past KV
  is a preallocated ``LayerKVCache`` (bf16 ``[B, n_kv, max_ctx, head_dim]``
  plus the filled length) written in place; a reference-style
  ``(keys, values)`` tuple or ``None`` is also accepted and answered with a
  tuple grown by the new positions, as ``torch.cat`` does in
  ``model.py:256-264`` (that form copies the past into a fresh cache every
  call: use ``LayerKVCache`` on a decode loop).

Nothing here computes on the CPU: a forward on a CPU tensor raises.  Device
weights are built on the first forward on a device (the reference likewise
unpacks its weights on the first forward, ``model.py:122-131``).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib
from . import weights as W
from .loaders import qparam_to_autogptq
from .synth import AutoGPTQLinear

_DT = {torch.bfloat16, torch.float16, torch.float32}


def _require_cuda(x: torch.Tensor, what: str) -> None:
    if not x.is_cuda:
        raise RuntimeError(f"{what} runs on the sm_100a kernels only (CUDA tensors); there is no CPU path")


def _dkey(device) -> str:
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return str(d)


def _ws(nbytes: int, device) -> tuple[torch.Tensor, int]:
    n = max(int(nbytes), 256)
    return torch.zeros(n, dtype=torch.uint8, device=device), n


# ---------------------------------------------------------------------------
# linear
# ---------------------------------------------------------------------------
class PackedW4A16Linear(nn.Module):
    """``y = x . dequant(W)^T`` on the GPU with the reference module's interface.

    Symmetric reference format (``packed_weight`` + bf16 ``scales``), or an
    asymmetric AutoGPTQ linear through ``from_autogptq``.  The device copy is
    the T2B layout (``t2b_repack_autogptq``; batch rows >= 2 then take the
    tcgen05 path for bf16 inputs); a bf16 scale fp16 cannot hold exactly
    keeps the reference's ``qparam`` rows on the device instead (the CUDA-core
    GEMV reads them as they are).
    """

    def __init__(self, *, packed_weight: torch.Tensor, scales: torch.Tensor, in_features: int, out_features: int,
                 group_size: int, compute_dtype: torch.dtype) -> None:
        super().__init__()
        self.in_features, self.out_features = int(in_features), int(out_features)
        self.group_size, self.compute_dtype = int(group_size), compute_dtype
        self._check_shape()
        if tuple(packed_weight.shape) != (self.out_features, self.in_features // 2) or packed_weight.dtype != torch.uint8:
            raise ValueError(f"packed_weight must be uint8 [{self.out_features}, {self.in_features // 2}], got "
                             f"{tuple(packed_weight.shape)} {packed_weight.dtype}")
        groups = self.in_features // self.group_size
        if tuple(scales.shape) != (self.out_features, groups):
            raise ValueError(f"scales must be [{self.out_features}, {groups}], got {tuple(scales.shape)}")
        self.register_buffer("packed_weight", packed_weight.contiguous())
        self.register_buffer("scales", scales.to(torch.bfloat16).contiguous())
        self._lin: AutoGPTQLinear | None = None
        self._dev: dict = {}

    def _check_shape(self) -> None:
        if self.compute_dtype not in _DT:
            raise ValueError(f"compute_dtype {self.compute_dtype} is not bf16, fp16 or fp32")
        if self.group_size != 128:
            raise ValueError("the B200 kernels take group_size=128")
        if self.in_features % 256 or self.out_features % 128:
            raise ValueError(f"the B200 kernels need in_features % 256 == 0 and out_features % 128 == 0, got "
                             f"[{self.out_features}, {self.in_features}]")

    @classmethod
    def from_store(cls, store, prefix: str, *, compute_dtype: torch.dtype) -> "PackedW4A16Linear":
        """From the reference's ``PackedInferenceStore`` (``linear_segments``) or
        this package's ``loaders.PackedArtifact`` (``qparam``)."""
        if hasattr(store, "linear_segments"):
            spec, packed, scales = store.linear_segments(prefix)
        else:
            spec, qp = store.qparam(prefix)
            k = int(spec["in_features"])
            packed = qp[:, :k // 2]
            scales = qp[:, k // 2:].contiguous().view(torch.bfloat16)
        return cls(packed_weight=packed, scales=scales, in_features=int(spec["in_features"]),
                   out_features=int(spec["out_features"]), group_size=int(spec["group_size"]),
                   compute_dtype=compute_dtype)

    @classmethod
    def from_autogptq(cls, lin: AutoGPTQLinear, *, compute_dtype: torch.dtype) -> "PackedW4A16Linear":
        """An AutoGPTQ-v1 linear (per-group zero points, fp16 scales)."""
        self = cls.__new__(cls)
        nn.Module.__init__(self)
        self.in_features, self.out_features = lin.in_features, lin.out_features
        self.group_size, self.compute_dtype = lin.group_size, compute_dtype
        self._check_shape()
        self.register_buffer("qweight", lin.qweight.contiguous())
        self.register_buffer("qzeros", lin.qzeros.contiguous())
        self.register_buffer("scales", lin.scales.contiguous())
        self._lin = None
        self._dev = {}
        return self

    def qparam(self) -> torch.Tensor:
        """The reference's runtime rows (``packed_format.py:195-205``)."""
        return torch.cat([self.packed_weight, self.scales.contiguous().view(torch.uint8)], dim=1).contiguous()

    def autogptq(self) -> AutoGPTQLinear:
        """The weights as AutoGPTQ-v1 tensors (host), for fusing into a decode layer."""
        if self._lin is None:
            if hasattr(self, "qweight"):
                self._lin = AutoGPTQLinear(self.qweight.cpu(), self.qzeros.cpu(), self.scales.cpu(),
                                           self.in_features, self.out_features, self.group_size)
            else:
                self._lin = qparam_to_autogptq(self.qparam().cpu(), self.in_features, self.out_features,
                                               self.group_size, what="PackedW4A16Linear")
        return self._lin

    def _device_weights(self, device):
        key = _dkey(device)
        if key not in self._dev:
            try:
                self._dev[key] = ("t2b", W.from_autogptq(self.autogptq(), device))
            except ValueError:
                if hasattr(self, "qweight"):
                    raise
                self._dev[key] = ("qparam", self.qparam().to(device))   # bf16 scales kept as they are
            torch.cuda.synchronize(device)    # repacked weights complete before a PDL launch reads them
        return self._dev[key]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _require_cuda(x, "PackedW4A16Linear")
        if x.shape[-1] != self.in_features:
            raise ValueError(f"x has {x.shape[-1]} features, the linear {self.in_features}")
        xf = x.reshape(-1, self.in_features)
        if xf.dtype not in _DT:
            xf = xf.to(torch.float32)
        xf = xf.contiguous()
        M = xf.shape[0]
        y = torch.empty(M, self.out_features, dtype=self.compute_dtype, device=x.device)
        if M:
            kind, w = self._device_weights(x.device)
            L = _lib.lib()
            ws, n = _ws(L.t2b_w4a16_gemm_workspace_bytes(M, self.out_features, self.in_features), x.device)
            if kind == "t2b":
                args = (_lib.ptr(w.qw), _lib.ptr(w.meta), _lib.WFMT_T2B)
            else:
                args = (_lib.ptr(w), None, _lib.WFMT_QPARAM)
            _lib.call("t2b_w4a16_gemm", *args, _lib.ptr(xf), _lib.DTYPE[xf.dtype], _lib.ptr(y),
                      _lib.DTYPE[y.dtype], M, self.out_features, self.in_features, self.group_size, _lib.ptr(ws), n,
                      _lib.stream())
        return y.reshape(*x.shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, group_size={self.group_size}, "
                f"compute_dtype={self.compute_dtype}")


# ---------------------------------------------------------------------------
# weights providers (model.py:149-169)
# ---------------------------------------------------------------------------
class T2BTensorWeights:
    """``PackedTensorWeights`` over a packed store: the reference's
    ``PackedInferenceStore`` or ``loaders.PackedArtifact``."""

    def __init__(self, store) -> None:
        self.store = store

    def dense(self, name: str) -> torch.Tensor:
        return self.store.dense(name)

    def has_linear(self, prefix: str) -> bool:
        return self.store.has_linear(prefix)

    def linear(self, prefix: str, *, compute_dtype: torch.dtype) -> nn.Module:
        return PackedW4A16Linear.from_store(self.store, prefix, compute_dtype=compute_dtype)


class AutoGPTQWeights:
    """The same provider over in-memory tensors: ``dense`` maps full tensor
    names (``model.layers.0.input_layernorm.weight``) to bf16 tensors,
    ``linears`` maps linear prefixes (``model.layers.0.self_attn.q_proj``) to
    ``AutoGPTQLinear``."""

    def __init__(self, dense: dict, linears: dict) -> None:
        self._dense, self._linears = dense, linears

    def dense(self, name: str) -> torch.Tensor:
        try:
            return self._dense[name]
        except KeyError as exc:
            raise KeyError(f"missing dense tensor {name!r}") from exc

    def has_linear(self, prefix: str) -> bool:
        return prefix in self._linears

    def linear(self, prefix: str, *, compute_dtype: torch.dtype) -> nn.Module:
        return PackedW4A16Linear.from_autogptq(self._linears[prefix], compute_dtype=compute_dtype)

    @classmethod
    def from_model(cls, model: dict) -> "AutoGPTQWeights":
        """From the model dict of ``synth.random_model`` / ``loaders``."""
        dense, linears = {"model.embed_tokens.weight": model["embed"], "model.norm.weight": model["final_norm"]}, {}
        for li, layer in enumerate(model["layers"]):
            pre = f"model.layers.{li}"
            for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
                linears[f"{pre}.self_attn.{n}"] = layer[n]
            for n in ("gate_proj", "up_proj", "down_proj"):
                linears[f"{pre}.mlp.{n}"] = layer[n]
            dense[f"{pre}.input_layernorm.weight"] = layer["input_layernorm"]
            dense[f"{pre}.post_attention_layernorm.weight"] = layer["post_attention_layernorm"]
            for n in ("q_norm", "k_norm"):
                if layer.get(n) is not None:
                    dense[f"{pre}.self_attn.{n}.weight"] = layer[n]
        lm = model.get("lm_head")
        if isinstance(lm, AutoGPTQLinear):
            linears["lm_head"] = lm
        elif lm is not None:
            dense["lm_head.weight"] = lm
        return cls(dense, linears)


def _autogptq_of(mod) -> AutoGPTQLinear:
    """The quantized weights behind a provider's linear: this package's module,
    or any module with the reference's ``packed_weight`` / ``scales`` buffers."""
    if hasattr(mod, "autogptq"):
        return mod.autogptq()
    if hasattr(mod, "packed_weight") and hasattr(mod, "scales"):
        qp = torch.cat([mod.packed_weight, mod.scales.to(torch.bfloat16).contiguous().view(torch.uint8)], dim=1)
        return qparam_to_autogptq(qp.cpu().contiguous(), int(mod.in_features), int(mod.out_features),
                                  int(mod.group_size), what=type(mod).__name__)
    raise TypeError(f"{type(mod).__name__} carries no W4A16 weights the fused layer can read")


# ---------------------------------------------------------------------------
# fused decoder layer
# ---------------------------------------------------------------------------
class LayerKVCache:
    """Preallocated KV cache of one layer: bf16 ``k``/``v`` ``[B, n_kv, max_ctx,
    head_dim]`` and ``length`` (positions filled, the same for every row)."""

    def __init__(self, batch: int, n_kv: int, max_ctx: int, head_dim: int, device="cuda") -> None:
        if max_ctx % 64:
            raise ValueError("max_ctx must be a multiple of 64")
        shape = (batch, n_kv, max_ctx, head_dim)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.length = 0

    @property
    def max_ctx(self) -> int:
        return self.k.shape[2]


class QuantizedQwenLayer(nn.Module):
    """``x += attn(ln1(x)); x += mlp(ln2(x))`` for ``x [B, S, H]`` as five fused launches.

    S = 1 (decode) runs ``t2b_qkv_norm_rope_kvwrite`` and
    ``t2b_decode_attention_after_kvwrite``; S > 1 (a prefill chunk) runs
    ``t2b_qkv_norm_rope_kvwrite_seq`` and the causal ``t2b_prefill_attention``;
    both then run ``t2b_oproj_residual``, ``t2b_upgate_swiglu`` and
    ``t2b_down_residual``.  The residual stream is fp32 inside the layer and
    returned in ``compute_dtype``; ``angles`` are the reference's rows for the
    S new positions (cos at even, sin at odd slots, ``model.py:351-358``).
    """

    def __init__(self, weights, layer_idx: int, config, *, compute_dtype: torch.dtype) -> None:
        super().__init__()
        if compute_dtype not in _DT:
            raise ValueError(f"compute_dtype {compute_dtype} is not bf16, fp16 or fp32")
        self.config, self.compute_dtype, self.layer_idx = config, compute_dtype, layer_idx
        pre = f"model.layers.{layer_idx}"
        kw = {"compute_dtype": compute_dtype}
        self.q_proj = weights.linear(f"{pre}.self_attn.q_proj", **kw)
        self.k_proj = weights.linear(f"{pre}.self_attn.k_proj", **kw)
        self.v_proj = weights.linear(f"{pre}.self_attn.v_proj", **kw)
        self.o_proj = weights.linear(f"{pre}.self_attn.o_proj", **kw)
        self.gate_proj = weights.linear(f"{pre}.mlp.gate_proj", **kw)
        self.up_proj = weights.linear(f"{pre}.mlp.up_proj", **kw)
        self.down_proj = weights.linear(f"{pre}.mlp.down_proj", **kw)

        def norm(name):
            return weights.dense(name).to(torch.bfloat16).contiguous()

        self.register_buffer("input_layernorm", norm(f"{pre}.input_layernorm.weight"))
        self.register_buffer("post_attention_layernorm", norm(f"{pre}.post_attention_layernorm.weight"))
        self.register_buffer("q_norm", norm(f"{pre}.self_attn.q_norm.weight"))
        self.register_buffer("k_norm", norm(f"{pre}.self_attn.k_norm.weight"))
        self._dev: dict = {}

    def device_status(self, device="cuda") -> int:
        """The status word of this layer's launches on ``device`` (0: no kernel
        timed out a wait; T2B_ERR_TIMEOUT otherwise).  Synchronises."""
        f = self._dev.get(_dkey(device))
        return 0 if f is None else int(f["err"].item())

    def _fused(self, device):
        key = _dkey(device)
        if key not in self._dev:
            q, k, v = (_autogptq_of(m) for m in (self.q_proj, self.k_proj, self.v_proj))
            self._dev[key] = {
                "qkv": W.concat_rows([q, k, v], device),
                "o": W.from_autogptq(_autogptq_of(self.o_proj), device),
                "gu": W.pair_blocks(_autogptq_of(self.gate_proj), _autogptq_of(self.up_proj), device),
                "down": W.from_autogptq(_autogptq_of(self.down_proj), device),
                **{n: getattr(self, n).to(device) for n in ("input_layernorm", "post_attention_layernorm",
                                                           "q_norm", "k_norm")},
                "err": torch.zeros(1, dtype=torch.int32, device=device),
            }
            torch.cuda.synchronize(device)
        return self._dev[key]

    def new_cache(self, batch: int, max_ctx: int, device="cuda") -> LayerKVCache:
        c = self.config
        return LayerKVCache(batch, c.n_kv_groups, max_ctx, c.head_dim, device)

    def forward(self, x: torch.Tensor, angles: torch.Tensor, past_key_value):
        _require_cuda(x, "QuantizedQwenLayer")
        c = self.config
        B, S, H = x.shape
        dev = x.device
        nq, nkv, hd, I = c.n_heads, c.n_kv_groups, c.head_dim, c.hidden_dim
        if H != c.emb_dim:
            raise ValueError(f"x has {H} features, the layer {c.emb_dim}")
        # the cache: in place, or a fresh one holding a reference-style past
        if isinstance(past_key_value, LayerKVCache):
            cache, as_tuple = past_key_value, False
        else:
            past = 0 if past_key_value is None else int(past_key_value[0].shape[2])
            cache, as_tuple = self.new_cache(B, ((past + S + 63) // 64) * 64, dev), True
            if past:
                cache.k[:, :, :past].copy_(past_key_value[0])
                cache.v[:, :, :past].copy_(past_key_value[1])
                cache.length = past
        p0 = cache.length
        if p0 + S > cache.max_ctx:
            raise ValueError(f"{p0} + {S} positions do not fit the cache ({cache.max_ctx})")
        if cache.k.shape[0] != B:
            raise ValueError(f"the cache holds {cache.k.shape[0]} rows, x {B}")
        ang = angles.reshape(-1, hd)
        if ang.shape[0] != S:
            raise ValueError(f"angles hold {ang.shape[0]} rows for {S} positions")
        table = torch.zeros(cache.max_ctx, hd, dtype=torch.float32, device=dev)   # rows p0..p0+S-1 used
        table[p0:p0 + S].copy_(ang)
        f = self._fused(dev)
        st = _lib.stream()
        with _lib.status_word(f["err"], st):
            out = self._launch(f, x, table, cache, B, S, p0, st)
        cache.length = p0 + S
        if as_tuple:
            n = cache.length
            present = (cache.k[:, :, :n].to(self.compute_dtype), cache.v[:, :, :n].to(self.compute_dtype))
        else:
            present = cache
        return out, present

    def _launch(self, f, x, table, cache, B, S, p0, st) -> torch.Tensor:
        c = self.config
        H, dev = c.emb_dim, x.device
        nq, nkv, hd, I = c.n_heads, c.n_kv_groups, c.head_dim, c.hidden_dim
        M = B * S
        L, p = _lib.lib(), _lib.ptr
        f32, bf = torch.float32, torch.bfloat16
        xin = x.reshape(M, H)
        if xin.dtype not in (f32, bf):
            xin = xin.to(f32)
        xin = xin.contiguous()
        xr = torch.zeros(M, H, dtype=f32, device=dev)
        ssq_a, ssq_b = torch.zeros(M, dtype=f32, device=dev), torch.zeros(M, dtype=f32, device=dev)
        act = _lib.ACT                                  # fp16 linear inputs (t2b.h)
        xw = torch.empty(M, H, dtype=act, device=dev)
        q = torch.empty(M, nq * hd, dtype=_lib.QDT if S == 1 else bf, device=dev)   # decode: fp32 q
        attn = torch.empty(M, nq * hd, dtype=act, device=dev)
        h = torch.empty(M, I, dtype=act, device=dev)
        eps = float(c.rms_norm_eps)
        # x -> residual stream + split norm input (bf16(x * ln1), sum of squares)
        _lib.call("t2b_residual_norm_input", p(xin), _lib.DTYPE[xin.dtype], p(xr), p(ssq_a), p(f["input_layernorm"]),
                  p(xw), M, H, st)
        ws = _ws(L.t2b_qkv_workspace_bytes(M, H, nq, nkv, hd), dev)
        if S == 1:
            pos = torch.full((B,), p0, dtype=torch.int32, device=dev)
            _lib.call("t2b_qkv_norm_rope_kvwrite", p(f["qkv"].qw), p(f["qkv"].meta), f["qkv"].fmt, p(xw), p(ssq_a), eps,
                      p(f["q_norm"]), p(f["k_norm"]), p(table), p(pos), p(q), _lib.DTYPE[q.dtype], p(cache.k),
                      p(cache.v), p(ssq_b), B, H, nq, nkv, hd, cache.max_ctx, p(ws[0]), ws[1], st)
            wa = _ws(L.t2b_decode_attention_workspace_bytes(B, nq, nkv, hd, cache.max_ctx), dev)
            _lib.call("t2b_decode_attention_after_kvwrite", p(q), _lib.DTYPE[q.dtype], p(cache.k), p(cache.v), p(pos),
                      p(attn), _lib.DTYPE[act], B, nq, nkv, hd, cache.max_ctx, p(wa[0]), wa[1], st)
        else:
            pos = (p0 + torch.arange(S, device=dev, dtype=torch.int32)).repeat(B)
            seq = torch.arange(B, device=dev, dtype=torch.int32).repeat_interleave(S)
            _lib.call("t2b_qkv_norm_rope_kvwrite_seq", p(f["qkv"].qw), p(f["qkv"].meta), f["qkv"].fmt, p(xw), p(ssq_a), eps,
                      p(f["q_norm"]), p(f["k_norm"]), p(table), p(pos), p(seq), B, p(q), p(cache.k), p(cache.v),
                      p(ssq_b), M, H, nq, nkv, hd, cache.max_ctx, p(ws[0]), ws[1], st)
            _lib.call("t2b_prefill_attention", p(q), p(cache.k), p(cache.v), p(attn), _lib.DTYPE[act], B, S, p0, nq,
                      nkv, hd,
                      cache.max_ctx, st)
        wo = _ws(L.t2b_oproj_residual_workspace_bytes(M, H, nq * hd), dev)
        _lib.call("t2b_oproj_residual", p(f["o"].qw), p(f["o"].meta), f["o"].fmt, p(attn), p(xr), p(ssq_b),
                  p(f["post_attention_layernorm"]), p(xw), M, H, nq * hd, p(wo[0]), wo[1], st)
        wu = _ws(L.t2b_upgate_swiglu_workspace_bytes(M, H, I), dev)
        _lib.call("t2b_upgate_swiglu", p(f["gu"].qw), p(f["gu"].meta), f["gu"].fmt, p(xw), p(ssq_b), eps, p(h), p(ssq_a), M, H, I,
                  p(wu[0]), wu[1], st)
        wd = _ws(L.t2b_down_residual_workspace_bytes(M, H, I), dev)
        _lib.call("t2b_down_residual", p(f["down"].qw), p(f["down"].meta), f["down"].fmt, p(h), p(xr), p(ssq_a), None, None, M, H,
                  I, p(wd[0]), wd[1], st)
        return xr.view(B, S, H).to(self.compute_dtype)

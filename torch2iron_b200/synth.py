"""Seeded synthetic AutoGPTQ-v1 W4A16 weights (the benchmark configurations' inputs).

The benchmark configurations quantize ``W ~ N(0, 0.02)`` with asymmetric round-to-nearest
int4 per group of 128 along K:

* ``scale = (max - min) / 15`` (stored fp16),
* ``zero = round(-min / scale)`` clamped to ``[1, 15]``,
* ``q = clamp(round(w / scale) + zero, 0, 15)``,

packed the AutoGPTQ-v1 way: ``qweight [K/8, N]`` int32 with nibble ``j`` of
word ``[k/8, n]`` holding ``q[n, 8*(k/8)+j]``; ``qzeros [G, N/8]`` int32 holding
``zero - 1`` (the v1 "+1" convention read back by
``src/models/quantized_qwen3/packed_format.py:103-106``); ``scales [G, N]``
fp16.  Works on CPU or CUDA tensors (generation is setup, never timed).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


def _pack_nibbles_last(v: torch.Tensor) -> torch.Tensor:
    """Pack groups of 8 nibbles along the last dim into int32 (nibble j at bits 4j)."""
    v = v.to(torch.int64).reshape(*v.shape[:-1], v.shape[-1] // 8, 8)
    shifts = torch.arange(0, 32, 4, device=v.device, dtype=torch.int64)
    words = (v << shifts).sum(dim=-1)
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words)
    return words.to(torch.int32)


@dataclass
class AutoGPTQLinear:
    qweight: torch.Tensor   # int32 [K/8, N]
    qzeros: torch.Tensor    # int32 [G, N/8]
    scales: torch.Tensor    # fp16  [G, N]
    in_features: int
    out_features: int
    group_size: int = 128

    def to(self, device) -> "AutoGPTQLinear":
        return AutoGPTQLinear(self.qweight.to(device), self.qzeros.to(device), self.scales.to(device),
                              self.in_features, self.out_features, self.group_size)


def quantize_rtn_autogptq(w: torch.Tensor, group_size: int = 128) -> AutoGPTQLinear:
    """Asymmetric RTN int4 of ``w [N, K]`` (fp32) into AutoGPTQ-v1 tensors."""
    n, k = w.shape
    if k % group_size or k % 8 or n % 8:
        raise ValueError(f"shape [{n},{k}] not divisible by group {group_size} / 8")
    g = k // group_size
    wg = w.to(torch.float32).reshape(n, g, group_size)
    mn = wg.amin(dim=-1)
    mx = wg.amax(dim=-1)
    scale = ((mx - mn) / 15.0).clamp(min=1e-6).to(torch.float16)
    sf = scale.to(torch.float32)
    zero = torch.round(-mn / sf).clamp(1, 15)
    q = torch.clamp(torch.round(wg / sf[..., None]) + zero[..., None], 0, 15).to(torch.int32)
    q = q.reshape(n, k)
    qweight = _pack_nibbles_last(q.t().contiguous().reshape(k // 8, 8, n).permute(0, 2, 1)).reshape(k // 8, n)
    qzeros = _pack_nibbles_last((zero.t() - 1).to(torch.int32).contiguous())      # [G, N/8]
    return AutoGPTQLinear(qweight.contiguous(), qzeros.contiguous(), scale.t().contiguous(), k, n, group_size)


def random_linear(out_features: int, in_features: int, gen: torch.Generator, device="cpu",
                  std: float = 0.02, group_size: int = 128) -> AutoGPTQLinear:
    w = torch.randn(out_features, in_features, generator=gen, device=device, dtype=torch.float32) * std
    return quantize_rtn_autogptq(w, group_size)


LINEAR_NAMES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def linear_shapes(cfg) -> dict:
    """``name -> (out_features, in_features)`` for one decoder layer."""
    h, hd = cfg.emb_dim, cfg.head_dim
    return {
        "q_proj": (cfg.n_heads * hd, h),
        "k_proj": (cfg.n_kv_groups * hd, h),
        "v_proj": (cfg.n_kv_groups * hd, h),
        "o_proj": (h, cfg.n_heads * hd),
        "gate_proj": (cfg.hidden_dim, h),
        "up_proj": (cfg.hidden_dim, h),
        "down_proj": (h, cfg.hidden_dim),
    }


def random_layer(cfg, gen: torch.Generator, device="cpu") -> dict:
    """AutoGPTQ linears + norm weights (``N(1, 0.02)``) for one layer."""
    out = {name: random_linear(o, i, gen, device, group_size=cfg.group_size)
           for name, (o, i) in linear_shapes(cfg).items()}
    h, hd = cfg.emb_dim, cfg.head_dim

    def norm(n):
        return (1.0 + 0.02 * torch.randn(n, generator=gen, device=device)).to(torch.bfloat16)

    out["input_layernorm"] = norm(h)
    out["post_attention_layernorm"] = norm(h)
    if cfg.qk_norm:
        out["q_norm"] = norm(hd)
        out["k_norm"] = norm(hd)
    return out


def random_model(cfg, seed: int = 0, device="cpu") -> dict:
    """Every tensor of a synthetic model: ``layers`` (list of dicts), ``embed``,
    ``final_norm`` and ``lm_head`` (``None`` when tied to ``embed``)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    layers = [random_layer(cfg, gen, device) for _ in range(cfg.n_layers)]
    embed = (torch.randn(cfg.vocab_size, cfg.emb_dim, generator=gen, device=device) * 0.02).to(torch.bfloat16)
    final_norm = (1.0 + 0.02 * torch.randn(cfg.emb_dim, generator=gen, device=device)).to(torch.bfloat16)
    lm_head = None
    if not cfg.tie_word_embeddings:
        lm_head = (torch.randn(cfg.vocab_size, cfg.emb_dim, generator=gen, device=device) * 0.02).to(torch.bfloat16)
    return {"layers": layers, "embed": embed, "final_norm": final_norm, "lm_head": lm_head}

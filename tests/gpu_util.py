"""Shared helpers for the GPU parity tests."""

import torch

import oracle
from torch2iron_b200 import synth


def rel_err(y: torch.Tensor, ref: torch.Tensor) -> float:
    """max |y - ref| / max |ref| (the GEMV/GEMM parity metric, bar 1e-2)."""
    y = y.detach().float().cpu()
    ref = ref.detach().float().cpu()
    return float((y - ref).abs().max() / ref.abs().max().clamp(min=1e-30))


def max_abs(y: torch.Tensor, ref: torch.Tensor) -> float:
    return float((y.detach().float().cpu() - ref.detach().float().cpu()).abs().max())


class Q4NXOracleLinear:
    """A stored Q4NX linear as the oracle computes it: fp32 ``x . W^T`` over the
    reference's dense dequantisation (``oracle.q4nx_dequantize_linear``)."""

    def __init__(self, lin):
        self.dense = oracle.q4nx_dequantize_linear(lin.data.numpy().tobytes(), lin.in_features, lin.out_features)
        self.in_features, self.out_features = lin.in_features, lin.out_features

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        y = x.reshape(-1, self.in_features).to(torch.float32) @ self.dense.t()
        return y.reshape(*x.shape[:-1], self.out_features)


def _oracle_linear(lin):
    if hasattr(lin, "padded_out_features"):
        return Q4NXOracleLinear(lin)
    return oracle.GroupedW4A16Linear(lin.qweight.cpu(), lin.qzeros.cpu(), lin.scales.cpu())


def oracle_layer(layer: dict, cfg) -> oracle.OracleLayer:
    lin = {n: _oracle_linear(layer[n]) for n in synth.LINEAR_NAMES}
    return oracle.OracleLayer(**lin, input_layernorm=layer["input_layernorm"].cpu(),
                              post_attention_layernorm=layer["post_attention_layernorm"].cpu(),
                              q_norm=layer["q_norm"].cpu() if cfg.qk_norm else None,
                              k_norm=layer["k_norm"].cpu() if cfg.qk_norm else None)


def oracle_shape(cfg) -> oracle.OracleShape:
    return oracle.OracleShape(vocab_size=cfg.vocab_size, emb_dim=cfg.emb_dim, n_layers=cfg.n_layers,
                              n_heads=cfg.n_heads, n_kv_groups=cfg.n_kv_groups, head_dim=cfg.head_dim,
                              hidden_dim=cfg.hidden_dim, rms_norm_eps=cfg.rms_norm_eps, rope_base=cfg.rope_base,
                              qk_norm=cfg.qk_norm)


def oracle_decoder(cfg, model: dict, batch: int, max_ctx: int, dense: bool = False) -> oracle.OracleDecoder:
    """The oracle model over ``model``'s weights (moved to the host); ``dense``
    keeps each linear's dequantised fp32 matrix (full-size model checks)."""
    layers = [oracle_layer(l, cfg) for l in model["layers"]]
    if dense:
        for ol in layers:
            for n in synth.LINEAR_NAMES:
                if hasattr(getattr(ol, n), "cache_dense"):
                    getattr(ol, n).cache_dense()
    emb = model["embed"].cpu()
    lm = emb if model.get("lm_head") is None else model["lm_head"].cpu()
    return oracle.OracleDecoder(oracle_shape(cfg), layers, embed=emb, final_norm=model["final_norm"].cpu(),
                                lm_head=lm, max_ctx=max_ctx, batch=batch)

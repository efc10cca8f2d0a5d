"""CPU restatement of torch2iron's W4A16 Qwen3 decode path (test oracle only).

All arithmetic is PyTorch-CPU fp32, following the reference line by line.
Reference paths are relative to the torch2iron project root.

Nothing here is product code: the CUDA path in ``torch2iron_b200`` never
imports this module.  It exists so that tests, ``smoke()`` and the CPU
baseline leg of ``bench.py`` can check / time the reference algorithm.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

__all__ = [
    "unpack_int32_nibbles",
    "unpack_autogptq_qweight",
    "unpack_autogptq_qzeros",
    "autogptq_linear_to_dense",
    "autogptq_gemv",
    "unpack_biased_int4",
    "packed_w4a16_linear",
    "split_qparam",
    "GroupedW4A16Linear",
    "rms_norm",
    "rotate_half_interleaved",
    "apply_rope",
    "apply_rope_rows",
    "rope_two_halves",
    "compute_rope_angles",
    "chunked_attention_packet",
    "gqa_attention",
    "Q4NX_GROUP",
    "Q4NX_OUT_CHUNK",
    "Q4NX_IN_CHUNK",
    "Q4NX_PATCH_ROWS",
    "Q4NX_CHUNK_BYTES",
    "q4nx_unpack_chunk",
    "q4nx_dequantize_linear",
    "q4nx_linear",
    "OracleShape",
    "OracleLayer",
    "OracleDecoder",
]


# ---------------------------------------------------------------------------
# AutoGPTQ unpack / dequant
# ---------------------------------------------------------------------------

def unpack_int32_nibbles(packed: torch.Tensor, values_per_word: int = 8) -> torch.Tensor:
    """Nibble j of each int32 word is ``(word >> 4j) & 0xF``.

    Follows ``src/models/quantized_qwen3/packed_format.py:88-91``.
    """
    shifts = torch.arange(0, values_per_word * 4, 4, dtype=torch.int32)
    unpacked = torch.bitwise_right_shift(packed.to(torch.int32).unsqueeze(-1), shifts)
    return torch.bitwise_and(unpacked, 0xF).to(torch.int16)


def unpack_autogptq_qweight(qweight: torch.Tensor, in_features: int, out_features: int) -> torch.Tensor:
    """``qweight [K/8, N]`` int32 -> unsigned nibbles ``[N, K]``: q[n, k] = nib(qweight[k/8, n], k%8).

    Follows ``src/models/quantized_qwen3/packed_format.py:94-100``.
    """
    unpacked = unpack_int32_nibbles(qweight)          # [K/8, N, 8]
    unpacked = unpacked.permute(1, 0, 2).reshape(out_features, -1)
    return unpacked[:, :in_features].contiguous()


def unpack_autogptq_qzeros(qzeros: torch.Tensor, out_features: int) -> torch.Tensor:
    """``qzeros [G, N/8]`` int32 -> zero points ``[G, N]`` with AutoGPTQ-v1's stored+1.

    Follows ``src/models/quantized_qwen3/packed_format.py:103-106``.
    """
    unpacked = unpack_int32_nibbles(qzeros).reshape(qzeros.shape[0], -1)
    return (unpacked[:, :out_features] + 1).contiguous()


def autogptq_linear_to_dense(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                             group_size: int = 128) -> torch.Tensor:
    """Dense fp32 ``W[n, k] = (q[n, k] - zero[k/g, n]) * scale[k/g, n]``.

    Follows ``src/models/fast_qwen3/fast_packed_format.py:132-161``.
    """
    scales = scales.detach().cpu().to(torch.float32).contiguous()
    in_features = int(qweight.shape[0] * 8)
    out_features = int(qweight.shape[1])
    qvalues = unpack_autogptq_qweight(qweight, in_features, out_features).to(torch.float32)
    zeros = unpack_autogptq_qzeros(qzeros, out_features).to(torch.float32)
    if scales.shape[0] != zeros.shape[0] and scales.shape[1] == zeros.shape[0]:
        scales = scales.t().contiguous()
    if scales.shape != zeros.shape:
        raise ValueError(f"scale/zero shape mismatch: scales={tuple(scales.shape)} zeros={tuple(zeros.shape)}")
    dense = torch.empty((out_features, in_features), dtype=torch.float32)
    for g in range(scales.shape[0]):
        start = g * group_size
        end = min(start + group_size, in_features)
        dense[:, start:end] = (qvalues[:, start:end] - zeros[g].view(out_features, 1)) * scales[g].view(out_features, 1)
    return dense


def autogptq_gemv(x: torch.Tensor, qweight, qzeros, scales, group_size: int = 128) -> torch.Tensor:
    """``y = x . dequant(W)^T`` in fp32 (the config-0 reference computation:
    ``_autogptq_linear_to_dense`` of ``fast_packed_format.py:132-161``
    followed by an fp32 matmul)."""
    w = autogptq_linear_to_dense(qweight, qzeros, scales, group_size)
    return x.to(torch.float32) @ w.t()


# ---------------------------------------------------------------------------
# Symmetric biased-int4 ("qparam") runtime linear
# ---------------------------------------------------------------------------

def unpack_biased_int4(packed: torch.Tensor, in_features: int) -> torch.Tensor:
    """Low nibble = even k, high nibble = odd k, signed = nibble - 8.

    Follows ``src/models/quantized_qwen3/model.py:122-131``.
    """
    low = torch.bitwise_and(packed, 0xF)
    high = torch.bitwise_and(torch.bitwise_right_shift(packed, 4), 0xF)
    nibbles = torch.stack((low, high), dim=-1).flatten(1)[:, :in_features]
    return (nibbles.to(torch.int16) - 8).to(torch.int8).contiguous()


def packed_w4a16_linear(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
                        in_features: int, out_features: int, group_size: int = 128) -> torch.Tensor:
    """Per-group fp32 accumulate of ``x[:, g] @ (signed[:, g] * s[:, g])^T``.

    Follows ``src/models/quantized_qwen3/model.py:133-146`` (returns fp32).
    """
    signed = unpack_biased_int4(packed, in_features)
    x_flat = x.reshape(-1, in_features).to(torch.float32)
    out = torch.zeros((x_flat.shape[0], out_features), dtype=torch.float32)
    sc = scales.to(torch.float32)
    for g in range(sc.shape[1]):
        start = g * group_size
        end = min(start + group_size, in_features)
        wg = signed[:, start:end].to(torch.float32) * sc[:, g].view(out_features, 1)
        out += x_flat[:, start:end].matmul(wg.t())
    return out.reshape(*x.shape[:-1], out_features)


def split_qparam(qparam: torch.Tensor, in_features: int, group_size: int = 128):
    """Split a ``qparam [N, K/2 + G*2]`` row (packed nibbles then bf16 scales).

    Inverse of ``src/models/quantized_qwen3/packed_format.py:195-205``.
    """
    n = qparam.shape[0]
    kb = in_features // 2
    packed = qparam[:, :kb].contiguous()
    scales = qparam[:, kb:].contiguous().view(torch.bfloat16).reshape(n, -1)
    return packed, scales


class GroupedW4A16Linear:
    """The reference runtime linear (``model.py:84-146``) generalised to the
    asymmetric AutoGPTQ zero of ``fast_packed_format.py:158-160``.

    Like ``PackedW4A16Linear.unpack_signed_weight`` (``model.py:122-131``) it
    unpacks once and caches the signed ``q - zero`` int8 matrix; ``__call__``
    runs the per-group fp32 loop of ``model.py:133-146``.
    """

    def __init__(self, qweight, qzeros, scales, group_size: int = 128):
        k = int(qweight.shape[0] * 8)
        n = int(qweight.shape[1])
        q = unpack_autogptq_qweight(qweight, k, n)
        z = unpack_autogptq_qzeros(qzeros, n)                       # [G, N]
        zf = z.t().repeat_interleave(group_size, dim=1)[:, :k]      # [N, K]
        self.signed = (q - zf).to(torch.int8).contiguous()          # in [-16, 14]
        self.scales = scales.to(torch.float32).t().contiguous()     # [N, G]
        self.in_features, self.out_features, self.group_size = k, n, group_size

    def dense(self) -> torch.Tensor:
        return self.signed.to(torch.float32) * self.scales.repeat_interleave(self.group_size, dim=1)

    def cache_dense(self) -> "GroupedW4A16Linear":
        """Keep the dequantised fp32 matrix and contract in one matmul: the
        same fp32 products, summed in one pass over K instead of one pass per
        group (only the association of the fp32 sum differs).  For the
        full-size model checks, where the per-group loop would re-dequantise
        every weight at every step."""
        self._dense = self.dense().contiguous()
        return self

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x_flat = x.reshape(-1, self.in_features).to(torch.float32)
        dense = getattr(self, "_dense", None)
        if dense is not None:
            return x_flat.matmul(dense.t()).reshape(*x.shape[:-1], self.out_features)
        out = torch.zeros((x_flat.shape[0], self.out_features), dtype=torch.float32)
        for g in range(self.scales.shape[1]):
            start = g * self.group_size
            end = min(start + self.group_size, self.in_features)
            wg = self.signed[:, start:end].to(torch.float32) * self.scales[:, g].view(-1, 1)
            out += x_flat[:, start:end].matmul(wg.t())
        return out.reshape(*x.shape[:-1], self.out_features)


# ---------------------------------------------------------------------------
# Norms and RoPE
# ---------------------------------------------------------------------------

def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``x * rsqrt(mean(x^2) + eps) * w``; follows ``model.py:178-181``."""
    variance = x.to(torch.float32).pow(2).mean(dim=-1, keepdim=True)
    x = x * torch.rsqrt(variance + eps).to(x.dtype)
    return x * weight.to(x.dtype)


def rotate_half_interleaved(x: torch.Tensor) -> torch.Tensor:
    """``rot(x)[2i] = -x[2i+1], rot(x)[2i+1] = x[2i]``; follows ``model.py:184-187``."""
    even = x[..., ::2]
    odd = x[..., 1::2]
    return torch.stack((-odd, even), dim=-1).flatten(-2)


def apply_rope(x: torch.Tensor, angles: torch.Tensor) -> torch.Tensor:
    """Interleaved RoPE with angles ``[seq, hd]`` (cos at even, sin at odd slots).

    ``x`` is ``[batch, seq, heads, hd]``; follows ``model.py:190-196``.
    """
    cos = angles[..., ::2].repeat_interleave(2, dim=-1)
    sin = angles[..., 1::2].repeat_interleave(2, dim=-1)
    view_shape = [1, angles.shape[-2], *([1] * (x.dim() - 3)), angles.shape[-1]]
    cos = cos.view(*view_shape)
    sin = sin.view(*view_shape)
    return x * cos.to(x.dtype) + rotate_half_interleaved(x) * sin.to(x.dtype)


def apply_rope_rows(x: torch.Tensor, angles: torch.Tensor) -> torch.Tensor:
    """``apply_rope`` with one angle row per batch row: x ``[B, heads, hd]``, angles ``[B, hd]``.

    Same arithmetic as ``model.py:190-196``; the reference broadcasts one
    angle row over the batch (all rows share a position), this form lets rows
    sit at different positions.
    """
    cos = angles[..., ::2].repeat_interleave(2, dim=-1)[:, None, :]
    sin = angles[..., 1::2].repeat_interleave(2, dim=-1)[:, None, :]
    return x * cos.to(x.dtype) + rotate_half_interleaved(x) * sin.to(x.dtype)


def rope_two_halves(x: torch.Tensor, angles: torch.Tensor) -> torch.Tensor:
    """HF-style two-halves RoPE used by the NPU ``RMSNormRoPE`` operator.

    ``out[i] = x[i] c_i - x[i+h] s_i``, ``out[i+h] = x[i+h] c_i + x[i] s_i`` with
    ``c_i = angles[2i]``, ``s_i = angles[2i+1]``; follows
    ``src/torch2iron/operators/rms_norm_rope/kernel.cc:39-67``.
    """
    half = x.shape[-1] // 2
    c = angles[..., 0::2]
    s = angles[..., 1::2]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1)


def compute_rope_angles(head_dim: int, context_length: int, rope_base: float) -> torch.Tensor:
    """``[ctx, hd]`` fp32 table, cos at even and sin at odd slots; follows ``model.py:351-358``."""
    inv_freq = 1.0 / (rope_base ** (torch.arange(0, head_dim, 2).float() / head_dim))
    position = torch.arange(context_length).float()
    freqs = torch.outer(position, inv_freq)
    angles = torch.empty(context_length, head_dim)
    angles[:, ::2] = torch.cos(freqs)
    angles[:, 1::2] = torch.sin(freqs)
    return angles


# ---------------------------------------------------------------------------
# Packet-cache attention (LlamaChunkedAttention's CPU twin)
# ---------------------------------------------------------------------------

def chunked_attention_packet(queries: torch.Tensor, packet: torch.Tensor, packet_seq_len: int,
                             chunk_size: int) -> torch.Tensor:
    """Masked GQA decode attention over the ``[group][chunk][K|V|mask]`` packet.

    Follows ``src/models/fast_qwen3/attention_reference.py:110-171`` with
    ``attend_seq_len = packet_seq_len`` (the NPU operator scans every chunk,
    ``src/torch2iron/operators/llama_chunked_attention/op.py:94-104``).
    Slots whose mask is <= 0.5 are skipped; a group with no live slot
    outputs zeros.  Returns bf16 ``[G, qh, hd]``.
    """
    groups, qh, hd = (int(s) for s in queries.shape)
    chunk_elems = 2 * chunk_size * hd + chunk_size
    per_group = packet_seq_len // chunk_size * chunk_elems
    out = torch.zeros((groups, qh, hd), dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(hd)
    for g in range(groups):
        keys, values = [], []
        for slot in range(packet_seq_len):
            base = g * per_group + (slot // chunk_size) * chunk_elems
            row = slot % chunk_size
            if float(packet[base + 2 * chunk_size * hd + row]) <= 0.5:
                continue
            keys.append(packet[base + row * hd: base + (row + 1) * hd].to(torch.float32))
            v0 = base + chunk_size * hd + row * hd
            values.append(packet[v0: v0 + hd].to(torch.float32))
        if not keys:
            continue
        km = torch.stack(keys)
        vm = torch.stack(values)
        scores = queries[g].to(torch.float32) @ km.t() * scale
        out[g] = (torch.softmax(scores, dim=-1) @ vm).to(torch.bfloat16)
    return out


# ---------------------------------------------------------------------------
# Decoder layer and model
# ---------------------------------------------------------------------------

# ---------------------------------------------------------------------------
# Q4NX group-32 layout of the fast Qwen3 path (src/models/fast_qwen3/q4nx_layout.py)
# ---------------------------------------------------------------------------
Q4NX_GROUP = 32          # k per (scale, zero point)            q4nx_layout.py:30
Q4NX_OUT_CHUNK = 32      # output rows per chunk                 :31
Q4NX_IN_CHUNK = 256      # k per chunk                           :32
Q4NX_PATCH_ROWS = 64     # output rows per patch (two chunks)    :33
Q4NX_CHUNK_BYTES = 2 * 2 * Q4NX_OUT_CHUNK * (Q4NX_IN_CHUNK // Q4NX_GROUP) + Q4NX_OUT_CHUNK * Q4NX_IN_CHUNK // 2


def q4nx_unpack_chunk(chunk) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """One 5120-byte chunk -> (q ``[32, 256]``, scale ``[32, 8]``, zero ``[32, 8]``):
    bf16 scales, then bf16 zero points, then 4-bit values two per byte, low
    nibble = even k (``q4nx_layout.py:92-113,159-174``)."""
    b = torch.frombuffer(bytearray(bytes(chunk)), dtype=torch.uint8)
    if b.numel() != Q4NX_CHUNK_BYTES:
        raise ValueError(f"a Q4NX chunk is {Q4NX_CHUNK_BYTES} bytes, got {b.numel()}")
    ng = Q4NX_OUT_CHUNK * (Q4NX_IN_CHUNK // Q4NX_GROUP)
    scale = b[:2 * ng].view(torch.bfloat16).to(torch.float32).view(Q4NX_OUT_CHUNK, -1)
    zero = b[2 * ng:4 * ng].view(torch.bfloat16).to(torch.float32).view(Q4NX_OUT_CHUNK, -1)
    packed = b[4 * ng:].view(Q4NX_OUT_CHUNK, Q4NX_IN_CHUNK // 2)
    q = torch.stack((packed & 0xF, packed >> 4), dim=-1).reshape(Q4NX_OUT_CHUNK, Q4NX_IN_CHUNK)
    return q, scale, zero


def q4nx_dequantize_linear(data, in_features: int, out_features: int) -> torch.Tensor:
    """Dense fp32 ``[out, in]`` of a Q4NX linear: output rows padded to 64-row
    patches, each patch stored K-chunk-major as (rows 0-31, rows 32-63) chunk
    pairs; ``w = (q - zero) * scale`` per 32-k group in fp32
    (``q4nx_layout.py:132-146,177-237``)."""
    if in_features % Q4NX_IN_CHUNK:
        raise ValueError(f"in_features must be a multiple of {Q4NX_IN_CHUNK}")
    padded = -(-out_features // Q4NX_PATCH_ROWS) * Q4NX_PATCH_ROWS
    raw = bytes(data)
    n_chunks = padded // Q4NX_OUT_CHUNK * (in_features // Q4NX_IN_CHUNK)
    if len(raw) != n_chunks * Q4NX_CHUNK_BYTES:
        raise ValueError(f"expected {n_chunks * Q4NX_CHUNK_BYTES} bytes, got {len(raw)}")
    w = torch.empty(padded, in_features, dtype=torch.float32)
    i = 0
    for r0 in range(0, padded, Q4NX_PATCH_ROWS):
        for k0 in range(0, in_features, Q4NX_IN_CHUNK):
            for half in (0, Q4NX_OUT_CHUNK):
                q, scale, zero = q4nx_unpack_chunk(raw[i * Q4NX_CHUNK_BYTES:(i + 1) * Q4NX_CHUNK_BYTES])
                i += 1
                g = q.to(torch.float32).view(Q4NX_OUT_CHUNK, -1, Q4NX_GROUP)
                w[r0 + half:r0 + half + Q4NX_OUT_CHUNK, k0:k0 + Q4NX_IN_CHUNK] = \
                    ((g - zero[..., None]) * scale[..., None]).view(Q4NX_OUT_CHUNK, Q4NX_IN_CHUNK)
    return w[:out_features]


def q4nx_linear(x: torch.Tensor, data, in_features: int, out_features: int) -> torch.Tensor:
    """fp32 ``x . W^T`` over the dense Q4NX weight (``q4nx_layout.py:292-303``
    before its final bf16 rounding)."""
    return x.to(torch.float32).reshape(-1, in_features) @ q4nx_dequantize_linear(data, in_features,
                                                                                 out_features).t()


def gqa_attention(q: torch.Tensor, keys: torch.Tensor, vals: torch.Tensor) -> torch.Tensor:
    """One query token: q ``[n_heads, hd]`` over ``keys``/``vals`` ``[n_kv, n, hd]``,
    q head h reading kv head ``h // (n_heads / n_kv)``; fp32 softmax(q k^T /
    sqrt(hd)) v (``model.py:266-279``, ``kv_plane_reference.py:122-187``)."""
    qpg = q.shape[0] // keys.shape[0]
    k = keys.to(torch.float32).repeat_interleave(qpg, dim=0)
    v = vals.to(torch.float32).repeat_interleave(qpg, dim=0)
    scores = torch.einsum("hd,hnd->hn", q.to(torch.float32), k) * q.shape[-1] ** -0.5
    return torch.einsum("hn,hnd->hd", torch.softmax(scores, dim=-1), v)


@dataclass(frozen=True)
class OracleShape:
    """Field-for-field subset of ``QuantizedQwenConfig`` (``model.py:330-348``) plus ``qk_norm``."""

    vocab_size: int
    emb_dim: int
    n_layers: int
    n_heads: int
    n_kv_groups: int
    head_dim: int
    hidden_dim: int
    rms_norm_eps: float
    rope_base: float
    qk_norm: bool = True
    group_size: int = 128

    @property
    def q_heads_per_group(self) -> int:
        return self.n_heads // self.n_kv_groups


@dataclass
class OracleLayer:
    """One decoder layer's weights; linears are ``GroupedW4A16Linear`` (or any callable)."""

    q_proj: object
    k_proj: object
    v_proj: object
    o_proj: object
    gate_proj: object
    up_proj: object
    down_proj: object
    input_layernorm: torch.Tensor
    post_attention_layernorm: torch.Tensor
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None


@dataclass
class OracleDecoder:
    """Embedding -> layers -> final norm -> lm_head, one token per row per step.

    Composition follows ``model.py:453-478`` (forward) and ``model.py:316-327``
    (layer).  The growing ``torch.cat`` past-KV of ``model.py:256-264`` is held
    here as a preallocated ``[B, kv, ctx, hd]`` cache written at ``pos``;
    attending to slots ``0..pos`` is the same causal set.  The cache stores
    bf16 values (``kv_dtype``) because the GPU cache is bf16; all arithmetic is
    fp32 (``model.py`` default ``compute_dtype=float32``).
    """

    shape: OracleShape
    layers: list
    embed: torch.Tensor            # [V, H] (bf16 in the benchmark configurations)
    final_norm: torch.Tensor       # [H]
    lm_head: torch.Tensor          # [V, H] (tied -> same tensor as embed)
    max_ctx: int
    batch: int
    kv_dtype: torch.dtype = torch.bfloat16
    k_cache: list = field(default_factory=list)
    v_cache: list = field(default_factory=list)

    def __post_init__(self):
        s = self.shape
        self.angles = compute_rope_angles(s.head_dim, self.max_ctx, s.rope_base)
        self.k_cache = [torch.zeros(self.batch, s.n_kv_groups, self.max_ctx, s.head_dim, dtype=self.kv_dtype)
                        for _ in range(s.n_layers)]
        self.v_cache = [torch.zeros_like(self.k_cache[0]) for _ in range(s.n_layers)]
        self._lm = self.lm_head.to(torch.float32)

    # model.py:240-280 for one new token per row
    def attention(self, li: int, layer: OracleLayer, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        s = self.shape
        b = x.shape[0]
        q = layer.q_proj(x).view(b, s.n_heads, s.head_dim)
        k = layer.k_proj(x).view(b, s.n_kv_groups, s.head_dim)
        v = layer.v_proj(x).view(b, s.n_kv_groups, s.head_dim)
        if s.qk_norm:
            q = rms_norm(q, layer.q_norm, s.rms_norm_eps)
            k = rms_norm(k, layer.k_norm, s.rms_norm_eps)
        ang = self.angles[pos]                                   # [B, hd]
        q = apply_rope_rows(q, ang)
        k = apply_rope_rows(k, ang)
        kc, vc = self.k_cache[li], self.v_cache[li]
        for r in range(b):
            kc[r, :, int(pos[r])] = k[r].to(self.kv_dtype)
            vc[r, :, int(pos[r])] = v[r].to(self.kv_dtype)
        ctx = torch.empty(b, s.n_heads, s.head_dim)
        for r in range(b):
            n = int(pos[r]) + 1
            ctx[r] = gqa_attention(q[r], kc[r, :, :n], vc[r, :, :n])
        return layer.o_proj(ctx.reshape(b, s.n_heads * s.head_dim))

    def layer_step(self, li: int, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        s = self.shape
        layer = self.layers[li]
        x = x + self.attention(li, layer, rms_norm(x, layer.input_layernorm, s.rms_norm_eps), pos)
        h = rms_norm(x, layer.post_attention_layernorm, s.rms_norm_eps)
        return x + layer.down_proj(F.silu(layer.gate_proj(h)) * layer.up_proj(h))   # model.py:215-216

    def hidden_after_embed(self, tokens: torch.Tensor) -> torch.Tensor:
        return self.embed[tokens].to(torch.float32)              # model.py:469

    def step(self, tokens: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """One decode step: tokens ``[B]`` at positions ``pos [B]`` -> logits ``[B, V]`` fp32."""
        x = self.hidden_after_embed(tokens)
        for li in range(self.shape.n_layers):
            x = self.layer_step(li, x, pos)
        return rms_norm(x, self.final_norm, self.shape.rms_norm_eps) @ self._lm.t()   # model.py:477

    def prefill_chunked(self, prompts: torch.Tensor, chunk: int, last_only: bool = False) -> torch.Tensor:
        """Chunked prefill of ``prompts [B, P]``: every chunk of ``chunk`` tokens per
        row goes through each layer at once, its K/V written into the cache
        first and each token attending keys ``0..its position`` -- the causal
        rule of the reference's chunked prefill (``prefill_runtime.py:95-164``,
        ``llama_chunked_prefill_attention/op.py:21-50``) and of the full-prompt
        forward (``model.py:453-478`` with a causal mask).  Returns the logits of
        every prompt token ``[B, P, V]``, or with ``last_only`` those of the last
        one ``[B, V]`` (the only row a greedy decode needs)."""
        s = self.shape
        B, P = prompts.shape
        out = []
        for c0 in range(0, P, chunk):
            n = min(chunk, P - c0)
            pos = torch.arange(c0, c0 + n)
            x = self.embed[prompts[:, c0:c0 + n]].to(torch.float32)            # [B, n, H]
            for li in range(s.n_layers):
                layer = self.layers[li]
                xn = rms_norm(x, layer.input_layernorm, s.rms_norm_eps).reshape(B * n, s.emb_dim)
                q = layer.q_proj(xn).view(B, n, s.n_heads, s.head_dim)
                k = layer.k_proj(xn).view(B, n, s.n_kv_groups, s.head_dim)
                v = layer.v_proj(xn).view(B, n, s.n_kv_groups, s.head_dim)
                if s.qk_norm:
                    q = rms_norm(q, layer.q_norm, s.rms_norm_eps)
                    k = rms_norm(k, layer.k_norm, s.rms_norm_eps)
                ang = self.angles[pos]                                         # [n, hd]
                q = apply_rope_rows(q.reshape(B * n, s.n_heads, s.head_dim), ang.repeat(B, 1)).view(q.shape)
                k = apply_rope_rows(k.reshape(B * n, s.n_kv_groups, s.head_dim), ang.repeat(B, 1)).view(k.shape)
                kc, vc = self.k_cache[li], self.v_cache[li]
                kc[:, :, c0:c0 + n] = k.permute(0, 2, 1, 3).to(self.kv_dtype)
                vc[:, :, c0:c0 + n] = v.permute(0, 2, 1, 3).to(self.kv_dtype)
                qpg = s.q_heads_per_group
                keys = kc[:, :, :c0 + n].to(torch.float32).repeat_interleave(qpg, dim=1)   # [B, nq, c0+n, hd]
                vals = vc[:, :, :c0 + n].to(torch.float32).repeat_interleave(qpg, dim=1)
                scores = torch.einsum("bihd,bhjd->bhij", q.to(torch.float32), keys) * s.head_dim ** -0.5
                mask = torch.arange(c0 + n)[None, :] > pos[:, None]           # key after the token
                scores = scores.masked_fill(mask[None, None], float("-inf"))
                ctx = torch.einsum("bhij,bhjd->bihd", torch.softmax(scores, dim=-1), vals)
                x = x + layer.o_proj(ctx.reshape(B * n, s.n_heads * s.head_dim)).view(B, n, s.emb_dim)
                h = rms_norm(x, layer.post_attention_layernorm, s.rms_norm_eps).reshape(B * n, s.emb_dim)
                x = x + layer.down_proj(F.silu(layer.gate_proj(h)) * layer.up_proj(h)).view(B, n, s.emb_dim)
            if last_only:
                if c0 + n == P:
                    return rms_norm(x[:, -1], self.final_norm, s.rms_norm_eps) @ self._lm.t()
                continue
            out.append(rms_norm(x, self.final_norm, s.rms_norm_eps) @ self._lm.t())
        return torch.cat(out, dim=1)

    def prefill(self, prompts: torch.Tensor) -> torch.Tensor:
        """Feed ``prompts [B, P]`` one position at a time; returns the last logits."""
        logits = None
        for p in range(prompts.shape[1]):
            logits = self.step(prompts[:, p], torch.full((prompts.shape[0],), p, dtype=torch.long))
        return logits

    def generate(self, prompts: torch.Tensor, new_tokens: int) -> torch.Tensor:
        """Greedy decode (``model.py:481-498``) for every row; returns ``[B, new_tokens]``."""
        logits = self.prefill(prompts)
        out = []
        p = prompts.shape[1]
        for i in range(new_tokens):
            nxt = torch.argmax(logits, dim=-1)
            out.append(nxt)
            if i + 1 < new_tokens:
                logits = self.step(nxt, torch.full((prompts.shape[0],), p + i, dtype=torch.long))
        return torch.stack(out, dim=1)

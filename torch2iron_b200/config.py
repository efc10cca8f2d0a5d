"""Model shapes for the decode hot path.

``QuantizedQwenConfig`` keeps the field names of the reference dataclass
(``src/models/quantized_qwen3/model.py:330-348``) and adds the two switches
the B200 path needs for Llama-3.2 shapes (``qk_norm``, ``tie_word_embeddings``).
"""

from __future__ import annotations

from dataclasses import dataclass, replace


@dataclass(frozen=True)
class QuantizedQwenConfig:
    vocab_size: int
    emb_dim: int
    n_layers: int
    n_heads: int
    n_kv_groups: int
    head_dim: int
    hidden_dim: int
    rms_norm_eps: float
    rope_base: float
    context_length: int = 40960
    eos_token_id: int | list[int] | None = None
    bos_token_id: int | None = None
    group_size: int = 128
    qk_norm: bool = True
    tie_word_embeddings: bool = True

    @property
    def q_heads_per_group(self) -> int:
        return self.n_heads // self.n_kv_groups

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_groups * self.head_dim

    def scaled(self, **kw) -> "QuantizedQwenConfig":
        return replace(self, **kw)

    def validate(self) -> None:
        g = self.group_size
        if g != 128:
            raise ValueError("only group_size=128 is supported")
        if self.n_heads % self.n_kv_groups:
            raise ValueError("n_heads must be a multiple of n_kv_groups")
        if self.head_dim not in (64, 128):
            raise ValueError("head_dim must be 64 or 128")
        for k in (self.emb_dim, self.q_dim, self.hidden_dim):
            if k % 256:
                raise ValueError(f"in_features {k} must be a multiple of 256")
        for n in (self.q_dim, self.kv_dim, self.emb_dim):
            if n % 128:
                raise ValueError(f"out_features {n} must be a multiple of 128")
        if self.hidden_dim % 64:
            raise ValueError("hidden_dim must be a multiple of 64")


# Model shapes of the benchmark configurations (decode configs 1-4).
QWEN3_0_6B = QuantizedQwenConfig(
    vocab_size=151936, emb_dim=1024, n_layers=28, n_heads=16, n_kv_groups=8, head_dim=128,
    hidden_dim=3072, rms_norm_eps=1e-6, rope_base=1e6, qk_norm=True, tie_word_embeddings=True)

LLAMA_3_2_1B = QuantizedQwenConfig(
    vocab_size=128256, emb_dim=2048, n_layers=16, n_heads=32, n_kv_groups=8, head_dim=64,
    hidden_dim=8192, rms_norm_eps=1e-5, rope_base=5e5, qk_norm=False, tie_word_embeddings=True)

QWEN3_8B = QuantizedQwenConfig(
    vocab_size=151936, emb_dim=4096, n_layers=36, n_heads=32, n_kv_groups=8, head_dim=128,
    hidden_dim=12288, rms_norm_eps=1e-6, rope_base=1e6, qk_norm=True, tie_word_embeddings=False)

PRESETS = {"qwen3-0.6b": QWEN3_0_6B, "llama-3.2-1b": LLAMA_3_2_1B, "qwen3-8b": QWEN3_8B}

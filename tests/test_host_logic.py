"""CPU-side host logic: operator validation (reference error behaviour), configs, synth."""

import pytest
import torch

import oracle
from torch2iron_b200 import synth
from torch2iron_b200.config import LLAMA_3_2_1B, QWEN3_0_6B, QWEN3_8B
from torch2iron_b200.operators import (LlamaChunkedAttention, RMSNormRoPE, ResidualAddRMSNorm, SiLUMul, W4A16GEMM,
                                       W4A16GEMV, W4A16KGroupGEMM)
from torch2iron_b200.rope import rope_angles


def test_reference_validation_errors():
    with pytest.raises(ValueError, match="K must be even"):
        W4A16GEMV(M=128, K=255)
    with pytest.raises(ValueError, match="multiple of group_size"):
        W4A16GEMV(M=128, K=200)
    with pytest.raises(ValueError, match="tile_k == group_size"):
        W4A16GEMM(M=8, K=1024, N=1024, tile_k=64)
    with pytest.raises(ValueError, match="k_tiles must be divisible"):
        W4A16KGroupGEMM(M=8, K=384, N=128, k_group=2)
    with pytest.raises(ValueError, match="cols must be divisible by 32"):
        RMSNormRoPE(rows=8, cols=100, angle_rows=8)
    with pytest.raises(ValueError, match="epsilon must be positive"):
        RMSNormRoPE(rows=8, cols=128, angle_rows=8, epsilon=0)
    with pytest.raises(ValueError, match="divisible by chunk_size"):
        LlamaChunkedAttention(max_seq_len=100)
    with pytest.raises(ValueError):
        ResidualAddRMSNorm(size=1000, num_aie_columns=8, tile_size=1024)
    with pytest.raises(ValueError):
        SiLUMul(size=1000, tile_size=512)


def test_arg_specs_follow_reference_shapes():
    op = W4A16GEMV(M=3072, K=1024)
    spec = op.get_arg_spec()
    assert spec[0].shape == (3072, 1024 // 2 + 8 * 2) and spec[0].dtype == torch.uint8
    assert spec[1].shape == (1024,) and spec[2].shape == (3072,)
    per_batch = W4A16GEMV(M=200, K=512, num_batches=3).get_arg_spec()     # ragged M, one qparam per batch row
    assert per_batch[0].shape == (3, 200, 256 + 8) and per_batch[1].shape == (3, 512)
    assert per_batch[2].shape == (3, 200)
    assert W4A16GEMV(M=256, K=512, num_batches=3, shared_qparam=True).get_arg_spec()[0].shape == (256, 264)
    a = LlamaChunkedAttention(max_seq_len=512, num_kv_groups=8, q_heads_per_group=2, head_dim=128)
    assert a.get_arg_spec()[1].shape == (8 * 8 * (2 * 64 * 128 + 64),)


def test_presets_validate():
    for cfg in (QWEN3_0_6B, LLAMA_3_2_1B, QWEN3_8B):
        cfg.validate()
    assert QWEN3_0_6B.q_heads_per_group == 2 and LLAMA_3_2_1B.q_heads_per_group == 4


def test_rope_table_is_the_reference_formula():
    assert torch.equal(rope_angles(128, 300, 1e6), oracle.compute_rope_angles(128, 300, 1e6))


def test_synth_recipe_properties():
    g = torch.Generator().manual_seed(0)
    lin = synth.random_linear(256, 512, g)
    assert lin.qweight.shape == (64, 256) and lin.qweight.dtype == torch.int32
    assert lin.qzeros.shape == (4, 32) and lin.scales.shape == (4, 256) and lin.scales.dtype == torch.float16
    z = oracle.unpack_autogptq_qzeros(lin.qzeros, 256)
    assert 1 <= int(z.min()) and int(z.max()) <= 15


def test_oracle_chunked_prefill_equals_stepwise():
    """Several sequences, a chunk that does not divide the prompt: the chunked
    restatement equals feeding one position per step (logits and KV caches)."""
    from tests.gpu_util import oracle_layer, oracle_shape
    from torch2iron_b200.config import QuantizedQwenConfig
    cfg = QuantizedQwenConfig(vocab_size=512, emb_dim=256, n_layers=2, n_heads=4, n_kv_groups=2, head_dim=64,
                              hidden_dim=512, rms_norm_eps=1e-6, rope_base=1e6)
    model = synth.random_model(cfg, seed=12)
    prompts = torch.randint(0, cfg.vocab_size, (3, 13), generator=torch.Generator().manual_seed(13))
    def dec():   # fp32 caches: only the order of fp32 sums differs between the two forms
        return oracle.OracleDecoder(oracle_shape(cfg), [oracle_layer(l, cfg) for l in model["layers"]],
                                    embed=model["embed"], final_norm=model["final_norm"], lm_head=model["embed"],
                                    max_ctx=64, batch=3, kv_dtype=torch.float32)
    a, b = dec(), dec()
    la = a.prefill_chunked(prompts, 4)[:, -1]
    lb = b.prefill(prompts)
    assert (la - lb).abs().max().item() <= 1e-5
    for li in range(cfg.n_layers):
        assert (a.k_cache[li] - b.k_cache[li]).abs().max().item() <= 1e-5
        assert (a.v_cache[li] - b.v_cache[li]).abs().max().item() <= 1e-5

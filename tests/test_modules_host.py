"""Host-side checks of the nn.Module surface (no GPU): construction and
validation, the CPU refusal, the providers' lookups, and -- where the
reference tree is present (the build container) -- that the reference's own
``QuantizedQwenLayer`` builds over this package's weights provider with every
linear a CUDA-backed ``PackedW4A16Linear``."""

import os
import sys

import pytest
import torch

from torch2iron_b200 import loaders as LD
from torch2iron_b200 import synth
from torch2iron_b200.config import QuantizedQwenConfig
from torch2iron_b200.modules import AutoGPTQWeights, PackedW4A16Linear, QuantizedQwenLayer, T2BTensorWeights

PACKED = os.path.join(os.path.dirname(__file__), "golden", "packed_tiny")
# the reference checkout beside this repository, when present (env T2B_REFERENCE_SRC overrides)
REF_SRC = os.environ.get("T2B_REFERENCE_SRC") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference", "src")


def test_packed_linear_validates_like_a_constructor_and_refuses_cpu():
    packed = torch.zeros(128, 128, dtype=torch.uint8)
    scales = torch.ones(128, 2, dtype=torch.bfloat16)
    lin = PackedW4A16Linear(packed_weight=packed, scales=scales, in_features=256, out_features=128, group_size=128,
                            compute_dtype=torch.float32)
    assert lin.qparam().shape == (128, 128 + 4)
    with pytest.raises(RuntimeError, match="no CPU path"):
        lin(torch.zeros(1, 256))
    with pytest.raises(ValueError, match="group_size"):
        PackedW4A16Linear(packed_weight=packed, scales=torch.ones(128, 4, dtype=torch.bfloat16), in_features=256,
                          out_features=128, group_size=64, compute_dtype=torch.float32)
    with pytest.raises(ValueError, match="packed_weight"):
        PackedW4A16Linear(packed_weight=packed[:, :64], scales=scales, in_features=256, out_features=128,
                          group_size=128, compute_dtype=torch.float32)
    with pytest.raises(ValueError, match="in_features % 256"):
        PackedW4A16Linear(packed_weight=torch.zeros(128, 64, dtype=torch.uint8),
                          scales=torch.ones(128, 1, dtype=torch.bfloat16), in_features=128, out_features=128,
                          group_size=128, compute_dtype=torch.float32)


def test_provider_over_the_packed_artifact_round_trips_the_weights():
    art = LD.PackedArtifact(LD.find_packed_dir(PACKED))
    prov = T2BTensorWeights(art)
    lin = prov.linear("model.layers.0.self_attn.q_proj", compute_dtype=torch.bfloat16)
    ref = art.linear("model.layers.0.self_attn.q_proj")
    got = lin.autogptq()
    assert torch.equal(got.qweight, ref.qweight) and torch.equal(got.scales, ref.scales)
    assert prov.dense("model.norm.weight").dtype == torch.bfloat16


def test_autogptq_provider_and_fused_layer_construct_on_the_host():
    cfg = QuantizedQwenConfig(vocab_size=512, emb_dim=256, n_layers=2, n_heads=4, n_kv_groups=2, head_dim=64,
                              hidden_dim=512, rms_norm_eps=1e-6, rope_base=1e6)
    model = synth.random_model(cfg, seed=4)
    prov = AutoGPTQWeights.from_model(model)
    assert prov.has_linear("model.layers.1.mlp.down_proj") and not prov.has_linear("lm_head")
    layer = QuantizedQwenLayer(prov, 1, cfg, compute_dtype=torch.float32)
    assert isinstance(layer.down_proj, PackedW4A16Linear)
    with pytest.raises(RuntimeError, match="no CPU path"):
        layer(torch.zeros(1, 1, 256), torch.zeros(1, 64), None)


@pytest.mark.skipif(not os.path.isdir(REF_SRC), reason="the reference tree is only in the build container")
def test_reference_layer_class_builds_over_this_provider():
    sys.path.insert(0, REF_SRC)
    try:
        import models.quantized_qwen3.model as ref_model
    except Exception as exc:       # its imports (transformers tokenizer) may be unavailable
        pytest.skip(f"reference model module does not import here: {exc}")
    finally:
        sys.path.remove(REF_SRC)
    art = LD.PackedArtifact(LD.find_packed_dir(PACKED))
    cfg = ref_model.QuantizedQwenConfig(vocab_size=512, emb_dim=256, n_layers=2, n_heads=4, n_kv_groups=2,
                                        head_dim=64, hidden_dim=512, rms_norm_eps=1e-6, rope_base=1e6,
                                        context_length=64, eos_token_id=None, bos_token_id=None, group_size=128)
    layer = ref_model.QuantizedQwenLayer(T2BTensorWeights(art), 0, cfg, compute_dtype=torch.float32)
    for mod in (layer.self_attn.q_proj, layer.self_attn.o_proj, layer.mlp.down_proj):
        assert isinstance(mod, PackedW4A16Linear)
    # the fused layer takes the reference's config object and the same provider
    fused = QuantizedQwenLayer(T2BTensorWeights(art), 0, cfg, compute_dtype=torch.float32)
    assert fused.q_proj.out_features == 256

"""The reference's nn.Module surface on the GPU (``torch2iron_b200.modules``).

* ``PackedW4A16Linear`` against the reference module's own output
  (``qparam_linear.npz``, written by ``model.PackedW4A16Linear``,
  ``model.py:84-146``): exact fp32 path held to 1e-4, bf16 activations
  (tcgen05 path, bf16 weight rounding) to 1e-2;
* the linear built from the reference's packed artifact through the weights
  provider (``from_store``), against the oracle's dequantisation;
* ``QuantizedQwenLayer`` against the reference layer's golden output
  (``layer_small.npz``, ``model.py:283-327``, batch 2, past length 7), with a
  reference-style past tuple and with the preallocated cache; a 5-token
  prefill chunk against five single-token calls.
"""

import os

import pytest
import torch

import oracle
from tests import golden_io as gio
from tests.gpu_util import max_abs, rel_err
from torch2iron_b200 import loaders as LD
from torch2iron_b200 import synth
from torch2iron_b200.config import QuantizedQwenConfig
from torch2iron_b200.modules import AutoGPTQWeights, LayerKVCache, PackedW4A16Linear, QuantizedQwenLayer, \
    T2BTensorWeights

pytestmark = pytest.mark.gpu

SMALL = QuantizedQwenConfig(vocab_size=512, emb_dim=256, n_layers=1, n_heads=4, n_kv_groups=2, head_dim=64,
                            hidden_dim=512, rms_norm_eps=1e-6, rope_base=1e6)


@pytest.mark.parametrize("dtype,bar", [(torch.float32, 1e-4), (torch.bfloat16, 1e-2)])
def test_packed_linear_matches_reference_module(dtype, bar):
    d = gio.load("qparam_linear.npz")
    qp = torch.from_numpy(d["qparam"])
    lin = PackedW4A16Linear(packed_weight=qp[:, :256], scales=qp[:, 256:].contiguous().view(torch.bfloat16),
                            in_features=512, out_features=256, group_size=128, compute_dtype=dtype)
    x = gio.bf16(d["x"]).to(dtype).cuda()
    y = lin(x)
    torch.cuda.synchronize()
    assert y.dtype == dtype and y.shape == (3, 256)
    assert rel_err(y, torch.from_numpy(d["y"])) <= bar
    y3 = lin(x.view(3, 1, 512))                        # leading dimensions kept, as F.linear does
    assert y3.shape == (3, 1, 256) and torch.equal(y3.view(3, 256), y)


def test_linear_from_packed_artifact_through_the_provider():
    art = LD.PackedArtifact(LD.find_packed_dir(os.path.join(gio.GOLDEN, "packed_tiny")))
    prov = T2BTensorWeights(art)
    prefix = "model.layers.0.mlp.down_proj"
    assert prov.has_linear(prefix) and not prov.has_linear("model.layers.0.mlp.nothing")
    lin = prov.linear(prefix, compute_dtype=torch.float32)
    ref = art.linear(prefix)
    x = torch.randn(4, lin.in_features, generator=torch.Generator().manual_seed(3))
    y = lin(x.cuda())
    want = oracle.GroupedW4A16Linear(ref.qweight, ref.qzeros, ref.scales)(x)
    assert rel_err(y, want) <= 1e-4


def _golden_layer(dtype=torch.float32):
    d = gio.load("layer_small.npz")
    pre = "model.layers.0"
    linears = {f"{pre}.{'self_attn' if n in ('q_proj', 'k_proj', 'v_proj', 'o_proj') else 'mlp'}.{n}": gio.linear(d, n)
               for n in synth.LINEAR_NAMES}
    dense = {f"{pre}.input_layernorm.weight": gio.bf16(d["input_layernorm"]),
             f"{pre}.post_attention_layernorm.weight": gio.bf16(d["post_attention_layernorm"]),
             f"{pre}.self_attn.q_norm.weight": gio.bf16(d["q_norm"]),
             f"{pre}.self_attn.k_norm.weight": gio.bf16(d["k_norm"])}
    return d, QuantizedQwenLayer(AutoGPTQWeights(dense, linears), 0, SMALL, compute_dtype=dtype)


def test_fused_layer_matches_reference_layer_golden():
    d, layer = _golden_layer()
    ang = oracle.compute_rope_angles(64, 64, 1e6)
    x = torch.from_numpy(d["x"]).cuda()
    past = (torch.from_numpy(d["past_k"]).cuda(), torch.from_numpy(d["past_v"]).cuda())
    out, (pk, pv) = layer(x, ang[7:8].cuda(), past)
    torch.cuda.synchronize()
    assert layer.device_status() == 0
    assert out.shape == (2, 1, 256) and out.dtype == torch.float32
    assert rel_err(out, torch.from_numpy(d["out"])) <= 1e-2
    assert pk.shape == (2, 2, 8, 64)
    assert max_abs(pk, torch.from_numpy(d["present_k"])) <= 5e-2
    assert max_abs(pv, torch.from_numpy(d["present_v"])) <= 5e-2
    # the preallocated cache gives the same result in place
    cache = LayerKVCache(2, 2, 64, 64)
    cache.k[:, :, :7].copy_(past[0])
    cache.v[:, :, :7].copy_(past[1])
    cache.length = 7
    out2, same = layer(x, ang[7:8].cuda(), cache)
    assert same is cache and cache.length == 8
    assert torch.equal(out2, out)
    assert torch.equal(cache.k[:, :, :8].float(), pk)


def test_fused_layer_prefill_chunk_equals_single_steps():
    """S = 5 new tokens in one call (causal prefill kernels) against five
    S = 1 calls (decode kernels) on the same layer."""
    _, layer = _golden_layer(torch.bfloat16)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(2, 5, 256, generator=g).to(torch.bfloat16).cuda()
    ang = oracle.compute_rope_angles(64, 64, 1e6).to(torch.bfloat16).cuda()
    a = LayerKVCache(2, 2, 64, 64)
    out_a, _ = layer(x, ang[0:5], a)
    b = LayerKVCache(2, 2, 64, 64)
    outs = [layer(x[:, t:t + 1], ang[t:t + 1], b)[0] for t in range(5)]
    torch.cuda.synchronize()
    assert a.length == b.length == 5
    assert rel_err(out_a, torch.cat(outs, dim=1)) <= 1e-2
    assert max_abs(a.k[:, :, :5], b.k[:, :, :5]) <= 5e-2
    assert layer.device_status() == 0

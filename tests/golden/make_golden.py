"""Generate golden vectors by running torch2iron's own CPU reference.

Run in a container where the reference project is mounted (its ``src`` on
``sys.path``)::

    python tests/golden/make_golden.py /path/to/torch2iron

Every output comes from the reference's functions and modules, called
unmodified:

* ``_autogptq_linear_to_dense`` (``src/models/fast_qwen3/fast_packed_format.py:132-161``)
  + fp32 matmul                                   -> gemv_autogptq.npz, config0.npz
* ``quantize_dense_to_biased_int4`` / ``make_qparam`` / ``PackedW4A16Linear``
  (``src/models/quantized_qwen3/packed_format.py:195-205,384-402``,
  ``src/models/quantized_qwen3/model.py:84-146``)  -> qparam_linear.npz
* ``RMSNorm`` / ``apply_rope`` / ``compute_rope_angles`` (``model.py:172-196,351-358``)
                                                  -> rope_norm.npz
* ``QuantizedQwenLayer`` (``model.py:283-327``)   -> layer_small.npz
* ``QuantizedQwenForCausalLM.forward/generate`` (``model.py:361-498``) -> model_tiny.npz
* ``write_decode_packet_slot`` / ``chunked_attention_reference``
  (``src/models/fast_qwen3/attention_reference.py:69-171``) -> attention_packet.npz

Weights are the benchmark recipe (``torch2iron_b200.synth``): asymmetric RTN
int4, AutoGPTQ-v1 packing.  The files are small; tests never need the
reference at run time.
"""

from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from torch2iron_b200 import synth  # noqa: E402


def bf16_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


def f16_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float16).contiguous().numpy()


def lin_arrays(prefix: str, lin: synth.AutoGPTQLinear) -> dict:
    return {f"{prefix}.qweight": lin.qweight.numpy(), f"{prefix}.qzeros": lin.qzeros.numpy(),
            f"{prefix}.scales": f16_np(lin.scales)}


class RefWeights:
    """Duck-typed weights provider (``model.py:149-169`` interface) whose
    ``.linear`` returns the reference's ``DenseLinear`` over the reference's
    own AutoGPTQ dequant."""

    def __init__(self, dense: dict, linears: dict, mods):
        self.dense_t, self.linears, self.mods = dense, linears, mods

    def dense(self, name):
        return self.dense_t[name]

    def has_linear(self, prefix):
        return prefix in self.linears

    def linear(self, prefix, *, compute_dtype):
        lin = self.linears[prefix]
        tensors = {f"{prefix}.qweight": lin.qweight, f"{prefix}.qzeros": lin.qzeros, f"{prefix}.scales": lin.scales}
        w = self.mods.fpf._autogptq_linear_to_dense(tensors, prefix, group_size=lin.group_size)
        return self.mods.model.DenseLinear(w, compute_dtype)


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    import models.fast_qwen3.attention_reference as attn_ref
    import models.fast_qwen3.fast_packed_format as fpf
    import models.quantized_qwen3.model as model
    import models.quantized_qwen3.packed_format as pf

    class M:
        pass

    mods = M()
    mods.fpf, mods.model = fpf, model

    # -- single GEMV, AutoGPTQ asymmetric (config-0 recipe, N reduced) --------
    g = torch.Generator().manual_seed(1608560892)
    w = torch.randn(512, 1024, generator=g) * 0.02
    lin = synth.quantize_rtn_autogptq(w)
    x = torch.randn(8, 1024, generator=g).to(torch.float16)
    t = {"p.qweight": lin.qweight, "p.qzeros": lin.qzeros, "p.scales": lin.scales}
    dense = fpf._autogptq_linear_to_dense(t, "p", group_size=128)
    y = x.to(torch.float32) @ dense.t()
    np.savez_compressed(HERE / "gemv_autogptq.npz", x=f16_np(x), y=y.numpy(), **lin_arrays("p", lin))

    # -- config 0 exactly: seed 0, x fp16 [1,1024], W [3072,1024] ------------
    g = torch.Generator().manual_seed(0)
    w = torch.randn(3072, 1024, generator=g) * 0.02
    x = torch.randn(1, 1024, generator=g).to(torch.float16)
    lin = synth.quantize_rtn_autogptq(w)
    t = {"p.qweight": lin.qweight, "p.qzeros": lin.qzeros, "p.scales": lin.scales}
    dense = fpf._autogptq_linear_to_dense(t, "p", group_size=128)
    y = x.to(torch.float32) @ dense.t()
    digest = hashlib.sha256(lin.qweight.numpy().tobytes() + lin.qzeros.numpy().tobytes()
                            + f16_np(lin.scales).tobytes()).hexdigest()
    np.savez_compressed(HERE / "config0.npz", x=f16_np(x), y=y.numpy(), weights_sha256=np.array(digest))

    # -- reference runtime format: symmetric biased int4 + bf16 scales -------
    g = torch.Generator().manual_seed(1608560892 + 1)
    w = torch.randn(256, 512, generator=g) * 0.02
    packed, scales = pf.quantize_dense_to_biased_int4(w, group_size=128)
    qparam = pf.make_qparam(packed, scales)
    x = torch.randn(3, 512, generator=g).to(torch.bfloat16)
    lin_mod = model.PackedW4A16Linear(packed_weight=packed, scales=scales, in_features=512, out_features=256,
                                      group_size=128, compute_dtype=torch.float32)
    y = lin_mod(x.to(torch.float32))
    np.savez_compressed(HERE / "qparam_linear.npz", qparam=qparam.numpy(), x=bf16_np(x), y=y.numpy())

    # -- RMSNorm + interleaved RoPE -----------------------------------------
    g = torch.Generator().manual_seed(7)
    angles = model.compute_rope_angles(128, 64, 1e6)
    xq = torch.randn(2, 1, 4, 128, generator=g)
    wn = 1.0 + 0.02 * torch.randn(128, generator=g)
    norm = model.RMSNorm(wn, 1e-6, torch.float32)
    yq = model.apply_rope(norm(xq), angles[5:6])
    np.savez_compressed(HERE / "rope_norm.npz", angles=angles.numpy(), x=xq.numpy(), w=wn.numpy(), y=yq.numpy(),
                        pos=np.array(5))

    # -- one decoder layer, batch 2, past length 7 ---------------------------
    cfg = model.QuantizedQwenConfig(vocab_size=512, emb_dim=256, n_layers=1, n_heads=4, n_kv_groups=2,
                                    head_dim=64, hidden_dim=512, rms_norm_eps=1e-6, rope_base=1e6,
                                    context_length=64, eos_token_id=None, bos_token_id=None, group_size=128)
    g = torch.Generator().manual_seed(1608560892 + 2)
    shapes = {"q_proj": (256, 256), "k_proj": (128, 256), "v_proj": (128, 256), "o_proj": (256, 256),
              "gate_proj": (512, 256), "up_proj": (512, 256), "down_proj": (256, 512)}
    linears, dense_t, arrays = {}, {}, {}
    pre = "model.layers.0"
    for name, (o, i) in shapes.items():
        sub = "self_attn" if name.endswith(("q_proj", "k_proj", "v_proj", "o_proj")) else "mlp"
        lin = synth.random_linear(o, i, g)
        linears[f"{pre}.{sub}.{name}"] = lin
        arrays.update(lin_arrays(name, lin))
    for nm, n in (("input_layernorm", 256), ("post_attention_layernorm", 256),
                  ("self_attn.q_norm", 64), ("self_attn.k_norm", 64)):
        v = (1.0 + 0.02 * torch.randn(n, generator=g)).to(torch.bfloat16)
        dense_t[f"{pre}.{nm}.weight"] = v
        arrays[nm.split(".")[-1]] = bf16_np(v)
    layer = model.QuantizedQwenLayer(RefWeights(dense_t, linears, mods), 0, cfg, compute_dtype=torch.float32)
    past_k = torch.randn(2, 2, 7, 64, generator=g).to(torch.bfloat16).to(torch.float32)
    past_v = torch.randn(2, 2, 7, 64, generator=g).to(torch.bfloat16).to(torch.float32)
    xin = torch.randn(2, 1, 256, generator=g)
    ang = model.compute_rope_angles(64, 64, 1e6)
    out, (pk, pv) = layer(xin, ang[7:8], (past_k, past_v))
    np.savez_compressed(HERE / "layer_small.npz", x=xin.numpy(), past_k=past_k.numpy(), past_v=past_v.numpy(),
                        out=out.numpy(), present_k=pk.numpy(), present_v=pv.numpy(), pos=np.array(7), **arrays)

    # -- tiny full model: forward + greedy generate ---------------------------
    hf_config = {"vocab_size": 512, "hidden_size": 256, "num_hidden_layers": 2, "num_attention_heads": 4,
                 "num_key_value_heads": 2, "head_dim": 64, "intermediate_size": 512, "rms_norm_eps": 1e-6,
                 "rope_theta": 1e6, "max_position_embeddings": 64,
                 "quantization_config": {"bits": 4, "sym": True, "group_size": 128}}
    g = torch.Generator().manual_seed(1608560892 + 3)
    linears, dense_t, arrays = {}, {}, {}
    for li in range(2):
        pre = f"model.layers.{li}"
        for name, (o, i) in shapes.items():
            sub = "self_attn" if name.endswith(("q_proj", "k_proj", "v_proj", "o_proj")) else "mlp"
            lin = synth.random_linear(o, i, g)
            linears[f"{pre}.{sub}.{name}"] = lin
            arrays.update(lin_arrays(f"l{li}.{name}", lin))
        for nm, n in (("input_layernorm", 256), ("post_attention_layernorm", 256),
                      ("self_attn.q_norm", 64), ("self_attn.k_norm", 64)):
            v = (1.0 + 0.02 * torch.randn(n, generator=g)).to(torch.bfloat16)
            dense_t[f"{pre}.{nm}.weight"] = v
            arrays[f"l{li}.{nm.split('.')[-1]}"] = bf16_np(v)
    emb = (torch.randn(512, 256, generator=g) * 0.02).to(torch.bfloat16)
    fnorm = (1.0 + 0.02 * torch.randn(256, generator=g)).to(torch.bfloat16)
    dense_t["model.embed_tokens.weight"] = emb
    dense_t["model.norm.weight"] = fnorm
    lm = model.QuantizedQwenForCausalLM(RefWeights(dense_t, linears, mods), hf_config, compute_dtype=torch.float32)
    prompt = torch.randint(0, 512, (1, 6), generator=g)
    logits, _ = lm(prompt)
    gen_ids = lm.generate(prompt, max_new_tokens=8)
    np.savez_compressed(HERE / "model_tiny.npz", prompt=prompt.numpy(), logits_last=logits[0, -1].numpy(),
                        generated=gen_ids[0, 6:].numpy(), embed=bf16_np(emb), final_norm=bf16_np(fnorm), **arrays)

    # -- packet-cache attention ----------------------------------------------
    g = torch.Generator().manual_seed(407895018)
    groups, qh, hd, seq, chunk = 2, 2, 64, 128, 64
    n_el = attn_ref.decode_packet_elements(groups, seq, chunk, hd)
    packet = torch.randn(n_el, generator=g).to(torch.bfloat16)
    # masks: slots 0..99 live, the rest dead, plus a few holes
    for gi in range(groups):
        for slot in range(seq):
            _, _, mo = attn_ref.decode_packet_slot_offsets(gi, slot, seq, chunk, hd)
            packet[mo] = 1.0 if (slot < 100 and slot % 17 != 3) else 0.0
    cur_k = torch.randn(groups, hd, generator=g).to(torch.bfloat16)
    cur_v = torch.randn(groups, hd, generator=g).to(torch.bfloat16)
    packet2 = attn_ref.write_decode_packet_slot(packet, cur_k, cur_v, 100, seq, chunk)
    q = torch.randn(groups, qh, hd, generator=g).to(torch.bfloat16)
    out = attn_ref.chunked_attention_reference(q, packet2, seq, seq, chunk)
    np.savez_compressed(HERE / "attention_packet.npz", packet=bf16_np(packet), cur_k=bf16_np(cur_k),
                        cur_v=bf16_np(cur_v), slot=np.array(100), packet_after=bf16_np(packet2), q=bf16_np(q),
                        out=bf16_np(out), seq=np.array(seq), chunk=np.array(chunk))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <torch2iron project root>")
    main(sys.argv[1])

"""Golden fixture for the artifact loaders, made by the reference itself.

Writes a tiny seeded symmetric AutoGPTQ Qwen3 checkpoint (config.json +
model.safetensors, untied dense head; weights N(0, 0.02) and norm weights
N(1, 0.02), the value distribution of the benchmark configurations), packs it
with the reference's own writer (``write_packed_inference_artifact``,
src/models/quantized_qwen3/packed_format.py:405-655) into
``tests/golden/packed_tiny/`` (config.json + qwen3_w4a16_packed/, the
checkpoint kept beside it), and records in ``tests/golden/packed_tiny.npz``
the reference model's logits over a prompt, its greedy tokens and the logits
each token was picked from (``QuantizedQwenForCausalLM`` on that artifact,
model.py:360-480, fp32).

Run once, in a container where the reference is mounted:
    python tests/golden/make_packed_artifact.py <reference root>
"""

import json
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch
from safetensors.torch import save_file

HERE = Path(__file__).resolve().parent
OUT = HERE / "packed_tiny"
CFG = {"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "vocab_size": 512, "hidden_size": 256,
       "num_hidden_layers": 2, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 64,
       "intermediate_size": 512, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0, "max_position_embeddings": 256,
       "tie_word_embeddings": False, "bos_token_id": 1, "eos_token_id": 2,
       "quantization_config": {"bits": 4, "group_size": 128, "sym": True, "quant_method": "gptq"}}


def sym_autogptq(w: torch.Tensor, g: int = 128):
    """Symmetric RTN int4 of w [N, K] in AutoGPTQ-v1 tensors (zero 8, stored 7)."""
    n, k = w.shape
    wg = w.reshape(n, k // g, g)
    scale = (wg.abs().amax(-1) / 7.0).clamp(min=1e-6).to(torch.float16)
    q = torch.clamp(torch.round(wg / scale.float()[..., None]) + 8, 0, 15).to(torch.int64).reshape(n, k)
    shifts = torch.arange(0, 32, 4, dtype=torch.int64)
    words = (q.t().reshape(k // 8, 8, n).permute(0, 2, 1) << shifts).sum(-1)
    qweight = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)
    zw = (torch.full((k // g, n // 8, 8), 7, dtype=torch.int64) << shifts).sum(-1)
    qzeros = torch.where(zw >= 2 ** 31, zw - 2 ** 32, zw).to(torch.int32)
    return qweight.contiguous(), qzeros.contiguous(), scale.t().contiguous()


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    from models.quantized_qwen3.packed_format import PackedInferenceStore, write_packed_inference_artifact
    from models.quantized_qwen3.model import PackedTensorWeights, QuantizedQwenForCausalLM

    gen = torch.Generator().manual_seed(1234)
    h, hd, nq, nkv, inter, v = 256, 64, 4, 2, 512, 512
    t = {}
    shapes = {"self_attn.q_proj": (nq * hd, h), "self_attn.k_proj": (nkv * hd, h), "self_attn.v_proj": (nkv * hd, h),
              "self_attn.o_proj": (h, nq * hd), "mlp.gate_proj": (inter, h), "mlp.up_proj": (inter, h),
              "mlp.down_proj": (h, inter)}
    for i in range(CFG["num_hidden_layers"]):
        p = f"model.layers.{i}"
        for name, (n, k) in shapes.items():
            qw, qz, sc = sym_autogptq(torch.randn(n, k, generator=gen) * 0.02)
            t[f"{p}.{name}.qweight"], t[f"{p}.{name}.qzeros"], t[f"{p}.{name}.scales"] = qw, qz, sc
        for nrm, size in (("input_layernorm", h), ("post_attention_layernorm", h), ("self_attn.q_norm", hd),
                          ("self_attn.k_norm", hd)):
            t[f"{p}.{nrm}.weight"] = (1.0 + 0.02 * torch.randn(size, generator=gen)).to(torch.bfloat16)
    t["model.embed_tokens.weight"] = (torch.randn(v, h, generator=gen) * 0.02).to(torch.bfloat16)
    t["model.norm.weight"] = (1.0 + 0.02 * torch.randn(h, generator=gen)).to(torch.bfloat16)
    # untied dense head: the packer quantizes it into the artifact's synthetic W4 lm_head
    t["lm_head.weight"] = (torch.randn(v, h, generator=gen) * 0.02).to(torch.bfloat16)

    if OUT.exists():
        shutil.rmtree(OUT)
    OUT.mkdir(parents=True)
    (OUT / "config.json").write_text(json.dumps(CFG, indent=2) + "\n")
    save_file(t, str(OUT / "model.safetensors"))
    with tempfile.TemporaryDirectory() as tmp:
        shutil.copy(OUT / "config.json", tmp)
        shutil.copy(OUT / "model.safetensors", tmp)
        write_packed_inference_artifact(tmp, OUT / "qwen3_w4a16_packed")
    manifest = json.loads((OUT / "qwen3_w4a16_packed" / "manifest.json").read_text())
    manifest["source_model_dir"] = "packed_tiny"          # the temp dir name is not reproducible
    (OUT / "qwen3_w4a16_packed" / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n")

    model = QuantizedQwenForCausalLM(PackedTensorWeights(PackedInferenceStore(OUT / "qwen3_w4a16_packed")), CFG,
                                     compute_dtype=torch.float32).eval()
    prompt = torch.randint(0, v, (1, 12), generator=gen)
    logits, past = model(prompt)
    toks, gen_logits, last = [], [], logits[:, -1]
    for _ in range(6):
        nxt = torch.argmax(last, dim=-1)
        toks.append(int(nxt))
        gen_logits.append(last[0].clone())
        lg, past = model(nxt.view(1, 1), past)
        last = lg[:, -1]
    # gen_logits[i]: the logits greedy token i was picked from (teacher-forced checks)
    np.savez_compressed(HERE / "packed_tiny.npz", prompt=prompt.numpy(), logits=logits[0].numpy(),
                        greedy=np.array(toks, dtype=np.int64), gen_logits=torch.stack(gen_logits).numpy())
    print("wrote", OUT, "and packed_tiny.npz;", len(toks), "greedy tokens:", toks)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_packed_artifact.py <reference root>")
    main(sys.argv[1])

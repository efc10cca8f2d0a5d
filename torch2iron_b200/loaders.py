"""Weight loaders: the reference's on-disk formats into this engine's model dict.

Three sources, each producing ``(QuantizedQwenConfig, model)`` where ``model``
has the layout ``synth.random_model`` returns (``layers`` of AutoGPTQ linears
and bf16 norms, bf16 ``embed`` / ``final_norm``, and ``lm_head`` = ``None``
(tied), a bf16 ``[V, H]`` tensor, or an ``AutoGPTQLinear`` for a W4A16 head):

* the packed inference artifact ``qwen3_w4a16_packed/`` (``manifest.json`` +
  ``weights.w4a16.bin``, format ``quantized_qwen3_w4a16_inference_v13``),
  written by ``write_packed_inference_artifact``
  (src/models/quantized_qwen3/packed_format.py:405-655) and read by
  ``PackedInferenceStore`` (:658-758).  Each linear's ``qparam`` segment is
  ``[N, K/2 + 2G]`` bytes: biased int4 (zero 8, low nibble = even k) then the
  bf16 scales of that row (``make_qparam``, :195-205).  The NPU tile streams
  (``gemm_w4_weight`` segments) are not read: the T2B layout is rebuilt from
  ``qparam`` on the GPU.  When the artifact carries a ``lm_head`` linear (the
  packer quantizes a dense or tied head, :583-648), it is loaded as a W4A16
  head, since that is what the reference runtime multiplies by
  (``model.py:410-414``);
* AutoGPTQ safetensors checkpoints (``config.json`` + ``model.safetensors``,
  or shards listed in ``model.safetensors.index.json``, as ``_load_safetensors``
  reads them, :71-85).  ``numerics="reference"`` reproduces what the reference
  runs after packing (scales rounded to bf16 by ``make_qparam``; a dense or
  tied head quantized like ``quantize_dense_to_biased_int4``, :384-402);
  ``numerics="checkpoint"`` keeps the checkpoint's fp16 scales and its bf16
  head;
* the fast Qwen3 artifact ``fast_qwen3_q4nx/`` (format
  ``fast_qwen3_q4nx_layer_v1``, ``fast_qwen3/fast_packed_format.py:178-300``):
  bf16 dense tensors and Q4NX group-32 linears (``Q4NXLinear``, bytes as
  stored), which the decode engine rearranges into its group-32 block
  layout at load (``weights.from_q4nx``).

The T2B meta word stores an fp16 scale, so a bf16 scale is accepted only when
fp16 holds it exactly (every bf16 value of magnitude >= 2**-17 does) or when
its group dequantizes to zeros whatever the scale; anything else raises.
Loading is host work done once; nothing here runs per token.
"""

from __future__ import annotations

import json
import sys
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from .config import QuantizedQwenConfig
from .synth import LINEAR_NAMES, AutoGPTQLinear

PACKED_FORMAT = "quantized_qwen3_w4a16_inference_v13"
PACKED_DIRNAME = "qwen3_w4a16_packed"
PACKED_MANIFEST = "manifest.json"
ZERO_BIAS = 8
_SYM_QZERO_WORD = 0x77777777          # eight stored zeros of 7 (= 8 under the AutoGPTQ-v1 "+1" rule)

_ATTN = ("q_proj", "k_proj", "v_proj", "o_proj")


def _linear_prefix(li: int, name: str) -> str:
    return f"model.layers.{li}.{'self_attn' if name in _ATTN else 'mlp'}.{name}"


# ---------------------------------------------------------------------------
# config
# ---------------------------------------------------------------------------
def check_quantization(hf_config: dict) -> int:
    """Bits / symmetry checks of the reference (``model.py:370-376``,
    ``packed_format.py:415-421``); returns the group size."""
    q = hf_config.get("quantization_config") or {}
    bits = int(q.get("bits", 4))
    if bits != 4:
        raise ValueError(f"only W4A16 checkpoints are supported, got bits={bits}")
    if not bool(q.get("sym", True)):
        raise ValueError("only symmetric AutoGPTQ W4A16 checkpoints are supported")
    return int(q.get("group_size", 128))


def config_from_hf(hf_config: dict, *, qk_norm: bool = True, tie_word_embeddings: bool = True) -> QuantizedQwenConfig:
    """``QuantizedQwenConfig`` from a Hugging Face ``config.json`` dict, with the
    defaults of ``QuantizedQwenForCausalLM.__init__`` (``model.py:378-393``)."""
    group = check_quantization(hf_config)
    h, nq = int(hf_config["hidden_size"]), int(hf_config["num_attention_heads"])
    rope = (hf_config.get("rope_parameters") or {}).get("rope_theta", hf_config.get("rope_theta", 1000000.0))
    return QuantizedQwenConfig(
        vocab_size=int(hf_config["vocab_size"]), emb_dim=h, n_layers=int(hf_config["num_hidden_layers"]),
        n_heads=nq, n_kv_groups=int(hf_config["num_key_value_heads"]),
        head_dim=int(hf_config.get("head_dim") or h // nq), hidden_dim=int(hf_config["intermediate_size"]),
        rms_norm_eps=float(hf_config.get("rms_norm_eps", 1e-6)), rope_base=float(rope),
        context_length=int(hf_config.get("max_position_embeddings", 40960)),
        eos_token_id=hf_config.get("eos_token_id"), bos_token_id=hf_config.get("bos_token_id"),
        group_size=group, qk_norm=qk_norm, tie_word_embeddings=tie_word_embeddings)


# ---------------------------------------------------------------------------
# qparam rows <-> AutoGPTQ tensors
# ---------------------------------------------------------------------------
def _scales_to_f16(scales: torch.Tensor, zero_groups: torch.Tensor | None, what: str) -> torch.Tensor:
    """bf16 / fp32 scales -> fp16, exact or raising (groups in ``zero_groups`` may round)."""
    f32 = scales.to(torch.float32)
    f16 = f32.to(torch.float16)
    bad = f16.to(torch.float32) != f32
    if zero_groups is not None:
        bad &= ~zero_groups
    if bool(bad.any()):
        i = tuple(int(v) for v in bad.nonzero()[0])
        raise ValueError(f"{what}: scale {float(f32[i])!r} at {i} has no exact fp16 value "
                         "(the T2B layout stores fp16 scales)")
    return f16


def qparam_to_autogptq(qparam: torch.Tensor, in_features: int, out_features: int,
                       group_size: int = 128, what: str = "qparam") -> AutoGPTQLinear:
    """One ``qparam`` segment (uint8 ``[N, K/2 + 2G]``) -> ``AutoGPTQLinear``.

    The biased nibbles are already AutoGPTQ's unsigned q with zero 8: four
    consecutive row bytes hold k = 8w..8w+7 in nibble order, i.e. the
    little-endian int32 word ``qweight[w, n]``.
    """
    n, k, g = out_features, in_features, group_size
    if k % 8 or k % g or n % 8:
        raise ValueError(f"{what}: shape [{n}, {k}] is not a multiple of 8 / the group size {g}")
    groups = k // g
    if tuple(qparam.shape) != (n, k // 2 + 2 * groups) or qparam.dtype != torch.uint8:
        raise ValueError(f"{what}: qparam is {tuple(qparam.shape)} {qparam.dtype}, "
                         f"expected ({n}, {k // 2 + 2 * groups}) uint8")
    if sys.byteorder != "little":
        raise RuntimeError("qparam rows are read as little-endian int32 words")
    packed = qparam[:, :k // 2].contiguous()
    qweight = packed.view(torch.int32).t().contiguous()                           # [K/8, N]
    scales_bf16 = qparam[:, k // 2:].contiguous().view(torch.bfloat16)           # [N, G]
    lo, hi = packed & 0xF, packed >> 4
    centred = ((lo == ZERO_BIAS) & (hi == ZERO_BIAS)).view(n, groups, g // 2).all(dim=-1)
    scales = _scales_to_f16(scales_bf16, centred, what)
    qzeros = torch.full((groups, n // 8), _SYM_QZERO_WORD, dtype=torch.int32)
    return AutoGPTQLinear(qweight, qzeros, scales.t().contiguous(), k, n, g)


def quantize_head_w4(weight: torch.Tensor, group_size: int = 128) -> AutoGPTQLinear:
    """Symmetric RTN int4 of a dense head ``[V, H]`` as the reference packer does it
    (``quantize_dense_to_biased_int4``, packed_format.py:384-402): per group
    ``s = max(|w|, 1e-8) / 7`` in fp32, ``q = clamp(round(w / s), -8, 7)``,
    stored scale ``bf16(s)``; returned with zero 8 (stored 7) and fp16 scales."""
    w = weight.detach().to("cpu", torch.float32)
    v, h = w.shape
    if h % group_size:
        raise ValueError(f"head width {h} is not a multiple of the group size {group_size}")
    wg = w.view(v, h // group_size, group_size)
    s = wg.abs().amax(dim=-1).clamp(min=1e-8) / 7.0
    q = torch.round(wg / s[..., None]).clamp(-8, 7).to(torch.int32) + ZERO_BIAS
    nib = q.view(v, h).to(torch.uint8)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).contiguous()
    qparam = torch.cat([packed, s.to(torch.bfloat16).contiguous().view(torch.uint8)], dim=1)
    return qparam_to_autogptq(qparam, h, v, group_size, what="lm_head (quantized from a dense head)")


def round_scales_bf16(lin: AutoGPTQLinear) -> AutoGPTQLinear:
    """The scale rounding of ``make_qparam`` (fp16 -> bf16), back in fp16."""
    s = lin.scales.to(torch.bfloat16)
    return AutoGPTQLinear(lin.qweight, lin.qzeros, _scales_to_f16(s, None, "scales"), lin.in_features,
                          lin.out_features, lin.group_size)


# ---------------------------------------------------------------------------
# packed artifact
# ---------------------------------------------------------------------------
def _supported_manifest(path: Path) -> bool:
    try:
        return json.loads(path.read_text()).get("format") == PACKED_FORMAT
    except (OSError, ValueError):
        return False


def find_packed_dir(path: str | Path) -> Path | None:
    """The artifact directory for ``path`` (itself, ``path/qwen3_w4a16_packed``,
    else the newest supported manifest below it), as ``find_packed_dir`` of
    packed_format.py:56-69 resolves it; ``None`` when there is none."""
    path = Path(path).expanduser().resolve()
    for cand in (path, path / PACKED_DIRNAME):
        if _supported_manifest(cand / PACKED_MANIFEST):
            return cand
    if not path.is_dir():
        return None
    found = [m.parent for m in path.rglob(PACKED_MANIFEST) if _supported_manifest(m)]
    found.sort(key=lambda d: (d / PACKED_MANIFEST).stat().st_mtime, reverse=True)
    return found[0] if found else None


class PackedArtifact:
    """Read-only view of one packed artifact (``PackedInferenceStore``, packed_format.py:658-758)."""

    def __init__(self, packed_dir: str | Path):
        self.dir = Path(packed_dir).expanduser().resolve()
        mpath = self.dir / PACKED_MANIFEST
        if not mpath.exists():
            raise FileNotFoundError(f"missing packed manifest: {mpath}")
        self.manifest = json.loads(mpath.read_text())
        fmt = self.manifest.get("format")
        if fmt != PACKED_FORMAT:
            raise RuntimeError(f"unsupported packed format {fmt!r}; expected {PACKED_FORMAT!r}")
        self.data_path = self.dir / self.manifest["data_file"]
        self._data = np.memmap(self.data_path, dtype=np.uint8, mode="r")

    def _bytes(self, seg: dict) -> np.ndarray:
        off, n = int(seg["byte_offset"]), int(seg["byte_length"])
        if off < 0 or off + n > self._data.size:
            raise ValueError(f"segment {seg.get('name')!r} [{off}, {off + n}) lies outside "
                             f"{self.data_path.name} ({self._data.size} bytes)")
        return self._data[off:off + n]

    def has_dense(self, name: str) -> bool:
        return name in self.manifest.get("dense", {})

    def has_linear(self, prefix: str) -> bool:
        return prefix in self.manifest.get("linears", {})

    def dense(self, name: str) -> torch.Tensor:
        """A bf16 dense tensor (copied out of the mapping)."""
        try:
            seg = self.manifest["dense"][name]
        except KeyError as exc:
            raise KeyError(f"missing dense tensor {name!r} in packed store") from exc
        if seg.get("dtype") != "bfloat16":
            raise ValueError(f"dense tensor {name!r} has dtype {seg.get('dtype')!r}, expected bfloat16")
        shape = tuple(int(d) for d in seg["shape"])
        raw = np.array(self._bytes(seg)).view(np.uint16)
        if raw.size != int(np.prod(shape)):
            raise ValueError(f"dense tensor {name!r}: {raw.size} values for shape {shape}")
        return torch.from_numpy(raw.reshape(shape)).view(torch.bfloat16)

    def qparam(self, prefix: str) -> tuple[dict, torch.Tensor]:
        """``(spec, uint8 [N, K/2 + 2G])`` of one linear."""
        try:
            spec = self.manifest["linears"][prefix]
        except KeyError as exc:
            raise KeyError(f"missing packed linear {prefix!r}") from exc
        seg = spec["qparam"]
        shape = tuple(int(d) for d in seg["shape"])
        raw = np.array(self._bytes(seg))
        if raw.size != shape[0] * shape[1]:
            raise ValueError(f"linear {prefix!r}: {raw.size} qparam bytes for shape {shape}")
        return spec, torch.from_numpy(raw.reshape(shape))

    def linear(self, prefix: str) -> AutoGPTQLinear:
        spec, qp = self.qparam(prefix)
        if int(spec.get("zero_bias", ZERO_BIAS)) != ZERO_BIAS:
            raise ValueError(f"linear {prefix!r}: zero_bias {spec['zero_bias']} (expected {ZERO_BIAS})")
        return qparam_to_autogptq(qp, int(spec["in_features"]), int(spec["out_features"]),
                                  int(spec["group_size"]), what=prefix)


def _hf_config_near(packed_dir: Path) -> dict:
    for cand in (packed_dir / "config.json", packed_dir.parent / "config.json"):
        if cand.exists():
            return json.loads(cand.read_text())
    raise FileNotFoundError(f"no config.json beside {packed_dir}; pass hf_config")


def _model_from(get_linear, get_dense, has_dense, n_layers: int) -> tuple[list, bool]:
    layers = []
    qk_norm = has_dense("model.layers.0.self_attn.q_norm.weight")
    for li in range(n_layers):
        p = f"model.layers.{li}"
        layer = {name: get_linear(_linear_prefix(li, name)) for name in LINEAR_NAMES}
        layer["input_layernorm"] = get_dense(f"{p}.input_layernorm.weight")
        layer["post_attention_layernorm"] = get_dense(f"{p}.post_attention_layernorm.weight")
        if qk_norm:
            layer["q_norm"] = get_dense(f"{p}.self_attn.q_norm.weight")
            layer["k_norm"] = get_dense(f"{p}.self_attn.k_norm.weight")
        layers.append(layer)
    return layers, qk_norm


def _check_shapes(cfg: QuantizedQwenConfig, model: dict) -> None:
    from .synth import linear_shapes
    want = linear_shapes(cfg)
    for li, layer in enumerate(model["layers"]):
        for name, (o, i) in want.items():
            lin = layer[name]
            if (lin.out_features, lin.in_features) != (o, i):
                raise ValueError(f"layer {li} {name}: [{lin.out_features}, {lin.in_features}] "
                                 f"does not match the config's [{o}, {i}]")
    if tuple(model["embed"].shape) != (cfg.vocab_size, cfg.emb_dim):
        raise ValueError(f"embedding {tuple(model['embed'].shape)} does not match the config")


def load_packed_artifact(path: str | Path, hf_config: dict | None = None) -> tuple[QuantizedQwenConfig, dict]:
    """Load a ``qwen3_w4a16_packed`` artifact (or a model dir holding one).

    ``hf_config`` defaults to the ``config.json`` beside the artifact (the
    model directory it was packed from); the manifest's ``model_config``
    must agree with it.
    """
    pdir = find_packed_dir(path)
    if pdir is None:
        raise FileNotFoundError(f"no {PACKED_FORMAT} artifact under {path}")
    art = PackedArtifact(pdir)
    hf = dict(hf_config) if hf_config is not None else _hf_config_near(pdir)
    for key, val in art.manifest.get("model_config", {}).items():
        if val is not None and key in hf and hf[key] is not None and int(hf[key]) != int(val):
            raise ValueError(f"manifest model_config {key}={val} disagrees with config.json ({hf[key]})")
    n_layers = int(hf["num_hidden_layers"])
    layers, qk_norm = _model_from(art.linear, art.dense, art.has_dense, n_layers)
    if art.has_linear("lm_head"):
        lm_head = art.linear("lm_head")
    elif art.has_dense("lm_head.weight"):
        lm_head = art.dense("lm_head.weight")
    else:
        lm_head = None
    model = {"layers": layers, "embed": art.dense("model.embed_tokens.weight"),
             "final_norm": art.dense("model.norm.weight"), "lm_head": lm_head}
    cfg = config_from_hf(hf, qk_norm=qk_norm, tie_word_embeddings=lm_head is None)
    _check_shapes(cfg, model)
    return cfg, model


# ---------------------------------------------------------------------------
# AutoGPTQ safetensors checkpoint
# ---------------------------------------------------------------------------
def load_safetensors_dir(model_dir: str | Path) -> dict[str, torch.Tensor]:
    """All tensors of ``model.safetensors`` or of the shards its index lists."""
    from safetensors.torch import load_file
    d = Path(model_dir)
    single = d / "model.safetensors"
    if single.exists():
        return load_file(str(single))
    index = d / "model.safetensors.index.json"
    if not index.exists():
        raise FileNotFoundError(f"missing safetensors file in {d}")
    out: dict[str, torch.Tensor] = {}
    for fname in sorted(set(json.loads(index.read_text())["weight_map"].values())):
        out.update(load_file(str(d / fname)))
    return out


def autogptq_linear(tensors: dict, prefix: str, group_size: int) -> AutoGPTQLinear:
    """``qweight [K/8, N]`` / ``qzeros [G, N/8]`` / ``scales [G, N]`` of one linear.

    A ``g_idx`` other than ``k // group_size`` (act-order checkpoints) is
    rejected: the T2B layout keeps groups contiguous along K.
    """
    qweight = tensors[f"{prefix}.qweight"].to(torch.int32)
    qzeros = tensors[f"{prefix}.qzeros"].to(torch.int32)
    scales = tensors[f"{prefix}.scales"]
    k, n = qweight.shape[0] * 8, qweight.shape[1]
    groups = -(-k // group_size)
    if tuple(qzeros.shape) != (groups, n // 8) or tuple(scales.shape) != (groups, n):
        raise ValueError(f"{prefix}: qzeros {tuple(qzeros.shape)} / scales {tuple(scales.shape)} "
                         f"do not fit qweight {tuple(qweight.shape)} with group size {group_size}")
    g_idx = tensors.get(f"{prefix}.g_idx")
    if g_idx is not None and not torch.equal(g_idx.to(torch.int64), torch.arange(k) // group_size):
        raise ValueError(f"{prefix}: act-order g_idx is not supported (groups must be contiguous along K)")
    if scales.dtype != torch.float16:
        scales = _scales_to_f16(scales, None, f"{prefix}.scales")
    return AutoGPTQLinear(qweight.contiguous(), qzeros.contiguous(), scales.contiguous(), k, n, group_size)


def load_autogptq_checkpoint(model_dir: str | Path, numerics: str = "reference") -> tuple[QuantizedQwenConfig, dict]:
    """Load a symmetric AutoGPTQ W4A16 checkpoint directory.

    ``numerics="reference"``: the weights the reference multiplies by after
    packing the same checkpoint (bf16-rounded scales; a quantized head
    when the checkpoint has none).  ``numerics="checkpoint"``: the stored
    fp16 scales and a bf16 head (tied to the embedding when absent).
    """
    if numerics not in ("reference", "checkpoint"):
        raise ValueError(f"numerics must be 'reference' or 'checkpoint', got {numerics!r}")
    d = Path(model_dir).expanduser()
    hf = json.loads((d / "config.json").read_text())
    group = check_quantization(hf)
    t = load_safetensors_dir(d)
    ref = numerics == "reference"

    def linear(prefix):
        lin = autogptq_linear(t, prefix, group)
        return round_scales_bf16(lin) if ref else lin

    def dense(name):
        if name not in t:
            raise KeyError(f"missing dense tensor {name!r} in {d}")
        return t[name].to(torch.bfloat16).contiguous()

    layers, qk_norm = _model_from(linear, dense, lambda n: n in t, int(hf["num_hidden_layers"]))
    embed = dense("model.embed_tokens.weight")
    if "lm_head.qweight" in t:
        lm_head = linear("lm_head")
    elif ref:
        lm_head = quantize_head_w4(dense("lm_head.weight") if "lm_head.weight" in t else embed, group)
    else:
        lm_head = dense("lm_head.weight") if "lm_head.weight" in t else None
    model = {"layers": layers, "embed": embed, "final_norm": dense("model.norm.weight"), "lm_head": lm_head}
    cfg = config_from_hf(hf, qk_norm=qk_norm, tie_word_embeddings=lm_head is None)
    _check_shapes(cfg, model)
    return cfg, model


# ---------------------------------------------------------------------------
# fast Qwen3 artifact (Q4NX group-32 weights)
# ---------------------------------------------------------------------------
FAST_FORMAT = "fast_qwen3_q4nx_layer_v1"
FAST_DIRNAME = "fast_qwen3_q4nx"
Q4NX_CHUNK_BYTES = 5120   # 32 rows x 256 k: 256 bf16 scales, 256 bf16 zero points, 4096 bytes of 4-bit values


@dataclass
class Q4NXLinear:
    """One linear of the fast Qwen3 artifact as stored: output rows padded to
    64-row patches, each patch K-chunk-major as pairs of 32-row x 256-k chunks,
    a chunk = bf16 scales and bf16 zero points per 32 k, then two 4-bit values
    per byte (low nibble = even k); ``w = (q - zero) * scale``
    (``fast_qwen3/q4nx_layout.py:14-38,115-237``).  ``data`` is uint8."""

    data: torch.Tensor
    in_features: int
    out_features: int
    padded_out_features: int
    group_size: int = 32

    @property
    def n_chunks(self) -> int:
        return self.padded_out_features // 32 * (self.in_features // 256)


def find_fast_dir(path: str | Path) -> Path | None:
    """The fast artifact directory for ``path`` (itself, ``path/fast_qwen3_q4nx``,
    else the newest fast manifest below it), as ``find_fast_dir`` of
    fast_packed_format.py:45-62 resolves it."""
    def ok(m: Path) -> bool:
        try:
            return json.loads(m.read_text()).get("format") == FAST_FORMAT
        except (OSError, ValueError):
            return False

    path = Path(path).expanduser().resolve()
    for cand in (path, path / FAST_DIRNAME):
        if ok(cand / PACKED_MANIFEST):
            return cand
    if not path.is_dir():
        return None
    found = [m.parent for m in path.rglob(PACKED_MANIFEST) if ok(m)]
    found.sort(key=lambda d: (d / PACKED_MANIFEST).stat().st_mtime, reverse=True)
    return found[0] if found else None


class FastArtifact(PackedArtifact):
    """Read-only view of a fast Qwen3 artifact (``FastQwen3Store``,
    fast_packed_format.py:265-300): bf16 dense tensors and Q4NX linears."""

    FORMAT = FAST_FORMAT

    def __init__(self, fast_dir: str | Path):
        self.dir = Path(fast_dir).expanduser().resolve()
        mpath = self.dir / PACKED_MANIFEST
        if not mpath.exists():
            raise FileNotFoundError(f"missing fast Qwen3 manifest: {mpath}")
        self.manifest = json.loads(mpath.read_text())
        if self.manifest.get("format") != FAST_FORMAT:
            raise RuntimeError(f"unsupported fast Qwen3 format {self.manifest.get('format')!r}")
        self.data_path = self.dir / self.manifest["data_file"]
        self._data = np.memmap(self.data_path, dtype=np.uint8, mode="r")

    def linear(self, prefix: str) -> Q4NXLinear:
        try:
            e = self.manifest["linears"][prefix]
        except KeyError as exc:
            raise KeyError(f"missing Q4NX linear {prefix!r}") from exc
        if int(e["group_size"]) != 32 or int(e["in_chunk"]) != 256 or int(e["out_chunk"]) != 32:
            raise ValueError(f"{prefix}: not the Q4NX group-32 layout")
        lin = Q4NXLinear(torch.empty(0, dtype=torch.uint8), int(e["in_features"]), int(e["out_features"]),
                         int(e["padded_out_features"]))
        want = lin.n_chunks * Q4NX_CHUNK_BYTES
        if int(e["byte_length"]) != want:
            raise ValueError(f"{prefix}: {e['byte_length']} bytes, the layout needs {want}")
        lin.data = torch.from_numpy(np.array(self._bytes({"name": prefix, **e})))
        return lin


def load_fast_qwen3_artifact(path: str | Path, hf_config: dict | None = None) -> tuple[QuantizedQwenConfig, dict]:
    """Load a ``fast_qwen3_q4nx`` artifact (or a model dir holding one): dense
    tensors as bf16, the linears as ``Q4NXLinear`` (run by the decode engine
    in the group-32 variant of its block layout, ``WFMT_Q4NX``)."""
    fdir = find_fast_dir(path)
    if fdir is None:
        raise FileNotFoundError(f"no {FAST_FORMAT} artifact under {path}")
    art = FastArtifact(fdir)
    hf = dict(hf_config) if hf_config is not None else _hf_config_near(fdir)
    for key, val in art.manifest.get("model_config", {}).items():
        if val is not None and key in hf and hf[key] is not None and float(hf[key]) != float(val):
            raise ValueError(f"manifest model_config {key}={val} disagrees with config.json ({hf[key]})")
    layers, qk_norm = _model_from(art.linear, art.dense, art.has_dense, int(hf["num_hidden_layers"]))
    if art.has_linear("lm_head"):
        lm_head = art.linear("lm_head")
    elif art.has_dense("lm_head.weight"):
        lm_head = art.dense("lm_head.weight")
    else:
        lm_head = None
    model = {"layers": layers, "embed": art.dense("model.embed_tokens.weight"),
             "final_norm": art.dense("model.norm.weight"), "lm_head": lm_head}
    cfg = config_from_hf(hf, qk_norm=qk_norm, tie_word_embeddings=lm_head is None)
    _check_shapes(cfg, model)
    return cfg, model


def load_model(path: str | Path, hf_config: dict | None = None) -> tuple[QuantizedQwenConfig, dict]:
    """The packed artifact under ``path`` when there is one, as
    ``QuantizedQwenForCausalLM.from_pretrained`` loads it (model.py:425-449).
    Where that raises for a checkpoint that was never packed, this loads the
    AutoGPTQ checkpoint with the numerics its packing would give."""
    if find_packed_dir(path) is not None:
        return load_packed_artifact(path, hf_config)
    return load_autogptq_checkpoint(path)

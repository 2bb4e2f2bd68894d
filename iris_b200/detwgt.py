"""Model bundles in the reference's `.detwgt` v3 format, loaded onto the device.

Both families: mistral-dense (below) and gemma-dense (`gemma_config`,
`load_gemma_bundle`: the shape of crates/model/import/src/gemma.rs:126-190,
the tensor names of gemma.rs:620-660, per-layer `layer_scalar` values, the
untied head when `tie_word_embeddings` is false). `load_bundle` picks the
family from the config (a per-layer input width makes it gemma-dense).

A bundle directory holds `model.detwgt` (the tensors) and `config.json` (the
Hugging Face text config). This module reads the file format
(crates/model/detwgt/src/write.rs:15-124: magic "DNWGTV0\\0", format version
3, det-num spec version 1, tensor count; per tensor its name, dims, element
count, element width — 16 or 32 for Q16.16 values stored as i16 / i32, 8 for
Q8_0 blocks kept exactly as GGUF stores them — payload length, row mass,
then the payload at the next 64-byte file offset), derives the mistral-dense
shape from the config as the importer does
(crates/model/import/src/mistral.rs:200-287: YaRN inverse frequencies from
`rope_parameters`, positions capped at `original_max_position_embeddings`
when `llama_4_scaling_beta` is set, since the query scaling past that point
is not built), and maps the tensor names onto the device model's tensor
kinds. The file is memory-mapped; Q8_0 payloads go to the device as raw
blocks (`iris_model_set_q8` repacks them into the tiled layout there).
"""
from __future__ import annotations

import json
import math
import mmap
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, List, Tuple

import numpy as np

from .shapes import GemmaConfig, MistralConfig, f32_to_acc

MAGIC = b"DNWGTV0\0"
VERSION = 3
SPEC_VERSION = 1
Q8_0_WIDTH = 8
ALIGNMENT = 64
BLOCK_BYTES = 34


@dataclass
class TensorEntry:
    name: str
    dims: List[int]
    width: int    # 16, 32 (Q16.16 values) or Q8_0_WIDTH (blocks)
    length: int   # payload bytes
    mass: int     # the writer's largest row sum of |value| (informational)
    offset: int   # payload's file offset


class Detwgt:
    """A memory-mapped `.detwgt` file: its tensor table and payload views."""

    def __init__(self, path):
        self.path = Path(path)
        with open(self.path, "rb") as f:
            self._map = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        self.tensors: Dict[str, TensorEntry] = {}
        buf = self._map
        if len(buf) < 24 or buf[:8] != MAGIC:
            raise ValueError(f"{self.path}: not a detwgt file")
        version, spec, count = struct.unpack_from("<IIQ", buf, 8)
        if version != VERSION or spec != SPEC_VERSION:
            raise ValueError(f"{self.path}: detwgt version {version} / spec {spec}, expected {VERSION} / {SPEC_VERSION}")
        off = 24
        for _ in range(count):
            (nlen,) = struct.unpack_from("<I", buf, off)
            name = bytes(buf[off + 4:off + 4 + nlen]).decode()
            off += 4 + nlen
            (ndims,) = struct.unpack_from("<I", buf, off)
            dims = list(struct.unpack_from(f"<{ndims}Q", buf, off + 4))
            off += 4 + 8 * ndims
            numel, width, length, mass = struct.unpack_from("<QIQQ", buf, off)
            off += 28
            off += (ALIGNMENT - off % ALIGNMENT) % ALIGNMENT
            if numel != math.prod(dims):
                raise ValueError(f"tensor {name!r}: {numel} elements for dims {dims}")
            if width in (16, 32):
                want = numel * width // 8
            elif width == Q8_0_WIDTH:
                cols = dims[-1] if dims else 0
                if cols == 0 or cols % 32:
                    raise ValueError(f"Q8_0 tensor {name!r}: rows are not whole blocks")
                want = numel // 32 * BLOCK_BYTES
            else:
                raise ValueError(f"tensor {name!r}: element width {width}")
            if length != want or off + length > len(buf):
                raise ValueError(f"tensor {name!r}: payload of {length} bytes, expected {want}")
            if name in self.tensors:
                raise ValueError(f"tensor {name!r} appears twice")
            self.tensors[name] = TensorEntry(name, dims, width, length, mass, off)
            off += length

    def is_q8(self, name: str) -> bool:
        return self.tensors[name].width == Q8_0_WIDTH

    def values(self, name: str) -> np.ndarray:
        """A Q16.16 tensor as int32 values (flattened)."""
        t = self.tensors[name]
        if t.width == Q8_0_WIDTH:
            raise ValueError(f"tensor {name!r} holds Q8_0 blocks, not values")
        dtype = "<i2" if t.width == 16 else "<i4"
        return np.frombuffer(self._map, dtype=dtype, count=math.prod(t.dims), offset=t.offset).astype(np.int32)

    def q8_blocks(self, name: str) -> np.ndarray:
        """A Q8_0 tensor's raw 34-byte blocks (a read-only view of the file)."""
        t = self.tensors[name]
        if t.width != Q8_0_WIDTH:
            raise ValueError(f"tensor {name!r} holds values, not Q8_0 blocks")
        return np.frombuffer(self._map, dtype=np.uint8, count=t.length, offset=t.offset)

    def close(self) -> None:
        """Unmaps the file, unless views of it are still alive (then the
        mapping goes with the last of them)."""
        try:
            self._map.close()
        except BufferError:
            pass


def _correction_dim(dims: float, original: float, rotations: float, base: float) -> float:
    return dims * math.log(original / (rotations * 2.0 * math.pi)) / (2.0 * math.log(base))


def _settled(v: float) -> float:
    if abs(v - round(v)) < 1e-6:
        raise ValueError(f"a YaRN bound of {v} is too close to a whole number")
    return v


def mistral_config(config: dict, name: str = "bundle") -> MistralConfig:
    """The mistral-dense shape of a config.json (mistral.rs:200-287 restated)."""
    text = config.get("text_config", config)
    if text.get("hidden_act") != "silu":
        raise ValueError("a mistral-dense model's hidden_act must be silu")
    if text.get("sliding_window") is not None:
        raise ValueError("a mistral-dense model has no sliding window")
    rope = text["rope_parameters"]
    if rope.get("rope_type") != "yarn":
        raise ValueError("a mistral-dense model's rope_type must be yarn")
    for key in ("mscale", "mscale_all_dim"):
        if float(rope[key]) != 1.0:
            raise ValueError(f"rope_parameters.{key} must be 1")
    head_dim = int(text["head_dim"])
    base, factor = float(rope["rope_theta"]), float(rope["factor"])
    original = float(rope["original_max_position_embeddings"])
    if base % 1 or factor % 1 or original % 1:
        raise ValueError("rope_theta, factor and original_max_position_embeddings must be whole")
    low = max(math.floor(_settled(_correction_dim(head_dim, original, float(rope["beta_fast"]), base))), 0)
    high = min(math.ceil(_settled(_correction_dim(head_dim, original, float(rope["beta_slow"]), base))), head_dim - 1)
    beta = rope.get("llama_4_scaling_beta")
    max_positions = int(original) if beta not in (None, 0, 0.0) else int(text["max_position_embeddings"])
    cfg = MistralConfig(name, layers=int(text["num_hidden_layers"]), hidden=int(text["hidden_size"]),
                        ffn=int(text["intermediate_size"]), heads=int(text["num_attention_heads"]),
                        kv_heads=int(text["num_key_value_heads"]), head_dim=head_dim,
                        vocab=int(text["vocab_size"]), rope_base=int(base), max_positions=max_positions,
                        eps=float(text["rms_norm_eps"]), tied=bool(text.get("tie_word_embeddings", False)),
                        yarn=(int(factor), int(low), int(high)))
    if cfg.freqs is None:
        raise ValueError("the model's rotation needs head_dim / 2 to be a power of two")
    return cfg


# Hugging Face tensor names of a mistral-dense model -> (kind, layer)
_PREFIX = "model.language_model."
_LAYER = {
    "self_attn.q_proj.weight": "W_Q", "self_attn.k_proj.weight": "W_K", "self_attn.v_proj.weight": "W_V",
    "self_attn.o_proj.weight": "W_O", "mlp.gate_proj.weight": "W_GATE", "mlp.up_proj.weight": "W_UP",
    "mlp.down_proj.weight": "W_DOWN", "input_layernorm.weight": "NORM_ATTN",
    "pre_feedforward_layernorm.weight": "NORM_FFN", "post_attention_layernorm.weight": "NORM_FFN",
}


def mistral_tensor_names(cfg: MistralConfig) -> Dict[Tuple[str, int], List[str]]:
    """Candidate file names of every tensor the device model takes."""
    out = {("EMBED", -1): [_PREFIX + "embed_tokens.weight"], ("FINAL_NORM", -1): [_PREFIX + "norm.weight"]}
    if not cfg.tied:
        out[("HEAD", -1)] = ["lm_head.weight", _PREFIX + "lm_head.weight"]
    for l in range(cfg.layers):
        for suffix, kind in _LAYER.items():
            out.setdefault((kind, l), []).append(f"{_PREFIX}layers.{l}.{suffix}")
    return out


def load_mistral_bundle(bundle) -> Tuple[MistralConfig, Dict[Tuple[str, int], np.ndarray], Detwgt]:
    """(shape, host tensors keyed as the device model's, the open file) of a
    mistral-dense bundle directory. The Q8_0 arrays are views of the mapped
    file: keep the Detwgt open while they are used."""
    bundle = Path(bundle)
    cfg = mistral_config(json.loads((bundle / "config.json").read_text()), bundle.name)
    f = Detwgt(bundle / "model.detwgt")
    from .model import tensor_table
    table = tensor_table(cfg)
    weights = {}
    for key, names in mistral_tensor_names(cfg).items():
        if key not in table:
            continue
        found = [n for n in names if n in f.tensors]
        if not found:
            raise ValueError(f"{bundle}: no tensor for {key} (looked for {names})")
        kind, rows, cols, _ = table[key]
        name = found[0]
        entry = f.tensors[name]
        if math.prod(entry.dims) != rows * cols or entry.dims[-1] != cols:
            raise ValueError(f"tensor {name!r}: dims {entry.dims}, expected [{rows}, {cols}]")
        if kind == "q8":
            weights[key] = f.q8_blocks(name)
        else:
            weights[key] = f.values(name)
    return cfg, weights, f


def open_mistral_bundle(bundle):
    """A DeviceModel holding a mistral-dense bundle's weights (uploaded as the
    file holds them; the mapping is closed afterwards)."""
    from .model import DeviceModel
    cfg, weights, f = load_mistral_bundle(bundle)
    try:
        return DeviceModel(cfg, weights=weights)
    finally:
        del weights
        f.close()


# ---- gemma-dense ----------------------------------------------------------

def _rope_param(text: dict, attention_type: str, key: str):
    """gemma.rs:21-26: rope_parameters.<attention_type>.<key>."""
    v = (text.get("rope_parameters") or {}).get(attention_type) or {}
    return v.get(key)


def gemma_config(config: dict, ffn: int, layer_scalars: List[int], name: str = "bundle") -> GemmaConfig:
    """The gemma-dense shape of a config.json (gemma.rs:126-190 restated);
    the FFN width is the gate projection's rows and the layer scalars come
    from the layers' `layer_scalar` tensors, as the importer takes them."""
    text = config.get("text_config", config)
    need = lambda k: int(text[k])
    head_dim = need("head_dim")
    if text.get("global_head_dim") not in (None, head_dim):
        raise ValueError("full-attention layers with their own head width are not supported")
    layers = need("num_hidden_layers")
    types = list(text.get("layer_types") or [])
    if len(types) != layers:  # gemma.rs:61-67: a layer without a declared type is full attention
        types = (types + ["full_attention"] * layers)[:layers]
    sliding_base = _rope_param(text, "sliding_attention", "rope_theta") or text.get("rope_local_base_freq") or 10_000
    full_base = _rope_param(text, "full_attention", "rope_theta") or text.get("rope_theta") or 1_000_000
    partial = _rope_param(text, "full_attention", "partial_rotary_factor")
    for base in (sliding_base, full_base):
        if float(base) % 1:
            raise ValueError("RoPE bases must be whole numbers")
    cfg = GemmaConfig(name, layers=layers, hidden=need("hidden_size"), ffn=ffn, heads=need("num_attention_heads"),
                      kv_heads=need("num_key_value_heads"), head_dim=head_dim, vocab=need("vocab_size"),
                      ple_width=need("hidden_size_per_layer_input"),
                      sliding_window=int(text.get("sliding_window") or 0), layer_types=types,
                      num_kv_shared_layers=int(text.get("num_kv_shared_layers") or 0),
                      rope_base_sliding=int(sliding_base), rope_base_full=int(full_base),
                      partial_rotary=float(partial) if partial is not None else 1.0,
                      softcap=float(text.get("final_logit_softcapping") or 0.0),
                      eps=float(text.get("rms_norm_eps") if text.get("rms_norm_eps") is not None else 1e-6),
                      layer_scalars=list(layer_scalars), tied=bool(text.get("tie_word_embeddings", False)))
    if cfg.norm_eps != f32_to_acc(float(np.float32(cfg.eps))):
        raise ValueError("rms_norm_eps does not survive the f32 conversion")
    donors = {cfg.kv_donor(l) for l in range(layers)} - {-1}
    if len(donors) > 2:  # gemma.rs:402-409
        raise ValueError("at most two K/V donor layers are supported")
    return cfg


_GEMMA_LAYER = {
    "self_attn.q_proj.weight": "W_Q", "self_attn.k_proj.weight": "W_K", "self_attn.v_proj.weight": "W_V",
    "self_attn.o_proj.weight": "W_O", "mlp.gate_proj.weight": "W_GATE", "mlp.up_proj.weight": "W_UP",
    "mlp.down_proj.weight": "W_DOWN", "input_layernorm.weight": "NORM_ATTN",
    "post_attention_layernorm.weight": "NORM_POST_ATTN", "pre_feedforward_layernorm.weight": "NORM_FFN",
    "post_feedforward_layernorm.weight": "NORM_POST_FFW", "post_per_layer_input_norm.weight": "PLE_POST_NORM",
    "self_attn.q_norm.weight": "Q_NORM", "self_attn.k_norm.weight": "K_NORM",
    "per_layer_input_gate.weight": "PLE_INPUT_GATE", "per_layer_projection.weight": "PLE_LAYER_PROJECTION",
}
_GEMMA_MODEL = {
    "embed_tokens.weight": "EMBED", "norm.weight": "FINAL_NORM", "embed_tokens_per_layer.weight": "PLE_EMBED",
    "per_layer_model_projection.weight": "PLE_MODEL_PROJECTION", "per_layer_projection_norm.weight": "PLE_NORM",
    "lm_head.weight": "HEAD",
}


def gemma_tensor_names(layers: int) -> Dict[Tuple[str, int], List[str]]:
    """Candidate file names of every tensor a gemma-dense device model takes
    (a layer without v_proj uses k_proj as V, gemma.rs:424-431)."""
    out = {(kind, -1): [_PREFIX + n] for n, kind in _GEMMA_MODEL.items()}
    out[("HEAD", -1)].append("lm_head.weight")
    for l in range(layers):
        for suffix, kind in _GEMMA_LAYER.items():
            out.setdefault((kind, l), []).append(f"{_PREFIX}layers.{l}.{suffix}")
        out[("W_V", l)].append(f"{_PREFIX}layers.{l}.self_attn.k_proj.weight")
    return out


def _known_gemma_tensor(name: str, layers: int) -> bool:
    """gemma.rs:659-675: a language-model tensor the import reads."""
    if not name.startswith(_PREFIX):
        return True
    rest = name[len(_PREFIX):]
    if not rest.startswith("layers."):
        return rest in _GEMMA_MODEL
    idx, _, suffix = rest[len("layers."):].partition(".")
    return idx.isdigit() and int(idx) < layers and (suffix in _GEMMA_LAYER or suffix == "layer_scalar")


def load_gemma_bundle(bundle) -> Tuple[GemmaConfig, Dict[Tuple[str, int], np.ndarray], Detwgt]:
    """(shape, host tensors keyed as the device model's, the open file) of a
    gemma-dense bundle directory (Q8_0 arrays are views of the mapped file)."""
    bundle = Path(bundle)
    config = json.loads((bundle / "config.json").read_text())
    text = config.get("text_config", config)
    f = Detwgt(bundle / "model.detwgt")
    layers = int(text["num_hidden_layers"])
    unknown = [n for n in f.tensors if not _known_gemma_tensor(n, layers)]
    if unknown:  # gemma.rs:677-700
        raise ValueError(f"{bundle}: language-model weights a gemma-dense import does not read: {unknown[:5]}")
    gate = f.tensors.get(f"{_PREFIX}layers.0.mlp.gate_proj.weight")
    if gate is None:
        raise ValueError(f"{bundle}: no layer 0 gate projection")
    scalars = []
    for l in range(layers):
        t = f.tensors.get(f"{_PREFIX}layers.{l}.layer_scalar")
        scalars.append(int(f.values(t.name)[0]) if t is not None else 0)
    cfg = gemma_config(config, int(gate.dims[0]), scalars, bundle.name)
    from .model import tensor_table
    table = tensor_table(cfg)
    weights = {}
    for key, names in gemma_tensor_names(layers).items():
        if key not in table:
            continue
        found = [n for n in names if n in f.tensors]
        if not found:
            raise ValueError(f"{bundle}: no tensor for {key} (looked for {names})")
        kind, rows, cols, _ = table[key]
        name = found[0]
        entry = f.tensors[name]
        if math.prod(entry.dims) != rows * cols or entry.dims[-1] != cols:
            raise ValueError(f"tensor {name!r}: dims {entry.dims}, expected [{rows}, {cols}]")
        weights[key] = f.q8_blocks(name) if kind == "q8" else f.values(name)
    return cfg, weights, f


def load_bundle(bundle):
    """load_mistral_bundle or load_gemma_bundle, by the config's family."""
    config = json.loads((Path(bundle) / "config.json").read_text())
    text = config.get("text_config", config)
    return load_gemma_bundle(bundle) if "hidden_size_per_layer_input" in text else load_mistral_bundle(bundle)


def open_bundle(bundle):
    """A DeviceModel holding a bundle's weights (either family)."""
    from .model import DeviceModel
    cfg, weights, f = load_bundle(bundle)
    try:
        return DeviceModel(cfg, weights=weights)
    finally:
        del weights
        f.close()

"""Model bundles in the reference's `.detwgt` v3 format, loaded onto the device.

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

from .shapes import MistralConfig

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

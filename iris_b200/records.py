"""Canonical checkpoint records of the teacher-forced chain's stages.

The reference commits each stage's outputs through Raster encodings
(crates/inference/artifacts/src/checkpoint.rs:32-204,
crates/inference/staged/src/artifact_io.rs:46-58); the Raster crate is not
available to this build, so those commitments cannot be reproduced. This
module defines a documented substitute that pins the same content: a stage's
output rows and its own K/V rows, byte for byte, under SHA-256.

Record layout (all integers little-endian):

    b"IRISREC1"
    u32 len(stage), stage name (UTF-8)      e.g. "layer_mistral/3"
    u32 start_position, u32 rows, u32 width
    rows x width int32                      the stage's output activations
    u32 kv_width (0 when there are none)
    rows x kv_width int32 (K), then the same for V

`chain_records` runs a claim's teacher-forced pass stage by stage on the
device (`iris_mistral_layer_range` per range and layer, K/V carried across
ranges, mistral/stage.rs:172-226) and returns each stage's record digest.
"""
from __future__ import annotations

import hashlib
import struct
from typing import List, Optional, Sequence, Tuple

import numpy as np

MAGIC = b"IRISREC1"


def stage_record(stage: str, start: int, rows: np.ndarray, k: Optional[np.ndarray] = None,
                 v: Optional[np.ndarray] = None) -> bytes:
    rows = np.ascontiguousarray(rows, "<i4")
    if rows.ndim != 2:
        raise ValueError("rows must be [n][width]")
    name = stage.encode()
    out = [MAGIC, struct.pack("<I", len(name)), name, struct.pack("<III", start, rows.shape[0], rows.shape[1]),
           rows.tobytes()]
    if k is None:
        out.append(struct.pack("<I", 0))
    else:
        k = np.ascontiguousarray(k, "<i4")
        v = np.ascontiguousarray(v, "<i4")
        if k.shape != v.shape or k.shape[0] != rows.shape[0]:
            raise ValueError("K and V must hold one row per output row")
        out += [struct.pack("<I", k.shape[1]), k.tobytes(), v.tobytes()]
    return b"".join(out)


def stage_digest(stage: str, start: int, rows: np.ndarray, k=None, v=None) -> str:
    return hashlib.sha256(stage_record(stage, start, rows, k, v)).hexdigest()


def chain_records(model, ids: Sequence[int], range_size: int = 512) -> List[Tuple[str, int, str]]:
    """(stage, start_position, SHA-256 of its record) for every (range, layer)
    stage of a mistral-dense claim whose prompt-and-output token ids are
    `ids`, ranges of `range_size` rows."""
    cfg = model.cfg
    kvd = cfg.kv_heads * cfg.head_dim
    carried_k = [np.zeros((0, kvd), np.int32) for _ in range(cfg.layers)]
    carried_v = [np.zeros((0, kvd), np.int32) for _ in range(cfg.layers)]
    out = []
    for start in range(0, len(ids), range_size):
        rows = model.embed(ids[start:start + range_size])
        for layer in range(cfg.layers):
            rows, own_k, own_v = model.layer_range(layer, rows, start, carried_k[layer], carried_v[layer])
            out.append((f"layer_mistral/{layer}", start, stage_digest(f"layer_mistral/{layer}", start, rows,
                                                                       own_k, own_v)))
            carried_k[layer] = np.concatenate([carried_k[layer], own_k])
            carried_v[layer] = np.concatenate([carried_v[layer], own_v])
    return out

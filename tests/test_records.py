"""Canonical checkpoint records (iris_b200/records.py): the documented byte
layout, digests pinned for a fixed record (a change of format changes them),
and refusals of malformed inputs."""
import hashlib
import struct

import numpy as np
import pytest


def test_layout_and_pinned_digests():
    from iris_b200 import records
    rows = np.arange(6, dtype=np.int32).reshape(2, 3) - 3
    k = np.array([[1, -2], [2**31 - 1, -(2**31)]], np.int32)
    v = np.array([[3, 4], [-5, 0]], np.int32)
    rec = records.stage_record("layer_mistral/0", 5, rows, k, v)
    want = (b"IRISREC1" + struct.pack("<I", 15) + b"layer_mistral/0" + struct.pack("<III", 5, 2, 3)
            + rows.astype("<i4").tobytes() + struct.pack("<I", 2) + k.astype("<i4").tobytes()
            + v.astype("<i4").tobytes())
    assert rec == want
    assert records.stage_digest("layer_mistral/0", 5, rows, k, v) == hashlib.sha256(want).hexdigest()
    assert records.stage_digest("s", 0, rows) == "018632a2a54573562657af76c9dba00c215a6886a6f228bf68af4d3f715c5344"
    assert records.stage_record("s", 0, rows).endswith(struct.pack("<I", 0))


def test_refusals():
    from iris_b200 import records
    with pytest.raises(ValueError):
        records.stage_record("s", 0, np.zeros(4, np.int32))
    with pytest.raises(ValueError):
        records.stage_record("s", 0, np.zeros((2, 3), np.int32), np.zeros((3, 2), np.int32), np.zeros((3, 2), np.int32))

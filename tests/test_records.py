"""Canonical checkpoint records (iris_b200/records.py): the documented byte
layout (a header, then the SHA-256 of every 4096-byte leaf of the rows, K
and V), digests pinned for fixed records (a change of format changes them),
refusals of malformed inputs, and the SHA-256 code the device hashes leaves
with (iris_b200/csrc/sha256.cuh, compiled here as host C++) against hashlib."""
import ctypes as C
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
    leaf = lambda a: hashlib.sha256(a.astype("<i4").tobytes()).digest()  # arrays under one leaf
    want = (b"IRISREC2" + struct.pack("<I", 15) + b"layer_mistral/0" + struct.pack("<IIIII", 5, 2, 3, 2, 4096)
            + leaf(rows) + leaf(k) + leaf(v))
    assert rec == want
    assert records.stage_digest("layer_mistral/0", 5, rows, k, v) == hashlib.sha256(want).hexdigest()
    assert records.stage_digest("s", 0, rows) == "b20af9c4c3bb922a7338588f21695ba3a7b1af549637ecdd856ab6e0d0cb8f08"
    # arrays over several leaves, the last one short
    big = (np.arange(3 * 1500, dtype=np.int64) * 2654435761 % (2**32)).astype(np.uint32).view(np.int32)
    big = big.reshape(3, 1500)
    assert len(records.leaf_digests(big)) == 32 * 5  # 18,000 bytes
    assert records.stage_digest("big", 7, big, big[:, :2], big[:, 2:4]) == \
        "7fced8b28b75529c4f54f48b98fa9e54dbe31e03ea436427e9693eb6a557e24d"
    leaves = records.leaf_digests(big) + records.leaf_digests(big[:, :2]) + records.leaf_digests(big[:, 2:4])
    assert records.digest_from_leaves("big", 7, 3, 1500, 2, leaves) == \
        records.stage_digest("big", 7, big, big[:, :2], big[:, 2:4])


def test_refusals():
    from iris_b200 import records
    with pytest.raises(ValueError):
        records.stage_record("s", 0, np.zeros(4, np.int32))
    with pytest.raises(ValueError):
        records.stage_record("s", 0, np.zeros((2, 3), np.int32), np.zeros((3, 2), np.int32), np.zeros((3, 2), np.int32))


@pytest.mark.parametrize("nbytes,leaf", [(0, 4096), (4, 4096), (52, 4096), (56, 4096), (60, 4096), (64, 4096),
                                         (116, 4096), (120, 64), (4096, 4096), (18000, 4096), (9000, 1024)])
def test_leaf_sha256_matches_hashlib(detnum_shim, nbytes, leaf):
    """The tail cases of the padding: the 0x80 marker in any of the last
    words, a second block when it lands in words 14-15, whole blocks."""
    data = np.random.default_rng(nbytes).integers(0, 2**32, size=max(nbytes // 4, 1), dtype=np.uint64)
    data = data.astype(np.uint32)[: nbytes // 4]
    n = (nbytes + leaf - 1) // leaf
    out = np.zeros(max(n, 1) * 32, np.uint8)
    buf = np.ascontiguousarray(data if nbytes else np.zeros(1, np.uint32))
    detnum_shim.shim_sha256_leaves(buf.ctypes.data_as(C.POINTER(C.c_uint32)), nbytes, leaf,
                                   out.ctypes.data_as(C.POINTER(C.c_uint8)))
    want = b"".join(hashlib.sha256(data.tobytes()[i:i + leaf]).digest() for i in range(0, nbytes, leaf))
    assert out[: 32 * n].tobytes() == want

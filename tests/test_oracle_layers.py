"""Layer-level pins of the CPU oracle against the reference's own layer tests.

crates/inference/direct/tests/executor.rs:191-350
(native_decode_rotary_outputs_match_prefill_across_chunks) and
crates/inference/kernels/src/prefill_range.rs:1040-1080: a one-block-wide
gemma-dense layer with identity Q8_0 and dense matrices, a two-lane rotary
prefix at base 10000, unit q/k norms. Position 1's key starts [35408, 55146],
and prefilling five rows at once equals prefill (1 row) + decode + decode +
a two-row chunk, rows and K/V alike.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

ONE = 1 << 16
W = 32


def identity_q8():
    """q8_exact of the W x W identity (executor.rs:764-782): scale 1.0, q = 1."""
    out = bytearray()
    for r in range(W):
        out += (0x3C00).to_bytes(2, "little") + bytes(1 if c == r else 0 for c in range(W))
    return np.frombuffer(bytes(out), np.uint8).copy()


@pytest.fixture(scope="module")
def layer():
    O.build()
    q8 = identity_q8()
    dense = np.zeros((W, W), np.int32)
    np.fill_diagonal(dense, ONE)
    norm = np.full(W, ONE, np.int32)
    unit = np.zeros(W, np.int32)
    unit[0] = ONE
    keep = [q8, dense, norm, unit]
    p = O.GemmaLayer(W, W, 1, 1, W, 0, ONE, 0, 0, 10_000 << 32, 2, 2, -1, -2, -3, W,
                     O.ptr(norm, C.c_int32), O.ptr(norm, C.c_int32), O.ptr(norm, C.c_int32),
                     O.ptr(norm, C.c_int32), O.ptr(unit, C.c_int32), O.ptr(unit, C.c_int32),
                     O.ptr(norm, C.c_int32),
                     *([O.ptr(q8, C.c_uint8)] * 7), O.ptr(dense, C.c_int32), O.ptr(dense, C.c_int32))
    return p, keep


def rows5():
    out = np.full((5, W), ONE, np.int32)
    for t in range(5):
        out[t, 1] = ONE if t % 2 == 0 else -ONE
    return out


def run(layer, rows, start, prior):
    p, _ = layer
    m = rows.shape[0]
    rows = np.ascontiguousarray(rows, np.int32)
    out = np.empty_like(rows)
    ok = np.empty((m, W), np.int32)
    ov = np.empty((m, W), np.int32)
    ple = np.full((m, W), ONE, np.int32)
    pos, pk, pv = prior
    pos = np.ascontiguousarray(pos, np.uint32)
    pk = np.ascontiguousarray(pk, np.int32).reshape(-1, W)
    pv = np.ascontiguousarray(pv, np.int32).reshape(-1, W)
    empty = O.Keys(0, None, None, None)
    prior_keys = O.Keys(len(pos), O.ptr(pos, C.c_uint32) if len(pos) else None,
                        O.ptr(pk, C.c_int32) if len(pos) else None, O.ptr(pv, C.c_int32) if len(pos) else None)
    rc = O.lib().oracle_gemma_layer(C.byref(p), O.ptr(rows, C.c_int32), m, start, prior_keys, empty, empty,
                                    O.ptr(ple, C.c_int32), O.ptr(out, C.c_int32), O.ptr(ok, C.c_int32),
                                    O.ptr(ov, C.c_int32), 2)
    assert rc == 0
    kv = (np.concatenate([pos, np.arange(start, start + m, dtype=np.uint32)]),
          np.concatenate([pk, ok]), np.concatenate([pv, ov]))
    return out, kv


def test_rope_answer_in_the_layer(layer):
    _, (pos, k, v) = run(layer, rows5(), 0, ([], np.zeros((0, W)), np.zeros((0, W))))
    assert list(k[1][:2]) == [35408, 55146]


def test_prefill_equals_chunked_decode(layer):
    rows = rows5()
    ref_rows, ref_kv = run(layer, rows, 0, ([], np.zeros((0, W)), np.zeros((0, W))))
    prior = ([], np.zeros((0, W)), np.zeros((0, W)))
    for s, e in [(0, 1), (1, 2), (2, 3), (3, 5)]:
        out, prior = run(layer, rows[s:e], s, prior)
        assert np.array_equal(out, ref_rows[s:e]), f"rows at start {s}"
        assert np.array_equal(prior[0], ref_kv[0][:e])
        assert np.array_equal(prior[1], ref_kv[1][:e]), f"keys at start {s}"
        assert np.array_equal(prior[2], ref_kv[2][:e])


def test_oracle_generate_is_deterministic_and_chunk_free():
    """The oracle's direct loop on a seeded parity-shaped Mistral model gives
    the same first token as its layer-by-layer pass over the whole prompt."""
    from iris_b200.model import synth_host_weights
    from iris_b200.shapes import parity_mistral
    from oracle.models import OracleModel
    cfg = parity_mistral()
    w = synth_host_weights(cfg, seed=11)
    om = OracleModel(cfg, w)
    prompt = [3, 17, 200, 5, 9, 400, 1]
    toks, logits = om.generate(prompt, 4)
    toks2, logits2 = om.generate(prompt, 4, threads=1)
    assert toks == toks2 and np.array_equal(logits, logits2)
    assert len(toks) == 4
    assert toks[0] == int(np.argmax(logits[0]))

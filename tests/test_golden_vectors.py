"""The reference's known-answer vectors (tests/golden/det_num_kats.json)
against the CPU oracle and against the device arithmetic header compiled for
the host (iris_b200/csrc/detnum.cuh via tests/native/detnum_shim.cc): both
implementations of the token-loop arithmetic must reproduce every vector."""
import ctypes as C
import json
import struct
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = json.loads((Path(__file__).parent / "golden" / "det_num_kats.json").read_text())


@pytest.fixture(scope="module")
def L():
    O.build()
    return O.lib()


@pytest.fixture(scope="module")
def S(detnum_shim):
    return detnum_shim


def block(scale_bits, weights):
    vals = [0] * 32
    for i, v in weights.items():
        vals[int(i)] = v
    return np.frombuffer(struct.pack("<H", scale_bits) + bytes(v & 0xFF for v in vals), np.uint8).copy()


def acts(d):
    a = np.zeros(32, np.int32)
    for i, v in d.items():
        a[int(i)] = v
    return a


def test_rounding_mac_saturation(L, S):
    for inp, exp in GOLDEN["rshift_round_ties_even_16"]["cases"]:
        assert L.oracle_rshift_round_ties_even(inp, 16) == exp
        assert L.oracle_requantize(inp) == exp
        assert S.shim_requantize(inp) == exp
    for acc, a, b, exp in GOLDEN["wrapping_mac"]["cases"]:
        assert L.oracle_mac_bits(acc, a, b) == exp
    for inp, exp in GOLDEN["requantize_saturates"]["cases"]:
        assert L.oracle_requantize(inp) == exp
        assert S.shim_requantize(inp) == exp
    for a, b, exp in GOLDEN["add_sub_saturate"]["add"]:
        assert L.oracle_add_sat(a, b) == exp
    for a, b, exp in GOLDEN["add_sub_saturate"]["sub"]:
        assert L.oracle_sub_sat(a, b) == exp


def test_fixed_point_conversions(L):
    for x, exp in GOLDEN["f32_to_fixed"]["act"]:
        assert L.oracle_f32_to_act(x) == exp
    for x, exp in GOLDEN["f32_to_fixed"]["acc"]:
        assert L.oracle_f32_to_acc(x) == exp


def test_q8_scales_and_dot_row(L, S):
    out = C.c_int64()
    for bits, exp in GOLDEN["scale_q24"]["cases"]:
        assert L.oracle_scale_q24(bits, C.byref(out)) == 0 and out.value == exp
    for bits in GOLDEN["scale_q24"]["rejected"]:
        assert L.oracle_scale_q24(bits, C.byref(out)) != 0
    for case in GOLDEN["dot_row"]["cases"]:
        row = block(case["scale_bits"], case["weights"])
        a = acts(case["activations"])
        assert O.dot_row(a, row) == case["expected"]
        assert S.shim_q8_dot(a.ctypes.data_as(C.POINTER(C.c_int32)), row.ctypes.data_as(C.POINTER(C.c_uint8)),
                             32) == case["expected"]


def test_silu_scale_yarn(L, S):
    for x, exp in GOLDEN["silu"]["cases"]:
        assert L.oracle_silu(x) == exp
        assert S.shim_silu(x) == exp
    for d, exp in GOLDEN["attention_scale_q32"]["cases"]:
        assert L.oracle_attention_scale_q32(d) == exp
    y = GOLDEN["yarn_first_frequency"]
    freqs = np.zeros(y["pairs"], np.int64)
    assert L.oracle_yarn_inverse_frequencies(y["base"], y["pairs"], y["factor"], y["low"], y["high"],
                                             O.ptr(freqs, C.c_int64)) == 0
    assert freqs[0] == y["first"]


def test_rope_answer_at_position_one(L, S):
    r = GOLDEN["rope_position_one"]
    for base in r["bases_acc"]:
        v = acts(r["input"])
        L.oracle_rope_rotate_pairs(O.ptr(v, C.c_int32), r["width"], r["rotary"], r["freq_base_dim"], base,
                                   r["position"])
        assert list(v[:2]) == r["expected_head"] and not v[2:].any()

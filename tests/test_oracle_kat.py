"""Pins the CPU oracle to the reference's own known-answer tests.

Every literal below is taken from the reference's Rust tests for this path:
- crates/det-num/tests/golden_vectors.rs:8-79 (ties at shift 16, wrapping MAC,
  saturation),
- crates/det-num/tests/equivalence.rs:21-67 (float conversions, partial rotary),
- crates/det-num/src/q8.rs:120-179 (scale decoding, dot_row, ties, dequant),
- crates/det-num/src/mistral.rs:222-285 (SiLU, rotation, YaRN, score scale),
- crates/det-num/src/convert.rs:131-145,
- crates/inference/kernels/src/prefill_range.rs:1040-1080 and
  crates/inference/direct/tests/executor.rs:318 (the RoPE answer [35408, 55146]),
- crates/inference/direct/src/generation.rs:64-94 (first maximum wins).
"""
import ctypes as C
import math
import struct

import numpy as np
import pytest

from oracle import oracle as O

I32_MIN, I32_MAX = -(2**31), 2**31 - 1
I64_MIN, I64_MAX = -(2**63), 2**63 - 1
ONE = 1 << 16


@pytest.fixture(scope="module")
def L():
    O.build()
    return O.lib()


# ---- golden_vectors.rs -------------------------------------------------------

def test_signed_rounding_ties_and_neighbors(L):
    for inp, exp in [(32767, 0), (32768, 0), (32769, 1), (98303, 1), (98304, 2), (163840, 2),
                     (-32767, 0), (-32768, 0), (-32769, -1), (-98303, -1), (-98304, -2),
                     (-163840, -2)]:
        assert L.oracle_rshift_round_ties_even(inp, 16) == exp
        assert L.oracle_requantize(inp) == exp


def test_wrapping_mac_and_partial_accumulators(L):
    for acc, a, b, exp in [(I64_MAX, 1, 1, I64_MIN), (I64_MIN, -1, 1, I64_MAX), (7, -3, 5, -8),
                           (0, I32_MIN, I32_MIN, 4_611_686_018_427_387_904),
                           (4_611_686_018_427_387_904, I32_MIN, I32_MIN, I64_MIN)]:
        assert L.oracle_mac_bits(acc, a, b) == exp


def test_activation_saturation_is_distinct_from_mac_wrapping(L):
    for inp, exp in [(I64_MAX, I32_MAX), (I64_MIN, I32_MIN), (140_737_488_289_792, I32_MAX),
                     (-140_737_488_355_328, I32_MIN)]:
        assert L.oracle_requantize(inp) == exp
    assert L.oracle_add_sat(I32_MAX, 1) == I32_MAX
    assert L.oracle_add_sat(I32_MIN, -1) == I32_MIN
    assert L.oracle_sub_sat(I32_MIN, 1) == I32_MIN
    assert L.oracle_sub_sat(I32_MAX, -1) == I32_MAX


# ---- equivalence.rs / convert.rs --------------------------------------------

def sample_bits(seed, n):
    """equivalence.rs:7-19: xorshift64 samples in (-8, 8) Q16.16."""
    state = (seed | 1) & (2**64 - 1)
    out = []
    for _ in range(n):
        state ^= (state << 13) & (2**64 - 1)
        state ^= state >> 7
        state ^= (state << 17) & (2**64 - 1)
        v = (state >> 24) & 0xFFFFFFFF
        v = v - 2**32 if v >= 2**31 else v
        out.append(int(math.fmod(v, 8 << 16)))  # Rust % truncates toward zero
    return out


def test_config_float_conversions_use_expected_fixed_widths(L):
    assert L.oracle_f32_to_act(1.0) == 1 << 16
    assert L.oracle_f32_to_act(-0.5) == -(1 << 15)
    assert L.oracle_f32_to_acc(1.0) == 1 << 32
    assert L.oracle_f32_to_acc(10_000.0) == 10_000 << 32
    assert L.oracle_f32_to_acc(1_000_000.0) == 1_000_000 << 32
    assert L.oracle_f32_to_acc(1e-6) != 0
    assert L.oracle_f32_to_act(1e-6) == 0
    # the eps values the synthetic configs use (import/src/mistral.rs:275-279)
    assert L.oracle_f32_to_acc(1e-5) == 42950
    assert L.oracle_f32_to_acc(1e-6) == 4295


def test_partial_rotary_leaves_the_tail_untouched(L):
    bits = np.array(sample_bits(0xABCD, 512), dtype=np.int32)
    out = bits.copy()
    L.oracle_rope_rotate_pairs(O.ptr(out, C.c_int32), 512, 128, 512, 1_000_000 << 32, 7)
    assert np.array_equal(out[128:], bits[128:])
    assert not np.array_equal(out[:128], bits[:128])


def test_rms_norm_shapes(L):
    for width in [4, 16, 256]:
        vals = np.array(sample_bits(0x5EED ^ width, width), dtype=np.int32)
        w = np.array(sample_bits(0xB1CE ^ width, width), dtype=np.int32)
        v = vals.copy()
        L.oracle_rms_norm(O.ptr(v, C.c_int32), O.ptr(w, C.c_int32), width, L.oracle_f32_to_acc(1e-6))
        assert v.shape == (width,)


# ---- q8.rs -------------------------------------------------------------------

def q8_block(scale_bits, values):
    return np.frombuffer(struct.pack("<H", scale_bits) + bytes(v & 0xFF for v in values),
                         dtype=np.uint8).copy()


def test_half_precision_scales_decode_exactly(L):
    out = C.c_int64()
    for bits, exp in [(0x3C00, 1 << 24), (0xBC00, -(1 << 24)), (0x0001, 1), (0x0400, 1 << 10),
                      (0x7BFF, 65504 << 24), (0x3555, (1024 + 0x155) << 12)]:
        assert L.oracle_scale_q24(bits, C.byref(out)) == 0
        assert out.value == exp
    assert L.oracle_scale_q24(0x7C00, C.byref(out)) != 0
    assert L.oracle_scale_q24(0x7E00, C.byref(out)) != 0


def test_dot_row_is_the_exact_product_rounded_once():
    vals = [0] * 32
    vals[0], vals[1] = 3, -5
    row = q8_block(0x2000, vals)
    a = np.zeros(32, np.int32)
    a[0], a[1] = 1 << 16, 3 << 15
    assert O.dot_row(a, row) == -2304
    one = [0] * 32
    one[0] = 1
    tiny = q8_block(0x0200, one)
    a = np.zeros(32, np.int32)
    a[0] = 1 << 14
    assert O.dot_row(a, tiny) == 0
    a[0] = 3 << 14
    assert O.dot_row(a, tiny) == 2
    a[0] = -(3 << 14)
    assert O.dot_row(a, tiny) == -2


def test_dequantized_rows_match_their_dot_products(L):
    vals = [(i - 16) * 7 for i in range(32)]
    row = q8_block(0x1E66, vals)
    w = np.zeros(32, np.int32)
    assert L.oracle_dequantize_row(O.ptr(row, C.c_uint8), 34, O.ptr(w, C.c_int32), 32) == 0
    for i in range(32):
        a = np.zeros(32, np.int32)
        a[i] = 1 << 16
        assert O.dot_row(a, row) == w[i]


def test_malformed_rows_are_rejected():
    row = q8_block(0x7C00, [1] * 32)
    with pytest.raises(ValueError):
        O.dot_row(np.zeros(32, np.int32), row)
    with pytest.raises(ValueError):
        O.dot_row(np.zeros(64, np.int32), row)


# ---- mistral.rs --------------------------------------------------------------

def real(bits):
    return bits / 65536.0


def test_silu_is_within_two_units_of_the_real_function(L):
    worst = 0.0
    x = -(24 << 16)
    while x <= 24 << 16:
        exact = real(x) / (1.0 + math.exp(-real(x)))
        worst = max(worst, abs(real(L.oracle_silu(x)) - exact))
        x += 977
    assert worst <= 2.0 / 65536.0
    assert L.oracle_silu(0) == 0
    assert L.oracle_silu(I32_MIN) == 0
    assert L.oracle_silu(I32_MAX) == I32_MAX


def yarn(L, base, pairs, factor, low, high):
    out = np.zeros(pairs, np.int64)
    rc = L.oracle_yarn_inverse_frequencies(base, pairs, factor, low, high, O.ptr(out, C.c_int64))
    return None if rc else out


def test_rotation_is_within_two_units_of_the_real_one(L):
    freqs = yarn(L, 1_000_000, 64, 16, 20, 37)
    for position in [1, 7, 513, 16_383]:
        values = np.array([(i - 64) * 9_173 for i in range(128)], np.int32)
        before = values.copy()
        L.oracle_rotate_consecutive_pairs(O.ptr(values, C.c_int32), 128, O.ptr(freqs, C.c_int64),
                                          64, position)
        for pair in range(64):
            angle = position * float(freqs[pair]) / 4294967296.0
            a, b = real(int(before[2 * pair])), real(int(before[2 * pair + 1]))
            e0 = a * math.cos(angle) - b * math.sin(angle)
            e1 = a * math.sin(angle) + b * math.cos(angle)
            assert abs(real(int(values[2 * pair])) - e0) <= 2.0 / 65536.0
            assert abs(real(int(values[2 * pair + 1])) - e1) <= 2.0 / 65536.0


def test_yarn_frequencies_follow_the_formula(L):
    freqs = yarn(L, 1_000_000, 64, 16, 20, 37)
    assert freqs[0] == 1 << 32
    for pair, bits in enumerate(freqs):
        plain = 1_000_000.0 ** (-(pair / 64.0))
        ramp = 1.0 - min(max((pair - 20.0) / 17.0, 0.0), 1.0)
        expected = plain * (1.0 / 16.0 + 15.0 / 16.0 * ramp)
        assert abs(float(bits) / 4294967296.0 - expected) <= 1e-8
    assert yarn(L, 1_000_000, 48, 16, 20, 37) is None


def test_plain_rope_table_is_the_factor_one_yarn_table(L):
    """Factor 1 reduces the YaRN table to base^(-j/pairs) (the configs' RoPE)."""
    freqs = yarn(L, 1_000_000, 64, 1, 0, 1)
    for pair, bits in enumerate(freqs):
        assert abs(float(bits) / 2**32 - 1_000_000.0 ** (-(pair / 64.0))) <= 1e-8


def test_the_score_scale_is_the_inverse_root(L):
    assert L.oracle_attention_scale_q32(128) == 379_625_062
    assert L.oracle_attention_scale_q32(1) == 2**32 - 1
    ones = np.full(128, 1 << 16, np.int32)
    s = L.oracle_scaled_score(O.ptr(ones, C.c_int32), O.ptr(ones, C.c_int32), 128,
                              L.oracle_attention_scale_q32(128))
    assert abs(real(s) - math.sqrt(128)) <= 2.0 / 65536.0


# ---- RoPE answer, prefill_range.rs:1073 / executor.rs:318 --------------------

def test_rope_known_answer_at_position_one(L):
    for base in [1 << 32, 10_000 << 32]:
        v = np.zeros(32, np.int32)
        v[0] = ONE
        L.oracle_rope_rotate_pairs(O.ptr(v, C.c_int32), 32, 2, 2, base, 1)
        assert list(v[:2]) == [35408, 55146]
        assert not v[2:].any()
    v = np.zeros(32, np.int32)
    v[0] = ONE
    L.oracle_rope_rotate_pairs(O.ptr(v, C.c_int32), 32, 2, 2, 10_000 << 32, 0)
    assert v[0] == ONE and v[1] == 0


# ---- softmax / selection -----------------------------------------------------

def test_softmax_weights_sum_to_one_with_the_residual_on_the_first_max(L):
    rng = np.random.default_rng(5)
    for n in [1, 2, 7, 100, 1000]:
        logits = rng.integers(-(8 << 16), 8 << 16, size=n, dtype=np.int64).astype(np.int32)
        if n > 3:
            logits[3] = logits.max()
        w = np.zeros(n, np.int32)
        L.oracle_attention_softmax(O.ptr(logits, C.c_int32), n, O.ptr(w, C.c_int32))
        assert int(w.astype(np.int64).sum()) == ONE
        # exact float reference within a few Q16.16 units per weight
        f = np.exp((logits - logits.max()) / 65536.0)
        f = f / f.sum() * 65536.0
        err = np.abs(f - w)
        first_max = int(np.argmax(logits))
        # every weight is within a few units except the first maximum, which
        # also carries the residual 1.0 - sum (ops.rs:255-260)
        assert np.delete(err, first_max).max(initial=0) <= 2.0
        assert err[first_max] <= 2.0 + n / 2.0
    # equal logits: ties go to the first maximum
    logits = np.array([5, 10, 10], np.int32)
    w = np.zeros(3, np.int32)
    L.oracle_attention_softmax(O.ptr(logits, C.c_int32), 3, O.ptr(w, C.c_int32))
    assert w[1] >= w[2]


def test_first_maximum_selects_the_lowest_token(L):
    """generation.rs:64-94: equal scores keep the earliest token."""
    logits = np.array([10, 10, 3], np.int32)
    assert int(np.argmax(logits)) == 0  # numpy argmax is also first-max

"""The product's exact-arithmetic header (iris_b200/csrc/detnum.cuh), compiled
as host C++, against the CPU oracle on seeded random and edge-case inputs.

The same header is what the CUDA kernels run, so these checks pin every
rounding rule of the device code without a GPU; tests/test_gpu_*.py repeat the
comparison on the device.
"""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

ROOT = Path(__file__).resolve().parent.parent
I32_MIN, I32_MAX = -(2**31), 2**31 - 1
EDGE32 = [0, 1, -1, 2, -2, 32767, 32768, -32768, 65535, 65536, -65536, 65537, 98304, -98304,
          3 << 16, -(3 << 16), (3 << 16) - 1, -(3 << 16) + 1, 1 << 24, -(1 << 24),
          I32_MAX, I32_MIN, I32_MAX - 1, I32_MIN + 1, 1 << 30, -(1 << 30)]


@pytest.fixture(scope="module")
def S(detnum_shim):
    return detnum_shim


@pytest.fixture(scope="module")
def L():
    O.build()
    return O.lib()


def rand32(rng, n, bits=32):
    return (rng.integers(-(2**(bits - 1)), 2**(bits - 1), size=n, dtype=np.int64)).tolist()


def test_requantize_mul_sat_div_act(S, L):
    rng = np.random.default_rng(1)
    xs = rng.integers(-(2**63), 2**63 - 1, size=2000, dtype=np.int64).tolist()
    xs += [v * 65536 + d for v in EDGE32 for d in (-32769, -32768, -1, 0, 1, 32768)]
    for x in xs:
        x = max(min(x, 2**63 - 1), -(2**63))
        assert S.shim_requantize(x) == L.oracle_requantize(x), x
    vals = EDGE32 + rand32(rng, 300) + rand32(rng, 300, 20)
    for a in vals[:120]:
        for b in vals[:120]:
            assert S.shim_mul_sat(a, b) == L.oracle_mul_sat(a, b)
            if b != 0:
                assert S.shim_div_act(a, b) == L.oracle_div_act(a, b), (a, b)


def test_mul_sat_rounding_ties_and_extremes(S, L):
    """mul_sat's one-addition rounding against the oracle where it matters:
    products exactly halfway (r = 2^15) with odd and even quotients of both
    signs, one unit either side of halfway, and the saturating extremes."""
    cases = []
    for f in range(-6, 7):
        for r in (0x7FFF, 0x8000, 0x8001, 0, 1, 0xFFFF):
            x = f * 65536 + r
            cases += [(x, 1), (-x, 1), (x, -1)]
    for a in (2**31 - 1, -(2**31), 2**30, -(2**30), 46341, -46341, 65535, 65536, 32768, 98304):
        for b in (2**31 - 1, -(2**31), 1, -1, 2, 3, 65536, 32768, 65537):
            cases.append((a, b))
    for a, b in cases:
        if -(2**31) <= a < 2**31 and -(2**31) <= b < 2**31:
            assert S.shim_mul_sat(a, b) == L.oracle_mul_sat(a, b), (a, b)


def test_inv_sqrt_and_rms_scale(S, L):
    rng = np.random.default_rng(2)
    xs = [1, 2, 3, 4, 42950, 4295, 2**32, 2**32 + 1, 2**62, 2**63 - 1, 7, 1 << 20]
    xs += rng.integers(1, 2**63 - 1, size=3000, dtype=np.int64).tolist()
    xs += (2 ** rng.uniform(0, 63, size=3000)).astype(np.int64).clip(1, 2**63 - 1).tolist()
    for x in xs:
        assert S.shim_inv_sqrt_acc(x) == L.oracle_inv_sqrt_acc(x), x
    assert S.shim_inv_sqrt_acc(0) == L.oracle_inv_sqrt_acc(0)
    for n in [1, 7, 64, 256, 4096]:
        for bits in [8, 16, 20, 24, 32]:
            v = np.array(rand32(rng, n, bits), np.int32)
            for eps in [0, 4295, 42950]:
                exp = L.oracle_rms_norm_scale(O.ptr(v, C.c_int32), n, eps)
                assert S.shim_rms_scale(O.ptr(v, C.c_int32), n, eps) == exp
    big = np.full(4096, I32_MIN, np.int32)  # saturating sum of squares
    assert S.shim_rms_scale(O.ptr(big, C.c_int32), 4096, 0) == L.oracle_rms_norm_scale(
        O.ptr(big, C.c_int32), 4096, 0)


def test_fast_inv_sqrt_and_width_division(S, L):
    """The norm prologues' inverse square root from a double estimate with
    exact steps, and the division by a power-of-two width as a shift, equal
    the oracle's binary search and the general rounded division."""
    rng = np.random.default_rng(21)
    xs = [0, 1, 2, 3, 4, 5, 42950, 4295, 2**32 - 1, 2**32, 2**32 + 1, 2**62, 2**63 - 1, 7, 1 << 20,
          (2**31 - 1) ** 2, (2**31 - 1) ** 2 - 1, 3 * 2**30, 2**34 - 1]
    xs += rng.integers(1, 2**63 - 1, size=20000, dtype=np.int64).tolist()
    xs += (2 ** rng.uniform(0, 63, size=20000)).astype(np.int64).clip(1, 2**63 - 1).tolist()
    sq = rng.integers(1, 2**31, size=5000, dtype=np.int64)  # around exact squares of the targets
    xs += [int(v) for c in sq for v in ((2**64 // (int(c) * int(c))), (2**64 // (int(c) * int(c))) + 1)
           if 0 < v < 2**63]
    for x in xs:
        assert S.shim_inv_sqrt_acc_fast(x) == L.oracle_inv_sqrt_acc(x), x
    for d in [1, 2, 3, 64, 96, 128, 2048, 4096, 14336, 16384, 1 << 20]:
        ns = [0, 1, d // 2, d // 2 + 1, d - 1, d, d + d // 2, 3 * d + d // 2, 2**64 - 1, 2**63]
        ns += rng.integers(0, 2**63, size=300, dtype=np.int64).tolist()
        for n in ns:
            assert S.shim_div_round_even_width(n, d) == S.shim_div_round_even_u64(n, d), (n, d)


def test_one_plane_row_rounding(S):
    """The one-plane GEMM's rounding of x m 2^e in 64 bits equals the
    128-bit formulation: every exponent, both signs, ties, saturation and the
    products past 2^62 that take the 128-bit path."""
    rng = np.random.default_rng(33)
    xs = rng.integers(-(2**56), 2**56, size=4000, dtype=np.int64).tolist()
    xs += (rng.choice([-1, 1], size=4000) * (2 ** rng.uniform(0, 56, size=4000))).astype(np.int64).tolist()
    xs += [0, 1, -1, 2**23, -(2**23), 2**24 + 2**23, 3 * 2**23, -(3 * 2**23), 2**55, -(2**55), 2**56 - 1]
    for x in xs:
        for m in (1, -1, 1024, 2047, -2047, int(rng.integers(-2047, 2048))):
            for e in (0, 1, 12, 23, 24, 25, 29, int(rng.integers(0, 30))):
                assert S.shim_round_q24_scaled(x, m, e) == S.shim_round_q24_scaled_ref(x, m, e), (x, m, e)


def test_mistral_functions(S, L):
    rng = np.random.default_rng(3)
    for x in EDGE32 + rand32(rng, 5000) + rand32(rng, 5000, 22):
        assert S.shim_silu(x) == L.oracle_silu(x), x
    s1, c1, s2, c2 = C.c_int64(), C.c_int64(), C.c_int64(), C.c_int64()
    angles = rng.integers(0, 2**62, size=3000, dtype=np.int64).tolist()
    angles += [0, 6746518852, 13493037705, 20239556557, 26986075409, 26986075408, 1, 2**32]
    for a in angles:
        S.shim_sin_cos_q30(a, C.byref(s1), C.byref(c1))
        L.oracle_sin_cos_q30(a, C.byref(s2), C.byref(c2))
        assert (s1.value, c1.value) == (s2.value, c2.value), a
    for d in [32, 64, 128]:
        scale = L.oracle_attention_scale_q32(d)
        for bits in [12, 20, 31, 32]:
            q = np.array(rand32(rng, d, bits), np.int32)
            k = np.array(rand32(rng, d, bits), np.int32)
            assert S.shim_scaled_score(O.ptr(q, C.c_int32), O.ptr(k, C.c_int32), d, scale) == \
                L.oracle_scaled_score(O.ptr(q, C.c_int32), O.ptr(k, C.c_int32), d, scale)


def test_softmax_pieces(S, L):
    rng = np.random.default_rng(4)
    for _ in range(3000):
        mx = int(rng.integers(-(2**31), 2**31))
        logit = int(rng.integers(-(2**31), mx + 1))
        if rng.random() < 0.5:
            logit = max(-(2**31), mx - int(rng.integers(0, 20 << 16)))
        d = max(-(2**31), logit - mx)
        exp = L.oracle_softmax_exp_term(d * 65536)
        assert S.shim_exp_term(logit, mx) == exp
    for n in [1, 3, 50, 700]:
        logits = np.array(rand32(rng, n, 22), np.int32)
        w = np.zeros(n, np.int32)
        L.oracle_attention_softmax(O.ptr(logits, C.c_int32), n, O.ptr(w, C.c_int32))
        mx = int(logits.max())
        terms = [S.shim_exp_term(int(x), mx) for x in logits]
        total = sum(terms)
        mine = [S.shim_softmax_weight(t, total) for t in terms]
        assert [S.shim_softmax_weight_inv(t, total) for t in terms] == mine
        first = int(np.argmax(logits))
        mine[first] += 65536 - sum(mine)
        assert mine == w.tolist()


def test_softmax_weight_by_reciprocal(S):
    """The device's reciprocal form of the weight division equals the plain
    division for every term in [0, 2^32] and sums in [2^32, 2^62)."""
    rng = np.random.default_rng(12)
    sums = [2**32, 2**32 + 1, 2**33 - 1, 3 << 31, 2**44 + 12345, 2**61 + 7, 2**62 - 1]
    sums += [int(x) for x in rng.integers(2**32, 2**40, size=300)]
    sums += [int(x) for x in rng.integers(2**32, 2**62, size=300)]
    for total in sums:
        terms = [0, 1, 2**32, 2**32 - 1, 2**31, total % 2**32]
        terms += [int(x) for x in rng.integers(0, 2**32 + 1, size=40)]
        for t in terms:
            assert S.shim_softmax_weight_inv(t, total) == S.shim_softmax_weight(t, total), (t, total)


def test_gemma_functions(S, L):
    rng = np.random.default_rng(5)
    for x in EDGE32 + rand32(rng, 5000) + rand32(rng, 5000, 20):
        assert S.shim_tanh(x) == L.oracle_tanh(x), x
        assert S.shim_gelu(x) == L.oracle_gelu(x), x
        assert S.shim_softcap(x, 1966080) == L.oracle_softcap(x, 1966080), x
        assert S.shim_softcap(x, 65536) == L.oracle_softcap(x, 65536), x
    c1, s1, c2, s2 = C.c_int32(), C.c_int32(), C.c_int32(), C.c_int32()
    for a in rng.integers(0, 2**62, size=3000, dtype=np.int64).tolist() + [0, 6746518852]:
        S.shim_sin_cos_acc(a, C.byref(c1), C.byref(s1))
        L.oracle_sin_cos_acc(a, C.byref(c2), C.byref(s2))
        assert (c1.value, s1.value) == (c2.value, s2.value), a


def test_rotate_half_matches_rope_rotate_pairs(S, L):
    """Rotate-half with a precomputed inverse-frequency table equals the
    reference's chained rope_rotate_pairs (ops.rs:154-199)."""
    rng = np.random.default_rng(6)
    for (d, rot, fbd, base) in [(64, 64, 64, 10_000 << 32), (256, 64, 256, 1_000_000 << 32),
                                (32, 2, 2, 10_000 << 32), (256, 256, 256, 10_000 << 32)]:
        step = L.oracle_rope_frequency_step(base, fbd)
        inv = [1 << 32]
        for _ in range(rot // 2 - 1):
            inv.append(L.oracle_acc_mul(inv[-1], step))
        for pos in [1, 2, 7, 511, 4095]:
            v = np.array(rand32(rng, d, 20), np.int32)
            ref = v.copy()
            L.oracle_rope_rotate_pairs(O.ptr(ref, C.c_int32), d, rot, fbd, base, pos)
            mine = v.copy()
            half = rot // 2
            for i in range(half):
                a, b = C.c_int32(int(mine[i])), C.c_int32(int(mine[i + half]))
                S.shim_rotate_half(C.byref(a), C.byref(b), inv[i], pos)
                mine[i], mine[i + half] = a.value, b.value
            assert np.array_equal(mine, ref), (d, rot, pos)


def test_q8_dot_plane_formulation(S, L):
    rng = np.random.default_rng(7)
    for cols in [32, 64, 256, 4096]:
        for max_exp in [30, 18, 5]:
            nb = cols // 32
            row = bytearray()
            for _ in range(nb):
                bits = (int(rng.integers(0, 2)) << 15) | (int(rng.integers(0, max_exp + 1)) << 10) \
                    | int(rng.integers(0, 1024))
                row += int(bits).to_bytes(2, "little")
                row += bytes(rng.integers(0, 256, size=32, dtype=np.uint8))
            row = np.frombuffer(bytes(row), np.uint8).copy()
            for bits in [32, 20, 12]:
                a = np.array(rand32(rng, cols, bits), np.int32)
                a[rng.integers(0, cols, size=3)] = [I32_MAX, I32_MIN, 0]
                assert S.shim_q8_dot(O.ptr(a, C.c_int32), O.ptr(row, C.c_uint8), cols) == \
                    O.dot_row(a, row)
    for bits in [0x3C00, 0x0001, 0x7BFF, 0xFBFF, 0x8001, 0x1E66]:
        row = np.frombuffer(int(bits).to_bytes(2, "little") + bytes(range(0, 256, 8)),
                            np.uint8).copy()
        w = np.zeros(32, np.int32)
        L.oracle_dequantize_row(O.ptr(row, C.c_uint8), 34, O.ptr(w, C.c_int32), 32)
        for j in range(32):
            assert S.shim_q8_dequant(int(np.int8(row[2 + j])), bits) == w[j]

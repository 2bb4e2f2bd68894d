"""The drop-in q8gpu_* products against the reference's own GPU kernel.

oracle/_ref/libq8ref.so is crates/inference/kernels/cuda/q8_product.cu built
unchanged for sm_100a (oracle/Makefile). Both libraries receive the same
weights and decoded Q.24 scales through the same five-function C ABI
(gpu.rs:45-62) and must return the same outputs bit for bit: the shapes and
scale regimes of the reference's device tests (gpu.rs:375-495) and the
Q8-sweep shapes (N, K) in {(2048, 2048), (16384, 2048), (4096, 4096),
(14336, 4096)} at M in {1, 16, 128}.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def libs():
    from iris_b200 import build, _lib
    from oracle import oracle
    build.build()
    ref = oracle.reference_q8()
    if ref is None:
        pytest.skip("oracle/_ref/libq8ref.so was not built (no reference checkout where build() ran)")
    mine = _lib.lib()
    assert mine.q8gpu_init() == 0 and ref.q8gpu_init() == 0, "no usable CUDA device"
    return mine, ref


def random_q8(rng, rows, cols, max_exp):
    nb = rows * cols // 32
    v = rng.integers(0, 2**62, size=nb, dtype=np.int64)
    exp = (v >> 20) % (max_exp + 1)
    bits = ((v & 1) << 15) | (exp << 10) | ((v >> 4) & 0x3FF)
    ex, man = (bits >> 10) & 0x1F, bits & 0x3FF
    mag = np.where(ex == 0, man, (1024 + man) << np.maximum(ex - 1, 0))
    scales = np.where(bits & 0x8000, -mag, mag).astype(np.int64)
    weights = rng.integers(-128, 128, size=rows * cols, dtype=np.int64).astype(np.int8)
    return weights, scales


def random_acts(rng, tokens, cols, bits):
    r = rng.integers(0, 2**63 - 1, size=tokens * cols, dtype=np.int64)
    vals = ((r >> 16) & 0xFFFFFFFF).astype(np.uint32).view(np.int32) >> (32 - bits)
    sel = r % 61
    vals = np.where(sel == 0, 2**31 - 1, np.where(sel == 1, -(2**31), np.where(sel == 2, 0, vals)))
    return vals.astype(np.int32)


def product(L, weights, scales, rows, cols, acts, tokens):
    h = C.c_void_p()
    rc = L.q8gpu_upload(weights.ctypes.data_as(C.POINTER(C.c_int8)), scales.ctypes.data_as(C.POINTER(C.c_int64)),
                        rows, cols, C.byref(h))
    assert rc == 0, rc
    out = np.empty(tokens * rows, np.int32)
    rc = L.q8gpu_product(h, acts.ctypes.data_as(C.POINTER(C.c_int32)), tokens, out.ctypes.data_as(C.POINTER(C.c_int32)))
    L.q8gpu_free(h)
    assert rc == 0, rc
    return out


@pytest.mark.parametrize("rows,cols,tokens,max_exp,bits", [
    (1, 32, 1, 30, 32), (7, 64, 3, 30, 32), (33, 96, 5, 14, 24), (128, 256, 17, 14, 20),
    (300, 1024, 2, 29, 31), (64, 4096, 1, 20, 32),
])
def test_reference_device_test_shapes(libs, rows, cols, tokens, max_exp, bits):
    mine, ref = libs
    rng = np.random.default_rng(rows * 7919 + cols)
    w, s = random_q8(rng, rows, cols, max_exp)
    a = random_acts(rng, tokens, cols, bits)
    assert np.array_equal(product(mine, w, s, rows, cols, a, tokens), product(ref, w, s, rows, cols, a, tokens))


@pytest.mark.parametrize("n,k", [(2048, 2048), (16384, 2048), (4096, 4096), (14336, 4096)])
@pytest.mark.parametrize("m", [1, 16, 128])
def test_q8_sweep_shapes(libs, n, k, m):
    mine, ref = libs
    rng = np.random.default_rng(n + k + m)
    w, s = random_q8(rng, n, k, 14)
    a = random_acts(rng, m, k, 21)
    assert np.array_equal(product(mine, w, s, n, k, a, m), product(ref, w, s, n, k, a, m))

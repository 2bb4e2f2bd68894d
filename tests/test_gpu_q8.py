"""GPU parity of the exact Q8_0 products against the CPU oracle.

Shapes, scale regimes, tie cases and the non-finite-scale refusal follow the
reference's own device tests (crates/inference/kernels/src/gpu.rs:375-495);
the sweep shapes are BASELINE config 2's (N, K) pairs. Every output is
compared, not sampled, except at M = 2048 where the oracle checks a seeded
sample and the tiled GEMM is checked against the per-token GEMV everywhere.
The bar is bit-exact.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

I32_MIN, I32_MAX = -(2**31), 2**31 - 1


@pytest.fixture(scope="module")
def L():
    from iris_b200 import build, _lib
    build.build()
    lib = _lib.lib()
    assert lib.q8gpu_init() == 0, "no usable CUDA device"
    return lib


@pytest.fixture(scope="module")
def O():
    from oracle import oracle
    oracle.build()
    return oracle


def rng_matrix(rng, rows, cols, max_exp):
    """gpu.rs:373-385: every weight byte, finite scales of either sign up to max_exp."""
    nb = rows * cols // 32
    v = rng.integers(0, 2**62, size=nb, dtype=np.int64)
    exp = (v >> 20) % (max_exp + 1)
    bits = ((v & 1) << 15) | (exp << 10) | ((v >> 4) & 0x3FF)
    out = np.empty((nb, 34), np.uint8)
    out[:, 0] = bits & 0xFF
    out[:, 1] = (bits >> 8) & 0xFF
    out[:, 2:] = rng.integers(0, 256, size=(nb, 32), dtype=np.uint8)
    return out.reshape(-1)


def rng_acts(rng, tokens, cols, magnitude_bits):
    """gpu.rs:387-398: i32::MAX / MIN / 0 mixed into values of a given size."""
    r = rng.integers(0, 2**63 - 1, size=tokens * cols, dtype=np.int64)
    vals = ((r >> 16) & 0xFFFFFFFF).astype(np.uint32).view(np.int32) >> (32 - magnitude_bits)
    sel = r % 61
    vals = np.where(sel == 0, I32_MAX, np.where(sel == 1, I32_MIN, np.where(sel == 2, 0, vals)))
    return vals.astype(np.int32).reshape(tokens, cols)


def scales_q24(blocks):
    b = blocks.reshape(-1, 34)
    bits = b[:, 0].astype(np.int64) | (b[:, 1].astype(np.int64) << 8)
    ex, man = (bits >> 10) & 0x1F, bits & 0x3FF
    mag = np.where(ex == 0, man, (1024 + man) << np.maximum(ex - 1, 0))
    return np.where(bits & 0x8000, -mag, mag).astype(np.int64), b[:, 2:].view(np.int8).reshape(-1)


def device_product(L, blocks, rows, cols, acts, via="blocks"):
    from iris_b200 import _lib
    h = C.c_void_p()
    if via == "blocks":
        _lib.check(L.iris_q8_upload_blocks(_lib.ptr(blocks, C.c_uint8), rows, cols, C.byref(h)), "upload")
    else:  # the reference's own call sequence: weights + decoded i64 scales
        sc, q = scales_q24(blocks)
        q = np.ascontiguousarray(q.reshape(rows, cols))
        _lib.check(L.q8gpu_upload(q.ctypes.data_as(C.POINTER(C.c_int8)), _lib.ptr(sc, C.c_int64), rows, cols,
                                  C.byref(h)), "q8gpu_upload")
    out = np.empty((acts.shape[0], rows), np.int32)
    a = np.ascontiguousarray(acts, np.int32)
    _lib.check(L.q8gpu_product(h, _lib.ptr(a, C.c_int32), a.shape[0], _lib.ptr(out, C.c_int32)), "product")
    L.q8gpu_free(h)
    return out


def test_device_products_equal_one_q8_dot_per_value(L, O):
    rng = np.random.default_rng(0x9E3779B97F4A7C15 % 2**63)
    for rows, cols, tokens in [(1, 32, 1), (16, 32, 16), (17, 64, 15), (130, 96, 33), (300, 1536, 70)]:
        for max_exp, mag in [(30, 32), (18, 20), (5, 12)]:
            blocks = rng_matrix(rng, rows, cols, max_exp)
            acts = rng_acts(rng, tokens, cols, mag)
            want = O.linear(acts, blocks, rows)
            for via in ("blocks", "q24"):
                got = device_product(L, blocks, rows, cols, acts, via)
                assert np.array_equal(got, want), (rows, cols, tokens, max_exp, via)
            # single tokens through the decode GEMV
            for t in range(min(tokens, 3)):
                got = device_product(L, blocks, rows, cols, acts[t:t + 1])
                assert np.array_equal(got[0], want[t])


def test_device_products_round_ties_to_even(L, O):
    """gpu.rs:420-444: scale 2^-15, activations in steps of 2^-2."""
    rows, cols, tokens = 64, 32, 96
    out = bytearray()
    for row in range(rows):
        w = [0] * 32
        w[row % 32] = [1, -1, 3, -3, 5, -7, 127, -128][row % 8]
        out += (0x0200).to_bytes(2, "little") + bytes(x & 0xFF for x in w)
    blocks = np.frombuffer(bytes(out), np.uint8).copy()
    idx = np.arange(tokens * cols)
    acts = (((idx // cols) - 48 + (idx % cols)) << 14).astype(np.int32).reshape(tokens, cols)
    want = O.linear(acts, blocks, rows)
    assert np.array_equal(device_product(L, blocks, rows, cols, acts), want)
    assert np.array_equal(device_product(L, blocks, rows, cols, acts[:1])[0], want[0])


def test_a_scale_that_is_not_finite_is_refused(L):
    from iris_b200 import _lib
    blocks = np.zeros(34, np.uint8)
    blocks[:2] = [0x00, 0x7C]  # +inf
    h = C.c_void_p()
    assert L.iris_q8_upload_blocks(_lib.ptr(blocks, C.c_uint8), 1, 32, C.byref(h)) == _lib.IRIS_ESCALE
    q = np.ones(32, np.int8)
    bad = np.array([3 << 40], np.int64)  # not the image of any fp16 scale
    assert L.q8gpu_upload(q.ctypes.data_as(C.POINTER(C.c_int8)), _lib.ptr(bad, C.c_int64), 1, 32,
                          C.byref(h)) == _lib.IRIS_ESCALE


def test_empty_and_malformed(L):
    from iris_b200 import _lib
    from iris_b200.tensor import Q8Matrix, Slab, linear_slab_from_source
    rng = np.random.default_rng(3)
    m = Q8Matrix("m", rng_matrix(rng, 4, 32, 10), 4, 32)
    assert linear_slab_from_source(Slab.zeroed(0, 32), m).rows() == 0
    with pytest.raises(ValueError):
        linear_slab_from_source(Slab.zeroed(2, 64), m)
    h = C.c_void_p()
    blocks = np.zeros(34, np.uint8)
    assert L.iris_q8_upload_blocks(_lib.ptr(blocks, C.c_uint8), 1, 33, C.byref(h)) == _lib.IRIS_EINVAL


@pytest.mark.parametrize("n,k", [(2048, 2048), (16384, 2048), (4096, 4096), (14336, 4096)])
def test_sweep_shapes(L, O, n, k):
    """BASELINE config 2 at M = 1 and 16 (all outputs vs the oracle), and at
    M = 128 for the smallest pair."""
    rng = np.random.default_rng(n * 7 + k)
    blocks = rng_matrix(rng, n, k, 14)
    for m, mag in [(1, 20), (16, 32)] + ([(128, 20)] if n == 2048 else []):
        acts = rng_acts(rng, m, k, mag)
        want = O.linear(acts, blocks, n)
        assert np.array_equal(device_product(L, blocks, n, k, acts), want), (n, k, m)


def test_gemm_at_2048_tokens_matches_gemv_and_oracle_sample(L, O):
    """M = 2048: the tiled GEMM against the decode GEMV token by token on a
    sample of tokens, and against the oracle on a seeded sample of outputs."""
    import torch
    from iris_b200 import _lib
    n, k, m = 2048, 2048, 2048
    rng = np.random.default_rng(99)
    blocks = rng_matrix(rng, n, k, 14)
    acts = rng_acts(rng, m, k, 20)
    h = C.c_void_p()
    _lib.check(L.iris_q8_upload_blocks(_lib.ptr(blocks, C.c_uint8), n, k, C.byref(h)), "upload")
    a = torch.from_numpy(acts).cuda()
    out = torch.empty((m, n), dtype=torch.int32, device="cuda")
    _lib.check(L.iris_q8_product_device_path(h, a.data_ptr(), m, out.data_ptr(), None, _lib.PATH_GEMM), "gemm")
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    one = torch.empty((1, n), dtype=torch.int32, device="cuda")
    for t in list(range(0, m, 97)) + [m - 1]:
        _lib.check(L.iris_q8_product_device_path(h, a[t:t + 1].data_ptr(), 1, one.data_ptr(), None,
                                                 _lib.PATH_GEMV), "gemv")
        torch.cuda.synchronize()
        assert np.array_equal(one.cpu().numpy()[0], got[t]), t
    rows_b = blocks.reshape(n, -1)
    for _ in range(300):
        t, r = int(rng.integers(0, m)), int(rng.integers(0, n))
        assert got[t, r] == O.dot_row(acts[t], rows_b[r])
    L.q8gpu_free(h)

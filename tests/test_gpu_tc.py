"""GPU parity of the tcgen05 tensor-core GEMM (many-token Q8_0 products over
the tensor-core copy of the weights) against the CPU oracle, bit for bit.

The product is the reference's dot_row per value (q8.rs:56-72). Both forms of
the copy are covered:
- three planes (block scales that differ within a row): rows whose
  block-scale exponents spread by the most the three weight planes hold (5),
  weights of -128 and 127, activations at i32::MIN / MAX (all four byte
  planes extreme), K up to the widest the int32 diagonal accumulators recover
  (18848), activations within 24 bits, ragged row and token counts, and a
  matrix one exponent too wide, which the tensor-core path refuses and the
  automatic path serves with the mma.sync GEMM;
- one plane (one scale a row, 128-token tiles): random signs, exponents from
  subnormal to the largest finite, blocks whose scale is +0 or -0 mixed into
  a row, rows with no non-zero scale, extreme weights and activations (totals
  that saturate), ragged shapes, K = 18848, 2048 tokens against the mma.sync
  GEMM, and the three-plane form of the same matrices.

The decode GEMV's one-scale-a-row form (one token; int32 plane sums over a
tile group, each row scaled once) is checked against the oracle and the
general GEMV over slice widths of 96 to 2048 columns and K up to 32768, with
extreme weights, scales and activations, and its refusals.
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


def spread_matrix(rng, rows, cols, base_ex, spread, q_extreme=False):
    """Q8_0 blocks whose fp16 scale exponents lie in [base_ex, base_ex + spread]
    for every row (random signs and mantissas); q uniform over all 256 byte
    values, or only -128 / 127 when q_extreme."""
    nb = rows * cols // 32
    ex = base_ex + rng.integers(0, spread + 1, size=nb)
    ex[:: max(1, cols // 32)] = base_ex + spread  # every row reaches both ends
    ex[1:: max(1, cols // 32)] = base_ex
    man = rng.integers(0, 1024, size=nb)
    sign = rng.integers(0, 2, size=nb)
    bits = (sign << 15) | (ex << 10) | man
    out = np.empty((nb, 34), np.uint8)
    out[:, 0] = bits & 0xFF
    out[:, 1] = (bits >> 8) & 0xFF
    if q_extreme:
        out[:, 2:] = np.where(rng.integers(0, 2, size=(nb, 32)) == 1, 0x7F, 0x80)
    else:
        out[:, 2:] = rng.integers(0, 256, size=(nb, 32), dtype=np.uint8)
    return out.reshape(-1)


def full_range_acts(rng, tokens, cols):
    r = rng.integers(I32_MIN, I32_MAX, size=(tokens, cols), dtype=np.int64, endpoint=True)
    sel = rng.integers(0, 17, size=(tokens, cols))
    r = np.where(sel == 0, I32_MAX, np.where(sel == 1, I32_MIN, np.where(sel == 2, 0, r)))
    return r.astype(np.int32)


def run(L, blocks, rows, cols, acts, path):
    import torch
    from iris_b200 import _lib
    h = C.c_void_p()
    _lib.check(L.iris_q8_upload_blocks(_lib.ptr(blocks, C.c_uint8), rows, cols, C.byref(h)), "upload")
    try:
        a = torch.from_numpy(np.ascontiguousarray(acts, np.int32)).cuda()
        out = torch.full((acts.shape[0], rows), 7, dtype=torch.int32, device="cuda")
        rc = L.iris_q8_product_device_path(h, a.data_ptr(), acts.shape[0], out.data_ptr(), None, path)
        torch.cuda.synchronize()
        return rc, out.cpu().numpy()
    finally:
        L.q8gpu_free(h)


@pytest.mark.parametrize("rows,cols,tokens,base_ex,spread", [
    (128, 128, 64, 10, 5),
    (200, 4096, 100, 1, 5),     # ragged rows and tokens; subnormal-adjacent exponents
    (130, 1536, 33, 25, 3),
    (64, 14336, 72, 12, 5),
    (40, 18848, 40, 20, 5),     # the widest K (a partial last K stage)
])
def test_tc_matches_oracle(L, O, rows, cols, tokens, base_ex, spread):
    from iris_b200 import _lib
    rng = np.random.default_rng(rows * 131 + cols + tokens)
    blocks = spread_matrix(rng, rows, cols, base_ex, spread)
    acts = full_range_acts(rng, tokens, cols)
    want = O.linear(acts, blocks, rows)
    rc, got = run(L, blocks, rows, cols, acts, _lib.PATH_TC)
    assert rc == 0, _lib.lib().iris_error(rc)
    assert np.array_equal(got, want), np.argwhere(got != want)[:5]


def test_tc_diagonal_sums_past_int32(L, O):
    """Activations i32::MAX / MIN (byte planes 255, 255, 255, 127 / 0, 0, 0,
    -128) against weights of 127 and -128 at the largest pre-scaled size:
    the diagonal sums leave the int32 range and come back exactly."""
    from iris_b200 import _lib
    rng = np.random.default_rng(5)
    rows, cols, tokens = 128, 14336, 64
    blocks = spread_matrix(rng, rows, cols, 15, 5, q_extreme=True)
    b = blocks.reshape(-1, 34)
    b[:, 0] = 0xFF  # mantissa 2047
    b[:, 1] = (b[:, 1] & 0xFC) | 0x03
    acts = np.where(rng.integers(0, 4, size=(tokens, cols)) == 0, I32_MIN, I32_MAX).astype(np.int32)
    acts[0, :] = I32_MAX
    want = O.linear(acts, blocks, rows)
    rc, got = run(L, blocks, rows, cols, acts, _lib.PATH_TC)
    assert rc == 0
    assert np.array_equal(got, want)


def test_tc_activations_within_24_bits(L, O):
    """Activations at the extremes of 24 bits (2^23 - 1, -2^23; byte plane 3
    the sign extension of plane 2) against the largest pre-scaled weights,
    then a 24-bit matrix with one full-range value in one stage of one token
    tile."""
    from iris_b200 import _lib
    rng = np.random.default_rng(23)
    rows, cols, tokens = 256, 14336, 128
    blocks = spread_matrix(rng, rows, cols, 15, 5, q_extreme=True)
    b = blocks.reshape(-1, 34)
    b[:, 0] = 0xFF
    b[:, 1] = (b[:, 1] & 0xFC) | 0x03
    acts = np.where(rng.integers(0, 2, size=(tokens, cols)) == 0, (1 << 23) - 1, -(1 << 23)).astype(np.int32)
    want = O.linear(acts, blocks, rows)
    rc, got = run(L, blocks, rows, cols, acts, _lib.PATH_TC)
    assert rc == 0 and np.array_equal(got, want)
    acts = rng.integers(-(1 << 23), 1 << 23, size=(tokens, cols)).astype(np.int32)
    acts[70, 5000] = 2**31 - 1
    acts[3, 9000] = -(2**31)
    want = O.linear(acts, blocks, rows)
    rc, got = run(L, blocks, rows, cols, acts, _lib.PATH_TC)
    assert rc == 0 and np.array_equal(got, want)


def test_tc_refuses_a_wider_spread_and_auto_falls_back(L, O):
    from iris_b200 import _lib
    rng = np.random.default_rng(11)
    rows, cols, tokens = 96, 512, 48
    blocks = spread_matrix(rng, rows, cols, 8, 6)
    acts = full_range_acts(rng, tokens, cols)
    want = O.linear(acts, blocks, rows)
    rc, _ = run(L, blocks, rows, cols, acts, _lib.PATH_TC)
    assert rc == 1  # cudaErrorInvalidValue: the matrix does not qualify
    rc, got = run(L, blocks, rows, cols, acts, _lib.PATH_AUTO)
    assert rc == 0 and np.array_equal(got, want)


def test_tc_equals_mma_gemm_at_2048_tokens(L):
    """M = 2048 (the sweep's largest): the tensor-core GEMM against the
    mma.sync GEMM on every output."""
    from iris_b200 import _lib
    rng = np.random.default_rng(2048)
    rows, cols, tokens = 2048, 2048, 2048
    blocks = spread_matrix(rng, rows, cols, 12, 4)
    acts = full_range_acts(rng, tokens, cols)
    rc, tc = run(L, blocks, rows, cols, acts, _lib.PATH_TC)
    assert rc == 0
    rc, mma = run(L, blocks, rows, cols, acts, _lib.PATH_GEMM)
    assert rc == 0
    assert np.array_equal(tc, mma)


def uniform_matrix(rng, rows, cols, q_extreme=False, exponents=(1, 30)):
    """Q8_0 blocks with one scale a row (random sign, exponent and mantissa),
    except blocks whose scale is +0 or -0 (about one in eight; their q stay
    random) and every seventh row with no non-zero scale at all."""
    nb_row = cols // 32
    ex = rng.integers(exponents[0], exponents[1] + 1, size=rows)
    ex[0], ex[-1] = exponents[1], 0  # the largest exponent; a subnormal row
    bits = (rng.integers(0, 2, size=rows) << 15) | (ex << 10) | rng.integers(0, 1024, size=rows)
    bits[0] = 0x7BFF  # 65504, the largest finite scale
    per_block = np.repeat(bits, nb_row).reshape(rows, nb_row)
    zero = rng.integers(0, 8, size=(rows, nb_row)) == 0
    per_block = np.where(zero, np.where(rng.integers(0, 2, size=(rows, nb_row)) == 0, 0x0000, 0x8000), per_block)
    per_block[::7] = 0x8000
    per_block = per_block.reshape(-1)
    nb = rows * nb_row
    out = np.empty((nb, 34), np.uint8)
    out[:, 0] = per_block & 0xFF
    out[:, 1] = (per_block >> 8) & 0xFF
    if q_extreme:
        out[:, 2:] = np.where(rng.integers(0, 2, size=(nb, 32)) == 1, 0x7F, 0x80)
    else:
        out[:, 2:] = rng.integers(0, 256, size=(nb, 32), dtype=np.uint8)
    return out.reshape(-1)


@pytest.mark.parametrize("rows,cols,tokens", [
    (128, 128, 128),
    (200, 4096, 100),   # ragged rows and tokens
    (130, 1536, 33),
    (64, 14336, 300),   # three 128-token tiles, the last partial
    (40, 18848, 129),   # the widest K
])
def test_one_plane_matches_oracle(L, O, rows, cols, tokens):
    from iris_b200 import _lib
    rng = np.random.default_rng(rows * 7 + cols + tokens)
    blocks = uniform_matrix(rng, rows, cols)
    acts = full_range_acts(rng, tokens, cols)
    want = O.linear(acts, blocks, rows)
    rc, got = run(L, blocks, rows, cols, acts, _lib.PATH_TC)
    assert rc == 0, _lib.lib().iris_error(rc)
    assert np.array_equal(got, want), np.argwhere(got != want)[:5]


def test_one_plane_extremes(L, O):
    """q of -128 / 127 under the largest scales against i32::MIN / MAX
    activations: every accumulator at its bound, totals far past the int32
    output (saturated by the rounding)."""
    from iris_b200 import _lib
    rng = np.random.default_rng(17)
    rows, cols, tokens = 256, 16384, 128
    blocks = uniform_matrix(rng, rows, cols, q_extreme=True, exponents=(28, 30))
    acts = np.where(rng.integers(0, 4, size=(tokens, cols)) == 0, I32_MIN, I32_MAX).astype(np.int32)
    acts[0, :] = I32_MAX
    acts[1, :] = I32_MIN
    want = O.linear(acts, blocks, rows)
    rc, got = run(L, blocks, rows, cols, acts, _lib.PATH_TC)
    assert rc == 0 and np.array_equal(got, want)


def test_one_plane_is_built_and_equals_three_planes_and_mma(L, O):
    """A one-scale-a-row matrix takes the one-plane form (asking the same
    handle for the three-plane form afterwards is refused); a fresh upload
    forced to three planes, and the mma.sync GEMM, give the same 2048 x 2048
    x 2048 product."""
    import torch
    from iris_b200 import _lib
    rng = np.random.default_rng(2049)
    rows, cols, tokens = 2048, 2048, 2048
    blocks = uniform_matrix(rng, rows, cols, exponents=(10, 16))
    acts = full_range_acts(rng, tokens, cols)
    h = C.c_void_p()
    _lib.check(L.iris_q8_upload_blocks(_lib.ptr(blocks, C.c_uint8), rows, cols, C.byref(h)), "upload")
    try:
        a = torch.from_numpy(acts).cuda()
        out = torch.zeros((tokens, rows), dtype=torch.int32, device="cuda")
        assert L.iris_q8_product_device_path(h, a.data_ptr(), tokens, out.data_ptr(), None, _lib.PATH_TC) == 0
        assert L.iris_q8_product_device_path(h, a.data_ptr(), tokens, out.data_ptr(), None, _lib.PATH_TC3) == 1
        torch.cuda.synchronize()
        one = out.cpu().numpy()
    finally:
        L.q8gpu_free(h)
    rc, three = run(L, blocks, rows, cols, acts, _lib.PATH_TC3)
    assert rc == 0
    rc, mma = run(L, blocks, rows, cols, acts, _lib.PATH_GEMM)
    assert rc == 0
    assert np.array_equal(one, mma) and np.array_equal(three, mma)
    sample = rng.choice(tokens, size=24, replace=False)
    assert np.array_equal(one[sample], O.linear(acts[sample], blocks, rows))


# ---- the decode GEMV's one-scale-a-row form (mma.sync on the byte planes) ----

def strict_row_matrix(rng, rows, cols, q_extreme=False, exponents=(0, 30)):
    """Q8_0 blocks where every block of a row has the same scale bits (the
    decode GEMV's one-scale-a-row condition): random signs, exponents and
    mantissas, row 0 at the largest finite scale (65504), row 1 subnormal,
    rows 2 and 3 at +0 and -0."""
    nb_row = cols // 32
    ex = rng.integers(exponents[0], exponents[1] + 1, size=rows)
    bits = (rng.integers(0, 2, size=rows) << 15) | (ex << 10) | rng.integers(0, 1024, size=rows)
    bits[0] = 0x7BFF
    if rows > 3:
        bits[1], bits[2], bits[3] = 0x03FF, 0x0000, 0x8000
    per_block = np.repeat(bits, nb_row)
    nb = rows * nb_row
    out = np.empty((nb, 34), np.uint8)
    out[:, 0] = per_block & 0xFF
    out[:, 1] = (per_block >> 8) & 0xFF
    if q_extreme:
        out[:, 2:] = np.where(rng.integers(0, 2, size=(nb, 32)) == 1, 0x7F, 0x80)
    else:
        out[:, 2:] = rng.integers(0, 256, size=(nb, 32), dtype=np.uint8)
    return out.reshape(-1)


@pytest.mark.parametrize("rows,cols", [
    (256, 4096),    # two 2048-column slices a tile group
    (100, 14336),   # seven slices, ragged rows
    (64, 3072),     # 1024-column slices
    (48, 384),      # one 384-column slice
    (40, 96),       # one 96-column slice: three blocks a row
    (32, 32768),    # the widest K
    (16, 2048),
])
def test_gemv_one_scale_a_row_matches_oracle(L, O, rows, cols):
    """The one-token product in the one-scale-a-row form against the oracle
    and against the general GEMV: full-range activations (all four byte
    planes, i32::MIN / MAX mixed in) and activations within 24 bits."""
    from iris_b200 import _lib
    rng = np.random.default_rng(rows * 3 + cols)
    blocks = strict_row_matrix(rng, rows, cols)
    for acts in (full_range_acts(rng, 1, cols), rng.integers(-(2**23), 2**23, size=(1, cols)).astype(np.int32)):
        want = O.linear(acts, blocks, rows)
        rc, got = run(L, blocks, rows, cols, acts, _lib.PATH_GEMV1)
        assert rc == 0, _lib.lib().iris_error(rc)
        assert np.array_equal(got, want), np.argwhere(got != want)[:5]
        rc, general = run(L, blocks, rows, cols, acts, _lib.PATH_GEMV)
        assert rc == 0 and np.array_equal(general, want)


def test_gemv_one_scale_a_row_extremes(L, O):
    """q of -128 / 127 under the largest scales against i32::MIN / MAX
    activations at K = 32768: row sums near 2^53 before the scale, totals far
    past the int32 output (saturated by the rounding)."""
    from iris_b200 import _lib
    rng = np.random.default_rng(5)
    rows, cols = 48, 32768
    blocks = strict_row_matrix(rng, rows, cols, q_extreme=True, exponents=(28, 30))
    for acts in (np.full((1, cols), I32_MIN, np.int32), np.full((1, cols), I32_MAX, np.int32),
                 np.where(rng.integers(0, 2, size=(1, cols)) == 0, I32_MIN, I32_MAX).astype(np.int32)):
        want = O.linear(acts, blocks, rows)
        rc, got = run(L, blocks, rows, cols, acts, _lib.PATH_GEMV1)
        assert rc == 0 and np.array_equal(got, want)


def test_gemv_one_scale_a_row_refusals(L):
    """Rows whose blocks differ in scale, and more than one token, are
    refused (cudaErrorInvalidValue)."""
    from iris_b200 import _lib
    rng = np.random.default_rng(6)
    mixed = spread_matrix(rng, 32, 2048, 10, 3)
    rc, _ = run(L, mixed, 32, 2048, full_range_acts(rng, 1, 2048), _lib.PATH_GEMV1)
    assert rc == 1
    ok = strict_row_matrix(rng, 32, 2048)
    rc, _ = run(L, ok, 32, 2048, full_range_acts(rng, 2, 2048), _lib.PATH_GEMV1)
    assert rc == 1

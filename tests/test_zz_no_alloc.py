"""The Q8_0 product entry point that allocates nothing, against the ordinary
device entry point on the same inputs.

iris_q8_product_device_noalloc keeps the GEMM path's byte planes in a fixed
16 MiB device array. Two calls are queued back to back on one stream with no
synchronisation between them, the second smaller than the first and on another
matrix, so that a stale plane from the first call would show in the second's
result. The file is named to be collected last, and passes alone too.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    from iris_b200 import build, _lib
    build.build()
    lib = _lib.lib()
    assert lib.q8gpu_init() == 0, "no usable CUDA device"
    return lib


def random_blocks(rng, rows, cols, max_exp=14):
    nb = rows * cols // 32
    v = rng.integers(0, 2**62, size=nb, dtype=np.int64)
    bits = ((v & 1) << 15) | (((v >> 20) % (max_exp + 1)) << 10) | ((v >> 4) & 0x3FF)
    out = np.empty((nb, 34), np.uint8)
    out[:, 0] = bits & 0xFF
    out[:, 1] = (bits >> 8) & 0xFF
    out[:, 2:] = rng.integers(0, 256, size=(nb, 32), dtype=np.uint8)
    return out.reshape(-1)


def random_acts(rng, tokens, cols):
    r = rng.integers(-(2**31), 2**31, size=(tokens, cols), dtype=np.int64)
    return (r >> rng.integers(0, 12, size=(tokens, cols))).astype(np.int32)


def upload(L, rng, rows, cols):
    from iris_b200 import _lib
    h = C.c_void_p()
    blocks = random_blocks(rng, rows, cols)
    _lib.check(L.iris_q8_upload_blocks(_lib.ptr(blocks, C.c_uint8), rows, cols, C.byref(h)), "upload")
    return h


def test_no_alloc_matches_the_device_entry_point_on_two_calls_in_a_row(L):
    import torch
    from iris_b200 import _lib
    rng = np.random.default_rng(0x5EED)
    cases = [(1024, 2048, 97), (512, 1024, 33), (768, 4096, 1)]  # (rows, cols, tokens)
    mats = [upload(L, rng, n, k) for n, k, _ in cases]
    acts = [torch.from_numpy(random_acts(rng, m, k)).cuda() for _, k, m in cases]
    stream = torch.cuda.Stream()
    got = [torch.full((m, n), -7, dtype=torch.int32, device="cuda") for n, _, m in cases]
    want = [torch.full((m, n), -7, dtype=torch.int32, device="cuda") for n, _, m in cases]
    torch.cuda.synchronize()
    for rep in range(2):
        # the no-alloc calls back to back on one stream, then the ordinary entry point
        for h, a, o, (n, k, m) in zip(mats, acts, got, cases):
            _lib.check(L.iris_q8_product_device_noalloc(h, a.data_ptr(), m, o.data_ptr(),
                                                        C.c_void_p(stream.cuda_stream)), "noalloc")
        stream.synchronize()
        for h, a, o, (n, k, m) in zip(mats, acts, want, cases):
            _lib.check(L.iris_q8_product_device(h, a.data_ptr(), m, o.data_ptr(), None), "device")
        torch.cuda.synchronize()
        for o, w, case in zip(got, want, cases):
            assert torch.equal(o, w), (rep, case)
            assert not torch.equal(o, torch.full_like(o, -7)), case
        for o in got:
            o.fill_(-7)
    for h in mats:
        L.q8gpu_free(h)


def test_no_alloc_refuses_inputs_beyond_its_scratch(L):
    import torch
    from iris_b200 import _lib
    rng = np.random.default_rng(7)
    rows, cols = 64, 4096
    h = upload(L, rng, rows, cols)
    tokens = _lib.NOALLOC_PLANES_BYTES // (cols * 4) + 1
    a = torch.zeros((tokens, cols), dtype=torch.int32, device="cuda")
    out = torch.full((tokens, rows), 5, dtype=torch.int32, device="cuda")
    code = L.iris_q8_product_device_noalloc(h, a.data_ptr(), tokens, out.data_ptr(), None)
    assert code == _lib.IRIS_ESCRATCH
    assert "16 MiB" in L.iris_error(code).decode()
    torch.cuda.synchronize()
    assert bool((out == 5).all())
    # the largest input that fits is accepted and equals the ordinary entry point
    tokens -= 1
    a = torch.from_numpy(random_acts(rng, tokens, cols)).cuda()
    got = torch.empty((tokens, rows), dtype=torch.int32, device="cuda")
    want = torch.empty_like(got)
    _lib.check(L.iris_q8_product_device_noalloc(h, a.data_ptr(), tokens, got.data_ptr(), None), "noalloc")
    _lib.check(L.iris_q8_product_device(h, a.data_ptr(), tokens, want.data_ptr(), None), "device")
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    L.q8gpu_free(h)

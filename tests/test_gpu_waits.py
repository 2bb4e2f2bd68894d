"""Bounded device waits on the GPU: a wait on a flag that nothing sets runs
out after about a second, the kernel records the give-up and returns, the
entry point reports IRIS_ESTALL, and the device stays usable: the next
product equals the oracle. Both kinds of wait the kernels use are covered
(an mbarrier phase, as the TMA and tensor-core pipelines wait; a global
arrival counter, as the persistent step's stages wait). No fault, trap or
endless loop is involved: the failure is a wait that gives up.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    from iris_b200 import build
    from oracle import oracle
    build.build()
    oracle.build()
    from iris_b200 import _lib
    lib = _lib.lib()
    assert lib.q8gpu_init() == 0
    return lib


@pytest.mark.parametrize("kind", [0, 1])
def test_a_wait_nothing_releases_reports_a_stall(L, kind):
    import time
    from iris_b200 import _lib
    assert L.iris_wait_probe(kind, 1) == 0  # released: completes
    t0 = time.monotonic()
    assert L.iris_wait_probe(kind, 0) == _lib.IRIS_ESTALL  # never released: gives up
    assert 0.5 < time.monotonic() - t0 < 30
    assert L.iris_wait_probe(kind, 1) == 0  # the fault word was cleared; the device still works


def test_products_after_a_stall_equal_the_oracle(L):
    from iris_b200 import _lib
    from iris_b200.tensor import Q8Matrix, Slab, linear_slab_from_source
    from oracle import oracle as O
    assert L.iris_wait_probe(1, 0) == _lib.IRIS_ESTALL
    rng = np.random.default_rng(5)
    w = _lib.synth_q8(5, 3, 0, 300, 512)
    x = rng.integers(-(1 << 20), 1 << 20, size=(40, 512)).astype(np.int32)
    m = Q8Matrix("w", w, 300, 512)
    got = linear_slab_from_source(Slab(x), m).data
    assert np.array_equal(got, O.linear(x, w, 300))

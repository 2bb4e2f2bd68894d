"""CPU checks of the product's boundary: the C-ABI library loads and exports
every symbol include/iris_b200.h declares, its host-side generator matches
itself, and the importer arithmetic in iris_b200.shapes matches the
reference's values. No compute call touches a GPU here."""
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def L():
    from iris_b200 import build
    build.build()
    from iris_b200 import _lib
    return _lib.lib()


def declared_functions():
    text = (ROOT / "include" / "iris_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b([a-z_][a-z0-9_]*)\s*\(", text)
    keywords = {"if", "defined", "sizeof"}
    return sorted({n for n in names if n not in keywords and (n.startswith("iris_") or n.startswith("q8gpu_"))})


def test_library_exports_every_declared_symbol(L):
    from iris_b200 import _lib
    names = declared_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), f"libiris_b200.so does not export {n}"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    # and nothing the binding declares is missing from the header
    assert set(_lib.SIGNATURES) == set(names)


def test_error_strings(L):
    from iris_b200 import _lib
    assert "not finite" in _lib.error_string(_lib.IRIS_ESCALE)
    assert _lib.error_string(0) == "no error"
    assert L.q8gpu_error(_lib.IRIS_EINVAL).decode() == _lib.error_string(_lib.IRIS_EINVAL)


def test_host_synth_is_deterministic_and_in_range(L):
    from iris_b200 import _lib
    a = _lib.synth_q8(7, 3, 0, 16, 64)
    b = _lib.synth_q8(7, 3, 0, 16, 64)
    c = _lib.synth_q8(8, 3, 0, 16, 64)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    blocks = a.reshape(-1, 34)
    q = blocks[:, 2:].view(np.int8)
    assert q.min() >= -127 and q.max() <= 127
    scales = blocks[:, 0].astype(np.uint16) | (blocks[:, 1].astype(np.uint16) << 8)
    assert ((scales >> 10) & 0x1F).max() < 31  # finite
    # one scale per output row (per-row variant)
    per_row = scales.reshape(16, 2)
    assert (per_row[:, 0] == per_row[:, 1]).all()
    pb = _lib.synth_q8(7, 3, 0, 16, 64, per_block=True).reshape(-1, 34)
    pbs = (pb[:, 0].astype(np.uint16) | (pb[:, 1].astype(np.uint16) << 8)).reshape(16, 2)
    assert (pbs[:, 0] != pbs[:, 1]).any()
    v = _lib.synth_values(7, 10, 0, 1000, 0)
    assert v.min() >= 65536 - 8192 and v.max() < 65536 + 8192


def test_importer_arithmetic_matches_the_reference():
    from iris_b200 import shapes
    assert shapes.attention_scale_q32(128) == 379_625_062  # mistral.rs:279
    assert shapes.attention_scale_q32(1) == 2**32 - 1
    f = shapes.yarn_inverse_frequencies(1_000_000, 64, 16, 20, 37)
    assert f[0] == 1 << 32 and shapes.yarn_inverse_frequencies(1_000_000, 48, 16, 20, 37) is None
    assert shapes.f32_to_acc(1e-5) == 42950 and shapes.f32_to_acc(1e-6) == 4295
    assert shapes.f32_to_act(1.0) == 65536 and shapes.f32_to_act(-0.5) == -32768
    # Gemma-4 E2B scalars from runtime/model-artifacts/gemma-4-E2B-q8/manifest.json
    e2b = shapes.GemmaConfig("e2b", layers=35, hidden=1536, ffn=6144, heads=8, kv_heads=1, head_dim=256,
                             vocab=262144, ple_width=256, softcap=30.0)
    assert e2b.embedding_scale == 2568476
    assert e2b.ple_embedding_scale == 1048576
    assert e2b.ple_projection_scalar == 1672
    assert e2b.ple_input_scale == 46341
    assert e2b.softcap_bits == 1966080


def test_against_the_oracle_tables():
    """The product's host tables equal the oracle's."""
    import ctypes as C
    from iris_b200 import shapes
    from oracle import oracle as O
    O.build()
    L = O.lib()
    for d in [32, 64, 128, 256]:
        assert shapes.attention_scale_q32(d) == L.oracle_attention_scale_q32(d)
    for args in [(1_000_000, 64, 1, 0, 1), (1_000_000, 64, 16, 20, 37), (10_000, 16, 1, 0, 1)]:
        out = np.zeros(args[1], np.int64)
        L.oracle_yarn_inverse_frequencies(*args, O.ptr(out, C.c_int64))
        assert shapes.yarn_inverse_frequencies(*args) == out.tolist()
    for x in [1e-5, 1e-6, 0.1, 3.0e-8, 30.0, 45.254833995939045, 2 ** -0.5]:
        assert shapes.f32_to_acc(x) == L.oracle_f32_to_acc(x)
        assert shapes.f32_to_act(x) == L.oracle_f32_to_act(x)


def test_shard_synthesis_is_a_block_of_the_full_tensor(L):
    """A tensor-parallel rank synthesizes its rows or columns of each tensor:
    the blocks equal the corresponding blocks of the full tensor (the shard
    layout of iris_model_create_mistral_tp)."""
    from iris_b200 import _lib
    seed, rows, cols = 77, 48, 256
    for per_block in (False, True):
        full = _lib.synth_q8(seed, 9, 3, rows, cols, per_block).reshape(rows, cols // 32, 34)
        for row0, nrows, col0, ncols in [(0, 48, 0, 256), (16, 16, 0, 256), (0, 48, 128, 128), (8, 24, 64, 96)]:
            blk = _lib.synth_q8_block(seed, 9, 3, nrows, ncols, row0, col0, cols, per_block)
            want = full[row0:row0 + nrows, col0 // 32:(col0 + ncols) // 32]
            assert np.array_equal(blk.reshape(nrows, ncols // 32, 34), want), (row0, nrows, col0, ncols, per_block)

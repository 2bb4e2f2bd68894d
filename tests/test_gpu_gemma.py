"""GPU parity of the gemma-dense path against the CPU oracle, bit for bit.

- the benchmark's config 3 shapes (Gemma-2B architecture: 2048 hidden, 8 query
  heads over one kv head of 256, GeGLU 16384, a 256,000-row tied head with
  softcap 30, PLE width 256, a 768-position sliding window), two of its 18
  layers: a short prompt and greedy steps (every logit of the 256k head), and
  a prompt longer than the window (two prefill ranges, the window cutting the
  prefix);
- the chain's gemma stage (iris_gemma_layer_range, prefill_range.rs:82-172)
  stage by stage against the oracle's stages: every stage's record digest
  (rows and own K/V), for the parity-shaped model (16-position window,
  layers sharing their donors' K/V, partial rotary, PLE) in ranges of 512,
  20 and 7 rows, and for the Gemma-2B slice across its window;
- PLE rows of token ids (iris_model_ple_rows, view_kernels.rs:59-99);
- the stage's refusal of carried keys that do not cover the window
  (IRIS_EWINDOW, the reference's cache-coverage fault);
- a gemma bundle in the .detwgt format with an untied head and layer
  scalars, read by iris_b200.detwgt, generating as the oracle does.
"""
import dataclasses

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def built():
    from iris_b200 import build
    from oracle import oracle
    build.build()
    oracle.build()


def seeded_prompt(seed, n, vocab):
    return np.random.default_rng(seed).integers(0, vocab, size=n).tolist()


def gemma_2b_slice():
    from iris_b200.shapes import gemma_2b
    return dataclasses.replace(gemma_2b(), name="gemma-2b-2l", layers=2)


@pytest.fixture(scope="module")
def g2b():
    from iris_b200.model import DeviceModel, synth_host_weights
    from oracle.models import OracleModel
    cfg = gemma_2b_slice()
    w = synth_host_weights(cfg, 0x2B)
    dm = DeviceModel(cfg, weights=w)
    yield cfg, w, dm, OracleModel(cfg, w)
    dm.close()


def assert_same(got, want):
    gt, gl = got
    wt, wl = want
    assert gt == wt, f"tokens differ: {gt} vs {wt}"
    for p in range(len(wt)):
        assert np.array_equal(gl[p], wl[p]), f"logits of pass {p} differ"


@pytest.mark.parametrize("n_prompt,steps", [(40, 6), (800, 2)])
def test_gemma_2b_decode_matches_the_oracle(g2b, n_prompt, steps):
    """40 tokens: one range on the tensor-core GEMM, then decode steps at
    head_dim 256 with the 256k softcapped head; 800 tokens: ranges of 512
    and 288, queries past position 767 seeing only their window."""
    cfg, w, dm, om = g2b
    prompt = seeded_prompt(n_prompt, n_prompt, cfg.vocab)
    want = om.generate(prompt, steps)
    sess = dm.session(n_prompt + steps + 8)
    assert_same(sess.generate(prompt, steps, want_logits=True), want)
    sess.close()


def test_gemma_2b_ple_rows_and_chain_stages_match_the_oracle(g2b):
    from iris_b200 import records
    from oracle.models import OracleStages, gemma_ple_rows
    cfg, w, dm, om = g2b
    ids = seeded_prompt(0x2B1, 800, cfg.vocab)
    assert np.array_equal(dm.ple_rows(ids[:40]), gemma_ple_rows(om, ids[:40]))
    got = records.chain_records(dm, ids, range_size=512)
    want = records.chain_records(OracleStages(om), ids, range_size=512)
    assert got == want and len(got) == 2 * cfg.layers


@pytest.mark.parametrize("range_size", [512, 20, 7])
def test_parity_gemma_chain_stages_match_the_oracle(range_size):
    """The window (16) is shorter than most ranges, so each range's carried
    keys are pruned; layers 2 and 3 attend over layers 0 and 1's keys."""
    from iris_b200 import records
    from iris_b200.model import DeviceModel, synth_host_weights
    from iris_b200.shapes import parity_gemma
    from oracle.models import OracleModel, OracleStages
    cfg = parity_gemma()
    w = synth_host_weights(cfg, 0x6E)
    dm = DeviceModel(cfg, weights=w)
    ids = seeded_prompt(0x6E + range_size, 600 if range_size == 512 else 45, cfg.vocab)
    got = records.chain_records(dm, ids, range_size=range_size)
    want = records.chain_records(OracleStages(OracleModel(cfg, w)), ids, range_size=range_size)
    assert got == want
    dm.close()


def test_gemma_stage_refuses_keys_that_do_not_cover_the_window():
    from iris_b200 import _lib
    from iris_b200.model import DeviceModel
    from iris_b200.shapes import parity_gemma
    cfg = parity_gemma()
    dm = DeviceModel(cfg, seed=3)
    kvd = cfg.kv_heads * cfg.head_dim
    rows = np.zeros((4, cfg.hidden), np.int32)
    ple = np.zeros((4, cfg.ple_width), np.int32)
    start = 30  # layer 0 slides over 16 positions: it needs carried keys 15..29
    k = np.zeros((15, kvd), np.int32)
    good = (np.arange(15, 30, dtype=np.uint32), k, k)
    dm.gemma_layer_range(0, rows, start, ple, prior=good)
    for bad in ((np.arange(16, 30, dtype=np.uint32), k[:14], k[:14]),               # starts too late
                (np.delete(np.arange(14, 30, dtype=np.uint32), 5), k, k),           # a gap
                (np.arange(15, 30, dtype=np.uint32)[::-1].copy(), k, k),            # out of order
                (np.arange(16, 31, dtype=np.uint32), k, k)):                        # past the range start
        with pytest.raises(_lib.IrisError) as e:
            dm.gemma_layer_range(0, rows, start, ple, prior=bad)
        assert e.value.code == _lib.IRIS_EWINDOW
    with pytest.raises(_lib.IrisError) as e:  # a sharing layer without its donor's keys of the range
        dm.gemma_layer_range(2, rows, start, ple, prior=good, donor=good)
    assert e.value.code == _lib.IRIS_EWINDOW
    dm.close()


@pytest.mark.parametrize("n_prompt,steps", [(5, 1), (15, 8), (34, 8)])
def test_gemma_detwgt_bundle_matches_the_oracle(tmp_path, n_prompt, steps):
    """A gemma-dense bundle in the reference's .detwgt format (written here
    from seeded weights under the import's tensor names, with per-layer
    `layer_scalar` tensors, one layer without one, and an untied lm_head;
    config.json shaped as the reference's gemma parity bundle) loaded
    through iris_b200.detwgt: every logit and token of a prompt short of,
    near and over the 16-key window and its greedy steps equals the
    oracle's on the same weights."""
    import json
    from iris_b200 import detwgt
    from iris_b200.model import DeviceModel, synth_host_weights, tensor_table
    from oracle.models import OracleModel
    from test_detwgt import gemma_text_config, write_detwgt
    config = {"model_type": "gemma3n", "text_config": gemma_text_config()}
    scalars = [1 << 16, 3 << 15, 0, 1 << 16]
    cfg = detwgt.gemma_config(config, 512, scalars)
    w = synth_host_weights(cfg, 0x6E)
    assert ("HEAD", -1) in w
    names = detwgt.gemma_tensor_names(cfg.layers)
    table = tensor_table(cfg)
    tensors = []
    for key, arr in w.items():
        kind, rows, cols, _ = table[key]
        dims = [cols] if kind == "values" and rows == 1 else [rows, cols]
        tensors.append((names[key][0], dims, 8 if kind == "q8" else 32, arr))
    for l, s in enumerate(scalars):
        if s:
            tensors.append((f"model.language_model.layers.{l}.layer_scalar", [1], 32, np.array([s])))
    write_detwgt(tmp_path / "model.detwgt", tensors)
    (tmp_path / "config.json").write_text(json.dumps(config))
    cfg2, w2, f = detwgt.load_bundle(tmp_path)
    assert cfg2.family == "gemma" and not cfg2.tied and cfg2.layer_scalars == scalars
    dm = DeviceModel(cfg2, weights=w2)
    prompt = seeded_prompt(n_prompt, n_prompt, cfg2.vocab)
    sess = dm.session(64)
    got = sess.generate(prompt, steps, want_logits=True)
    want = OracleModel(cfg2, {k: np.array(v) for k, v in w2.items()}).generate(prompt, steps)
    assert_same(got, want)
    sess.close()
    dm.close()
    del w2
    f.close()

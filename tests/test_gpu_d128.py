"""GPU parity at head_dim 128: the shapes the Mistral-7B benchmark times,
against the CPU oracle, bit for bit.

Ranges of 32 or more queries at head_dim 128 run the prefill attention on the
tensor cores (byte-plane scores into seven int32 diagonals, the exp-term
table, the integer softmax to weight planes, weights x values into six
diagonals); every test here checks that those kernels ran (the model's
attention-range counters) and that their results equal the oracle's
(kernels/src/mistral/layer.rs:274-318, det-num ops.rs:233-276,508-556,
mistral.rs:130-145).

- a small head_dim-128 model (2 layers, 4 query heads over 1 kv head, the
  7B model's group of 4): prompts that cross the 128-key tiles and the
  512-row ranges, every logit of the prefill and of the decode steps on both
  decode paths, and the tensor-core against the CUDA-core prefill attention;
- one Mistral-7B layer (4096 hidden, 14336 FFN, 32 heads over 8 kv heads)
  through the chain's layer-range entry point at the starts and lengths of a
  4096-token claim;
- two Mistral-7B layers with the 7B vocabulary: a 64-token prompt and 8
  greedy steps on the persistent step (the instantiation the benchmark
  times) and on the kernel graph;
- the exp-term table, every entry, against softmax_exp_term.
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


def small_d128():
    from iris_b200.shapes import MistralConfig
    return MistralConfig("mistral-d128-small", layers=2, hidden=256, ffn=512, heads=4, kv_heads=1,
                         head_dim=128, vocab=512, rope_base=1_000_000, max_positions=16384, tied=True)


def assert_same(got, want):
    gt, gl = got
    wt, wl = want
    assert gt == wt, f"tokens differ: {gt} vs {wt}"
    for p in range(len(wt)):
        assert np.array_equal(gl[p], wl[p]), f"logits of pass {p} differ"


@pytest.mark.parametrize("n_prompt", [40, 300, 600])
def test_small_d128_model_matches_the_oracle(n_prompt):
    """40 tokens: one 64-query tile over one 128-key tile; 300: three key
    tiles; 600: two ranges (512 + 88), the second over 512 cached rows. Every
    logit of the prefill and of 8 decode steps, both decode paths."""
    from iris_b200.model import DeviceModel, synth_host_weights
    from oracle.models import OracleModel
    cfg = small_d128()
    w = synth_host_weights(cfg, 0xD128 + n_prompt)
    prompt = seeded_prompt(n_prompt, n_prompt, cfg.vocab)
    want = OracleModel(cfg, w).generate(prompt, 8)
    dm = DeviceModel(cfg, weights=w)
    for path in ("step", "graph"):
        sess = dm.session(n_prompt + 16)
        sess.set_decode_path(path)
        assert sess.decode_path == path
        assert_same(sess.generate(prompt, 8, want_logits=True), want)
        sess.close()
    tc, cc = dm.attention_ranges()
    ranges = 2 * cfg.layers if n_prompt > 512 else cfg.layers
    assert (tc, cc) == (2 * ranges, 0), (tc, cc)  # both sessions' prefills on the tensor cores
    dm.close()


def test_small_d128_layer_ranges_match_the_oracle():
    """The chain stage (mistral/stage.rs:172-226) at head_dim 128 with carried
    K/V of random values: rows and own K/V. Starts that are not multiples of
    the 64-query or 128-key tiles; lengths from the 32-row minimum up."""
    from iris_b200.model import DeviceModel, synth_host_weights
    from oracle.models import OracleModel
    cfg = small_d128()
    w = synth_host_weights(cfg, 0xD1)
    dm = DeviceModel(cfg, weights=w)
    om = OracleModel(cfg, w)
    rng = np.random.default_rng(0xD1)
    kvd = cfg.kv_heads * cfg.head_dim
    rows = rng.integers(-(4 << 16), 4 << 16, size=(512, cfg.hidden)).astype(np.int32)
    cases = [(0, 0, 32), (1, 0, 512), (0, 100, 200), (1, 511, 64), (0, 1000, 33), (1, 1337, 97)]
    for layer, start, m in cases:
        prior_k = rng.integers(-(1 << 22), 1 << 22, size=(start, kvd)).astype(np.int32)
        prior_v = rng.integers(-(1 << 22), 1 << 22, size=(start, kvd)).astype(np.int32)
        got = dm.layer_range(layer, rows[:m], start, prior_k, prior_v)
        want = om.mistral_layer_range(layer, rows[:m], start, prior_k, prior_v)
        for g, wnt, what in zip(got, want, ("rows", "k", "v")):
            assert np.array_equal(g, wnt), (layer, start, m, what)
    assert dm.attention_ranges() == (len(cases), 0)


def test_small_d128_tensor_core_and_cuda_core_attention_agree():
    """The same 600-token prefill with the tensor-core products and attention
    and with the mma.sync products and the CUDA-core attention
    (attn_prefill_group_kernel): every logit and K/V row equal."""
    from iris_b200.model import DeviceModel, synth_host_weights
    cfg = small_d128()
    w = synth_host_weights(cfg, 0xD3)
    prompt = seeded_prompt(0xD3, 600, cfg.vocab)
    out = {}
    for mode in ("auto", "mma"):
        dm = DeviceModel(cfg, weights=w)
        dm.set_gemm(mode)
        sess = dm.session(len(prompt) + 8)
        tok, logits = sess.prefill(prompt, want_logits=True)
        out[mode] = [tok, logits] + [x for l in range(cfg.layers) for x in sess.kv(l, 0, len(prompt))]
        tc, cc = dm.attention_ranges()
        assert (tc > 0, cc > 0) == ((True, False) if mode == "auto" else (False, True))
        sess.close()
        dm.close()
    for x, y in zip(out["auto"], out["mma"]):
        assert np.array_equal(np.asarray(x), np.asarray(y))


def test_mistral_7b_layer_ranges_match_the_oracle():
    """One Mistral-7B layer over the ranges of a 4096-token claim (first
    range, a whole 512-row range, the middle, the last range over 3584
    carried rows), with random carried K/V: rows and own K/V bit for bit. The
    products run on the tcgen05 GEMM at K = 4096 and 14336, the attention on
    the tensor-core kernels at head_dim 128 and a GQA group of 4."""
    from iris_b200.model import DeviceModel, synth_host_weights
    from iris_b200.shapes import mistral_7b
    from oracle.models import OracleModel
    cfg = dataclasses.replace(mistral_7b(), name="mistral-7b-1l", layers=1)
    w = synth_host_weights(cfg, 0x7B1)
    dm = DeviceModel(cfg, weights=w)
    om = OracleModel(cfg, w)
    rng = np.random.default_rng(0x7B1)
    kvd = cfg.kv_heads * cfg.head_dim
    rows = rng.integers(-(4 << 16), 4 << 16, size=(512, cfg.hidden)).astype(np.int32)
    cases = [(0, 32), (0, 512), (1792, 256), (3584, 512)]
    for start, m in cases:
        prior_k = rng.integers(-(1 << 20), 1 << 20, size=(start, kvd)).astype(np.int32)
        prior_v = rng.integers(-(1 << 20), 1 << 20, size=(start, kvd)).astype(np.int32)
        got = dm.layer_range(0, rows[:m], start, prior_k, prior_v)
        want = om.mistral_layer_range(0, rows[:m], start, prior_k, prior_v)
        for g, wnt, what in zip(got, want, ("rows", "k", "v")):
            assert np.array_equal(g, wnt), (start, m, what)
    assert dm.attention_ranges() == (len(cases), 0)
    assert dm.tc_matrices()[0] == 4  # q|k|v, o, gate|up, down on the tensor-core copy


def test_mistral_7b_two_layers_decode_matches_the_oracle():
    """Two Mistral-7B layers with the 7B head (32000 x 4096, untied): a
    64-token prompt (tensor-core prefill) and 8 greedy steps on the
    persistent step kernel (blocks of 16 positions x 4 heads, the benchmark's
    instantiation) and on the kernel graph; every logit of every pass."""
    from iris_b200.model import DeviceModel, synth_host_weights
    from iris_b200.shapes import mistral_7b
    from oracle.models import OracleModel
    cfg = dataclasses.replace(mistral_7b(), name="mistral-7b-2l", layers=2)
    w = synth_host_weights(cfg, 0x7B2)
    prompt = seeded_prompt(0x7B2, 64, cfg.vocab)
    want = OracleModel(cfg, w).generate(prompt, 8)
    dm = DeviceModel(cfg, weights=w)
    for path in ("step", "graph"):
        sess = dm.session(len(prompt) + 16)
        sess.set_decode_path(path)
        assert sess.decode_path == path
        if path == "step":
            assert sess.step_plan["why"] == 0 and sess.attention_plan["heads_per_block"] == 4
        assert_same(sess.generate(prompt, 8, want_logits=True), want)
        sess.close()
    assert dm.attention_ranges()[0] == 2 * cfg.layers
    dm.close()


def test_exp_term_table_matches_softmax_exp_term():
    """Every distance the many-query softmax looks up (ops.rs:508-556 via
    softmax_exp_term_act): 0 gives 2^32, 1 .. 2^20 - 1 the table's entries,
    2^20 (16.0 in Q16.16) and beyond give 0."""
    import ctypes as C
    from iris_b200 import _lib
    from oracle import oracle as O
    n = (1 << 20) + 64
    got = np.empty(n, np.uint64)
    _lib.check(_lib.lib().iris_softmax_exp_terms(0, n, got.ctypes.data_as(C.POINTER(C.c_uint64))),
               "iris_softmax_exp_terms")
    f = O.lib().oracle_softmax_exp_term
    # the oracle takes delta = sub_sat(logit, max) << 16 as an Acc value
    for i in (0, 1, 2, 3, 1000, 65535, 65536, (1 << 20) - 1, 1 << 20, (1 << 20) + 1, n - 1):
        assert int(got[i]) == f(-(i << 16)) & ((1 << 64) - 1), i
    want = np.fromiter((f(-(i << 16)) for i in range(n)), np.int64, n).astype(np.uint64)
    assert np.array_equal(got, want)
    far = np.empty(4, np.uint64)
    _lib.check(_lib.lib().iris_softmax_exp_terms((1 << 31) - 4, 4, far.ctypes.data_as(C.POINTER(C.c_uint64))),
               "iris_softmax_exp_terms")
    assert not far.any()

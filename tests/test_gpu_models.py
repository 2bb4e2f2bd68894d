"""GPU parity of whole passes: the direct decode loop (prefill, decode steps,
greedy selection, EOS) and the chain's per-layer stage, against the CPU
oracle on the same seeded weights. Bit-exact: every logit of every pass,
every selected token, every K/V row and every output activation.

Configurations: BASELINE config 1 (tiny Gemma: 32-token prompt, 64 greedy
steps), a parity-bundle-shaped mistral-dense model, and a small gemma-dense
model with a sliding window, K/V-sharing layers, partial rotary and softcap.
"""
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


def run_both(cfg, seed, prompt, steps, per_block=False, eos=(), attn="auto", path="auto"):
    from iris_b200.model import DeviceModel, synth_host_weights
    from oracle.models import OracleModel
    w = synth_host_weights(cfg, seed, per_block)
    dm = DeviceModel(cfg, weights=w)
    sess = dm.session(len(prompt) + steps + 8)
    sess.set_attention(attn)
    sess.set_decode_path(path)
    got = sess.generate(prompt, steps, eos, want_logits=True)
    want = OracleModel(cfg, w).generate(prompt, steps, eos)
    return dm, sess, w, got, want


def assert_same(got, want):
    gt, gl = got
    wt, wl = want
    assert gt == wt, f"tokens differ: {gt} vs {wt}"
    for p in range(len(wt)):
        assert np.array_equal(gl[p], wl[p]), f"logits of pass {p} differ"


def test_device_synthesis_equals_host_synthesis():
    from iris_b200.model import DeviceModel, synth_host_weights, tensor_table
    from iris_b200.shapes import parity_gemma
    cfg = parity_gemma()
    dm = DeviceModel(cfg, seed=5)
    w = synth_host_weights(cfg, 5)
    for key in tensor_table(cfg):
        assert np.array_equal(dm.get(key), w[key]), key


def test_tiny_gemma_config_1():
    from iris_b200.shapes import tiny_gemma
    cfg = tiny_gemma()
    prompt = seeded_prompt(1, 32, cfg.vocab)
    _, _, _, got, want = run_both(cfg, 0x11, prompt, 64)
    assert_same(got, want)
    assert len(got[0]) == 64


def test_parity_mistral_prefill_and_decode():
    """Both decode paths: the persistent step (the default for
    mistral-dense) and the graph of one kernel per operation."""
    from iris_b200.shapes import parity_mistral
    cfg = parity_mistral()
    for seed, per_block in [(3, False), (4, True)]:
        prompt = seeded_prompt(seed, 19, cfg.vocab)
        for path in ("auto", "graph"):
            dm, sess, w, got, want = run_both(cfg, seed, prompt, 12, per_block, path=path)
            assert sess.decode_path == ("step" if path == "auto" else "graph"), sess.step_plan
            assert_same(got, want)


def test_saturating_residual_norms():
    """Embedding rows near the Q16.16 limit (every block scale 16000): the
    residual stream's sum of squares saturates at i64::MAX in every norm
    (add_sat_nonneg, ops.rs:98-114). Both decode paths against the oracle:
    the persistent step takes that sum from the residual epilogues, the graph
    path from a block-wide reduction."""
    from iris_b200.model import DeviceModel, synth_host_weights
    from iris_b200.shapes import parity_mistral
    from oracle.models import OracleModel
    cfg = parity_mistral()
    w = synth_host_weights(cfg, 41)
    emb = w[("EMBED", -1)].reshape(-1, 34).copy()
    emb[:, 0:2] = np.frombuffer(np.float16(16000.0).tobytes(), np.uint8)
    w[("EMBED", -1)] = emb.reshape(-1)
    prompt = seeded_prompt(41, 9, cfg.vocab)
    want = OracleModel(cfg, w).generate(prompt, 6)
    for path in ("auto", "graph"):
        dm = DeviceModel(cfg, weights=w)
        sess = dm.session(32)
        sess.set_decode_path(path)
        assert sess.decode_path == ("step" if path == "auto" else "graph")
        assert_same(sess.generate(prompt, 6, want_logits=True), want)
        sess.close()
        dm.close()


def test_wide_ffn_model():
    """A parity-bundle-shaped model with an 8192-wide FFN (four 2048-column
    slices a down row, 32 KB of input planes) against the oracle, on both
    decode paths."""
    import dataclasses
    from iris_b200.shapes import parity_mistral
    cfg = dataclasses.replace(parity_mistral(), name="parity-mistral-ffn8192", ffn=8192)
    prompt = seeded_prompt(43, 17, cfg.vocab)
    for path in ("auto", "graph"):
        dm, sess, w, got, want = run_both(cfg, 43, prompt, 8, path=path)
        assert sess.decode_path == ("step" if path == "auto" else "graph")
        assert_same(got, want)


def test_step_matches_graph_on_mistral_7b_shapes():
    """The persistent step against the kernel-per-operation pass (itself
    pinned to the oracle) on the Mistral-7B layer shapes (2 of its 32 layers):
    4096 hidden, 14336 FFN, 32 heads over 8 kv heads of 128, 32000 vocab;
    a 700-token prompt so that every attention block holds several rows.
    Every logit of every pass, every token and the K/V rows agree."""
    import dataclasses
    from iris_b200.model import DeviceModel
    from iris_b200.shapes import mistral_7b
    cfg = dataclasses.replace(mistral_7b(), name="mistral-7b-2l", layers=2)
    dm = DeviceModel(cfg, seed=0x7B)
    prompt = seeded_prompt(0x7B, 700, cfg.vocab)
    out = {}
    for path in ("step", "graph"):
        sess = dm.session(len(prompt) + 16)
        sess.set_decode_path(path)
        assert sess.decode_path == path
        toks, logits = sess.generate(prompt, 10, want_logits=True)
        batched, _ = sess.generate(prompt, 10)  # device-resident loop with history
        assert batched == toks
        out[path] = (toks, logits, sess.kv(1, len(prompt) - 2, 10))
        sess.close()
    assert out["step"][0] == out["graph"][0]
    assert np.array_equal(out["step"][1], out["graph"][1])
    for a, b in zip(out["step"][2], out["graph"][2]):
        assert np.array_equal(a, b)


def test_parity_gemma_window_donors_softcap():
    from iris_b200.shapes import parity_gemma
    cfg = parity_gemma()
    prompt = seeded_prompt(7, 21, cfg.vocab)  # crosses the 16-position window
    _, _, _, got, want = run_both(cfg, 7, prompt, 14)
    assert_same(got, want)


def test_single_token_prompt():
    """A one-row prompt pass takes the single-row attention path with a host
    position (both families)."""
    from iris_b200.shapes import parity_gemma, parity_mistral
    for cfg in (parity_mistral(), parity_gemma()):
        prompt = seeded_prompt(13, 1, cfg.vocab)
        _, _, _, got, want = run_both(cfg, 13, prompt, 5)
        assert_same(got, want)


def test_three_launch_decode_attention():
    """The split (three-launch) decode attention, kept for shapes the cluster
    kernel does not serve, on both families."""
    from iris_b200.shapes import parity_gemma, parity_mistral
    for cfg, seed in ((parity_mistral(), 21), (parity_gemma(), 22)):
        prompt = seeded_prompt(seed, 23, cfg.vocab)
        _, _, _, got, want = run_both(cfg, seed, prompt, 9, attn="split")
        assert_same(got, want)


def test_cluster_decode_attention():
    """The thread-block-cluster decode attention (the path for capacities the
    whole-GPU launch does not hold), on both families."""
    from iris_b200.shapes import parity_gemma, parity_mistral
    for cfg, seed in ((parity_mistral(), 23), (parity_gemma(), 24)):
        prompt = seeded_prompt(seed, 45, cfg.vocab)
        _, _, _, got, want = run_both(cfg, seed, prompt, 7, attn="cluster")
        assert_same(got, want)


def test_long_context_attention():
    """1100 positions: the whole-GPU launch holds tens of positions a block,
    and every block of a cluster streams several 32-position key and value
    tiles."""
    from iris_b200.shapes import parity_mistral
    cfg = parity_mistral()
    prompt = seeded_prompt(31, 1100, cfg.vocab)
    for attn in ("auto", "cluster"):
        _, _, _, got, want = run_both(cfg, 31, prompt, 4, attn=attn)
        assert_same(got, want)


def test_long_prompt_crosses_device_ranges():
    """A 600-token prompt is processed as two device ranges (512 + 88), both
    through the tensor-core GEMM (ranges of 32 or more tokens)."""
    from iris_b200.shapes import parity_mistral
    cfg = parity_mistral()
    prompt = seeded_prompt(9, 600, cfg.vocab)
    dm, _, _, got, want = run_both(cfg, 9, prompt, 3)
    assert_same(got, want)
    n, nbytes = dm.tc_matrices()
    assert n == 4 * cfg.layers and nbytes > 0  # every layer product took the tensor-core copy


@pytest.mark.parametrize("per_block", [False, True])
def test_prefill_tensor_core_and_mma_gemms_agree(per_block):
    """The same prefill (ranges of 512 and 88 tokens) through the tcgen05 GEMM
    and through the mma.sync GEMM: every logit and every K/V row equal."""
    from iris_b200.model import DeviceModel, synth_host_weights
    from iris_b200.shapes import parity_mistral
    cfg = parity_mistral()
    w = synth_host_weights(cfg, 41, per_block)
    prompt = seeded_prompt(41, 600, cfg.vocab)
    out = {}
    for mode in ("auto", "mma"):
        dm = DeviceModel(cfg, weights=w)
        dm.set_gemm(mode)
        sess = dm.session(len(prompt) + 8)
        tok, logits = sess.prefill(prompt, want_logits=True)
        kvs = [sess.kv(l, 0, len(prompt)) for l in range(cfg.layers)]
        out[mode] = (tok, logits, *[x for kv in kvs for x in kv])
        assert (dm.tc_matrices()[0] > 0) == (mode == "auto")
    a, b = out["auto"], out["mma"]
    assert a[0] == b[0]
    for x, y in zip(a[1:], b[1:]):
        assert np.array_equal(np.asarray(x), np.asarray(y))


def test_eos_stops_the_loop_and_batches_agree():
    """generate without logits runs batched graph replays; with an EOS id the
    loop stops after it (executor.rs:163-168), as the oracle does."""
    from iris_b200.model import DeviceModel, synth_host_weights
    from iris_b200.shapes import parity_mistral
    from oracle.models import OracleModel
    cfg = parity_mistral()
    w = synth_host_weights(cfg, 21)
    dm = DeviceModel(cfg, weights=w)
    om = OracleModel(cfg, w)
    prompt = seeded_prompt(21, 9, cfg.vocab)
    want, _ = om.generate(prompt, 40)
    sess = dm.session(64)
    got, _ = sess.generate(prompt, 40)
    assert got == want
    eos = want[5]
    first = want.index(eos)
    got, _ = sess.generate(prompt, 40, eos=[eos])
    assert got == want[:first + 1]
    assert sess.length == len(prompt) + first
    # host-driven steps through the C-ABI decode entry point
    sess.reset()
    tok, _ = sess.prefill(prompt)
    seq = [tok]
    for _ in range(6):
        tok, _ = sess.decode(tok)
        seq.append(tok)
    assert seq == want[:7]


def test_kv_cache_matches_the_oracle_layer_stage():
    """The chain's per-layer stage (mistral/stage.rs:172-226) over a range
    with carried K/V, on the device, against the oracle: rows and K/V."""
    from iris_b200.model import DeviceModel, synth_host_weights
    from iris_b200.shapes import parity_mistral
    from oracle.models import OracleModel
    cfg = parity_mistral()
    w = synth_host_weights(cfg, 31)
    dm = DeviceModel(cfg, weights=w)
    om = OracleModel(cfg, w)
    rng = np.random.default_rng(31)
    kvd = cfg.kv_heads * cfg.head_dim
    rows = rng.integers(-(4 << 16), 4 << 16, size=(300, cfg.hidden)).astype(np.int32)
    for layer, start, m in [(0, 0, 300), (2, 0, 7), (1, 37, 260), (3, 100, 1)]:
        prior_k = rng.integers(-(1 << 18), 1 << 18, size=(start, kvd)).astype(np.int32)
        prior_v = rng.integers(-(1 << 18), 1 << 18, size=(start, kvd)).astype(np.int32)
        got = dm.layer_range(layer, rows[:m], start, prior_k, prior_v)
        want = om.mistral_layer_range(layer, rows[:m], start, prior_k, prior_v)
        for g, wnt, what in zip(got, want, ("rows", "k", "v")):
            assert np.array_equal(g, wnt), (layer, start, m, what)


def test_refusals():
    from iris_b200 import _lib
    from iris_b200.model import DeviceModel
    from iris_b200.shapes import parity_mistral
    cfg = parity_mistral()
    dm = DeviceModel(cfg, seed=1)
    sess = dm.session(16)
    with pytest.raises(_lib.IrisError) as e:
        sess.decode(3)
    assert e.value.code == _lib.IRIS_ESTATE
    with pytest.raises(_lib.IrisError) as e:
        sess.prefill(list(range(17)))
    assert e.value.code == _lib.IRIS_ERANGE
    with pytest.raises(_lib.IrisError) as e:
        sess.prefill([cfg.vocab])
    assert e.value.code == _lib.IRIS_EINVAL


@pytest.mark.parametrize("family", ["mistral", "gemma"])
def test_sequence_check_select_matches_oracle(family):
    """The chain's head check (sequence_check.rs:232-300): rms_norm(final),
    dot_row over the head, softcap (the gemma model's is on), first maximum,
    for every predicting row; 600 rows cross the device's 512-row ranges (both
    on the tensor-core GEMM) and 5 rows take the mma.sync GEMM. A zero row
    ties every score and selects token 0."""
    from iris_b200.model import DeviceModel, synth_host_weights
    from iris_b200.shapes import parity_gemma, parity_mistral
    from oracle.models import OracleModel
    cfg = parity_mistral() if family == "mistral" else parity_gemma()
    w = synth_host_weights(cfg, 51)
    dm = DeviceModel(cfg, weights=w)
    om = OracleModel(cfg, w)
    rng = np.random.default_rng(51)
    rows = rng.integers(-(1 << 21), 1 << 21, size=(600, cfg.hidden)).astype(np.int32)
    rows[7] = 0
    rows[8, :3] = [2**31 - 1, -(2**31), 2**31 - 1]
    for sel in (rows, rows[:5]):
        tok, val = dm.sequence_check_select(sel)
        want_tok, want_val = om.head_select(sel)
        assert np.array_equal(tok, want_tok) and np.array_equal(val, want_val)
    assert dm.sequence_check_select(rows[7:8])[0][0] == 0


def test_detwgt_bundle_matches_the_oracle(tmp_path):
    """A model bundle in the reference's .detwgt format (written here from
    seeded weights under their file names, with a YaRN config.json shaped as
    the reference's parity bundle) loaded through iris_b200.detwgt: every
    logit and token of a prefill and 8 decode steps equals the oracle's on
    the same weights and rotary table."""
    import json
    from iris_b200 import detwgt
    from iris_b200.model import DeviceModel, synth_host_weights, tensor_table
    from iris_b200.shapes import parity_mistral
    from oracle.models import OracleModel
    from test_detwgt import write_detwgt
    config = {"model_type": "mistral3", "text_config": {
        "hidden_act": "silu", "hidden_size": 128, "intermediate_size": 2048, "num_hidden_layers": 4,
        "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 32, "vocab_size": 512,
        "max_position_embeddings": 262144, "sliding_window": None, "rms_norm_eps": 1e-05,
        "tie_word_embeddings": True,
        "rope_parameters": {"beta_fast": 32.0, "beta_slow": 1.0, "factor": 16.0, "llama_4_scaling_beta": 0.1,
                            "mscale": 1.0, "mscale_all_dim": 1.0, "original_max_position_embeddings": 16384,
                            "rope_theta": 1000000.0, "rope_type": "yarn"}}}
    cfg = detwgt.mistral_config(config)
    w = synth_host_weights(parity_mistral(), 61)
    names = detwgt.mistral_tensor_names(cfg)
    tensors = []
    for key, arr in w.items():
        kind, rows, cols, _ = tensor_table(cfg)[key]
        dims = [cols] if kind == "values" and rows == 1 else [rows, cols]
        tensors.append((names[key][0], dims, 8 if kind == "q8" else 32, arr))
    write_detwgt(tmp_path / "model.detwgt", tensors)
    (tmp_path / "config.json").write_text(json.dumps(config))
    cfg2, w2, f = detwgt.load_mistral_bundle(tmp_path)
    assert cfg2.yarn == (16, 5, 10) and cfg2.freqs != parity_mistral().freqs
    dm = DeviceModel(cfg2, weights=w2)
    prompt = seeded_prompt(61, 40, cfg2.vocab)
    got = dm.session(64).generate(prompt, 8, want_logits=True)
    want = OracleModel(cfg2, {k: np.array(v) for k, v in w2.items()}).generate(prompt, 8)
    assert_same(got, want)
    del w2
    f.close()


def test_chain_records_match_the_oracle():
    """A claim's teacher-forced pass stage by stage (600 tokens in ranges of
    512: 2 ranges x 4 layers, K/V carried) through iris_mistral_layer_range,
    starting from iris_model_embed's rows: every stage's canonical record
    digest (iris_b200/records.py) equals the digest of the oracle's rows and
    K/V for the same stage."""
    import ctypes as C
    from iris_b200 import records
    from iris_b200.model import DeviceModel, synth_host_weights
    from iris_b200.shapes import parity_mistral
    from oracle import oracle as O
    from oracle.models import OracleModel
    cfg = parity_mistral()
    w = synth_host_weights(cfg, 71)
    dm = DeviceModel(cfg, weights=w)
    om = OracleModel(cfg, w)
    ids = seeded_prompt(71, 600, cfg.vocab)
    emb = np.asarray(w[("EMBED", -1)]).reshape(cfg.vocab, -1)
    want_rows = np.empty((len(ids), cfg.hidden), np.int32)
    for i, t in enumerate(ids):
        assert O.lib().oracle_dequantize_row(O.ptr(np.ascontiguousarray(emb[t]), C.c_uint8), emb.shape[1],
                                              O.ptr(want_rows[i], C.c_int32), cfg.hidden) == 0
    assert np.array_equal(dm.embed(ids), want_rows)
    got = records.chain_records(dm, ids, range_size=512)
    kvd = cfg.kv_heads * cfg.head_dim
    ck = [np.zeros((0, kvd), np.int32) for _ in range(cfg.layers)]
    cv = [np.zeros((0, kvd), np.int32) for _ in range(cfg.layers)]
    want = []
    for start in range(0, len(ids), 512):
        rows = want_rows[start:start + 512]
        for l in range(cfg.layers):
            rows, ok, ov = om.mistral_layer_range(l, rows, start, ck[l], cv[l])
            want.append((f"layer_mistral/{l}", start, records.stage_digest(f"layer_mistral/{l}", start, rows, ok, ov)))
            ck[l] = np.concatenate([ck[l], ok])
            cv[l] = np.concatenate([cv[l], ov])
    assert got == want and len(got) == 2 * cfg.layers

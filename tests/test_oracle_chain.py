"""CPU checks of the chain driver (iris_b200.records.chain_records) on the
oracle: a claim run stage by stage in ranges, with the carried K/V handed on
as the reference does (pruned to each gemma layer's window, a sharing layer
attending over its donor's keys of the same range), gives every row the same
values whatever the range size, and its last row's head scores equal the
oracle decode loop's prompt pass. So the per-range calls and the hand-off
are those of one whole pass (prefill_range.rs:82-172, 849-860;
mistral/stage.rs:172-226)."""
import numpy as np
import pytest


@pytest.fixture(scope="module", autouse=True)
def built():
    from iris_b200 import build
    from oracle import oracle
    build.build()
    oracle.build()


class Recorder:
    """Wraps an OracleStages and keeps the last layer's output rows."""

    def __init__(self, inner):
        self.inner, self.cfg, self.rows = inner, inner.cfg, {}

    def __getattr__(self, name):
        return getattr(self.inner, name)

    def layer_range(self, layer, rows, start, pk, pv):
        out = self.inner.layer_range(layer, rows, start, pk, pv)
        if layer == self.cfg.layers - 1:
            self.rows[start] = out[0]
        return out

    def gemma_layer_range(self, layer, rows, start, ple, prior=None, donor=None):
        out = self.inner.gemma_layer_range(layer, rows, start, ple, prior=prior, donor=donor)
        if layer == self.cfg.layers - 1:
            self.rows[start] = out[0]
        return out


@pytest.mark.parametrize("family", ["mistral", "gemma"])
def test_chain_ranges_equal_one_pass(family):
    import ctypes as C
    from iris_b200 import records
    from iris_b200.model import synth_host_weights
    from iris_b200.shapes import parity_gemma, parity_mistral
    from oracle import oracle as O
    from oracle.models import OracleModel, OracleStages
    cfg = parity_gemma() if family == "gemma" else parity_mistral()
    w = synth_host_weights(cfg, 91)
    om = OracleModel(cfg, w)
    ids = np.random.default_rng(91).integers(0, cfg.vocab, size=37).tolist()  # past the 16-position window
    finals, digests = [], []
    for rs in (37, 16, 7):
        rec = Recorder(OracleStages(om))
        digests.append(records.chain_records(rec, ids, range_size=rs))
        finals.append(np.concatenate([rec.rows[s] for s in sorted(rec.rows)]))
    assert np.array_equal(finals[0], finals[1]) and np.array_equal(finals[0], finals[2])
    assert len(digests[2]) == 6 * cfg.layers
    want_tokens, want_logits = om.generate(ids, 1)
    logits = np.empty(cfg.vocab, np.int32)
    last = np.ascontiguousarray(finals[0][-1])
    assert O.lib().oracle_head_logits(C.byref(om.model.head), O.ptr(last, C.c_int32), O.ptr(logits, C.c_int32),
                                      O.threads_default()) == 0
    assert np.array_equal(logits, want_logits[0])

"""The claim's teacher-forced pass on a session, range by range and
device-resident (iris_session_range_begin / _layer / _end, driven by
iris_b200.records.chain_claim, the stage records hashed while the device
runs on: their leaves on the device (iris_session_range_layer_leaves,
SHA-256 of every 4096-byte piece of the rows and K/V where they live) or
everything on host threads from copies): every stage's record digest equals the oracle's
stage by stage (chain_records over oracle/models.OracleStages), and the head
check's selection of every row equals the oracle's first maximum over its
final rows (sequence_check.rs:232-300). Both families; mistral ranges of 512
(the tensor-core GEMM and attention) and of 100, gemma ranges of 20 (the
window pruning the carried keys, layers sharing their donors' keys)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def built():
    from iris_b200 import build
    from oracle import oracle
    build.build()
    oracle.build()


class FinalRows:
    """An OracleStages that keeps the last layer's output rows of each range."""

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


@pytest.mark.parametrize("device_hash", [True, False])
@pytest.mark.parametrize("family,n,range_size", [("mistral", 600, 512), ("mistral", 250, 100),
                                                 ("gemma", 45, 20)])
def test_device_chain_matches_the_oracle(family, n, range_size, device_hash):
    from iris_b200 import records
    from iris_b200.model import DeviceModel, synth_host_weights
    from iris_b200.shapes import parity_gemma, parity_mistral
    from oracle.models import OracleModel, OracleStages
    cfg = parity_gemma() if family == "gemma" else parity_mistral()
    w = synth_host_weights(cfg, 0xC5)
    dm = DeviceModel(cfg, weights=w)
    om = OracleModel(cfg, w)
    ids = np.random.default_rng(n).integers(0, cfg.vocab, size=n).tolist()
    sess = dm.session(n + 8)
    got, selected, scores = records.chain_claim(sess, ids, range_size=range_size, slots=3, workers=2,
                                                device_hash=device_hash)
    assert sess.length == n
    oracle = FinalRows(OracleStages(om))
    want = records.chain_records(oracle, ids, range_size=range_size)
    assert got == want and len(got) == cfg.layers * ((n + range_size - 1) // range_size)
    final = np.concatenate([oracle.rows[s] for s in sorted(oracle.rows)])
    want_tok, want_val = om.head_select(final)
    assert np.array_equal(selected, want_tok) and np.array_equal(scores, want_val)
    # the session refuses a layer out of order and a range past its capacity
    from iris_b200 import _lib
    sess.reset()
    with pytest.raises(_lib.IrisError) as e:
        records.chain_claim(sess, ids + ids, range_size=range_size, slots=2, workers=1, device_hash=device_hash)
    assert e.value.code == _lib.IRIS_ERANGE
    sess.close()
    dm.close()

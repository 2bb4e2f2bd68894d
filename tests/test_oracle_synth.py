"""CPU checks of the CPU legs' inputs: the oracle's seeded generator gives
the same bytes as the product's (so the reference arm and the CPU baseline
run on the device's weights without loading the product library), the
Mistral-7B shape derived by the oracle's scalar functions equals the host
mirror's, and the oracle's one-token decode pass reproduces the oracle's
decode loop."""
import numpy as np
import pytest


@pytest.fixture(scope="module", autouse=True)
def built():
    from iris_b200 import build
    from oracle import oracle
    build.build()
    oracle.build()


@pytest.mark.parametrize("name,layer,rows,cols,per_block", [
    ("W_Q", 0, 48, 256, False), ("W_DOWN", 3, 130, 2048, True), ("EMBED", -1, 70, 4096, False),
    ("HEAD", -1, 65, 14336, True)])
def test_q8_generator_matches_the_product(name, layer, rows, cols, per_block):
    from iris_b200 import _lib
    from iris_b200.model import T
    from oracle.models import SYNTH_IDS, synth_q8
    assert SYNTH_IDS[name] == T[name]
    want = _lib.synth_q8(0xABC, T[name], layer, rows, cols, per_block)
    for threads in (1, 5):
        assert np.array_equal(synth_q8(0xABC, name, layer, rows, cols, per_block, threads), want)


@pytest.mark.parametrize("name,layer,count,fan_in", [("NORM_ATTN", 2, 4096, 0), ("FINAL_NORM", -1, 300, 0),
                                                     ("NORM_FFN", 0, 1000, 2048), ("W_Q", 1, 777, 3)])
def test_value_generator_matches_the_product(name, layer, count, fan_in):
    from iris_b200 import _lib
    from iris_b200.model import T
    from oracle.models import synth_values
    want = _lib.synth_values(0x5EED, T[name], layer, count, fan_in)
    assert np.array_equal(synth_values(0x5EED, name, layer, count, fan_in, threads=3), want)


def test_mistral_7b_shape_matches_the_host_mirror():
    from iris_b200.shapes import mistral_7b
    from oracle.models import mistral_7b_shape
    a, b = mistral_7b_shape(), mistral_7b()
    for k in ("layers", "hidden", "ffn", "heads", "kv_heads", "head_dim", "vocab", "tied", "max_positions",
              "norm_eps", "scale_q32", "freqs"):
        assert getattr(a, k) == getattr(b, k), k


def test_cpu_decoder_reproduces_the_decode_loop():
    """Token by token through CpuDecoder (the prompt too) gives the oracle
    decode loop's selections (a prompt pass equals its rows one at a time)."""
    from iris_b200.shapes import parity_mistral
    from oracle.models import CpuDecoder, OracleModel, synth_mistral_weights
    cfg = parity_mistral()
    w = synth_mistral_weights(cfg, 77)
    om = OracleModel(cfg, w)
    prompt = np.random.default_rng(77).integers(0, cfg.vocab, size=9).tolist()
    want, _ = om.generate(prompt, 6)
    dec = CpuDecoder(om, 32)
    for t in prompt:
        tok = dec.step(t)
    got = [tok]
    for _ in range(5):
        got.append(dec.step(got[-1]))
    assert got == want

"""The `.detwgt` v3 reader and the mistral-dense config import (host side).

The format follows crates/model/detwgt/src/write.rs:15-124; the shape
derivation crates/model/import/src/mistral.rs:200-287. The reference's own
parity bundle (model-bundles/parity-mistral) is read when the reference tree
is present: its file checksum (checksums.json), tensor table and derived
shape, with the YaRN table's first inverse frequency 2^32 (the importer's
known answer for its first pair). A file written here in the same format
reads back value for value, and malformed files are refused.
"""
import hashlib
import json
import math
import os
import struct

import numpy as np
import pytest

def _bundle():
    from oracle.oracle import reference_root
    root = reference_root()
    return str(root / "model-bundles" / "parity-mistral") if root else ""


BUNDLE = _bundle()


def write_detwgt(path, tensors):
    """tensors: (name, dims, width, payload array); width 16 / 32 (values) or 8
    (raw Q8_0 blocks). The row-mass field is written for values and left 0
    for blocks (the reader does not use it)."""
    out = bytearray(b"DNWGTV0\0" + struct.pack("<IIQ", 3, 1, len(tensors)))
    for name, dims, width, data in tensors:
        nb = name.encode()
        if width == 8:
            payload, mass = np.asarray(data, np.uint8).tobytes(), 0
        else:
            v = np.asarray(data, np.int64).reshape(-1, dims[-1])
            mass = int(np.abs(v).sum(axis=1).max())
            payload = v.astype("<i2" if width == 16 else "<i4").tobytes()
        out += struct.pack("<I", len(nb)) + nb + struct.pack("<I", len(dims))
        out += struct.pack(f"<{len(dims)}Q", *dims) + struct.pack("<QIQQ", math.prod(dims), width, len(payload), mass)
        out += bytes((64 - len(out) % 64) % 64)
        out += payload
    with open(path, "wb") as f:
        f.write(out)


def test_round_trip(tmp_path):
    from iris_b200 import detwgt
    rng = np.random.default_rng(4)
    blocks = rng.integers(0, 256, size=3 * 2 * 34, dtype=np.uint8)
    narrow = rng.integers(-30000, 30000, size=(2, 5))
    wide = rng.integers(-(1 << 30), 1 << 30, size=(7,))
    write_detwgt(tmp_path / "m.detwgt", [("narrow", [2, 5], 16, narrow), ("q", [3, 64], 8, blocks),
                                         ("wide", [7], 32, wide)])
    f = detwgt.Detwgt(tmp_path / "m.detwgt")
    assert list(f.tensors) == ["narrow", "q", "wide"]
    assert np.array_equal(f.values("narrow"), narrow.reshape(-1))
    assert np.array_equal(f.values("wide"), wide)
    assert np.array_equal(f.q8_blocks("q"), blocks) and f.is_q8("q")
    with pytest.raises(ValueError):
        f.values("q")
    f.close()


def test_malformed_files_are_refused(tmp_path):
    from iris_b200 import detwgt
    (tmp_path / "a").write_bytes(b"NOTDETWG" + bytes(16))
    with pytest.raises(ValueError):
        detwgt.Detwgt(tmp_path / "a")
    write_detwgt(tmp_path / "b", [("q", [2, 48], 8, np.zeros(2 * 34, np.uint8))])  # rows not whole blocks
    with pytest.raises(ValueError):
        detwgt.Detwgt(tmp_path / "b")
    write_detwgt(tmp_path / "c", [("v", [4], 32, np.arange(4))])
    raw = bytearray((tmp_path / "c").read_bytes())
    (tmp_path / "c").write_bytes(raw[:-4])  # truncated payload
    with pytest.raises(ValueError):
        detwgt.Detwgt(tmp_path / "c")


def test_config_import_refusals():
    from iris_b200 import detwgt
    base = {"hidden_act": "silu", "hidden_size": 128, "intermediate_size": 256, "num_hidden_layers": 1,
            "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 32, "vocab_size": 64,
            "max_position_embeddings": 4096, "rms_norm_eps": 1e-5, "sliding_window": None,
            "rope_parameters": {"rope_type": "yarn", "rope_theta": 1000000.0, "factor": 16.0,
                                "original_max_position_embeddings": 16384, "beta_fast": 32.0, "beta_slow": 1.0,
                                "mscale": 1.0, "mscale_all_dim": 1.0}}
    cfg = detwgt.mistral_config(base)
    assert cfg.max_positions == 4096 and cfg.yarn == (16, 5, 10) and cfg.freqs[0] == 1 << 32
    for bad in ({"hidden_act": "gelu"}, {"sliding_window": 4096}):
        with pytest.raises(ValueError):
            detwgt.mistral_config({**base, **bad})
    with pytest.raises(ValueError):
        detwgt.mistral_config({**base, "rope_parameters": {**base["rope_parameters"], "mscale": 2.0}})
    scaled = {**base, "rope_parameters": {**base["rope_parameters"], "llama_4_scaling_beta": 0.1}}
    assert detwgt.mistral_config(scaled).max_positions == 16384  # mistral.rs:255-266


@pytest.mark.skipif(not BUNDLE or not os.path.isdir(BUNDLE), reason="the reference's parity bundle is not present")
def test_reference_parity_bundle():
    from iris_b200 import detwgt
    sums = json.load(open(os.path.join(BUNDLE, "checksums.json")))
    data = open(os.path.join(BUNDLE, "model.detwgt"), "rb").read()
    assert hashlib.sha256(data).hexdigest() == sums["model.detwgt"]
    cfg, weights, f = detwgt.load_mistral_bundle(BUNDLE)
    assert (cfg.layers, cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.vocab, cfg.tied) == \
        (4, 128, 2048, 4, 2, 32, 512, True)
    assert cfg.freqs[0] == 1 << 32 and cfg.max_positions == 16384
    assert len(f.tensors) == 2 + 4 * 9 and len(weights) == len(f.tensors)
    assert weights[("W_GATE", 0)].size == 2048 * 128 // 32 * 34
    assert weights[("FINAL_NORM", -1)].dtype == np.int32
    f.close()


# ---- gemma-dense ----------------------------------------------------------

def _gemma_bundle():
    from oracle.oracle import reference_root
    root = reference_root()
    return str(root / "model-bundles" / "parity-gemma") if root else ""


GEMMA_BUNDLE = _gemma_bundle()


def gemma_text_config(**over):
    """A gemma-dense config.json text section of the parity shape: two
    sliding and two full layers, the last two sharing K/V, a 16-key window,
    PLE 32, partial rotary on the full layers, softcap, an untied head."""
    text = {"hidden_size": 128, "intermediate_size": 512, "num_hidden_layers": 4, "num_attention_heads": 4,
            "num_key_value_heads": 2, "head_dim": 32, "hidden_size_per_layer_input": 32, "vocab_size": 512,
            "sliding_window": 16, "num_kv_shared_layers": 2, "rms_norm_eps": 1e-06, "tie_word_embeddings": False,
            "final_logit_softcapping": 1.0,
            "layer_types": ["sliding_attention", "full_attention", "sliding_attention", "full_attention"],
            "rope_parameters": {"sliding_attention": {"rope_theta": 10000},
                                "full_attention": {"rope_theta": 1000000, "partial_rotary_factor": 0.5}}}
    text.update(over)
    return text


def test_gemma_config_import():
    """gemma.rs:126-190: the shape, rotary split, K/V donors and head tying
    derived from a config.json, and the refusals."""
    from iris_b200 import detwgt
    cfg = detwgt.gemma_config({"text_config": gemma_text_config()}, 512, [65536, 1 << 15, 0, 65536])
    assert (cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ple_width) == (4, 128, 4, 2, 32, 32)
    assert cfg.tied is False and cfg.softcap == 1.0 and cfg.layer_scalars == [65536, 1 << 15, 0, 65536]
    assert [cfg.kv_donor(l) for l in range(4)] == [-1, -1, 0, 1]
    assert cfg.rope(0) == (10_000 << 32, 32, 32) and cfg.rope(1) == (1_000_000 << 32, 16, 32)
    assert cfg.window(0) == 16 and cfg.window(1) == 0
    # a layer without a declared type is full attention; bases fall back to the defaults
    bare = gemma_text_config(layer_types=["sliding_attention"], rope_parameters=None, num_kv_shared_layers=0)
    cfg = detwgt.gemma_config(bare, 512, [0] * 4)
    assert cfg.types() == ["sliding_attention"] + ["full_attention"] * 3
    assert (cfg.rope_base_sliding, cfg.rope_base_full, cfg.partial_rotary) == (10_000, 1_000_000, 1.0)
    assert detwgt.gemma_config(gemma_text_config(tie_word_embeddings=True), 512, [0] * 4).tied
    for bad in ({"global_head_dim": 64},
                {"rope_parameters": {"sliding_attention": {"rope_theta": 10000.5}}},
                {"num_hidden_layers": 6, "num_kv_shared_layers": 3,
                 "layer_types": ["sliding_attention", "full_attention", "local", "sliding_attention",
                                 "full_attention", "local"]}):
        with pytest.raises(ValueError):
            detwgt.gemma_config(gemma_text_config(**bad), 512, [0] * 6)


@pytest.mark.skipif(not GEMMA_BUNDLE or not os.path.isdir(GEMMA_BUNDLE),
                    reason="the reference's gemma parity bundle is not present")
def test_reference_parity_gemma_bundle():
    """The reference's gemma parity bundle: its file checksum, every tensor
    the import reads placed, the derived shape, and the oracle generating
    from it on the bundle's own prompts (cases.json: short, near the window,
    over the window)."""
    from iris_b200 import detwgt
    from oracle.models import OracleModel
    sums = json.load(open(os.path.join(GEMMA_BUNDLE, "checksums.json")))
    data = open(os.path.join(GEMMA_BUNDLE, "model.detwgt"), "rb").read()
    assert hashlib.sha256(data).hexdigest() == sums["model.detwgt"]
    cfg, weights, f = detwgt.load_gemma_bundle(GEMMA_BUNDLE)
    try:
        assert (cfg.layers, cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.vocab, cfg.ple_width) \
            == (4, 128, 2048, 4, 2, 32, 512, 32)
        assert cfg.tied is False and ("HEAD", -1) in weights and cfg.sliding_window == 16
        assert [cfg.kv_donor(l) for l in range(4)] == [-1, -1, 0, 1] and cfg.rope(1)[1] == 16
        assert len(f.tensors) == 74 and len(weights) == 2 + 3 + 1 + 4 * 16
        om = OracleModel(cfg, {k: np.array(v) for k, v in weights.items()})
        for case in json.load(open(os.path.join(GEMMA_BUNDLE, "cases.json"))):
            toks, _ = om.generate(case["input_token_ids"], case["tokens"])
            assert len(toks) == case["tokens"] and all(0 <= t < cfg.vocab for t in toks)
    finally:
        del weights
        f.close()

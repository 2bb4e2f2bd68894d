"""Tensor-parallel decode on 2, 4 and 8 GPUs (iris_model_create_mistral_tp):
the row-parallel o and down products exchange exact partial sums (one-token
passes through the peers' memory over NVLink, or over NCCL; many-token
passes over NCCL), the head's vocabulary shards meet in a first-maximum
reduction. Every token and every logit of an N-way model must equal the CPU
oracle's on the full model, through both decode loops (logits copied each
pass; batched graph replays). Each case is skipped when the machine has fewer
GPUs than its ranks."""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def gpu_count():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange,path", [("peer", "step"), ("peer", "graph"), ("nccl", "graph")])
@pytest.mark.parametrize("config,seed,prompt_len,steps", [("parity-mistral", 41, 19, 10),
                                                         ("parity-mistral", 43, 100, 4)])
def test_two_way_tensor_parallel_decode_matches_the_oracle(tmp_path, config, seed, prompt_len, steps, exchange, path):
    """exchange "peer" with path "step": the persistent step on each rank,
    the o / down partial sums exchanged inside it over peer memory and the
    head's first maximum through peer key slots; "graph": one kernel per
    operation (peer-memory finish kernel, or NCCL sums). The 100-token prompt
    runs its products on the tensor-core GEMM, the row-parallel ones ending in
    partial limbs summed over NCCL."""
    run_tp(tmp_path, 2, config, seed, prompt_len, steps, exchange, path)


@pytest.mark.parametrize("world", [4, 8])
@pytest.mark.parametrize("exchange,path", [("peer", "step"), ("nccl", "graph")])
def test_wider_tensor_parallel_decode_matches_the_oracle(tmp_path, world, exchange, path):
    """4 and 8 ranks (one or two kv heads a rank, 256 or 128 FFN rows, 256 or
    128 vocabulary rows): a 70-token prompt on the tensor-core GEMM, then
    greedy steps on the persistent step (peer-memory exchange stages) or the
    kernel graph (NCCL sums)."""
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    run_tp(tmp_path, world, "tp-mistral", 47, 70, 6, exchange, path)


def run_tp(tmp_path, world, config, seed, prompt_len, steps, exchange, path):
    from iris_b200 import _lib, build
    from iris_b200.model import synth_host_weights
    from iris_b200.shapes import CONFIGS
    from oracle import oracle
    from oracle.models import OracleModel
    build.build()
    oracle.build()
    nccl_id = _lib.tp_unique_id().hex()
    out = tmp_path / "tp.npz"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, "-m", "iris_b200.tp_worker", "--rank", str(r), "--world", str(world),
                               "--id", nccl_id, "--config", config, "--seed", str(seed), "--prompt-seed", "3",
                               "--prompt-len", str(prompt_len), "--steps", str(steps), "--out", str(out), "--untied",
                               "--exchange", exchange, "--path", path],
                              cwd=ROOT, env=env) for r in range(world)]
    try:
        codes = [p.wait(timeout=600) for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    assert codes == [0] * world, codes
    got = np.load(out)
    assert str(got["path"]) == path
    cfg = CONFIGS[config]
    cfg = type(cfg)(**{**cfg.__dict__, "tied": False})  # the head is sharded by vocabulary
    want_tokens, want_logits = OracleModel(cfg, synth_host_weights(cfg, seed)).generate(got["prompt"].tolist(), steps)
    assert got["tokens"].tolist() == want_tokens
    assert got["tokens_graph"].tolist() == want_tokens
    for p in range(len(want_tokens)):
        assert np.array_equal(got["logits"][p], want_logits[p]), f"logits of pass {p}"

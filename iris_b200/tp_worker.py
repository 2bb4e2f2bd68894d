"""One rank of a tensor-parallel decode, as a process (tests and tools).

  python -m iris_b200.tp_worker --rank R --world W --id HEX --config NAME \\
      --seed S --prompt-seed P --prompt-len N --steps K --out FILE.npz [--untied] [--exchange peer|nccl]

Rank R uses CUDA device R, builds its shard of the seeded synthetic model,
runs `Session.generate` twice (every pass's logits copied out, then the
batched graph-replay loop) and rank 0 writes the tokens and logits to FILE.
Every rank must be started with the same arguments except --rank.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--rank", type=int, required=True)
    p.add_argument("--world", type=int, required=True)
    p.add_argument("--id", required=True, help="NCCL unique id, hex")
    p.add_argument("--config", required=True)
    p.add_argument("--seed", type=int, required=True)
    p.add_argument("--prompt-seed", type=int, default=1)
    p.add_argument("--prompt-len", type=int, default=16)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--out", required=True)
    p.add_argument("--untied", action="store_true", help="a separate head matrix (tensor parallelism shards it)")
    p.add_argument("--exchange", choices=["peer", "nccl"], default="peer")
    p.add_argument("--path", choices=["auto", "graph", "step"], default="auto", help="decode path")
    a = p.parse_args()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import numpy as np
    import torch
    torch.cuda.set_device(a.rank)
    from iris_b200.model import DeviceModel
    from iris_b200.shapes import CONFIGS
    cfg = CONFIGS[a.config]
    if a.untied:
        cfg = type(cfg)(**{**cfg.__dict__, "tied": False})
    prompt = np.random.default_rng(a.prompt_seed).integers(0, cfg.vocab, size=a.prompt_len).tolist()
    dm = DeviceModel(cfg, seed=a.seed, tp=(a.rank, a.world, bytes.fromhex(a.id)))
    dm.set_tp_exchange(a.exchange)
    sess = dm.session(a.prompt_len + a.steps + 8)
    sess.set_decode_path(a.path)
    path = sess.decode_path
    toks, logits = sess.generate(prompt, a.steps, want_logits=True)
    toks2, _ = sess.generate(prompt, a.steps)
    sess.close()
    dm.close()
    if a.rank == 0:
        np.savez(a.out, tokens=np.array(toks), logits=logits, tokens_graph=np.array(toks2), prompt=np.array(prompt),
                 path=np.array(path))


if __name__ == "__main__":
    main()

"""The tensor-parallel exact partial-sum exchange on CPU ranks (gloo), with
the product's own arithmetic: each rank's row-parallel shard (whole 32-value
blocks of the input columns, as the tensor-parallel model splits o and down)
leaves its unrounded 128-bit row sums as four int64 limbs
(limbs_from_acc128, the EPI_PARTIAL output), the ranks sum the limbs (an
all-reduce SUM, as the NCCL exchange does), and every rank rebuilds the
128-bit total and rounds it once (acc128_add_limbs + acc128_round_q24, as
tp_finish does). The result must equal the oracle's dot_row over the whole
row (q8.rs:56-72) bit for bit, for shards whose own sums leave the int64
range (the largest scales against i32::MIN / MAX activations) and for any
order of the ranks. The device code is compiled as host C++
(tests/native/detnum_shim.cc); no GPU is involved.
"""
import ctypes as C
import os

import numpy as np
import pytest


def rank_main(rank, world, port, shim_path, data_path, result_path):
    import torch
    import torch.distributed as dist
    from conftest import declare_shim_limbs
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L = C.CDLL(shim_path)
        declare_shim_limbs(L)
        d = np.load(data_path)
        acts, blocks, bounds = d["acts"], d["blocks"], d["bounds"]
        tokens, rows = acts.shape[0], blocks.shape[0]
        b0, b1 = int(bounds[rank]), int(bounds[rank + 1])
        limbs = np.zeros((tokens, rows, 4), np.int64)
        for t in range(tokens):
            a = np.ascontiguousarray(acts[t])
            for r in range(rows):
                row = np.ascontiguousarray(blocks[r])
                L.shim_partial_limbs(a.ctypes.data_as(C.POINTER(C.c_int32)), row.ctypes.data_as(C.POINTER(C.c_uint8)),
                                     b0, b1, limbs[t, r].ctypes.data_as(C.POINTER(C.c_int64)))
        summed = torch.from_numpy(limbs.copy())
        dist.all_reduce(summed, op=dist.ReduceOp.SUM)
        summed = summed.numpy()
        out = np.empty((tokens, rows), np.int32)
        for t in range(tokens):
            for r in range(rows):
                out[t, r] = L.shim_round_limb_sums(np.ascontiguousarray(summed[t, r]).ctypes.data_as(
                    C.POINTER(C.c_int64)))
        np.save(f"{result_path}.{rank}.npy", out)
    finally:
        dist.destroy_process_group()


def free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_limb_exchange_matches_the_oracle(world, tmp_path, detnum_shim):
    import torch.multiprocessing as mp
    from oracle import oracle as O
    O.build()
    rng = np.random.default_rng(world)
    tokens, rows, cols = 3, 6, 1024
    nb = cols // 32
    bits = rng.integers(0, 0x7C00, size=(rows, nb))  # finite fp16 scales, random signs below
    bits[0] = 0x7BFF                                  # the largest scale everywhere in row 0
    bits[1, ::3] = 0x0000
    bits = bits | (rng.integers(0, 2, size=(rows, nb)) << 15)
    blocks = np.empty((rows, nb, 34), np.uint8)
    blocks[:, :, 0] = bits & 0xFF
    blocks[:, :, 1] = (bits >> 8) & 0xFF
    blocks[:, :, 2:] = rng.integers(0, 256, size=(rows, nb, 32), dtype=np.uint8)
    blocks[0, :, 2:] = 0x7F  # q = 127 against the extreme activations
    blocks = blocks.reshape(rows, nb * 34)
    acts = rng.integers(-(2**31), 2**31, size=(tokens, cols), dtype=np.int64).astype(np.int32)
    acts[0] = 2**31 - 1
    acts[1, ::2] = -(2**31)
    # uneven shards at block boundaries; the middle ranks' shards may be small
    cuts = np.sort(rng.choice(np.arange(1, nb), size=world - 1, replace=False))
    bounds = np.concatenate([[0], cuts, [nb]]).astype(np.int64)
    want = np.array([[O.dot_row(acts[t], blocks[r]) for r in range(rows)] for t in range(tokens)], np.int32)
    assert abs(int(want[0, 0])) == 2**31 - 1 or want[0, 0] in (2**31 - 1, -(2**31))  # row 0 saturates
    data = tmp_path / "case.npz"
    np.savez(data, acts=acts, blocks=blocks, bounds=bounds)
    res = str(tmp_path / "out")
    mp.start_processes(rank_main, args=(world, free_port(), detnum_shim.path, str(data), res), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        got = np.load(f"{res}.{r}.npy")
        assert np.array_equal(got, want), (r, np.argwhere(got != want)[:4])

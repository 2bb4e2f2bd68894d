"""Single-kernel timings, for tuning and for profiler captures of one kernel.

  python -m iris_b200.microbench gemv [--rows 28672 --cols 4096 --iters 20]
      the decode GEMV (one token) over one Q8_0 matrix;
  python -m iris_b200.microbench attention [--context 2560 --layers 1]
      one single-query attention over a mistral-7b-shaped cache;
  python -m iris_b200.microbench gemm [--rows 6144 --cols 4096 --tokens 256]
      the many-token product.

Each prints one JSON line (average device time a launch, bytes or ops a
launch, the implied rate). Inputs are seeded synthetic values; timings use
CUDA events on the stream the kernels run on.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def _events(torch):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def gemv(args):
    import torch
    from iris_b200 import _lib
    L = _lib.lib()
    _lib.check(L.q8gpu_init(), "q8gpu_init")
    blocks = _lib.synth_q8(args.seed, 7, 0, args.rows, args.cols)
    mats = []
    for i in range(args.copies):  # distinct matrices so that nothing is served from L2
        h = C.c_void_p()
        _lib.check(L.iris_q8_upload_blocks(_lib.ptr(blocks, C.c_uint8), args.rows, args.cols, C.byref(h)), "upload")
        mats.append(h)
    x = torch.randint(-(1 << 20), 1 << 20, (1, args.cols), dtype=torch.int32, device="cuda")
    out = torch.empty((1, args.rows), dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    run = lambda h: _lib.check(L.iris_q8_product_device_path(h, x.data_ptr(), 1, out.data_ptr(), stream.cuda_stream,
                                                             _lib.PATH_GEMV), "gemv")
    for h in mats:
        run(h)
    torch.cuda.synchronize()
    e0, e1 = _events(torch)
    e0.record(stream)
    for i in range(args.iters):
        run(mats[i % len(mats)])
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.iters
    nbytes = args.rows * args.cols * 34 // 32 + 4 * args.cols + 4 * args.rows
    for h in mats:
        L.q8gpu_free(h)
    return {"kernel": "q8_gemv_tma_kernel<IN_RAW, EPI_STORE>", "rows": args.rows, "cols": args.cols,
            "us_per_launch": us, "bytes_per_launch": nbytes, "GB_s": nbytes / us / 1e3}


def attention(args):
    import torch
    from iris_b200.model import DeviceModel
    from iris_b200.shapes import mistral_7b
    cfg = mistral_7b()
    cfg = type(cfg)(**{**cfg.__dict__, "layers": args.layers, "vocab": 512})
    model = DeviceModel(cfg, seed=args.seed)
    sess = model.session(args.context + 8)
    prompt = np.random.default_rng(args.seed).integers(0, cfg.vocab, size=args.context).tolist()
    sess.prefill(prompt)
    stream = torch.cuda.ExternalStream(sess.stream_ptr)
    for _ in range(3):
        sess.attention(0)
    sess.synchronize()
    e0, e1 = _events(torch)
    e0.record(stream)
    for i in range(args.iters):
        sess.attention(i % args.layers)
    e1.record(stream)
    sess.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.iters
    kvd = cfg.kv_heads * cfg.head_dim
    nbytes = 2 * args.context * kvd * 4
    return {"kernel": "attn_scores+attn_exp+attn_out (decode)", "context": args.context, "us_per_attention": us,
            "kv_bytes": nbytes, "GB_s": nbytes / us / 1e3}


def gemm(args):
    import torch
    from iris_b200 import _lib
    L = _lib.lib()
    _lib.check(L.q8gpu_init(), "q8gpu_init")
    blocks = _lib.synth_q8(args.seed, 7, 0, args.rows, args.cols)
    h = C.c_void_p()
    _lib.check(L.iris_q8_upload_blocks(_lib.ptr(blocks, C.c_uint8), args.rows, args.cols, C.byref(h)), "upload")
    x = torch.randint(-(1 << 20), 1 << 20, (args.tokens, args.cols), dtype=torch.int32, device="cuda")
    out = torch.empty((args.tokens, args.rows), dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    run = lambda: _lib.check(L.iris_q8_product_device_path(h, x.data_ptr(), args.tokens, out.data_ptr(),
                                                           stream.cuda_stream, _lib.PATH_GEMM), "gemm")
    run()
    torch.cuda.synchronize()
    e0, e1 = _events(torch)
    e0.record(stream)
    for _ in range(args.iters):
        run()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.iters
    ops = 2 * args.rows * args.cols * args.tokens
    L.q8gpu_free(h)
    return {"kernel": "planes_kernel + q8_gemm_kernel<EPI_STORE>", "rows": args.rows, "cols": args.cols,
            "tokens": args.tokens, "us_per_launch": us, "TOPS": ops / us / 1e6}


def main():
    p = argparse.ArgumentParser()
    p.add_argument("which", choices=["gemv", "attention", "gemm"])
    p.add_argument("--rows", type=int, default=28672)
    p.add_argument("--cols", type=int, default=4096)
    p.add_argument("--tokens", type=int, default=256)
    p.add_argument("--copies", type=int, default=1)
    p.add_argument("--context", type=int, default=2560)
    p.add_argument("--layers", type=int, default=1)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--seed", type=int, default=7)
    args = p.parse_args()
    from iris_b200 import build
    build.build()
    print(json.dumps({"gemv": gemv, "attention": attention, "gemm": gemm}[args.which](args)), flush=True)


if __name__ == "__main__":
    main()

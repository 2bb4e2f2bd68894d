"""Single-kernel timings, for tuning and for profiler captures of one kernel.

  python -m iris_b200.microbench gemv [--rows 28672 --cols 4096 --iters 20]
      the decode GEMV (one token) over one Q8_0 matrix;
  python -m iris_b200.microbench attention [--context 2560 --layers 1]
      one single-query attention over a mistral-7b-shaped cache;
  python -m iris_b200.microbench gemm [--rows 6144 --cols 4096 --tokens 256]
      the many-token product;
  python -m iris_b200.microbench sweep
      the Q8 sweep (M in 1, 16, 128, 2048 x (N, K) pairs): this library's
      device products, and both this library's and the reference's
      q8gpu_product (host buffers in and out) when oracle/_ref holds the
      reference kernel;
  python -m iris_b200.microbench product [--product 2 --layers 2]
      one of the decode pass's own products (0 q|k|v, 1 o, 2 gate|up,
      3 down, 4 head) of a mistral-7b-shaped session, layer after layer;
  python -m iris_b200.microbench step [--context 2048 --layers 32]
      the persistent decode step's timeline: per stage kind, how long the
      stage took end to end and the median block's intervals between its
      stamps (wake-up after the stage before, prologue, streaming, tail;
      attention: key slots, scores, the two group exchanges, value sums).

Each prints one JSON line (average device time a launch, bytes or ops a
launch, the implied rate). Inputs are seeded synthetic values; the launches
are captured into a CUDA graph and timed with CUDA events around one replay
on the stream they run on.
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


def device_us(torch, stream, launches, iters):
    """Average device time of launches(i) over i < iters: the launches are
    captured into one CUDA graph on `stream` (through the library's own
    capture entry points) and replayed, so host launch overhead does not
    enter the figure."""
    from iris_b200 import _lib
    L = _lib.lib()
    sp = C.c_void_p(stream.cuda_stream)
    _lib.check(L.iris_capture_begin(sp), "iris_capture_begin")
    try:
        for i in range(iters):
            launches(i)
    finally:
        g = C.c_void_p()
        end = L.iris_capture_end(sp, C.byref(g))
    _lib.check(end, "iris_capture_end")
    try:
        _lib.check(L.iris_graph_launch(g, sp), "iris_graph_launch")
        stream.synchronize()
        e0, e1 = _events(torch)
        e0.record(stream)
        _lib.check(L.iris_graph_launch(g, sp), "iris_graph_launch")
        e1.record(stream)
        stream.synchronize()
    finally:
        L.iris_graph_free(g)
    return e0.elapsed_time(e1) * 1e3 / iters


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
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    run = lambda h: _lib.check(L.iris_q8_product_device_path(h, x.data_ptr(), 1, out.data_ptr(), stream.cuda_stream,
                                                             _lib.PATH_GEMV), "gemv")
    for h in mats:
        run(h)
    torch.cuda.synchronize()
    us = device_us(torch, stream, lambda i: run(mats[i % len(mats)]), args.iters)
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
    sess.set_attention(args.attn)
    if args.shape:
        c, h, r = (int(v) for v in args.shape.split(","))
        sess.set_attention_shape(c, h, r)
    stream = torch.cuda.ExternalStream(sess.stream_ptr)
    for _ in range(3):
        sess.attention(0)
    sess.synchronize()
    us = device_us(torch, stream, lambda i: sess.attention(i % args.layers), args.iters)
    kvd = cfg.kv_heads * cfg.head_dim
    nbytes = 2 * args.context * kvd * 4
    kernel = {"auto": "attn_decode_grid_kernel (where planned)", "cluster": "attn_decode_cluster_kernel",
              "split": "attn_scores+attn_exp+attn_out"}[args.attn]
    return {"kernel": kernel, "attn": args.attn, "shape": args.shape, "context": args.context, "us_per_attention": us,
            "kv_bytes": nbytes, "GB_s": nbytes / us / 1e3}


def prefill(args):
    """A prefill of --context seeded tokens through an --layers-layer model of
    the Mistral-7B layer shapes (vocabulary 512): whole-call time, and the
    kernels of its ranges for ncu (attention and tensor-core GEMMs)."""
    import time
    from iris_b200.model import DeviceModel
    from iris_b200.shapes import mistral_7b
    cfg = mistral_7b()
    cfg = type(cfg)(**{**cfg.__dict__, "layers": args.layers, "vocab": 512})
    model = DeviceModel(cfg, seed=args.seed)
    model.prepare_gemm()
    prompt = np.random.default_rng(args.seed).integers(0, cfg.vocab, size=args.context).tolist()
    times = []
    for _ in range(max(1, args.iters)):
        sess = model.session(args.context + 8)
        t0 = time.perf_counter()
        sess.prefill(prompt)
        times.append(time.perf_counter() - t0)
        sess.close()
    model.close()
    best = min(times)
    return {"layers": args.layers, "context": args.context, "ms": best * 1e3, "tok_s": args.context / best}


def decode(args):
    """Greedy decode of the Gemma-2B architecture (seeded weights) after a
    --context-token prompt: one warm pass, then --iters passes inside an
    NVTX range named "decode" (for ncu's --nvtx-include "decode/"), timed by
    the host around a synchronisation."""
    import time
    import torch
    from iris_b200.model import DeviceModel
    from iris_b200.shapes import gemma_2b
    cfg = gemma_2b()
    model = DeviceModel(cfg, seed=args.seed)
    model.prepare_gemm()
    prompt = np.random.default_rng(args.seed).integers(0, cfg.vocab, size=args.context).tolist()
    sess = model.session(args.context + args.iters + 8)
    sess.prefill(prompt)
    sess.decode_steps(1)
    sess.synchronize()
    torch.cuda.nvtx.range_push("decode")
    t0 = time.perf_counter()
    sess.decode_steps(args.iters)
    sess.synchronize()
    dt = time.perf_counter() - t0
    torch.cuda.nvtx.range_pop()
    out = {"model": cfg.name, "context": args.context, "steps": args.iters, "ms_per_step": dt * 1e3 / args.iters,
           "tok_s": args.iters / dt, "kernels_per_step": sess.kernels_per_pass}
    sess.close()
    model.close()
    return out


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
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    if args.gemm in ("tc", "tc3"):  # builds the tensor-core copy; the no-alloc calls below then take it
        path = _lib.PATH_TC if args.gemm == "tc" else _lib.PATH_TC3
        _lib.check(L.iris_q8_product_device_path(h, x.data_ptr(), args.tokens, out.data_ptr(), None, path),
                   "tensor-core gemm")
    # the no-alloc entry point: the tiled GEMM path without a synchronisation
    run = lambda: _lib.check(L.iris_q8_product_device_noalloc(h, x.data_ptr(), args.tokens, out.data_ptr(),
                                                              stream.cuda_stream), "gemm")
    run()
    torch.cuda.synchronize()
    us = device_us(torch, stream, lambda i: run(), args.iters)
    ops = 2 * args.rows * args.cols * args.tokens
    L.q8gpu_free(h)
    kernel = {"tc": "q8_gemm_tc_kernel<EPI_STORE, 1> (one-plane copy: one scale a row)",
              "tc3": "q8_gemm_tc_kernel<EPI_STORE, 3> (three-plane copy: per-block scales)",
              "mma": "q8_gemm_mma_kernel<EPI_STORE>"}[args.gemm]
    return {"kernel": "planes_kernel + " + kernel, "rows": args.rows, "cols": args.cols,
            "tokens": args.tokens, "us_per_launch": us, "TOPS": ops / us / 1e6}


def product(args):
    import torch
    from iris_b200.model import DeviceModel
    from iris_b200.shapes import mistral_7b
    cfg = mistral_7b()
    cfg = type(cfg)(**{**cfg.__dict__, "layers": args.layers})
    model = DeviceModel(cfg, seed=args.seed)
    sess = model.session(64)
    sess.prefill(np.random.default_rng(args.seed).integers(0, cfg.vocab, size=16).tolist())
    stream = torch.cuda.ExternalStream(sess.stream_ptr)
    for l in range(args.layers):
        sess.product(l, args.product_which)
    sess.synchronize()
    us = device_us(torch, stream, lambda i: sess.product(i % args.layers, args.product_which), args.iters)
    H, F, qd, kvd, V = cfg.hidden, cfg.ffn, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.vocab
    rows, cols, outb = {0: (qd + 2 * kvd, H, 4 * (qd + 2 * kvd)), 1: (H, qd, 4 * H), 2: (2 * F, H, 4 * F),
                        3: (H, F, 4 * H), 4: (V, H, 4 * V)}[args.product_which]
    nbytes = rows * cols * 34 // 32 + 4 * cols + outb
    sess.close()
    model.close()
    names = {0: "IN_NORM, EPI_STORE", 1: "IN_PLANES, EPI_STORE", 2: "IN_NORM, EPI_SILU_MUL",
             3: "IN_PLANES, EPI_STORE", 4: "IN_NORM, EPI_LOGITS"}
    return {"kernel": f"q8_gemv_tma_kernel<{names[args.product_which]}>", "rows": rows, "cols": cols,
            "us_per_launch": us, "bytes_per_launch": nbytes, "GB_s": nbytes / us / 1e3}


kTcWarmTokens = 64  # a many-token product: builds a matrix's tensor-core copy


def sweep(args):
    """Q8 sweep: one JSON line a (M, N, K). `device_us`: this library's
    product on device buffers (GEMV for M = 1, tiled GEMM otherwise);
    `host_us` / `ref_host_us`: q8gpu_product of this library / of the
    reference's kernel with host activations and outputs (copies included)."""
    import time
    import torch
    from iris_b200 import _lib
    from oracle import oracle
    L = _lib.lib()
    _lib.check(L.q8gpu_init(), "q8gpu_init")
    ref = oracle.reference_q8()
    if ref is not None:
        assert ref.q8gpu_init() == 0
    rng = np.random.default_rng(args.seed)
    lines = []
    for n, k in [(2048, 2048), (16384, 2048), (4096, 4096), (14336, 4096)]:
        nb = n * k // 32
        bits = (rng.integers(0, 64, size=nb) + 0x2400).astype(np.int64)  # finite positive scales
        if args.scales == "row":  # one scale an output row, in every block of the row
            bits = np.repeat(bits[:: k // 32], k // 32)
        ex, man = (bits >> 10) & 0x1F, bits & 0x3FF
        scales = ((1024 + man) << np.maximum(ex - 1, 0)).astype(np.int64)
        weights = rng.integers(-127, 128, size=n * k).astype(np.int8)
        h = C.c_void_p()
        _lib.check(L.q8gpu_upload(weights.ctypes.data_as(C.POINTER(C.c_int8)), _lib.ptr(scales, C.c_int64), n, k,
                                  C.byref(h)), "upload")
        # the tensor-core copy is built once per matrix, outside the timed calls
        warm = torch.zeros((kTcWarmTokens, k), dtype=torch.int32, device="cuda")
        wout = torch.empty((kTcWarmTokens, n), dtype=torch.int32, device="cuda")
        _lib.check(L.iris_q8_product_device(h, warm.data_ptr(), kTcWarmTokens, wout.data_ptr(), None), "warm")
        del warm, wout
        hr = C.c_void_p()
        if ref is not None:
            assert ref.q8gpu_upload(weights.ctypes.data_as(C.POINTER(C.c_int8)),
                                    scales.ctypes.data_as(C.POINTER(C.c_int64)), n, k, C.byref(hr)) == 0
        for m in [1, 16, 128, 2048]:
            acts = rng.integers(-(1 << 20), 1 << 20, size=(m, k)).astype(np.int32)
            x = torch.from_numpy(acts).cuda()
            out = torch.empty((m, n), dtype=torch.int32, device="cuda")
            stream = torch.cuda.Stream()
            torch.cuda.synchronize()
            iters = max(2, min(args.iters, int(2e9 / (2 * m * n * k)) + 2))
            if m * k * 4 <= _lib.NOALLOC_PLANES_BYTES:  # captured: no host launch overhead
                run = lambda i: _lib.check(L.iris_q8_product_device_noalloc(h, x.data_ptr(), m, out.data_ptr(),
                                                                            stream.cuda_stream), "product")
                run(0)
                stream.synchronize()
                dev = device_us(torch, stream, run, iters)
            else:  # large M: the GEMM dominates the eager call
                run = lambda: _lib.check(L.iris_q8_product_device(h, x.data_ptr(), m, out.data_ptr(),
                                                                  stream.cuda_stream), "product")
                run()
                stream.synchronize()
                e0, e1 = _events(torch)
                e0.record(stream)
                for _ in range(iters):
                    run()
                e1.record(stream)
                stream.synchronize()
                dev = e0.elapsed_time(e1) * 1e3 / iters
            host_out = np.empty(m * n, np.int32)
            def host_time(lib, handle):
                lib.q8gpu_product(handle, _lib.ptr(acts, C.c_int32), m, _lib.ptr(host_out, C.c_int32))
                reps = max(1, min(5, int(5e8 / (2 * m * n * k)) + 1))
                t0 = time.perf_counter()
                for _ in range(reps):
                    rc = lib.q8gpu_product(handle, _lib.ptr(acts, C.c_int32), m, _lib.ptr(host_out, C.c_int32))
                    assert rc == 0, rc
                return (time.perf_counter() - t0) / reps * 1e6
            mine_host = host_time(L, h)
            mine_vals = host_out.copy()
            line = {"m": m, "n": n, "k": k, "scales": args.scales, "device_us": dev, "host_us": mine_host,
                    "bytes": n * k * 34 // 32 + 4 * m * k + 4 * m * n, "ops": 2 * m * n * k}
            line["GB_s"] = line["bytes"] / dev / 1e3
            line["TOPS"] = line["ops"] / dev / 1e6
            if ref is not None:
                line["ref_host_us"] = host_time(ref, hr)
                line["equal_to_reference"] = bool(np.array_equal(mine_vals, host_out))
            lines.append(line)
            print(json.dumps(line), flush=True)
        L.q8gpu_free(h)
        if ref is not None:
            ref.q8gpu_free(hr)
    return {"sweep": len(lines)}


def step(args):
    """Timeline of one persistent decode pass (global-timer stamps per block
    and stage), summarised per stage kind (µs)."""
    from iris_b200.model import DeviceModel
    from iris_b200.shapes import mistral_7b
    cfg = mistral_7b()
    cfg = type(cfg)(**{**cfg.__dict__, "layers": args.layers})
    model = DeviceModel(cfg, seed=args.seed)
    sess = model.session(args.context + 8 + args.iters)
    sess.set_decode_path("step")
    sess.prefill(np.random.default_rng(args.seed).integers(0, cfg.vocab, size=args.context).tolist())
    sess.step_trace(True)
    sess.decode_steps(args.iters)
    sess.synchronize()
    tr = sess.get_step_trace().astype(np.int64)  # [blocks][stages][8]
    sess.step_trace(False)
    if args.raw:
        np.save(args.raw, tr)
    kinds = ["embed"] + ["qkv", "attn", "o", "gate_up", "down"] * cfg.layers + ["head"]
    stages = tr.shape[1]
    end = np.array([tr[:, k, 7].max() for k in range(stages)])
    t0 = tr[:, 0, 7][tr[:, 0, 7] > 0].min()
    # intervals between stamps (events of step.cuh's timeline), medians over
    # the blocks that worked at the stage, then means over the layers
    spans = {"product": [("wake", None, 0), ("prologue", 0, 1), ("consume", 1, 2), ("tail", 2, 7),
                         ("producer_done", None, 6)],
             "norm": [("wake", None, 0), ("norm_scale", 0, 3), ("norm_emit", 3, 4), ("norm_sync", 4, 1),
                      ("consume", 1, 2), ("tail", 2, 7), ("producer_done", None, 6)],
             "attn": [("wake", None, 0), ("first_key_slot", 0, 1), ("scores", 1, 2), ("exchange1", 2, 3),
                      ("exchange2", 3, 4), ("values", 4, 5), ("finish", 5, 7), ("producer_done", None, 6)]}
    acc = {}
    for k in range(1, stages):
        kind = kinds[k]
        st = tr[:, k, :]
        lst = spans["attn" if kind == "attn" else "norm" if kind in ("qkv", "gate_up", "head") else "product"]
        need = [e for _, a, b in lst for e in (a, b) if e is not None and e != 6]
        act = np.all(st[:, sorted(set(need))] > 0, axis=1)
        d = acc.setdefault(kind, {"stage": [], **{n: [] for n, _, _ in lst}})
        d["stage"].append((end[k] - end[k - 1]) / 1e3)
        if not act.any():
            continue
        for name, a, b in lst:
            va = end[k - 1] if a is None else st[act, a]
            vb = st[act, b]
            if b == 6 and not (vb > 0).any():
                continue
            d[name].append(float(np.median(vb - va)) / 1e3)
    out = {kind: {n: round(float(np.mean(v)), 2) for n, v in d.items() if v} for kind, d in acc.items()}
    sess.close()
    model.close()
    return {"kernel": "decode_step_kernel", "context": args.context, "layers": cfg.layers,
            "pass_us": (end[-1] - t0) / 1e3, "per_kind_us": out}


def main():
    p = argparse.ArgumentParser()
    p.add_argument("which", choices=["gemv", "attention", "gemm", "product", "sweep", "step", "prefill",
                                      "decode"])
    p.add_argument("--product", type=int, default=2, dest="product_which")
    p.add_argument("--rows", type=int, default=28672)
    p.add_argument("--cols", type=int, default=4096)
    p.add_argument("--tokens", type=int, default=256)
    p.add_argument("--scales", choices=["block", "row"], default="block",
                   help="sweep: random scales per block (as GGUF) or one scale a row (BASELINE's weights)")
    p.add_argument("--gemm", choices=["tc", "tc3", "mma"], default="tc", help="gemm: the tcgen05 or the mma.sync GEMM")
    p.add_argument("--copies", type=int, default=1)
    p.add_argument("--context", type=int, default=2560)
    p.add_argument("--layers", type=int, default=1)
    p.add_argument("--attn", choices=["auto", "split", "cluster"], default="auto")
    p.add_argument("--shape", default="", help="cluster,hpc,ring of the one-launch attention")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--seed", type=int, default=7)
    p.add_argument("--raw", default="", help="step: also save the raw stamps (.npy)")
    args = p.parse_args()
    from iris_b200 import build
    build.build()
    print(json.dumps({"gemv": gemv, "attention": attention, "gemm": gemm, "product": product, "sweep": sweep, "step": step, "prefill": prefill,
                      "decode": decode}[args.which](args)), flush=True)


if __name__ == "__main__":
    main()

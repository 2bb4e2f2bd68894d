#!/usr/bin/env python
"""Bit-exact Q8 decode tok/s of a Mistral-7B-architecture model on B200.

Workload (BASELINE.json config 4 at N=1): seeded synthetic Q8_0 weights
(L32, H4096, 32q/8kv, d128, SwiGLU 14336, V32000, untied head, RoPE 1e6),
a 2048-token seeded prompt prefilled on the device, then greedy decode
passes. A step is one decode pass (32 layers + head + first-maximum
selection) at the next position; the first-maximum token feeds the next pass
on the device. Inputs: every pass streams ~7.6 GB of weights (larger than
the 126 MB L2), so no flush is needed between steps.

  python bench.py [--gpus N --steps K --warmup W]      this framework
  python bench.py --impl reference ...                 the CPU reference path

With N > 1 (torchrun), the one sequence is decoded by an N-way
tensor-parallel model (kv groups, FFN rows and vocabulary split; the
row-parallel products' exact partial sums summed over NCCL): strong scaling.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "bit-exact Q8 decode tok/s (Mistral-7B arch)"
UNIT = "tok/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=256)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", default="iris", choices=["iris", "reference"])
    p.add_argument("--prompt", type=int, default=2048)
    p.add_argument("--seed", type=int, default=0x1215B200)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--tp-exchange", choices=["peer", "nccl"], default="peer",
                   help="N > 1: how decode passes exchange partial sums")
    p.add_argument("--chain-tokens", type=int, default=4096,
                   help="tokens of the chain-shaped prefill measured after the decode (0: skip)")
    p.add_argument("--decode-path", choices=["auto", "graph", "step"], default="auto",
                   help="decode passes as the persistent step kernel (auto where the model allows) "
                        "or as a CUDA graph of one kernel per operation")
    return p.parse_args()


def bf16_peak():
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0  # the profiling recipe's fallback burst figure


def peaks():
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self, index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-i", str(index), "-lms", "100"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        sm, mx, reasons = [], [], set()
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"],
                                 parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def profiled_traffic(name):
    """DRAM bytes (read + write) a launch of the roofline kernel moved in its
    committed ncu capture (profiles/<name>, line traffic_bytes_per_launch),
    or None."""
    path = ROOT / "profiles" / name
    try:
        for line in path.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1])
    except (OSError, ValueError):
        pass
    return None


def algorithmic_bytes_per_step(cfg, context_positions):
    """Bytes a decode pass must move: every Q8_0 weight once (34 bytes per 32
    weights), the norm vectors, the embedding row, the K/V rows it reads and
    the one it writes, its activations."""
    H, F, V, L = cfg.hidden, cfg.ffn, cfg.vocab, cfg.layers
    qd, kvd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    q8 = lambda r, c: r * c * 34 // 32
    layer_w = q8(qd + 2 * kvd, H) + q8(H, qd) + q8(2 * F, H) + q8(H, F) + 2 * H * 4
    head = q8(V, H) + H * 4
    kv_read = 2 * kvd * 4 * context_positions * L
    kv_write = 2 * kvd * 4 * L
    return layer_w * L + head + q8(1, H) + kv_read + kv_write


def cpu_baseline(cfg, seed, prompt_len, budget_s=12.0, sample_layers=2):
    """The oracle (C++ restatement of the reference's Rust CPU path) on the
    host cores: decode passes of `sample_layers` layers at context
    `prompt_len`, plus the head; tok/s extrapolated to all layers."""
    import ctypes as C
    from iris_b200 import _lib
    from iris_b200.model import synth_host_weights
    from oracle import oracle as O
    from oracle.models import OracleModel
    O.build()
    keys = [("EMBED", -1), ("FINAL_NORM", -1), ("HEAD", -1)]
    for l in range(sample_layers):
        keys += [(n, l) for n in ("W_Q", "W_K", "W_V", "W_O", "W_GATE", "W_UP", "W_DOWN", "NORM_ATTN", "NORM_FFN")]
    w = synth_host_weights(cfg, seed, only=keys)
    sub = type(cfg)(**{**cfg.__dict__, "layers": sample_layers})
    om = OracleModel(sub, w)
    threads = O.threads_default()
    rng = np.random.default_rng(seed)
    kvd = cfg.kv_heads * cfg.head_dim
    pk = rng.integers(-(1 << 17), 1 << 17, size=(prompt_len, kvd)).astype(np.int32)
    pv = rng.integers(-(1 << 17), 1 << 17, size=(prompt_len, kvd)).astype(np.int32)
    x = rng.integers(-(2 << 16), 2 << 16, size=(1, cfg.hidden)).astype(np.int32)
    layer_times, t_start = [], time.perf_counter()
    while time.perf_counter() - t_start < budget_s or len(layer_times) < sample_layers:
        l = len(layer_times) % sample_layers
        t0 = time.perf_counter()
        x2, _, _ = om.mistral_layer_range(l, x, prompt_len, pk, pv, threads)
        layer_times.append(time.perf_counter() - t0)
    logits = np.empty(cfg.vocab, np.int32)
    t0 = time.perf_counter()
    rc = O.lib().oracle_head_logits(C.byref(om.model.head), O.ptr(np.ascontiguousarray(x2[0]), C.c_int32),
                                    O.ptr(logits, C.c_int32), threads)
    head_t = time.perf_counter() - t0
    assert rc == 0
    per_token = statistics.mean(layer_times) * cfg.layers + head_t
    return {"value": 1.0 / per_token, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{len(layer_times)} single-layer decode passes (M=1) at context {prompt_len} over "
                      f"{sample_layers} layers + 1 head pass, extrapolated to {cfg.layers} layers; "
                      f"C++ oracle (Rust reference not buildable here), {threads} threads"}


def run_reference(args):
    """--impl reference: the CPU reference path (the oracle port) timed on the
    host cores; each step is one single-layer decode pass at context 2048
    (rotating over 2 layers), the head timed once; tok/s extrapolated."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import ctypes as C
    from iris_b200.model import synth_host_weights
    from iris_b200.shapes import mistral_7b
    from oracle import oracle as O
    from oracle.models import OracleModel
    cfg = mistral_7b()
    O.build()
    sample_layers = 2
    keys = [("EMBED", -1), ("FINAL_NORM", -1), ("HEAD", -1)]
    for l in range(sample_layers):
        keys += [(n, l) for n in ("W_Q", "W_K", "W_V", "W_O", "W_GATE", "W_UP", "W_DOWN", "NORM_ATTN", "NORM_FFN")]
    w = synth_host_weights(cfg, args.seed, only=keys)
    sub = type(cfg)(**{**cfg.__dict__, "layers": sample_layers})
    om = OracleModel(sub, w)
    threads = O.threads_default()
    rng = np.random.default_rng(args.seed)
    kvd = cfg.kv_heads * cfg.head_dim
    pk = rng.integers(-(1 << 17), 1 << 17, size=(args.prompt, kvd)).astype(np.int32)
    pv = rng.integers(-(1 << 17), 1 << 17, size=(args.prompt, kvd)).astype(np.int32)
    x = rng.integers(-(2 << 16), 2 << 16, size=(1, cfg.hidden)).astype(np.int32)
    logits = np.empty(cfg.vocab, np.int32)
    t0 = time.perf_counter()
    O.lib().oracle_head_logits(C.byref(om.model.head), O.ptr(np.ascontiguousarray(x[0]), C.c_int32),
                               O.ptr(logits, C.c_int32), threads)
    head_t = time.perf_counter() - t0
    for i in range(args.warmup):
        om.mistral_layer_range(i % sample_layers, x, args.prompt, pk, pv, threads)
    t0 = time.perf_counter()
    for i in range(args.steps):
        om.mistral_layer_range(i % sample_layers, x, args.prompt, pk, pv, threads)
    layer_t = (time.perf_counter() - t0) / max(args.steps, 1)
    per_token = layer_t * cfg.layers + head_t
    value = 1.0 / per_token
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": layer_t * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int64",
            "data": "synthetic (seeded Q8_0 weights and tokens)",
            "config": {"workload": "mistral-7b-arch decode, 2048-token context, CPU reference path",
                       "model": "mistral-7b-arch", "context": args.prompt, "parallelism": "replicas"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"each step: one single-layer decode pass (M=1) at context {args.prompt}; "
                                       f"tok/s = 1/(32 x mean layer step + head pass); C++ oracle "
                                       f"(the Rust reference cannot be built: no cargo, absent ../raster)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    from iris_b200 import build
    build.build()
    from iris_b200 import _lib
    from iris_b200.model import DeviceModel
    from iris_b200.shapes import mistral_7b
    _lib.check(_lib.lib().q8gpu_init(), "q8gpu_init")

    cfg = mistral_7b()
    seed = args.seed
    if world > 1:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        idt = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            idt.copy_(torch.frombuffer(bytearray(_lib.tp_unique_id()), dtype=torch.uint8))
        dist.broadcast(idt, 0)
        model = DeviceModel(cfg, seed=seed, tp=(rank, world, bytes(idt.cpu().numpy().tobytes())))
        model.set_tp_exchange(args.tp_exchange)
    else:
        model = DeviceModel(cfg, seed=seed)
    e2e_steps = args.steps
    cap = args.prompt + args.warmup + args.steps + e2e_steps + 8
    sess = model.session(cap)
    sess.set_decode_path(args.decode_path)
    prompt = np.random.default_rng(seed).integers(0, cfg.vocab, size=args.prompt).tolist()
    model.prepare_gemm()  # the prefill GEMM's pre-scaled weight copies, built once per model
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    tok, _ = sess.prefill(prompt)
    prefill_s = time.perf_counter() - t0

    # warm-up passes, then exactly `steps` timed passes (events on the session's stream)
    sess.decode_steps(args.warmup)
    sess.synchronize()
    stream = torch.cuda.ExternalStream(sess.stream_ptr)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx0 = sess.length
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    ev0.record(stream)
    sess.decode_steps(args.steps)
    ev1.record(stream)
    sess.synchronize()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    value = args.steps / (ms / 1e3)  # one sequence (tensor-parallel over the N GPUs)
    ms_per_step = ms / args.steps

    # e2e through the C-ABI decode call: host token in, host token out, per step
    tok_in = int(np.random.default_rng(seed + 1).integers(0, cfg.vocab))
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        tok_in, _ = sess.decode(tok_in)
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = e2e_steps / e2e_s

    # The decode GEMV over the fused gate|up matrix (28672 x 4096 Q8_0) as its
    # own launch, once per layer (32 distinct 125 MB matrices, so nothing is
    # served from L2), timed with events on the session's stream: the roofline
    # kernel of the graph path, reported beside the step kernel's.
    sess.product(0, 2)
    sess.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record(stream)
    for _ in range(reps):
        for l in range(cfg.layers):
            sess.product(l, 2)
    e1.record(stream)
    sess.synchronize()
    gemv_ms = e0.elapsed_time(e1) / (reps * cfg.layers)
    n_rows, k = 2 * cfg.ffn // world, cfg.hidden  # this rank's gate|up shard
    gemv_bytes = n_rows * k * 34 // 32 + 4 * k + (n_rows // 2) * 4  # weights + activation row + gated output
    peak, peak_kind = peaks()
    achieved = gemv_bytes / (gemv_ms / 1e3) / 1e9
    mean_ctx = ctx0 + (args.steps - 1) / 2.0 + 1
    step_bytes = algorithmic_bytes_per_step(cfg, mean_ctx)
    step_gbs = step_bytes / (ms_per_step / 1e3) / 1e9  # all ranks' bytes
    gemv_roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": profiled_traffic("q8_gemv_gate_up_28672x4096.md"),
                     "algorithmic_bytes": gemv_bytes,
                     "kernel": "q8_gemv_tma_kernel<IN_NORM, EPI_SILU_MUL> (fused gate|up, 28672x4096)",
                     "peak_kind": peak_kind}
    path = sess.decode_path
    if path == "step":
        # the whole pass is one launch: its algorithmic bytes over the
        # launch's average duration (events around the K timed launches)
        roofline = {"bound": "hbm", "achieved": step_gbs, "peak": peak, "unit": "GB/s",
                    "frac": step_gbs / peak, "traffic": profiled_traffic("decode_step_mistral7b.md"),
                    "algorithmic_bytes": step_bytes,
                    "kernel": "decode_step_kernel<16, 4> (persistent: the whole decode pass, one launch)",
                    "peak_kind": peak_kind}
    else:
        roofline = gemv_roofline

    # The teacher-forced chain's pass: claims are
    # independent, so with N GPUs each rank runs its own claim on its own
    # whole-model copy (replicas; the decode model above is tensor-parallel):
    # 4096 seeded tokens a claim through the device-resident prefill in ranges
    # of 512 rows, every layer's products on the tcgen05 GEMM and attention on
    # the tensor cores. Whole-call time (ids in, first-maximum token out), the
    # maximum over ranks; tok_s counts every rank's tokens.
    chain = None
    if args.chain_tokens > 0:
        cmodel = model
        if world > 1:
            cmodel = DeviceModel(cfg, seed=seed)
            cmodel.prepare_gemm()
        csess = cmodel.session(args.chain_tokens + 8)
        cprompt = np.random.default_rng(seed + 5 + rank).integers(0, cfg.vocab, size=args.chain_tokens).tolist()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        csess.prefill(cprompt)
        cs = time.perf_counter() - t0
        if dist:
            t = torch.tensor([cs], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            cs = float(t.item())
        csess.close()
        if cmodel is not model:
            cmodel.close()
        chain = {"tokens_per_claim": args.chain_tokens, "claims": world, "tok_s": world * args.chain_tokens / cs,
                 "ms": cs * 1e3, "parallelism": "replicas (one claim a GPU)" if world > 1 else "single",
                 "range_rows": 512, "gemm": "q8_gemm_tc_kernel (tcgen05 kind::i8)",
                 "note": "the chain stages' arithmetic through iris_session_prefill; the canonical stage "
                         "records (iris_b200/records.py) are not computed in the timed region"}
    # The prefill GEMM on its own (gate|up shape, 512 tokens: one range, the tensor-core
    # copy of a seeded matrix), timed with events over a captured graph of
    # launches: algorithmic int8 ops 2*M*N*K against the dense int8 peak,
    # which is taken as twice the measured bf16 cuBLAS figure (the nominal
    # int8:bf16 ratio of B200; no int8 GEMM is measured here). The twelve
    # byte-plane MMAs a product issues are reported beside it.
    gemm_roofline = None
    if rank == 0 and world == 1:
        from iris_b200 import microbench
        g = microbench.gemm(argparse.Namespace(seed=seed, rows=2 * cfg.ffn, cols=cfg.hidden, tokens=512,
                                               iters=10, gemm="tc"))
        bf16 = bf16_peak()
        if bf16:
            int8_peak = 2 * bf16
            gemm_roofline = {"bound": "tensor", "achieved": g["TOPS"], "peak": int8_peak, "unit": "TOPS",
                             "frac": g["TOPS"] / int8_peak, "plane_mma_frac": 12 * g["TOPS"] / int8_peak,
                             "us_per_launch": g["us_per_launch"], "shape": [512, 2 * cfg.ffn, cfg.hidden],
                             "kernel": "q8_gemm_tc_kernel<EPI_STORE> (+ planes_kernel)",
                             "peak_kind": "2 x measured bf16 (MEASURED_PEAKS.json)",
                             "traffic": profiled_traffic("q8_gemm_tc_gateup_28672x4096_512tok.md")}

    kernels = sess.kernels_per_pass
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "int64",
        "data": "synthetic (seeded Q8_0 weights, seeded prompt tokens)",
        "config": {"workload": "mistral-7b-arch greedy decode after a 2048-token prompt (BASELINE config 4)",
                   "model": "mistral-7b-arch", "prompt": args.prompt, "context_at_start": ctx0,
                   "global_batch": 1, "parallelism": f"tp{world}" if world > 1 else "single",
                   "tp_exchange": args.tp_exchange if world > 1 else None,
                   "l2": "not flushed: every step streams ~7.6 GB of weights (> 126 MB L2)"},
        "roofline": roofline,
        "gemv_roofline": gemv_roofline,
        "decode_path": path,
        "step_roofline": {"achieved": step_gbs, "peak": peak * world, "unit": "GB/s",
                          "frac": step_gbs / (peak * world), "bytes_per_step": step_bytes},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                "api": "iris_session_decode (host token id in, host token id out)"},
        "gpu_launches": kernels * args.steps,
        "kernels_per_step": kernels,
        "attention": sess.attention_plan,
        "prefill_tok_s": args.prompt / prefill_s,
        "chain_prefill": chain,
        "prefill_gemm_roofline": gemm_roofline,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, seed, args.prompt)
    sess.close()
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()

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
    p.add_argument("--warmup", type=int, default=4)
    p.add_argument("--impl", default="iris", choices=["iris", "reference"])
    p.add_argument("--prompt", type=int, default=2048)
    p.add_argument("--seed", type=int, default=0x1215B200)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-other-configs", action="store_true",
                   help="skip BASELINE configs 1 and 3 (tiny Gemma, Gemma-2B decode) after the main line")
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


def int8_peak_tops(torch):
    """Dense int8 tensor peak measured here: cuBLASLt's int8 GEMM through
    torch._int_mm at 8192^3 (2 N^3 ops), best of 10 launches timed with
    events; twice the measured bf16 figure if that call is unavailable."""
    try:
        a = torch.randint(-128, 128, (8192, 8192), dtype=torch.int8, device="cuda")
        b = torch.randint(-128, 128, (8192, 8192), dtype=torch.int8, device="cuda")
        for _ in range(3):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b
        return 2 * 8192 ** 3 / (best / 1e3) / 1e12, "measured int8 (cuBLASLt via torch._int_mm, 8192^3, this run)"
    except Exception:
        return 2 * bf16_peak(), "2 x measured bf16 (MEASURED_PEAKS.json)"


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
                                       "-i", str(index), "-lms", "50"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        # nvidia-smi takes a moment to start: the timed region begins once it
        # has written its first sample (at most ~10 s)
        t0 = time.monotonic()
        while self.p and self.p.poll() is None and time.monotonic() - t0 < 10:
            if os.path.getsize(self.f.name) > 0:
                break
            time.sleep(0.02)

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


def layer_weights(cfg):
    """Weights of one mistral-dense layer (q, k, v, o, gate, up, down)."""
    H, F = cfg.hidden, cfg.ffn
    qd, kvd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    return H * (qd + 2 * kvd) + qd * H + 3 * H * F


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


def gemma_decode_bytes(cfg, context):
    """Algorithmic bytes of one gemma-dense decode pass: every Q8_0 weight
    once (layers and the tied head), the per-layer dense PLE matrices and the
    model projection (int32), the token's PLE embedding row, the norm
    vectors, the K/V rows each layer's window reads and the row it writes."""
    H, F, V, L, P = cfg.hidden, cfg.ffn, cfg.vocab, cfg.layers, cfg.ple_width
    qd, kvd, d = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.head_dim
    q8 = lambda r, c: r * c * 34 // 32
    layer = q8(qd + 2 * kvd, H) + q8(H, qd) + q8(2 * F, H) + q8(H, F) + 2 * P * H * 4 + (5 * H + 2 * d) * 4
    kv = sum(2 * kvd * 4 * (min(context, cfg.window(l)) if cfg.window(l) else context) for l in range(L))
    return L * layer + q8(V, H) + L * P * H * 4 + q8(1, L * P) + P * 4 + H * 4 + kv + 2 * kvd * 4 * L


def other_configs(torch, seed, peak):
    """BASELINE configs 1 and 3 on this GPU (device-resident decode loop,
    CUDA events on the session stream around the timed passes):
    - config 1, tiny Gemma: 32-token prompt, 64 greedy steps; the same
      workload through the oracle's decode loop on the host cores beside it;
    - config 3, Gemma-2B architecture (18 layers, 256k tied head, PLE 256):
      512-token prompt, 256 greedy steps, with the HBM fraction of the passes'
      algorithmic bytes (no CPU figure: the oracle's 512-token prompt pass
      alone takes minutes)."""
    from iris_b200.model import DeviceModel, synth_host_weights
    from iris_b200.shapes import gemma_2b, tiny_gemma
    from oracle.models import OracleModel
    out = {}
    for name, cfg, n_prompt, steps in (("config1_tiny_gemma", tiny_gemma(), 32, 64),
                                       ("config3_gemma_2b", gemma_2b(), 512, 256)):
        tiny = name.startswith("config1")
        w = synth_host_weights(cfg, seed) if tiny else None
        dm = DeviceModel(cfg, weights=w) if tiny else DeviceModel(cfg, seed=seed)
        dm.prepare_gemm()
        prompt = np.random.default_rng(seed + 3).integers(0, cfg.vocab, size=n_prompt).tolist()
        sess = dm.session(n_prompt + steps + 8)
        stream = torch.cuda.ExternalStream(sess.stream_ptr)
        times = []
        for _ in range(2):  # the first run warms the captured pass up
            sess.reset()
            sess.prefill(prompt)
            sess.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            sess.decode_steps(steps)
            e1.record(stream)
            sess.synchronize()
            times.append(e0.elapsed_time(e1) / 1e3)
        t = times[-1]
        t0 = time.perf_counter()
        toks, _ = sess.generate(prompt, steps)
        e2e = time.perf_counter() - t0
        r = {"workload": f"{cfg.name}: {n_prompt}-token prompt, {steps} greedy steps",
             "decode_tok_s": steps / t, "ms_per_step": t * 1e3 / steps,
             "e2e_generate_s": e2e, "api_e2e": "iris_generate (prompt in, tokens out, prefill included)",
             "decode_path": sess.decode_path, "kernels_per_step": sess.kernels_per_pass}
        mean_ctx = n_prompt + (steps + 1) / 2
        nbytes = gemma_decode_bytes(cfg, mean_ctx)
        r["roofline"] = {"bound": "hbm", "achieved": nbytes / (t / steps) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": nbytes / (t / steps) / 1e9 / peak, "bytes_per_step": nbytes}
        if tiny:
            t0 = time.perf_counter()
            want, _ = OracleModel(cfg, w).generate(prompt, steps, want_logits=False)
            cpu = time.perf_counter() - t0
            r["cpu_baseline"] = {"value": steps / cpu, "unit": "tok/s", "kind": "port", "cores": os.cpu_count(),
                                 "sample": "the oracle's decode loop (prompt pass included) on all host threads"}
            r["tokens_equal_oracle"] = toks == want
        sess.close()
        dm.close()
        out[name] = r
    return out


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def decode_config(prompt, warmup, world, tp_exchange):
    """The `config` object of the decode line, the same for both arms."""
    return {"workload": f"mistral-7b-arch greedy decode after a {prompt}-token prompt (BASELINE config 4)",
            "model": "mistral-7b-arch", "prompt": prompt, "context_at_start": prompt + warmup,
            "global_batch": 1, "parallelism": f"tp{world}" if world > 1 else "single",
            "tp_exchange": tp_exchange if world > 1 else None,
            "l2": "not flushed: every step streams ~7.6 GB of weights (> 126 MB L2)"}


def cpu_decode(seed, prompt_len, warmup, steps):
    """Whole decode passes of the Mistral-7B-architecture model on the host
    cores through the oracle (the C++ restatement of the reference's Rust CPU
    path, row-sharded over all host threads as tensor.rs:175-185): the same
    seeded weights as the device model, generated by the oracle's own copy of
    the generator (the product library is not loaded). The K/V of the
    `prompt_len` context positions are seeded random rows in place of a CPU
    prompt pass (a pass's arithmetic does not depend on their values); each
    pass then runs the token at the next position through all 32 layers and
    the head and selects the first maximum, which feeds the next pass.
    Returns (seconds a pass over `steps` timed passes, threads)."""
    from oracle import oracle as O
    from oracle.models import CpuDecoder, OracleModel, mistral_7b_shape, synth_mistral_weights
    O.build()
    threads = O.threads_default()
    cfg = mistral_7b_shape()
    om = OracleModel(cfg, synth_mistral_weights(cfg, seed, threads=threads))
    dec = CpuDecoder(om, prompt_len + warmup + steps + 1, threads)
    dec.fill(prompt_len, seed)
    tok = int(np.random.default_rng(seed).integers(0, cfg.vocab))
    for _ in range(warmup):
        tok = dec.step(tok)
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = dec.step(tok)
    return (time.perf_counter() - t0) / max(steps, 1), threads


def cpu_baseline(seed, prompt_len, steps=4):
    """The GPU arm's reported CPU baseline: a bounded sample (one untimed and
    `steps` timed whole decode passes, ~10 s of CPU work on 16 cores)."""
    per_pass, threads = cpu_decode(seed, prompt_len, 1, steps)
    return {"value": 1.0 / per_pass, "unit": UNIT, "cores": threads, "kind": "port",
            "cpu_model": cpu_model(), "nproc": os.cpu_count(),
            "sample": f"{steps} whole 32-layer decode passes (+ head, first maximum) at context {prompt_len + 2}.."
                      f"{prompt_len + steps + 1}, seeded random K/V in place of the CPU prompt pass; C++ oracle "
                      f"(the Rust reference is not buildable here), {threads} threads"}


def run_reference(args):
    """--impl reference: the reference's CPU path (the oracle port: the Rust
    workspace cannot be built here) timed on the host cores, on this arm's
    metric and config: W untimed and K timed whole decode passes of the
    Mistral-7B-architecture model (32 layers + head + first maximum) after a
    `prompt`-token context, all host threads. Rank 0 alone runs and prints;
    the other ranks of a torchrun launch exit without work. Imports only the
    oracle (no product library)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    per_pass, threads = cpu_decode(args.seed, args.prompt, args.warmup, args.steps)
    value = 1.0 / per_pass
    sample = (f"each step: one whole 32-layer decode pass (+ head, first maximum) at context "
              f"{args.prompt + args.warmup + 1}..{args.prompt + args.warmup + args.steps}, seeded random K/V "
              f"in place of the CPU prompt pass; C++ oracle (the Rust reference cannot be built: no cargo, "
              f"absent ../raster), {threads} threads")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_pass * 1e3,
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "int64", "data": "synthetic (seeded Q8_0 weights, seeded prompt tokens)",
            "config": decode_config(args.prompt, args.warmup, world, args.tp_exchange),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "cpu_model": cpu_model(), "nproc": os.cpu_count(), "sample": sample},
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
    sess.prefill(prompt)  # warm: the session's attention scratch is sized on first use
    sess.reset()
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
    clocks = Clocks(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
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
                    "kernel": "decode_step_kernel<16, 4, true> (persistent: the whole decode pass, one launch; "
                              "the one-scale-a-row form the benchmark's weights take)",
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
        from iris_b200 import records
        csess = cmodel.session(args.chain_tokens + 8)
        cprompt = np.random.default_rng(seed + 5 + rank).integers(0, cfg.vocab, size=args.chain_tokens).tolist()
        # warm: buffers, pinned memory, kernels, and the attention scratch every
        # range position of the claim needs (sized on first use)
        records.chain_claim(csess, cprompt, range_size=512)
        csess.reset()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        recs, selected, _ = records.chain_claim(csess, cprompt, range_size=512)
        cs = time.perf_counter() - t0
        # the stages' arithmetic alone: the same claim through iris_session_prefill
        csess.reset()
        t0 = time.perf_counter()
        csess.prefill(cprompt)
        arith = time.perf_counter() - t0
        if dist:
            t = torch.tensor([cs, arith], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            cs, arith = (float(x) for x in t.tolist())
        csess.close()
        if cmodel is not model:
            cmodel.close()
        import hashlib
        T, L = args.chain_tokens, cfg.layers
        ops = 2 * T * layer_weights(cfg) * L + 4 * cfg.heads * cfg.head_dim * T * (T + 1) // 2 * L  # + QK and PV
        int8_peak_c = int8_peak_tops(torch)[0] if rank == 0 else None
        chain = {"tokens_per_claim": T, "claims": world, "tok_s": world * T / cs, "ms": cs * 1e3,
                 "tok_s_per_gpu": T / cs, "stages": len(recs), "range_rows": 512,
                 "records_digest": hashlib.sha256("".join(d for _, _, d in recs).encode()).hexdigest(),
                 "selected_first": [int(x) for x in selected[:4]],
                 "parallelism": "replicas (one claim a GPU)" if world > 1 else "single",
                 "api": "iris_session_range_begin/_layer_leaves/_end per range and layer (records.chain_claim)",
                 "in_timed_region": "every stage (32 layers x 8 ranges) on the device, its rows and own K/V "
                                    "hashed on the device into the canonical record's SHA-256 leaf digests "
                                    "(4096-byte leaves), the leaves copied out and the record digest taken on "
                                    "host threads, the head check's first maximum for every row",
                 "arith_only_ms": arith * 1e3, "arith_only_tok_s": T / arith,
                 "algorithmic_int8_ops": ops,
                 "int8_frac": (ops / cs / 1e12 / int8_peak_c) if int8_peak_c else None,
                 "gemm": "q8_gemm_tc_kernel (tcgen05 kind::i8)"}
    # The prefill GEMM on its own (gate|up shape, 512 tokens: one range), timed
    # with events over a captured graph of launches: algorithmic int8 ops
    # 2*M*N*K against the dense int8 peak measured in this run (cuBLASLt int8
    # GEMM through torch._int_mm, 8192^3). Two forms of the tensor-core copy:
    # one plane (the benchmark's weights have one scale a row: four byte-plane
    # MMAs a product) and three planes (what per-block scales need: twelve).
    gemm_roofline = gemm_roofline3 = None
    if rank == 0 and world == 1:
        from iris_b200 import microbench
        int8_peak, int8_kind = int8_peak_tops(torch)
        for form, planes_mmas in (("tc", 4), ("tc3", 12)):
            g = microbench.gemm(argparse.Namespace(seed=seed, rows=2 * cfg.ffn, cols=cfg.hidden, tokens=512,
                                                   iters=10, gemm=form))
            r = {"bound": "tensor", "achieved": g["TOPS"], "peak": int8_peak, "unit": "TOPS",
                 "frac": g["TOPS"] / int8_peak, "plane_mma_frac": planes_mmas * g["TOPS"] / int8_peak,
                 "us_per_launch": g["us_per_launch"], "shape": [512, 2 * cfg.ffn, cfg.hidden],
                 "kernel": "planes_kernel + " + g["kernel"].split("planes_kernel + ")[-1], "peak_kind": int8_kind,
                 "traffic": profiled_traffic("q8_gemm_tc1_gateup_28672x4096_512tok.md" if form == "tc"
                                             else "q8_gemm_tc3_gateup_28672x4096_512tok.md")}
            if form == "tc":
                gemm_roofline = r
            else:
                gemm_roofline3 = r

    kernels = sess.kernels_per_pass
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "int64",
        "data": "synthetic (seeded Q8_0 weights, seeded prompt tokens)",
        "config": decode_config(args.prompt, args.warmup, world, args.tp_exchange),
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
        "prefill_gemm_roofline_per_block_scales": gemm_roofline3,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_other_configs:
        line["other_configs"] = other_configs(torch, seed, peak)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(seed, args.prompt)
    sess.close()
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()

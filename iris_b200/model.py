"""Device-resident models and decoding sessions (the direct-infer path).

Host-side mirror of the reference's direct executor
(crates/inference/direct/src/executor.rs:41-186): a model is loaded once into
HBM; a Session keeps every layer's K/V on the device; `generate` is the decode
loop (prefill, then greedy first-maximum selection until EOS or the budget).
All arithmetic runs in libiris_b200.so.
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib
from ._lib import T, check, lib, ptr
from .shapes import GemmaConfig, MistralConfig

Key = Tuple[str, int]  # (tensor name, layer or -1)
KeyRows = Tuple[np.ndarray, np.ndarray, np.ndarray]  # (positions, k rows, v rows)


def tensor_table(cfg) -> Dict[Key, tuple]:
    """(kind, rows, cols, fan_in) of every tensor; kind is 'q8' or 'values'."""
    H, F, V, L = cfg.hidden, cfg.ffn, cfg.vocab, cfg.layers
    qd, kvd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    t: Dict[Key, tuple] = {("EMBED", -1): ("q8", V, H, 0), ("FINAL_NORM", -1): ("values", 1, H, 0)}
    if not cfg.tied:
        t[("HEAD", -1)] = ("q8", V, H, 0)
    for l in range(L):
        t[("W_Q", l)] = ("q8", qd, H, 0)
        t[("W_K", l)] = ("q8", kvd, H, 0)
        t[("W_V", l)] = ("q8", kvd, H, 0)
        t[("W_O", l)] = ("q8", H, qd, 0)
        t[("W_GATE", l)] = ("q8", F, H, 0)
        t[("W_UP", l)] = ("q8", F, H, 0)
        t[("W_DOWN", l)] = ("q8", H, F, 0)
        t[("NORM_ATTN", l)] = ("values", 1, H, 0)
        t[("NORM_FFN", l)] = ("values", 1, H, 0)
        if cfg.family == "gemma":
            P, d = cfg.ple_width, cfg.head_dim
            for n in ("NORM_POST_ATTN", "NORM_POST_FFW", "PLE_POST_NORM"):
                t[(n, l)] = ("values", 1, H, 0)
            t[("Q_NORM", l)] = ("values", 1, d, 0)
            t[("K_NORM", l)] = ("values", 1, d, 0)
            t[("PLE_INPUT_GATE", l)] = ("values", P, H, H)
            t[("PLE_LAYER_PROJECTION", l)] = ("values", H, P, P)
    if cfg.family == "gemma":
        P = cfg.ple_width
        t[("PLE_EMBED", -1)] = ("q8", V, L * P, 0)
        t[("PLE_MODEL_PROJECTION", -1)] = ("values", L * P, H, H)
        t[("PLE_NORM", -1)] = ("values", 1, P, 0)
    return t


def synth_host_weights(cfg, seed: int, per_block: bool = False,
                       only: Optional[Iterable[Key]] = None) -> Dict[Key, np.ndarray]:
    """The seeded synthetic tensors, generated on the host by the same code the
    device runs in `DeviceModel.synthesize` (iris_b200/csrc/synth.cuh); Q8_0
    tensors in row chunks on a thread pool (the C calls run without the GIL)."""
    import os
    from concurrent.futures import ThreadPoolExecutor
    out = {}
    table = tensor_table(cfg)
    keys = list(only) if only is not None else list(table)
    jobs = []
    for key in keys:
        kind, rows, cols, fan = table[key]
        name, layer = key
        if kind == "q8":
            buf = np.empty(rows * (cols // 32) * 34, np.uint8)
            out[key] = buf
            step = max(1, (1 << 22) // cols)  # ~4 MB of weights a job
            for r0 in range(0, rows, step):
                n = min(step, rows - r0)
                view = buf[r0 * (cols // 32) * 34:(r0 + n) * (cols // 32) * 34]
                jobs.append((T[name], layer, n, cols, r0, view))
        else:
            out[key] = _lib.synth_values(seed, T[name], layer, rows * cols, fan)

    def run(job):
        tensor, layer, n, cols, r0, view = job
        check(lib().iris_synth_q8_block(seed, tensor, layer, n, cols, r0, 0, cols, int(per_block),
                                        ptr(view, C.c_uint8)), "iris_synth_q8_block")

    with ThreadPoolExecutor(max_workers=min(32, os.cpu_count() or 1)) as pool:
        list(pool.map(run, jobs))
    return out


class DeviceModel:
    """A model whose weights live in HBM (IrisModel)."""

    def __init__(self, cfg, weights: Optional[Dict[Key, np.ndarray]] = None, seed: Optional[int] = None,
                 per_block: bool = False, tp: Optional[Tuple[int, int, bytes]] = None):
        """`tp` = (rank, world, nccl_id): this process's shard of a tensor-parallel
        mistral-dense model (weights synthesized on the device from `seed`;
        every rank makes the same calls in the same order)."""
        self.cfg = cfg
        self.tp = tp
        self._h = C.c_void_p()
        L = lib()
        if cfg.family == "mistral":
            self._freqs = np.array(cfg.freqs, dtype=np.int64)
            shape = _lib.MistralShape(cfg.layers, cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.head_dim,
                                      cfg.vocab, cfg.max_positions, cfg.norm_eps, cfg.scale_q32, int(cfg.tied),
                                      ptr(self._freqs, C.c_int64))
            if tp is not None and tp[1] > 1:
                if weights is not None or seed is None:
                    raise ValueError("tensor-parallel shards are synthesized on the device: give `seed`")
                rank, world, nccl_id = tp
                idb = np.frombuffer(bytes(nccl_id), np.uint8).copy()
                check(L.iris_model_create_mistral_tp(C.byref(shape), rank, world, ptr(idb, C.c_uint8),
                                                     C.byref(self._h)), "iris_model_create_mistral_tp")
            else:
                check(L.iris_model_create_mistral(C.byref(shape), C.byref(self._h)), "iris_model_create_mistral")
        else:
            n = cfg.layers
            self._win = np.array([cfg.window(l) for l in range(n)], np.uint32)
            rope = [cfg.rope(l) for l in range(n)]
            self._base = np.array([r[0] for r in rope], np.int64)
            self._rot = np.array([r[1] for r in rope], np.uint32)
            self._fbd = np.array([r[2] for r in rope], np.uint32)
            self._donor = np.array([cfg.kv_donor(l) for l in range(n)], np.int32)
            self._scal = np.array(cfg.layer_scalars or [0] * n, np.int32)
            shape = _lib.GemmaShape(n, cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.vocab,
                                    cfg.ple_width, cfg.norm_eps, cfg.embedding_scale, cfg.ple_embedding_scale,
                                    cfg.ple_projection_scalar, cfg.ple_input_scale, cfg.softcap_bits,
                                    ptr(self._win, C.c_uint32), ptr(self._base, C.c_int64),
                                    ptr(self._rot, C.c_uint32), ptr(self._fbd, C.c_uint32),
                                    ptr(self._donor, C.c_int32), ptr(self._scal, C.c_int32), int(cfg.tied))
            check(L.iris_model_create_gemma(C.byref(shape), C.byref(self._h)), "iris_model_create_gemma")
        if weights is not None:
            self.load(weights)
        elif seed is not None:
            self.synthesize(seed, per_block)

    @property
    def handle(self):
        return self._h

    def set_tp_exchange(self, mode: str) -> None:
        """'peer' (NVLink loads of the peers' partial sums; default) or 'nccl'."""
        check(lib().iris_model_set_tp_exchange(self._h, {"peer": 0, "nccl": 1}[mode]), "iris_model_set_tp_exchange")

    def load(self, weights: Dict[Key, np.ndarray]) -> None:
        table = tensor_table(self.cfg)
        for key, arr in weights.items():
            name, layer = key
            kind = table[key][0]
            if kind == "q8":
                a = np.ascontiguousarray(arr, dtype=np.uint8)
                check(lib().iris_model_set_q8(self._h, T[name], layer, ptr(a, C.c_uint8), a.size),
                      f"iris_model_set_q8 {key}")
            else:
                a = np.ascontiguousarray(arr, dtype=np.int32)
                check(lib().iris_model_set_values(self._h, T[name], layer, ptr(a, C.c_int32), a.size),
                      f"iris_model_set_values {key}")

    def synthesize(self, seed: int, per_block: bool = False) -> None:
        check(lib().iris_model_synthesize(self._h, seed, int(per_block)), "iris_model_synthesize")

    def get(self, key: Key) -> np.ndarray:
        kind, rows, cols, _ = tensor_table(self.cfg)[key]
        name, layer = key
        if kind == "q8":
            out = np.empty(rows * (cols // 32) * 34, np.uint8)
            check(lib().iris_model_get_q8(self._h, T[name], layer, ptr(out, C.c_uint8), out.size), "get_q8")
        else:
            out = np.empty(rows * cols, np.int32)
            check(lib().iris_model_get_values(self._h, T[name], layer, ptr(out, C.c_int32), out.size),
                  "get_values")
        return out

    @property
    def weight_bytes(self) -> int:
        return int(lib().iris_model_weight_bytes(self._h))

    def set_gemm(self, mode: str) -> None:
        """Many-token products: 'auto' (tcgen05 tensor-core GEMM where a matrix
        qualifies, default) or 'mma' (the mma.sync GEMM only)."""
        check(lib().iris_model_set_gemm(self._h, {"auto": 0, "mma": 1}[mode]), "iris_model_set_gemm")

    def prepare_gemm(self) -> None:
        """Builds the tensor-core copies of the layer matrices now (not on first use)."""
        check(lib().iris_model_prepare_gemm(self._h), "iris_model_prepare_gemm")

    def embed(self, ids: Sequence[int]) -> np.ndarray:
        """The embedding rows [n][hidden] of token ids (the chain's first input)."""
        a = np.ascontiguousarray(ids, np.uint32)
        out = np.empty((a.size, self.cfg.hidden), np.int32)
        check(lib().iris_model_embed(self._h, ptr(a, C.c_uint32), a.size, ptr(out, C.c_int32)), "iris_model_embed")
        return out

    def sequence_check_select(self, rows: np.ndarray):
        """The chain's head check over predicting rows [n][hidden]: the
        first-maximum token id and its score for each row."""
        r = np.ascontiguousarray(rows, np.int32)
        n = r.shape[0]
        tok = np.empty(n, np.uint32)
        val = np.empty(n, np.int32)
        check(lib().iris_sequence_check_select(self._h, ptr(r, C.c_int32), n, ptr(tok, C.c_uint32),
                                               ptr(val, C.c_int32)), "iris_sequence_check_select")
        return tok, val

    def tc_matrices(self):
        """(number of matrices with a tensor-core copy, device bytes of those copies)."""
        b = C.c_uint64(0)
        n = lib().iris_model_tc_matrices(self._h, C.byref(b))
        return int(n), int(b.value)

    def attention_ranges(self):
        """(many-query attention launches on the tensor cores, on CUDA cores) so far."""
        v = (C.c_uint64 * 2)()
        check(lib().iris_model_attention_ranges(self._h, v), "iris_model_attention_ranges")
        return int(v[0]), int(v[1])

    def session(self, max_positions: int) -> "Session":
        return Session(self, max_positions)

    def layer_range(self, layer: int, rows: np.ndarray, start: int, prior_k: Optional[np.ndarray],
                    prior_v: Optional[np.ndarray]):
        """One mistral-dense layer over a range (mistral/stage.rs:172-226):
        returns (rows_out, own_k, own_v)."""
        rows = np.ascontiguousarray(rows, np.int32)
        m = rows.shape[0]
        kvd = self.cfg.kv_heads * self.cfg.head_dim
        out = np.empty_like(rows)
        ok = np.empty((m, kvd), np.int32)
        ov = np.empty((m, kvd), np.int32)
        pk = np.ascontiguousarray(prior_k if prior_k is not None else np.zeros((0, kvd)), np.int32)
        pv = np.ascontiguousarray(prior_v if prior_v is not None else np.zeros((0, kvd)), np.int32)
        check(lib().iris_mistral_layer_range(self._h, layer, ptr(rows, C.c_int32), m, start,
                                             ptr(pk, C.c_int32) if start else None,
                                             ptr(pv, C.c_int32) if start else None,
                                             ptr(out, C.c_int32), ptr(ok, C.c_int32), ptr(ov, C.c_int32)),
              "iris_mistral_layer_range")
        return out, ok, ov

    def ple_rows(self, ids: Sequence[int]) -> np.ndarray:
        """gemma-dense: the PLE rows [n][layers][ple] of token ids (view_kernels.rs:59-99)."""
        a = np.ascontiguousarray(ids, np.uint32)
        out = np.empty((a.size, self.cfg.layers, self.cfg.ple_width), np.int32)
        check(lib().iris_model_ple_rows(self._h, ptr(a, C.c_uint32), a.size, ptr(out, C.c_int32)),
              "iris_model_ple_rows")
        return out

    def gemma_layer_range(self, layer: int, rows: np.ndarray, start: int, ple_rows: np.ndarray,
                          prior: Optional[KeyRows] = None, donor: Optional[KeyRows] = None):
        """One gemma-dense layer over a range (prefill_range.rs:82-172):
        returns (rows_out, own_k, own_v). `prior`: the layer's carried keys
        (positions, k, v); `donor`: the donor layer's keys for a layer that
        shares them."""
        rows = np.ascontiguousarray(rows, np.int32)
        m = rows.shape[0]
        kvd = self.cfg.kv_heads * self.cfg.head_dim
        ple = np.ascontiguousarray(ple_rows, np.int32)
        out = np.empty_like(rows)
        ok = np.empty((m, kvd), np.int32)
        ov = np.empty((m, kvd), np.int32)
        args, keep = [], []  # keep: the arrays behind the pointers, alive until the call returns
        for keys in (prior, donor):
            if keys is None or len(keys[0]) == 0:
                args += [0, None, None, None]
            else:
                pos = np.ascontiguousarray(keys[0], np.uint32)
                k = np.ascontiguousarray(keys[1], np.int32)
                v = np.ascontiguousarray(keys[2], np.int32)
                keep += [pos, k, v]
                args += [pos.size, ptr(pos, C.c_uint32), ptr(k, C.c_int32), ptr(v, C.c_int32)]
        check(lib().iris_gemma_layer_range(self._h, layer, ptr(rows, C.c_int32), m, start, ptr(ple, C.c_int32),
                                           *args, ptr(out, C.c_int32), ptr(ok, C.c_int32), ptr(ov, C.c_int32)),
              "iris_gemma_layer_range")
        return out, ok, ov

    def close(self) -> None:
        if self._h:
            lib().iris_model_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """A decoding session: the K/V cache of every layer, in HBM."""

    def __init__(self, model: DeviceModel, max_positions: int):
        self.model = model
        self._h = C.c_void_p()
        check(lib().iris_session_create(model.handle, max_positions, C.byref(self._h)), "iris_session_create")

    @property
    def handle(self):
        return self._h

    def set_tp_exchange(self, mode: str) -> None:
        """'peer' (NVLink loads of the peers' partial sums; default) or 'nccl'."""
        check(lib().iris_model_set_tp_exchange(self._h, {"peer": 0, "nccl": 1}[mode]), "iris_model_set_tp_exchange")

    def reset(self) -> None:
        check(lib().iris_session_reset(self._h), "iris_session_reset")

    def prefill(self, ids: Sequence[int], want_logits: bool = False):
        a = np.ascontiguousarray(ids, np.uint32)
        logits = np.empty(self.model.cfg.vocab, np.int32) if want_logits else None
        tok = C.c_uint32()
        check(lib().iris_session_prefill(self._h, ptr(a, C.c_uint32), a.size,
                                         ptr(logits, C.c_int32) if logits is not None else None,
                                         C.byref(tok)), "iris_session_prefill")
        return tok.value, logits

    def decode(self, token: int, want_logits: bool = False):
        logits = np.empty(self.model.cfg.vocab, np.int32) if want_logits else None
        tok = C.c_uint32()
        check(lib().iris_session_decode(self._h, token, ptr(logits, C.c_int32) if logits is not None else None,
                                        C.byref(tok)), "iris_session_decode")
        return tok.value, logits

    def generate(self, prompt: Sequence[int], max_tokens: int, eos: Sequence[int] = (),
                 want_logits: bool = False):
        p = np.ascontiguousarray(prompt, np.uint32)
        e = np.ascontiguousarray(list(eos) or [0], np.uint32)
        out = np.zeros(max(max_tokens, 1), np.uint32)
        count = C.c_uint32()
        logits = np.zeros((max(max_tokens, 1), self.model.cfg.vocab), np.int32) if want_logits else None
        check(lib().iris_generate(self._h, ptr(p, C.c_uint32), p.size, max_tokens, ptr(e, C.c_uint32),
                                  len(list(eos)), ptr(out, C.c_uint32), C.byref(count),
                                  ptr(logits, C.c_int32) if logits is not None else None), "iris_generate")
        n = count.value
        return out[:n].tolist(), (logits[:n] if logits is not None else None)

    @property
    def length(self) -> int:
        return int(lib().iris_session_length(self._h))

    def decode_steps(self, steps: int) -> None:
        """Replays the captured decode pass `steps` times without waiting."""
        check(lib().iris_session_decode_steps(self._h, steps), "iris_session_decode_steps")

    def synchronize(self) -> None:
        check(lib().iris_session_synchronize(self._h), "iris_session_synchronize")

    @property
    def stream_ptr(self) -> int:
        return int(lib().iris_session_stream(self._h) or 0)

    @property
    def kernels_per_pass(self) -> int:
        return int(lib().iris_session_graph_kernels(self._h))

    def product(self, layer: int, which: int) -> None:
        check(lib().iris_session_product(self._h, layer, which), "iris_session_product")

    def attention(self, layer: int) -> None:
        """Launches one single-query attention of `layer` (for timing)."""
        check(lib().iris_session_attention(self._h, layer), "iris_session_attention")

    def set_attention(self, mode: str) -> None:
        """'auto' (whole-GPU launch, else cluster, else split), 'split' (three
        launches) or 'cluster' (the cluster launch where possible)."""
        check(lib().iris_session_set_attention(self._h, {"auto": 0, "split": 1, "cluster": 2}[mode]),
              "iris_session_set_attention")

    @property
    def attention_plan(self) -> dict:
        """The decode attention in use (path, heads a block, blocks, positions a block)."""
        plan = (C.c_uint32 * 4)()
        check(lib().iris_session_attention_plan(self._h, plan), "iris_session_attention_plan")
        return {"path": {4: "step", 3: "grid", 2: "cluster", 1: "split"}[plan[0]], "heads_per_block": plan[1],
                "blocks": plan[2], "positions_per_block": plan[3]}

    def set_decode_path(self, mode: str) -> None:
        """'auto' (the persistent step where the model allows it), 'graph'
        (a CUDA graph of one kernel per operation) or 'step' (one cooperative
        launch a pass; refused where the model does not allow it)."""
        check(lib().iris_session_set_decode_path(self._h, {"auto": 0, "graph": 1, "step": 2}[mode]),
              "iris_session_set_decode_path")

    @property
    def decode_path(self) -> str:
        return {1: "graph", 2: "step"}[lib().iris_session_decode_path(self._h)]

    def step_trace(self, enable: bool) -> None:
        """Per-stage timeline of every persistent-step pass (profiling)."""
        check(lib().iris_session_step_trace(self._h, int(enable)), "iris_session_step_trace")

    def get_step_trace(self):
        """The last pass's stamps as [blocks][stages][8] uint64 ns."""
        plan = self.step_plan
        stages = 2 + 5 * self.model.cfg.layers
        out = np.zeros((plan["blocks"], stages, 8), np.uint64)
        check(lib().iris_session_get_step_trace(self._h, out.ctypes.data_as(C.POINTER(C.c_uint64)), out.size),
              "iris_session_get_step_trace")
        return out

    @property
    def step_plan(self) -> dict:
        """The persistent step's plan (why 0 when usable)."""
        v = (C.c_uint32 * 8)()
        check(lib().iris_session_step_plan(self._h, v), "iris_session_step_plan")
        keys = ("why", "blocks", "ring_slots", "slot_bytes", "planes_bytes", "smem", "chunks", "span_max")
        return dict(zip(keys, list(v)))

    def set_attention_shape(self, cluster: int, hpc: int, ring: int) -> None:
        """Explicit one-launch decode attention shape (tuning)."""
        check(lib().iris_session_set_attention_shape(self._h, cluster, hpc, ring), "iris_session_set_attention_shape")

    def kv(self, layer: int, first: int, count: int):
        kvd = self.model.cfg.kv_heads * self.model.cfg.head_dim
        k = np.empty((count, kvd), np.int32)
        v = np.empty((count, kvd), np.int32)
        check(lib().iris_session_get_kv(self._h, layer, first, count, ptr(k, C.c_int32), ptr(v, C.c_int32)),
              "iris_session_get_kv")
        return k, v

    def close(self) -> None:
        for sets in getattr(self, "_pinned_sets", {}).values():  # records.chain_claim's buffers
            for group in sets:
                for b in group:
                    b.free()
        self._pinned_sets = {}
        if self._h:
            lib().iris_session_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

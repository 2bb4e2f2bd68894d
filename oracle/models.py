"""TEST INFRASTRUCTURE ONLY: builds the oracle's model structs from host
tensors (the same bytes the device model is loaded with), the seeded
synthetic weights of the benchmark configurations, and the CPU decode pass
the CPU legs time.

Used by tests/, __graft_entry__.smoke() and bench.py's CPU legs (its
reference arm and CPU baseline); nothing here loads the product library.
"""
from __future__ import annotations

import ctypes as C
from types import SimpleNamespace

import numpy as np

from . import oracle as O

# Tensor ids of the seeded generator: the numbering of the product's tensor
# kinds, so that both sides hash the same (tensor, layer, index).
SYNTH_IDS = {"EMBED": 0, "HEAD": 1, "FINAL_NORM": 2, "W_Q": 3, "W_K": 4, "W_V": 5, "W_O": 6, "W_GATE": 7,
             "W_UP": 8, "W_DOWN": 9, "NORM_ATTN": 10, "NORM_FFN": 11}


def synth_q8(seed, name, layer, rows, cols, per_block=False, threads=None):
    out = np.empty(rows * (cols // 32) * 34, np.uint8)
    if O.lib().oracle_synth_q8(seed, SYNTH_IDS[name], layer, rows, cols, int(per_block), O.ptr(out, C.c_uint8),
                               threads or O.threads_default()):
        raise ValueError("oracle_synth_q8: bad shape")
    return out


def synth_values(seed, name, layer, count, fan_in=0, threads=None):
    out = np.empty(count, np.int32)
    if O.lib().oracle_synth_values(seed, SYNTH_IDS[name], layer, count, fan_in, O.ptr(out, C.c_int32),
                                   threads or O.threads_default()):
        raise ValueError("oracle_synth_values: bad arguments")
    return out


def mistral_7b_shape(layers=32):
    """BASELINE config 4's mistral-dense shape (L32, H4096, F14336, 32q/8kv,
    d128, V32000, untied head, RoPE base 1e6 as the factor-1 YaRN table,
    eps 1e-5), its derived values computed by the oracle's own restatements
    of mistral.rs:148-160 / 185-214 and convert.rs."""
    d = 128
    freqs = np.zeros(d // 2, np.int64)
    if O.lib().oracle_yarn_inverse_frequencies(1_000_000, d // 2, 1, 0, 1, O.ptr(freqs, C.c_int64)):
        raise ValueError("yarn_inverse_frequencies refused the plain table")
    return SimpleNamespace(name="mistral-7b-arch", family="mistral", layers=layers, hidden=4096, ffn=14336,
                           heads=32, kv_heads=8, head_dim=d, vocab=32000, tied=False, max_positions=32768,
                           norm_eps=int(O.lib().oracle_f32_to_acc(1e-5)),
                           scale_q32=int(O.lib().oracle_attention_scale_q32(d)), freqs=freqs.tolist())


def synth_mistral_weights(cfg, seed, per_block=False, threads=None):
    """Every tensor of a mistral-dense model from the seeded generator."""
    H, F, V = cfg.hidden, cfg.ffn, cfg.vocab
    qd, kvd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    w = {("EMBED", -1): synth_q8(seed, "EMBED", -1, V, H, per_block, threads),
         ("FINAL_NORM", -1): synth_values(seed, "FINAL_NORM", -1, H, 0, threads)}
    if not cfg.tied:
        w[("HEAD", -1)] = synth_q8(seed, "HEAD", -1, V, H, per_block, threads)
    for l in range(cfg.layers):
        for name, rows, cols in (("W_Q", qd, H), ("W_K", kvd, H), ("W_V", kvd, H), ("W_O", H, qd),
                                 ("W_GATE", F, H), ("W_UP", F, H), ("W_DOWN", H, F)):
            w[(name, l)] = synth_q8(seed, name, l, rows, cols, per_block, threads)
        w[("NORM_ATTN", l)] = synth_values(seed, "NORM_ATTN", l, H, 0, threads)
        w[("NORM_FFN", l)] = synth_values(seed, "NORM_FFN", l, H, 0, threads)
    return w


class CpuDecoder:
    """The direct decode step on the CPU (executor.rs:172-184): the token's
    embedding row, every layer at the next position with the K/V of the
    positions before it, the head and the first maximum. The K/V cache is
    held here ([layer][position][kv]); `fill` seeds positions 0..n-1 with
    random rows in place of a prompt pass."""

    def __init__(self, om, capacity, threads=None):
        c = om.cfg
        self.om, self.threads = om, threads or O.threads_default()
        kvd = c.kv_heads * c.head_dim
        self.k = np.zeros((c.layers, capacity, kvd), np.int32)
        self.v = np.zeros((c.layers, capacity, kvd), np.int32)
        self.pos = 0
        self.logits = np.empty(c.vocab, np.int32)
        self.emb = np.asarray(om.w[("EMBED", -1)]).reshape(c.vocab, -1)

    def fill(self, n, seed):
        rng = np.random.default_rng(seed)
        self.k[:, :n] = rng.integers(-(1 << 17), 1 << 17, size=self.k[:, :n].shape, dtype=np.int32)
        self.v[:, :n] = rng.integers(-(1 << 17), 1 << 17, size=self.v[:, :n].shape, dtype=np.int32)
        self.pos = n

    def step(self, token):
        c, p = self.om.cfg, self.pos
        x = np.empty((1, c.hidden), np.int32)
        row = np.ascontiguousarray(self.emb[token])
        if O.lib().oracle_dequantize_row(O.ptr(row, C.c_uint8), row.size, O.ptr(x[0], C.c_int32), c.hidden):
            raise RuntimeError("dequantize_row failed")
        for l in range(c.layers):
            x, ok, ov = self.om.mistral_layer_range(l, x, p, self.k[l, :p], self.v[l, :p], self.threads)
            self.k[l, p], self.v[l, p] = ok[0], ov[0]
        if O.lib().oracle_head_logits(C.byref(self.om.model.head), O.ptr(x[0], C.c_int32),
                                      O.ptr(self.logits, C.c_int32), self.threads):
            raise RuntimeError("oracle_head_logits failed")
        self.pos = p + 1
        return int(np.argmax(self.logits))  # the first maximum


class OracleModel:
    """Keeps the numpy buffers alive for as long as the ctypes structs exist."""

    def __init__(self, cfg, w):
        self.cfg, self.w = cfg, {k: np.ascontiguousarray(v) for k, v in w.items()}
        self._keep = []
        L = cfg.layers
        m = O.Model()
        m.layers, m.hidden, m.vocab = L, cfg.hidden, cfg.vocab
        m.embed = self.u8("EMBED", -1)
        if cfg.family == "mistral":
            m.family = 0
            self.freqs = np.array(cfg.freqs, np.int64)
            layers = (O.MistralLayer * L)()
            for l in range(L):
                layers[l] = self.mistral_layer(l)
            m.mistral = layers
            head_key = ("EMBED", -1) if cfg.tied else ("HEAD", -1)
            m.head = O.Head(cfg.hidden, cfg.vocab, cfg.norm_eps, 0, self.i32("FINAL_NORM", -1),
                            self.u8(*head_key))
        else:
            m.family = 1
            m.embedding_scale = cfg.embedding_scale
            layers = (O.GemmaLayer * L)()
            for l in range(L):
                layers[l] = self.gemma_layer(l)
            m.gemma = layers
            m.head = O.Head(cfg.hidden, cfg.vocab, cfg.norm_eps, cfg.softcap_bits, self.i32("FINAL_NORM", -1),
                            self.u8(*(("EMBED", -1) if cfg.tied else ("HEAD", -1))))
            m.ple = O.Ple(cfg.hidden, cfg.ple_width, cfg.ple_embedding_scale, cfg.ple_projection_scalar,
                          cfg.ple_input_scale, cfg.norm_eps, self.i32("PLE_NORM", -1), self.u8("PLE_EMBED", -1),
                          self.i32("PLE_MODEL_PROJECTION", -1))
        self._keep.append(layers)
        self.model = m

    def u8(self, name, layer):
        return O.ptr(self.w[(name, layer)], C.c_uint8)

    def i32(self, name, layer):
        return O.ptr(self.w[(name, layer)], C.c_int32)

    def mistral_layer(self, l):
        c = self.cfg
        return O.MistralLayer(c.hidden, c.ffn, c.heads, c.kv_heads, c.head_dim, c.max_positions, c.norm_eps,
                              c.scale_q32, c.head_dim // 2, O.ptr(self.freqs, C.c_int64),
                              self.i32("NORM_ATTN", l), self.i32("NORM_FFN", l),
                              self.u8("W_Q", l), self.u8("W_K", l), self.u8("W_V", l), self.u8("W_O", l),
                              self.u8("W_GATE", l), self.u8("W_UP", l), self.u8("W_DOWN", l))

    def gemma_layer(self, l):
        c = self.cfg
        base, rot, fbd = c.rope(l)
        da, db = c.donor_candidates()
        scal = (c.layer_scalars or [0] * c.layers)[l]
        return O.GemmaLayer(c.hidden, c.ffn, c.heads, c.kv_heads, c.head_dim, c.window(l), 0, scal,
                            c.norm_eps, base, rot, fbd, c.kv_donor(l), da, db, c.ple_width,
                            self.i32("NORM_ATTN", l), self.i32("NORM_POST_ATTN", l), self.i32("NORM_FFN", l),
                            self.i32("NORM_POST_FFW", l), self.i32("Q_NORM", l), self.i32("K_NORM", l),
                            self.i32("PLE_POST_NORM", l),
                            self.u8("W_Q", l), self.u8("W_K", l), self.u8("W_V", l), self.u8("W_O", l),
                            self.u8("W_GATE", l), self.u8("W_UP", l), self.u8("W_DOWN", l),
                            self.i32("PLE_INPUT_GATE", l), self.i32("PLE_LAYER_PROJECTION", l))

    def generate(self, prompt, max_tokens, eos=(), threads=None, want_logits=True):
        p = np.ascontiguousarray(prompt, np.uint32)
        e = np.ascontiguousarray(list(eos) or [0], np.uint32)
        out = np.zeros(max(max_tokens, 1), np.uint32)
        count = C.c_uint32()
        logits = np.zeros((max(max_tokens, 1), self.cfg.vocab), np.int32) if want_logits else None
        rc = O.lib().oracle_generate(C.byref(self.model), O.ptr(p, C.c_uint32), p.size, max_tokens,
                                     O.ptr(e, C.c_uint32), len(list(eos)), O.ptr(out, C.c_uint32),
                                     C.byref(count), O.ptr(logits, C.c_int32) if logits is not None else None,
                                     threads or O.threads_default())
        if rc:
            raise RuntimeError(f"oracle_generate failed: {rc}")
        n = count.value
        return out[:n].tolist(), (logits[:n] if logits is not None else None)

    def head_select(self, rows, threads=None):
        """sequence_check.rs:274-288 per row: rms_norm(final), dot_row over the
        head, softcap, first maximum -> (token ids, scores)."""
        rows = np.ascontiguousarray(rows, np.int32)
        tok = np.empty(rows.shape[0], np.uint32)
        val = np.empty(rows.shape[0], np.int32)
        logits = np.empty(self.cfg.vocab, np.int32)
        for i in range(rows.shape[0]):
            rc = O.lib().oracle_head_logits(C.byref(self.model.head), O.ptr(rows[i], C.c_int32),
                                            O.ptr(logits, C.c_int32), threads or O.threads_default())
            if rc:
                raise RuntimeError(f"oracle_head_logits failed: {rc}")
            tok[i] = int(np.argmax(logits))  # the first maximum
            val[i] = logits[tok[i]]
        return tok, val

    def mistral_layer_range(self, l, rows, start, prior_k, prior_v, threads=None):
        c = self.cfg
        kvd = c.kv_heads * c.head_dim
        rows = np.ascontiguousarray(rows, np.int32)
        m = rows.shape[0]
        out = np.empty_like(rows)
        ok = np.empty((m, kvd), np.int32)
        ov = np.empty((m, kvd), np.int32)
        layer = self.model.mistral[l]
        pk = np.ascontiguousarray(prior_k if start else np.zeros((1, kvd)), np.int32)
        pv = np.ascontiguousarray(prior_v if start else np.zeros((1, kvd)), np.int32)
        rc = O.lib().oracle_mistral_layer(C.byref(layer), O.ptr(rows, C.c_int32), m, start, O.ptr(pk, C.c_int32),
                                          O.ptr(pv, C.c_int32), O.ptr(out, C.c_int32), O.ptr(ok, C.c_int32),
                                          O.ptr(ov, C.c_int32), threads or O.threads_default())
        if rc:
            raise RuntimeError(f"oracle_mistral_layer failed: {rc}")
        return out, ok, ov


def _keys(keys):
    """OracleKeys over (positions, k, v) arrays (kept alive by the caller)."""
    if keys is None or len(keys[0]) == 0:
        return O.Keys(0, None, None, None)
    pos, k, v = keys
    return O.Keys(len(pos), O.ptr(pos, C.c_uint32), O.ptr(k, C.c_int32), O.ptr(v, C.c_int32))


def gemma_ple_rows(om, ids):
    """PLE rows [n][layers][ple] of token ids (view_kernels.rs:59-99) from the
    embedding rows times embedding_scale (model.rs:316-330)."""
    c = om.cfg
    emb = np.asarray(om.w[("EMBED", -1)]).reshape(c.vocab, -1)
    out = np.empty((len(ids), c.layers, c.ple_width), np.int32)
    row = np.empty(c.hidden, np.int32)
    for i, t in enumerate(ids):
        e = np.ascontiguousarray(emb[t])
        if O.lib().oracle_dequantize_row(O.ptr(e, C.c_uint8), e.size, O.ptr(row, C.c_int32), c.hidden):
            raise RuntimeError("dequantize_row failed")
        seed = np.array([O.lib().oracle_mul_sat(int(x), c.embedding_scale) for x in row], np.int32)
        for l in range(c.layers):
            if O.lib().oracle_ple_prepare(C.byref(om.model.ple), c.layers, l, O.ptr(seed, C.c_int32), int(t),
                                          O.ptr(out[i, l], C.c_int32)):
                raise RuntimeError("oracle_ple_prepare failed")
    return out


def gemma_layer_range(om, l, rows, start, ple, prior=None, donor_a=None, donor_b=None, threads=None):
    """One gemma-dense layer over a range (prefill_range.rs:307-333):
    (rows_out, own_k, own_v). prior / donor_*: (positions uint32, k, v)."""
    c = om.cfg
    kvd = c.kv_heads * c.head_dim
    rows = np.ascontiguousarray(rows, np.int32)
    ple = np.ascontiguousarray(ple, np.int32)
    m = rows.shape[0]
    out = np.empty_like(rows)
    ok = np.empty((m, kvd), np.int32)
    ov = np.empty((m, kvd), np.int32)
    keep = [tuple(np.ascontiguousarray(a, t) for a, t in zip(ks, (np.uint32, np.int32, np.int32)))
            if ks is not None and len(ks[0]) else None for ks in (prior, donor_a, donor_b)]
    rc = O.lib().oracle_gemma_layer(C.byref(om.model.gemma[l]), O.ptr(rows, C.c_int32), m, start,
                                    _keys(keep[0]), _keys(keep[1]), _keys(keep[2]), O.ptr(ple, C.c_int32),
                                    O.ptr(out, C.c_int32), O.ptr(ok, C.c_int32), O.ptr(ov, C.c_int32),
                                    threads or O.threads_default())
    if rc:
        raise RuntimeError(f"oracle_gemma_layer failed: {rc}")
    return out, ok, ov


class OracleStages:
    """The chain-stage calls of a device model (embed, layer_range,
    ple_rows, gemma_layer_range) computed by the oracle, so that one driver
    (iris_b200.records.chain_records) runs a claim stage by stage on either."""

    def __init__(self, om, threads=None):
        self.om, self.cfg, self.threads = om, om.cfg, threads

    def embed(self, ids):
        c = self.cfg
        emb = np.asarray(self.om.w[("EMBED", -1)]).reshape(c.vocab, -1)
        out = np.empty((len(ids), c.hidden), np.int32)
        for i, t in enumerate(ids):
            e = np.ascontiguousarray(emb[t])
            if O.lib().oracle_dequantize_row(O.ptr(e, C.c_uint8), e.size, O.ptr(out[i], C.c_int32), c.hidden):
                raise RuntimeError("dequantize_row failed")
            if c.family == "gemma":  # model.rs:316-330
                out[i] = [O.lib().oracle_mul_sat(int(x), c.embedding_scale) for x in out[i]]
        return out

    def layer_range(self, layer, rows, start, prior_k, prior_v):
        return self.om.mistral_layer_range(layer, rows, start, prior_k, prior_v, self.threads)

    def ple_rows(self, ids):
        return gemma_ple_rows(self.om, ids)

    def gemma_layer_range(self, layer, rows, start, ple, prior=None, donor=None):
        da, db = self.cfg.donor_candidates()
        d = self.cfg.kv_donor(layer)
        return gemma_layer_range(self.om, layer, rows, start, ple, prior=prior,
                                 donor_a=donor if d >= 0 and d == da else None,
                                 donor_b=donor if d >= 0 and d == db else None, threads=self.threads)

"""TEST INFRASTRUCTURE ONLY: builds the oracle's model structs from host
tensors (the same bytes the device model is loaded with).

Used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import oracle as O


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
                            self.u8("EMBED", -1))
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

"""TEST INFRASTRUCTURE ONLY: ctypes binding of the CPU oracle (liboracle.so).

The oracle restates the reference's Rust CPU path (det-num, the mistral-dense
and gemma-dense layers, the head and the direct decode loop) in C++. Only
tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this
module, and only as the checker; the product path never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
# The reference's GPU product kernel, built unchanged from its own source
# where the reference checkout is present (oracle/Makefile, _ref/ target).
REF_Q8_RELPATH = "crates/inference/kernels/cuda/q8_product.cu"
REF_Q8_LIB = HERE / "_ref" / "libq8ref.so"


def reference_root() -> Path | None:
    """The reference checkout: $IRIS_REFERENCE, else the `reference_path`
    that BASELINE.json at the repository root records; None when neither
    names an existing directory (the GPU box has no checkout)."""
    cand = os.environ.get("IRIS_REFERENCE")
    if not cand:
        try:
            import json
            cand = json.loads((HERE.parent / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            cand = None
    return Path(cand) if cand and Path(cand).is_dir() else None

i32p = C.POINTER(C.c_int32)
i64p = C.POINTER(C.c_int64)
u8p = C.POINTER(C.c_uint8)
u32p = C.POINTER(C.c_uint32)


class MistralLayer(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("ffn", C.c_uint32), ("heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("max_positions", C.c_uint32),
                ("norm_eps", C.c_int64), ("attention_scale_q32", C.c_uint32),
                ("n_freqs", C.c_uint32), ("rope_freqs", i64p),
                ("norm_attention", i32p), ("norm_feed_forward", i32p),
                ("w_q", u8p), ("w_k", u8p), ("w_v", u8p), ("w_o", u8p),
                ("w_gate", u8p), ("w_up", u8p), ("w_down", u8p)]


class GemmaLayer(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("ffn", C.c_uint32), ("heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("sliding_window", C.c_uint32),
                ("attn_scale", C.c_int32), ("layer_scalar", C.c_int32),
                ("norm_eps", C.c_int64), ("rope_base", C.c_int64),
                ("rotary_dim", C.c_uint32), ("rope_freq_base_dim", C.c_uint32),
                ("kv_donor_layer", C.c_int32), ("donor_a_layer", C.c_int32),
                ("donor_b_layer", C.c_int32), ("ple_width", C.c_uint32),
                ("norm_input", i32p), ("norm_post_attn", i32p), ("norm_pre_ffw", i32p),
                ("norm_post_ffw", i32p), ("q_norm", i32p), ("k_norm", i32p),
                ("ple_post_norm", i32p),
                ("w_q", u8p), ("w_k", u8p), ("w_v", u8p), ("w_o", u8p),
                ("w_gate", u8p), ("w_up", u8p), ("w_down", u8p),
                ("ple_input_gate", i32p), ("ple_layer_projection", i32p)]


class Head(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("vocab", C.c_uint32), ("norm_eps", C.c_int64),
                ("softcap", C.c_int32), ("norm", i32p), ("projection", u8p)]


class Ple(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("ple_width", C.c_uint32),
                ("embedding_scale", C.c_int32), ("projection_scalar", C.c_int32),
                ("input_scale", C.c_int32), ("norm_eps", C.c_int64), ("norm", i32p),
                ("embeddings", u8p), ("projection", i32p)]


class Model(C.Structure):
    _fields_ = [("family", C.c_uint32), ("layers", C.c_uint32), ("hidden", C.c_uint32),
                ("vocab", C.c_uint32), ("embedding_scale", C.c_int32), ("embed", u8p),
                ("mistral", C.POINTER(MistralLayer)), ("gemma", C.POINTER(GemmaLayer)),
                ("head", Head), ("ple", Ple)]


class Keys(C.Structure):
    _fields_ = [("n", C.c_size_t), ("positions", u32p), ("k", i32p), ("v", i32p)]


def build(force: bool = False, reference: bool = False) -> Path:
    """Compile liboracle.so with the committed Makefile (g++, seconds); with
    `reference`, also the reference's own GPU product kernel into _ref/ when
    the reference checkout is present (nvcc). Tests and the GPU box only use
    the prebuilt _ref/ file."""
    sources = [HERE / n for n in ("det_num.cc", "layers.cc", "synth.cc", "det_num.h", "oracle_abi.h", "Makefile")]
    if force or not LIB_PATH.exists() or any(
            s.stat().st_mtime > LIB_PATH.stat().st_mtime for s in sources):
        subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    root = reference_root() if reference else None
    if root is not None and (root / REF_Q8_RELPATH).exists() and (force or not REF_Q8_LIB.exists()):
        subprocess.run(["make", "-s", "-C", str(HERE), f"REFERENCE={root}", "_ref/libq8ref.so"], check=True)
    return LIB_PATH


def reference_q8():
    """The reference's q8gpu_* library (crates/inference/kernels/cuda/
    q8_product.cu built unchanged for sm_100a), or None when it was not built."""
    if not REF_Q8_LIB.exists():
        return None
    L = C.CDLL(str(REF_Q8_LIB))
    vp = C.c_void_p
    L.q8gpu_init.restype = C.c_int
    L.q8gpu_upload.restype = C.c_int
    L.q8gpu_upload.argtypes = [C.POINTER(C.c_int8), C.POINTER(C.c_int64), C.c_uint32, C.c_uint32, C.POINTER(vp)]
    L.q8gpu_product.restype = C.c_int
    L.q8gpu_product.argtypes = [vp, C.POINTER(C.c_int32), C.c_uint32, C.POINTER(C.c_int32)]
    L.q8gpu_free.restype = None
    L.q8gpu_free.argtypes = [vp]
    L.q8gpu_error.restype = C.c_char_p
    L.q8gpu_error.argtypes = [C.c_int]
    return L


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = C.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


def _declare(L):
    sig = {
        "oracle_requantize": (C.c_int32, [C.c_int64]),
        "oracle_rshift_round_ties_even": (C.c_int64, [C.c_int64, C.c_uint32]),
        "oracle_mac_bits": (C.c_int64, [C.c_int64, C.c_int32, C.c_int32]),
        "oracle_add_sat": (C.c_int32, [C.c_int32, C.c_int32]),
        "oracle_sub_sat": (C.c_int32, [C.c_int32, C.c_int32]),
        "oracle_mul_sat": (C.c_int32, [C.c_int32, C.c_int32]),
        "oracle_div_act": (C.c_int32, [C.c_int32, C.c_int32]),
        "oracle_div_acc": (C.c_int64, [C.c_int64, C.c_int64]),
        "oracle_acc_mul": (C.c_int64, [C.c_int64, C.c_int64]),
        "oracle_inv_sqrt_acc": (C.c_int32, [C.c_int64]),
        "oracle_tanh": (C.c_int32, [C.c_int32]),
        "oracle_gelu": (C.c_int32, [C.c_int32]),
        "oracle_softcap": (C.c_int32, [C.c_int32, C.c_int32]),
        "oracle_softmax_exp_term": (C.c_int64, [C.c_int64]),
        "oracle_silu": (C.c_int32, [C.c_int32]),
        "oracle_sigmoid_q32": (C.c_uint64, [C.c_int32]),
        "oracle_exp_neg_q32": (C.c_uint64, [C.c_uint64]),
        "oracle_sin_cos_q30": (None, [C.c_int64, i64p, i64p]),
        "oracle_sin_cos_acc": (None, [C.c_int64, i32p, i32p]),
        "oracle_rope_frequency_step": (C.c_int64, [C.c_int64, C.c_uint32]),
        "oracle_nth_root_acc": (C.c_int64, [C.c_int64, C.c_uint32]),
        "oracle_attention_scale_q32": (C.c_uint32, [C.c_uint32]),
        "oracle_yarn_inverse_frequencies": (C.c_int, [C.c_uint64, C.c_uint32, C.c_uint32,
                                                       C.c_uint32, C.c_uint32, i64p]),
        "oracle_scaled_score": (C.c_int32, [i32p, i32p, C.c_size_t, C.c_uint32]),
        "oracle_dot_bits": (C.c_int32, [i32p, i32p, C.c_size_t]),
        "oracle_f32_to_act": (C.c_int32, [C.c_float]),
        "oracle_f32_to_acc": (C.c_int64, [C.c_float]),
        "oracle_scale_q24": (C.c_int, [C.c_uint16, i64p]),
        "oracle_dot_row": (C.c_int, [i32p, C.c_size_t, u8p, C.c_size_t, i32p]),
        "oracle_dequantize_row": (C.c_int, [u8p, C.c_size_t, i32p, C.c_size_t]),
        "oracle_rms_norm": (None, [i32p, i32p, C.c_size_t, C.c_int64]),
        "oracle_value_rms_norm": (None, [i32p, C.c_size_t, C.c_int64]),
        "oracle_rms_norm_scale": (C.c_int32, [i32p, C.c_size_t, C.c_int64]),
        "oracle_rope_rotate_pairs": (None, [i32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int64,
                                            C.c_size_t]),
        "oracle_rotate_consecutive_pairs": (None, [i32p, C.c_size_t, i64p, C.c_size_t,
                                                   C.c_uint32]),
        "oracle_attention_softmax": (None, [i32p, C.c_size_t, i32p]),
        "oracle_linear": (C.c_int, [i32p, C.c_size_t, C.c_size_t, u8p, C.c_size_t, i32p, C.c_int]),
        "oracle_linear_dense": (C.c_int, [i32p, C.c_size_t, C.c_size_t, i32p, C.c_size_t, i32p,
                                          C.c_int]),
        "oracle_mistral_layer": (C.c_int, [C.POINTER(MistralLayer), i32p, C.c_size_t, C.c_uint32,
                                           i32p, i32p, i32p, i32p, i32p, C.c_int]),
        "oracle_gemma_layer": (C.c_int, [C.POINTER(GemmaLayer), i32p, C.c_size_t, C.c_uint32,
                                         Keys, Keys, Keys, i32p, i32p, i32p, i32p, C.c_int]),
        "oracle_head_logits": (C.c_int, [C.POINTER(Head), i32p, i32p, C.c_int]),
        "oracle_ple_prepare": (C.c_int, [C.POINTER(Ple), C.c_uint32, C.c_uint32, i32p, C.c_uint32,
                                         i32p]),
        "oracle_generate": (C.c_int, [C.POINTER(Model), u32p, C.c_size_t, C.c_uint32, u32p,
                                      C.c_size_t, u32p, u32p, i32p, C.c_int]),
        "oracle_synth_q8": (C.c_int, [C.c_uint64, C.c_uint32, C.c_int32, C.c_uint32, C.c_uint32, C.c_int,
                                      u8p, C.c_int]),
        "oracle_synth_values": (C.c_int, [C.c_uint64, C.c_uint32, C.c_int32, C.c_uint64, C.c_uint32, i32p,
                                          C.c_int]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args


def threads_default() -> int:
    return max(1, os.cpu_count() or 1)


def ptr(a: np.ndarray, ctype):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be contiguous"
    return a.ctypes.data_as(C.POINTER(ctype))


# ---- thin numpy-level helpers --------------------------------------------

def linear(inp: np.ndarray, q8: np.ndarray, rows: int, threads: int | None = None) -> np.ndarray:
    """out[t, r] = dot_row(inp[t], q8 row r); q8 is raw Q8_0 bytes."""
    inp = np.ascontiguousarray(inp, dtype=np.int32)
    q8 = np.ascontiguousarray(q8, dtype=np.uint8)
    tokens, cols = inp.shape
    out = np.zeros((tokens, rows), dtype=np.int32)
    rc = lib().oracle_linear(ptr(inp, C.c_int32), tokens, cols, ptr(q8, C.c_uint8), rows,
                             ptr(out, C.c_int32), threads or threads_default())
    if rc:
        raise ValueError("oracle_linear: malformed Q8_0 matrix or non-finite scale")
    return out


def dot_row(act: np.ndarray, row: np.ndarray) -> int:
    act = np.ascontiguousarray(act, dtype=np.int32)
    row = np.ascontiguousarray(row, dtype=np.uint8)
    out = C.c_int32()
    rc = lib().oracle_dot_row(ptr(act, C.c_int32), act.size, ptr(row, C.c_uint8), row.size,
                              C.byref(out))
    if rc:
        raise ValueError("dot_row error")
    return out.value

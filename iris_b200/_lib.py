"""ctypes binding of libiris_b200.so (include/iris_b200.h).

The library is the product: there is no Python or CPU fallback. Loading fails
loudly when the shared object is missing, and every call that returns a
non-zero status raises IrisError with the library's own message.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libiris_b200.so"

IRIS_EINVAL, IRIS_ESCALE, IRIS_ERANGE, IRIS_ESTATE, IRIS_EWINDOW, IRIS_ESTALL = 10001, 10002, 10003, 10004, 10005, 10006
IRIS_ESCRATCH = 10007
NOALLOC_PLANES_BYTES = 16 << 20
PATH_AUTO, PATH_GEMV, PATH_GEMM, PATH_TC, PATH_TC3, PATH_GEMV1 = 0, 1, 2, 3, 4, 5
GEMM_AUTO, GEMM_MMA = 0, 1
ATTN_AUTO, ATTN_SPLIT, ATTN_CLUSTER = 0, 1, 2
DECODE_AUTO, DECODE_GRAPH, DECODE_STEP = 0, 1, 2

# Tensor kinds (include/iris_b200.h)
T = dict(EMBED=0, HEAD=1, FINAL_NORM=2, W_Q=3, W_K=4, W_V=5, W_O=6, W_GATE=7, W_UP=8, W_DOWN=9,
         NORM_ATTN=10, NORM_FFN=11, NORM_POST_ATTN=12, NORM_POST_FFW=13, Q_NORM=14, K_NORM=15,
         PLE_POST_NORM=16, PLE_INPUT_GATE=17, PLE_LAYER_PROJECTION=18, PLE_EMBED=19,
         PLE_MODEL_PROJECTION=20, PLE_NORM=21)

i32p = C.POINTER(C.c_int32)
i64p = C.POINTER(C.c_int64)
u8p = C.POINTER(C.c_uint8)
u32p = C.POINTER(C.c_uint32)
vp = C.c_void_p


class IrisError(RuntimeError):
    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what}: {error_string(code)} (status {code})")


class MistralShape(C.Structure):
    _fields_ = [("layers", C.c_uint32), ("hidden", C.c_uint32), ("ffn", C.c_uint32),
                ("heads", C.c_uint32), ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("vocab", C.c_uint32), ("max_positions", C.c_uint32), ("norm_eps", C.c_int64),
                ("attention_scale_q32", C.c_uint32), ("tied_head", C.c_uint32),
                ("rope_inverse_frequencies", i64p)]


class GemmaShape(C.Structure):
    _fields_ = [("layers", C.c_uint32), ("hidden", C.c_uint32), ("ffn", C.c_uint32),
                ("heads", C.c_uint32), ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("vocab", C.c_uint32), ("ple_width", C.c_uint32), ("norm_eps", C.c_int64),
                ("embedding_scale", C.c_int32), ("ple_embedding_scale", C.c_int32),
                ("ple_projection_scalar", C.c_int32), ("ple_input_scale", C.c_int32),
                ("final_logit_softcap", C.c_int32),
                ("sliding_window", u32p), ("rope_base", i64p), ("rotary_dim", u32p),
                ("rope_freq_base_dim", u32p), ("kv_donor_layer", i32p), ("layer_scalar", i32p),
                ("tied_head", C.c_uint32)]


# name -> (restype, argtypes); every symbol include/iris_b200.h declares.
SIGNATURES = {
    "q8gpu_error": (C.c_char_p, [C.c_int]),
    "q8gpu_init": (C.c_int, []),
    "q8gpu_free": (None, [vp]),
    "q8gpu_upload": (C.c_int, [C.POINTER(C.c_int8), i64p, C.c_uint32, C.c_uint32, C.POINTER(vp)]),
    "q8gpu_product": (C.c_int, [vp, i32p, C.c_uint32, i32p]),
    "iris_q8_upload_blocks": (C.c_int, [u8p, C.c_uint32, C.c_uint32, C.POINTER(vp)]),
    "iris_q8_product_device": (C.c_int, [vp, vp, C.c_uint32, vp, vp]),
    "iris_q8_product_device_path": (C.c_int, [vp, vp, C.c_uint32, vp, vp, C.c_int]),
    "iris_q8_product_device_noalloc": (C.c_int, [vp, vp, C.c_uint32, vp, vp]),
    "iris_model_create_mistral": (C.c_int, [C.POINTER(MistralShape), C.POINTER(vp)]),
    "iris_model_create_gemma": (C.c_int, [C.POINTER(GemmaShape), C.POINTER(vp)]),
    "iris_model_create_mistral_tp": (C.c_int, [C.POINTER(MistralShape), C.c_uint32, C.c_uint32, u8p, C.POINTER(vp)]),
    "iris_tp_unique_id": (C.c_int, [u8p]),
    "iris_model_set_tp_exchange": (C.c_int, [vp, C.c_int]),
    "iris_synth_q8_block": (C.c_int, [C.c_uint64, C.c_uint32, C.c_int32, C.c_uint32, C.c_uint32, C.c_uint32,
                                      C.c_uint32, C.c_uint32, C.c_int, u8p]),
    "iris_model_set_q8": (C.c_int, [vp, C.c_int, C.c_int32, u8p, C.c_uint64]),
    "iris_model_set_values": (C.c_int, [vp, C.c_int, C.c_int32, i32p, C.c_uint64]),
    "iris_model_synthesize": (C.c_int, [vp, C.c_uint64, C.c_int]),
    "iris_model_get_q8": (C.c_int, [vp, C.c_int, C.c_int32, u8p, C.c_uint64]),
    "iris_model_get_values": (C.c_int, [vp, C.c_int, C.c_int32, i32p, C.c_uint64]),
    "iris_model_weight_bytes": (C.c_uint64, [vp]),
    "iris_model_set_gemm": (C.c_int, [vp, C.c_int]),
    "iris_model_prepare_gemm": (C.c_int, [vp]),
    "iris_sequence_check_select": (C.c_int, [vp, i32p, C.c_uint32, C.POINTER(C.c_uint32), i32p]),
    "iris_model_embed": (C.c_int, [vp, C.POINTER(C.c_uint32), C.c_uint32, i32p]),
    "iris_model_tc_matrices": (C.c_int, [vp, C.POINTER(C.c_uint64)]),
    "iris_model_attention_ranges": (C.c_int, [vp, C.POINTER(C.c_uint64)]),
    "iris_softmax_exp_terms": (C.c_int, [C.c_uint32, C.c_uint32, C.POINTER(C.c_uint64)]),
    "iris_wait_probe": (C.c_int, [C.c_int, C.c_int]),
    "iris_model_free": (None, [vp]),
    "iris_session_create": (C.c_int, [vp, C.c_uint32, C.POINTER(vp)]),
    "iris_session_reset": (C.c_int, [vp]),
    "iris_session_prefill": (C.c_int, [vp, u32p, C.c_uint32, i32p, u32p]),
    "iris_session_decode": (C.c_int, [vp, C.c_uint32, i32p, u32p]),
    "iris_generate": (C.c_int, [vp, u32p, C.c_uint32, C.c_uint32, u32p, C.c_uint32, u32p, u32p, i32p]),
    "iris_session_length": (C.c_uint32, [vp]),
    "iris_session_decode_steps": (C.c_int, [vp, C.c_uint32]),
    "iris_session_synchronize": (C.c_int, [vp]),
    "iris_session_stream": (vp, [vp]),
    "iris_session_graph_kernels": (C.c_uint32, [vp]),
    "iris_session_product": (C.c_int, [vp, C.c_uint32, C.c_int]),
    "iris_session_attention": (C.c_int, [vp, C.c_uint32]),
    "iris_session_set_attention": (C.c_int, [vp, C.c_int]),
    "iris_session_attention_plan": (C.c_int, [vp, C.POINTER(C.c_uint32)]),
    "iris_session_set_decode_path": (C.c_int, [vp, C.c_int]),
    "iris_session_decode_path": (C.c_int, [vp]),
    "iris_session_step_plan": (C.c_int, [vp, C.POINTER(C.c_uint32)]),
    "iris_session_step_trace": (C.c_int, [vp, C.c_int]),
    "iris_session_get_step_trace": (C.c_int, [vp, C.POINTER(C.c_uint64), C.c_uint64]),
    "iris_session_set_attention_shape": (C.c_int, [vp, C.c_uint32, C.c_uint32, C.c_uint32]),
    "iris_session_get_kv": (C.c_int, [vp, C.c_uint32, C.c_uint32, C.c_uint32, i32p, i32p]),
    "iris_session_free": (None, [vp]),
    "iris_capture_begin": (C.c_int, [vp]),
    "iris_capture_end": (C.c_int, [vp, C.POINTER(vp)]),
    "iris_graph_launch": (C.c_int, [vp, vp]),
    "iris_graph_free": (None, [vp]),
    "iris_mistral_layer_range": (C.c_int, [vp, C.c_uint32, i32p, C.c_uint32, C.c_uint32, i32p, i32p,
                                           i32p, i32p, i32p]),
    "iris_model_ple_rows": (C.c_int, [vp, C.POINTER(C.c_uint32), C.c_uint32, i32p]),
    "iris_gemma_layer_range": (C.c_int, [vp, C.c_uint32, i32p, C.c_uint32, C.c_uint32, i32p,
                                         C.c_uint32, C.POINTER(C.c_uint32), i32p, i32p,
                                         C.c_uint32, C.POINTER(C.c_uint32), i32p, i32p, i32p, i32p, i32p]),
    "iris_session_range_begin": (C.c_int, [vp, C.POINTER(C.c_uint32), C.c_uint32]),
    "iris_session_range_layer": (C.c_int, [vp, C.c_uint32, vp, vp, vp, C.POINTER(C.c_uint32)]),
    "iris_session_range_layer_leaves": (C.c_int, [vp, C.c_uint32, C.c_uint32, vp, C.POINTER(C.c_uint32)]),
    "iris_session_range_layers_leaves": (C.c_int, [vp, C.c_uint32, C.c_uint32, C.POINTER(vp),
                                                   C.POINTER(C.c_uint32)]),
    "iris_session_ticket_wait": (C.c_int, [vp, C.c_uint32]),
    "iris_session_range_end": (C.c_int, [vp, C.POINTER(C.c_uint32), i32p]),
    "iris_host_alloc": (C.c_int, [C.c_uint64, C.POINTER(vp)]),
    "iris_host_free": (None, [vp]),
    "iris_synth_q8": (C.c_int, [C.c_uint64, C.c_uint32, C.c_int32, C.c_uint32, C.c_uint32, C.c_int, u8p]),
    "iris_synth_values": (C.c_int, [C.c_uint64, C.c_uint32, C.c_int32, C.c_uint64, C.c_uint32, i32p]),
    "iris_error": (C.c_char_p, [C.c_int]),
}

_lib = None


def lib() -> C.CDLL:
    """The loaded library; raises when it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m iris_b200.build` "
                              "(there is no CPU fallback)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def tp_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for a tensor-parallel model."""
    out = np.zeros(128, np.uint8)
    check(lib().iris_tp_unique_id(ptr(out, C.c_uint8)), "iris_tp_unique_id")
    return out.tobytes()


def synth_q8_block(seed: int, tensor: int, layer: int, rows: int, cols: int, row0: int, col0: int,
                   full_cols: int, per_block: bool = False) -> np.ndarray:
    out = np.empty(rows * (cols // 32) * 34, np.uint8)
    check(lib().iris_synth_q8_block(seed, tensor, layer, rows, cols, row0, col0, full_cols, int(per_block),
                                    ptr(out, C.c_uint8)), "iris_synth_q8_block")
    return out


def error_string(code: int) -> str:
    return lib().iris_error(code).decode()


def check(code: int, what: str) -> None:
    if code:
        raise IrisError(code, what)


def ptr(a: np.ndarray, ctype):
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the library must be contiguous"
    return a.ctypes.data_as(C.POINTER(ctype))


def synth_q8(seed: int, tensor: int, layer: int, rows: int, cols: int, per_block: bool = False) -> np.ndarray:
    """Host copy of the device's synthetic Q8_0 generator (raw 34-byte blocks)."""
    out = np.empty(rows * (cols // 32) * 34, dtype=np.uint8)
    check(lib().iris_synth_q8(seed, tensor, layer, rows, cols, int(per_block), ptr(out, C.c_uint8)),
          "iris_synth_q8")
    return out


def synth_values(seed: int, tensor: int, layer: int, count: int, fan_in: int) -> np.ndarray:
    out = np.empty(count, dtype=np.int32)
    check(lib().iris_synth_values(seed, tensor, layer, count, fan_in, ptr(out, C.c_int32)),
          "iris_synth_values")
    return out

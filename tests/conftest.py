"""Shared pytest setup: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device and the built libiris_b200.so; the rest
run on a CPU-only machine (oracle known-answer tests, host logic, the C-ABI
symbol check, and multi-process gloo tests).
"""
import ctypes as C
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# torch first: its own CUDA and NCCL libraries are then the process's copies,
# whatever a test loads before its first use of torch.
try:
    import torch  # noqa: F401
except Exception:  # the CPU-only tests do not need it
    pass


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built CUDA library")


@pytest.fixture(scope="session")
def detnum_shim(tmp_path_factory):
    """iris_b200/csrc/detnum.cuh compiled as host C++ (tests/native/detnum_shim.cc)."""
    out = tmp_path_factory.mktemp("shim") / "libdetnum_shim.so"
    subprocess.run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-o", str(out),
                    os.path.join(ROOT, "tests", "native", "detnum_shim.cc")], check=True)
    L = C.CDLL(str(out))
    i32p, i64p = C.POINTER(C.c_int32), C.POINTER(C.c_int64)
    sig = {
        "shim_sha256_leaves": (None, [C.POINTER(C.c_uint32), C.c_uint32, C.c_uint32, C.POINTER(C.c_uint8)]),
        "shim_requantize": (C.c_int32, [C.c_int64]),
        "shim_mul_sat": (C.c_int32, [C.c_int32, C.c_int32]),
        "shim_div_act": (C.c_int32, [C.c_int32, C.c_int32]),
        "shim_inv_sqrt_acc": (C.c_int32, [C.c_int64]),
        "shim_inv_sqrt_acc_fast": (C.c_int32, [C.c_int64]),
        "shim_round_q24_scaled": (C.c_int32, [C.c_int64, C.c_int32, C.c_int32]),
        "shim_round_q24_scaled_ref": (C.c_int32, [C.c_int64, C.c_int32, C.c_int32]),
        "shim_div_round_even_width": (C.c_uint64, [C.c_uint64, C.c_uint32]),
        "shim_div_round_even_u64": (C.c_uint64, [C.c_uint64, C.c_uint64]),
        "shim_rms_scale": (C.c_int32, [i32p, C.c_uint32, C.c_int64]),
        "shim_silu": (C.c_int32, [C.c_int32]),
        "shim_sin_cos_q30": (None, [C.c_int64, i64p, i64p]),
        "shim_sin_cos_acc": (None, [C.c_int64, i32p, i32p]),
        "shim_scaled_score": (C.c_int32, [i32p, i32p, C.c_uint32, C.c_uint32]),
        "shim_exp_term": (C.c_int64, [C.c_int32, C.c_int32]),
        "shim_softmax_weight": (C.c_int32, [C.c_int64, C.c_uint64]),
        "shim_softmax_weight_inv": (C.c_int32, [C.c_int64, C.c_uint64]),
        "shim_tanh": (C.c_int32, [C.c_int32]),
        "shim_gelu": (C.c_int32, [C.c_int32]),
        "shim_softcap": (C.c_int32, [C.c_int32, C.c_int32]),
        "shim_q8_dot": (C.c_int32, [i32p, C.POINTER(C.c_uint8), C.c_uint32]),
        "shim_q8_dequant": (C.c_int32, [C.c_int8, C.c_uint16]),
        "shim_rotate_half": (None, [i32p, i32p, C.c_int64, C.c_uint32]),
    }
    declare_shim_limbs(L)
    for name, (res, args) in sig.items():
        getattr(L, name).restype = res
        getattr(L, name).argtypes = args
    L.path = str(out)
    return L


def declare_shim_limbs(L):
    """Signatures of the shim's tensor-parallel limb functions (also used by
    child processes that load the shim by path)."""
    i32p, i64p = C.POINTER(C.c_int32), C.POINTER(C.c_int64)
    L.shim_partial_limbs.restype = None
    L.shim_partial_limbs.argtypes = [i32p, C.POINTER(C.c_uint8), C.c_uint32, C.c_uint32, i64p]
    L.shim_round_limb_sums.restype = C.c_int32
    L.shim_round_limb_sums.argtypes = [i64p]

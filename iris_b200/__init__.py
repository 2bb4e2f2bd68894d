"""iris_b200: B200-native exact-integer inference for iris's token loop.

The direct-infer decode step and the teacher-forced per-layer prefill of the
reference (casettek/iris), bit-exact with its det-num arithmetic, on
hand-written sm_100a CUDA kernels behind the C ABI of include/iris_b200.h.

- iris_b200.tensor  — Slab / Q8Matrix / linear_slab_from_source (tensor.rs)
- iris_b200.model   — DeviceModel / Session / generate (direct executor)
- iris_b200.shapes  — the benchmark configurations and importer arithmetic
- iris_b200.build   — nvcc build of libiris_b200.so
"""
from .shapes import CONFIGS, GemmaConfig, MistralConfig  # noqa: F401

__all__ = ["CONFIGS", "GemmaConfig", "MistralConfig"]

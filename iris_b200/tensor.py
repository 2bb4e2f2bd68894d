"""The reference's operator API for weight products, on the device.

Mirrors crates/inference/kernels/src/tensor.rs: `Slab` (token rows of Q16.16
values, :26-88), `Q8Matrix` (committed Q8_0 rows, :329-417) and
`linear_slab_from_source` (:437-520), the one weight-product site of a layer.
Every output equals `det_num::q8::dot_row` (q8.rs:56-72); the product runs in
libiris_b200.so (decode GEMV for one token, tiled GEMM for more).
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from . import _lib
from ._lib import check, lib, ptr

BLOCK, BLOCK_BYTES = 32, 34


def row_bytes(cols: int) -> Optional[int]:
    """q8.rs:21-23."""
    return cols // BLOCK * BLOCK_BYTES if cols > 0 and cols % BLOCK == 0 else None


class Slab:
    """Rows of Q16.16 activations (tensor.rs:26-88)."""

    def __init__(self, data: np.ndarray):
        self.data = np.ascontiguousarray(data, dtype=np.int32)
        assert self.data.ndim == 2

    @classmethod
    def zeroed(cls, rows: int, cols: int) -> "Slab":
        return cls(np.zeros((rows, cols), np.int32))

    def rows(self) -> int:
        return self.data.shape[0]

    def cols(self) -> int:
        return self.data.shape[1]

    def row(self, i: int) -> np.ndarray:
        return self.data[i]


class Q8Matrix:
    """A Q8_0 matrix uploaded to HBM from its committed bytes (tensor.rs:329-417)."""

    def __init__(self, name: str, blocks: np.ndarray, rows: int, cols: int):
        rb = row_bytes(cols)
        if rb is None:
            raise ValueError(f"{name} rows of {cols} values are not whole Q8_0 blocks")
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        if blocks.size != rows * rb:
            raise ValueError(f"{name} has {blocks.size} bytes, expected {rows * rb} ({rows} x {cols} Q8_0)")
        self.name, self._rows, self._cols = name, rows, cols
        self.blocks = blocks
        self._h = C.c_void_p()
        check(lib().iris_q8_upload_blocks(ptr(blocks, C.c_uint8), rows, cols, C.byref(self._h)),
              f"upload {name}")

    @classmethod
    def from_bytes(cls, name: str, blocks, rows: int, cols: int) -> "Q8Matrix":
        return cls(name, np.frombuffer(bytes(blocks), np.uint8) if isinstance(blocks, (bytes, bytearray))
                   else blocks, rows, cols)

    def rows(self) -> int:
        return self._rows

    def cols(self) -> int:
        return self._cols

    @property
    def handle(self):
        return self._h

    def __del__(self):
        try:
            if self._h:
                lib().q8gpu_free(self._h)
        except Exception:
            pass


def linear_slab_from_source(inp: Slab, matrix: Q8Matrix) -> Slab:
    """out[t][r] = dot_row(inp[t], matrix row r), computed on the device."""
    if inp.cols() != matrix.cols():
        raise ValueError(f"deterministic linear input row 0 has width {inp.cols()}, expected {matrix.cols()}")
    out = np.empty((inp.rows(), matrix.rows()), np.int32)
    if inp.rows() == 0:
        return Slab(out)
    check(lib().q8gpu_product(matrix.handle, ptr(inp.data, C.c_int32), inp.rows(), ptr(out, C.c_int32)),
          "q8gpu_product")
    return Slab(out)

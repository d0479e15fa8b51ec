"""Host-side mirror of dianoia's GpuLinear (lib/src/gpu.dart:1269-1368) over the
lab_gpu_* C-ABI of libdianoia_b200.so.

GpuLinear keeps each uploaded matrix in a GPU buffer of its own (qs, then
the scales at the next 64-byte boundary), and for every ``apply`` copies the
inputs into a growing input buffer, records one product in its own command
buffer, commits and waits, and copies the outputs out. The same names,
argument meaning and errors as the Dart class (``ArgumentError`` for an
unknown matrix or short lists, ``StateError`` after ``dispose`` or when the
command buffer fails).
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional

import numpy as np

from . import _lib
from .native import ArgumentError, NativeQ4Matrix, StateError


def live_buffers() -> int:
    """GPU buffers not yet released (GpuForward.liveBuffers, gpu.dart:455)."""
    return int(_lib.lib().lab_gpu_live_buffers())


class _Buffer:
    """A GPU buffer of `floats` f32 with a numpy view of its contents."""

    def __init__(self, floats: int):
        L = _lib.lib()
        self.handle = int(L.lab_gpu_buffer(floats * 4))
        if self.handle < 0:
            raise StateError(f"GPU buffer of {floats * 4} bytes failed")
        self.length = floats
        ptr = L.lab_gpu_contents(self.handle)
        self.view = np.ctypeslib.as_array((ctypes.c_float * max(floats, 1)).from_address(ptr))


class _Matrix:
    def __init__(self, q4: bool, buffer: int, qs_at: int, scales_at: int, rows: int, cols: int):
        self.q4, self.buffer, self.qs_at, self.scales_at = q4, buffer, qs_at, scales_at
        self.rows, self.cols = rows, cols

    def encode(self, x: int, y: int, offset: int, n: int) -> None:
        enc = _lib.lib().lab_gpu_enc_matmul_q4 if self.q4 else _lib.lib().lab_gpu_enc_matmul_q8
        enc(self.buffer, self.qs_at, self.scales_at, x, offset, y, offset, self.rows, self.cols, n)


class GpuLinear:
    """Quantized products on the GPU outside a forward pass (gpu.dart:1269)."""

    def __init__(self):
        self._matrices: Dict[str, _Matrix] = {}
        self._owned: List[int] = []
        self._x: Optional[_Buffer] = None
        self._y: Optional[_Buffer] = None
        self._disposed = False

    @classmethod
    def start(cls) -> Optional["GpuLinear"]:
        """A GpuLinear, or None where the GPU does not start."""
        return cls() if _lib.lib().lab_gpu_init() == 1 else None

    @property
    def names(self):
        return self._matrices.keys()

    def upload(self, name: str, matrix) -> None:
        """Copies `matrix` (NativeQ8Matrix or NativeQ4Matrix) into a buffer of its own."""
        self._check_open()
        qs, scales = matrix.qs_bytes, matrix.scale_bytes
        scales_at = (qs.size + 63) // 64 * 64
        nbytes = scales_at + scales.size
        L = _lib.lib()
        handle = int(L.lab_gpu_buffer(nbytes))
        if handle < 0:
            raise StateError(f"GPU buffer of {nbytes} bytes failed")
        self._owned.append(handle)
        view = np.ctypeslib.as_array((ctypes.c_uint8 * nbytes).from_address(L.lab_gpu_contents(handle)))
        view[:qs.size] = qs
        view[scales_at:scales_at + scales.size] = scales
        previous = self._matrices.get(name)
        if previous is not None:
            self._owned.remove(previous.buffer)
            L.lab_gpu_release(previous.buffer)
        self._matrices[name] = _Matrix(isinstance(matrix, NativeQ4Matrix), handle, 0, scales_at,
                                       matrix.rows, matrix.cols)

    def apply(self, name: str, xs: np.ndarray, ys: np.ndarray, n: int) -> None:
        """ys[t * rows + r] = (W xs[t])[r] for t < n, W the matrix uploaded as `name`."""
        self._check_open()
        w = self._matrices.get(name)
        if w is None:
            raise ArgumentError(f"no GPU matrix named {name}")
        if n < 1 or xs.size < n * w.cols or ys.size < n * w.rows:
            raise ArgumentError(f"GPU product: bad shapes for n={n}")
        x = self._x = self._grow(self._x, n * w.cols)
        y = self._y = self._grow(self._y, n * w.rows)
        x.view[:n * w.cols] = xs[:n * w.cols]
        L = _lib.lib()
        L.lab_gpu_begin()
        w.encode(x.handle, y.handle, 0, n)
        if L.lab_gpu_commit(1) != 1:
            raise StateError("GPU command buffer failed")
        ys[:n * w.rows] = y.view[:n * w.rows]

    def _grow(self, buffer: Optional[_Buffer], floats: int) -> _Buffer:
        if buffer is not None and buffer.length >= floats:
            return buffer
        if buffer is not None:
            self._owned.remove(buffer.handle)
            _lib.lib().lab_gpu_release(buffer.handle)
        grown = _Buffer(floats)
        self._owned.append(grown.handle)
        return grown

    def _check_open(self) -> None:
        if self._disposed:
            raise StateError("the GPU products are disposed")

    def dispose(self) -> None:
        """Releases every GPU buffer. Using this afterwards throws."""
        if self._disposed:
            return
        self._disposed = True
        for h in self._owned:
            _lib.lib().lab_gpu_release(h)
        self._owned.clear()
        self._matrices.clear()
        self._x = self._y = None

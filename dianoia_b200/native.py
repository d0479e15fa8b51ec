"""Host-side mirror of dianoia's native quantized matrices (lib/src/native.dart).

The reference's Dart classes own weight memory from ``lab_alloc``, keep a
process-wide quantization scratch, check shapes and call ``lab_gemm_q8`` /
``lab_gemm_q4`` through dart:ffi (native.dart:499-868). Dart is not
available here, so this module restates that layer in Python over the same
C-ABI, served by the CUDA library: the same class and method names (in
Python spelling), the same argument meaning, and the same errors
(``ArgumentError`` for bad shapes, ``StateError`` for use before ``load``
or after ``free``).

Weights live in ``lab_alloc`` memory, which is CUDA managed memory: after the
first product they stay in HBM, while ``qs_bytes`` / ``weight_at`` still read
them from the host. Activations and outputs are ordinary host arrays, copied
to and from the GPU inside each call, or CUDA tensors used in place.
"""
from __future__ import annotations

import ctypes
import math
from typing import Callable, Optional

import numpy as np

from . import _lib


class ArgumentError(ValueError):
    """Dart's ArgumentError: a bad shape or argument."""


class StateError(RuntimeError):
    """Dart's StateError: an object used in a state that does not allow it."""


def _addr(a) -> int:
    """Address of a numpy array or a torch tensor (host or CUDA)."""
    if isinstance(a, np.ndarray):
        if not a.flags["C_CONTIGUOUS"]:
            raise ArgumentError("arrays must be contiguous")
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        if not a.is_contiguous():
            raise ArgumentError("tensors must be contiguous")
        return a.data_ptr()
    raise ArgumentError(f"unsupported buffer type {type(a)!r}")


def _len(a) -> int:
    return a.size if isinstance(a, np.ndarray) else a.numel()


def _check_call(what: str) -> None:
    code = _lib.lib().dn_last_error()
    if code != _lib.DN_OK:
        raise StateError(f"{what} failed on the GPU: {_lib.lib().dn_error_string(code).decode()}")


def _view(ptr: int, ctype, count: int) -> np.ndarray:
    """A numpy view of native memory (managed memory is host-addressable)."""
    if count == 0 or not ptr:
        return np.zeros(0, dtype=np.dtype(ctype))
    return np.ctypeslib.as_array((ctype * count).from_address(ptr))


def half_to_double(bits: int) -> float:
    """An IEEE half-precision bit pattern as a float (native.dart:871-880)."""
    sign = -1.0 if bits & 0x8000 else 1.0
    exponent = (bits >> 10) & 0x1F
    mantissa = bits & 0x3FF
    if exponent == 0:
        return sign * mantissa * 5.960464477539063e-8  # 2^-24
    if exponent == 31:
        return sign * math.inf if mantissa == 0 else math.nan
    return sign * (1 + mantissa / 1024) * 2.0 ** (exponent - 15)


class NativeKernels:
    """Process-wide settings of the kernels (native.dart:499-596)."""

    _instance: Optional["NativeKernels"] = None

    def __init__(self, threads: int, int8_inputs: bool):
        self.threads = threads
        self.int8_inputs = int8_inputs
        self._xq = 0
        self._xsc = 0
        self._capacity = 0

    @classmethod
    def load(cls, path: Optional[str] = None, threads: int = 4, int8_inputs: bool = True) -> None:
        """Enables the kernels. ``path`` is accepted for the reference's signature;
        the library is always the in-tree libdianoia_b200.so."""
        if not cls.is_available():
            raise StateError("the CUDA kernels cannot run here (no sm_100 device)")
        cls._instance = NativeKernels(threads, int8_inputs)

    @classmethod
    def instance(cls) -> "NativeKernels":
        if cls._instance is None:
            raise StateError("native kernels are not loaded (NativeKernels.load)")
        return cls._instance

    @classmethod
    def is_loaded(cls) -> bool:
        return cls._instance is not None

    @staticmethod
    def is_available() -> bool:
        return _lib.lib().lab_cpu_supported() == 1

    def _ensure_scratch(self, values: int) -> None:
        if values <= self._capacity:
            return
        L = _lib.lib()
        # The old scratch is not freed, as in the reference (native.dart:582-587).
        self._xq = L.lab_alloc(values) or 0
        self._xsc = L.lab_alloc(values // 32 * 4 + 4) or 0
        if not self._xq or not self._xsc:
            raise StateError(f"native allocation of {values} bytes failed")
        self._capacity = values

    @staticmethod
    def allocate(nbytes: int) -> int:
        p = _lib.lib().lab_alloc(nbytes)
        if not p:
            raise StateError(f"native allocation of {nbytes} bytes failed")
        return p


class _NativeMatrix:
    format = ""

    def __init__(self, rows: int, cols: int, qs: int, scales: int, owned: bool = True):
        self.rows = rows
        self.cols = cols
        self._qs = qs
        self._scales = scales
        self._owned = owned
        self._freed = False

    def free(self) -> None:
        """Frees the memory of a matrix made by quantizing (native.dart:700-708)."""
        if not self._owned:
            raise StateError("this matrix does not own its memory")
        if self._freed:
            return
        self._freed = True
        L = _lib.lib()
        L.lab_free(self._qs)
        L.lab_free(self._scales)

    def _check_live(self):
        if self._freed:
            raise StateError("the matrix was freed")

    def apply(self, xs, ys, n: int, int8_inputs: Optional[bool] = None) -> None:
        """ys[t * rows + r] = (W xs[t])[r] for t < n, xs as [n, cols]."""
        k = NativeKernels.instance()
        self._check_live()
        if _len(xs) < n * self.cols or _len(ys) < n * self.rows:
            raise ArgumentError(f"{self.format.upper()} product: bad shapes for n={n}")
        k._ensure_scratch(n * self.cols)
        mode = 1 if (k.int8_inputs if int8_inputs is None else int8_inputs) else 0
        fn = _lib.lib().lab_gemm_q4 if self.format == "q4" else _lib.lib().lab_gemm_q8
        fn(self._qs, self._scales, _addr(xs), k._xq, k._xsc, _addr(ys), self.rows, self.cols, n,
           k.threads, mode)
        _check_call(f"{self.format.upper()} product")


class NativeQ8Matrix(_NativeMatrix):
    """A row-major [rows, cols] matrix quantized to Q8 (native.dart:624-752)."""

    format = "q8"

    @classmethod
    def quantize(cls, w, rows: int, cols: int) -> "NativeQ8Matrix":
        if cols % 32 != 0:
            raise ArgumentError(f"Q8 needs cols to be a multiple of 32, got {cols}")
        w = np.ascontiguousarray(w, dtype=np.float32)
        qs = NativeKernels.allocate(rows * cols)
        scales = NativeKernels.allocate(rows * cols // 32 * 4)
        _lib.lib().lab_quantize_q8(w.ctypes.data, qs, scales, rows, cols)
        _check_call("Q8 quantization")
        return cls(rows, cols, qs, scales)

    @classmethod
    def quantize_rows(cls, rows: int, cols: int, fill: Callable[[int, int, np.ndarray], None],
                      chunk: int = 1024) -> "NativeQ8Matrix":
        """Quantizes a matrix too large to hold in f32 at once: ``fill(first,
        count, out)`` writes ``count`` rows starting at ``first`` into ``out``."""
        L = _lib.lib()
        qs = NativeKernels.allocate(rows * cols)
        scales = NativeKernels.allocate(rows * cols // 32 * 4)
        try:
            buffer = np.zeros(chunk * cols, np.float32)
            for first in range(0, rows, chunk):
                count = min(chunk, rows - first)
                fill(first, count, buffer)
                L.lab_quantize_q8(buffer.ctypes.data, qs + first * cols,
                                  scales + first * cols // 32 * 4, count, cols)
                _check_call("Q8 quantization")
        except BaseException:
            L.lab_free(qs)
            L.lab_free(scales)
            raise
        return cls(rows, cols, qs, scales)

    @classmethod
    def from_pointers(cls, rows: int, cols: int, qs: int, scales: int) -> "NativeQ8Matrix":
        """Wraps Q8 data that already exists (not owned)."""
        return cls(rows, cols, qs, scales, owned=False)

    @property
    def bytes(self) -> int:
        return self.rows * self.cols + self.rows * self.cols // 32 * 4

    @property
    def qs_bytes(self) -> np.ndarray:
        return _view(self._qs, ctypes.c_uint8, self.rows * self.cols)

    @property
    def scale_bytes(self) -> np.ndarray:
        return _view(self._scales, ctypes.c_uint8, self.rows * self.cols // 32 * 4)

    def weight_at(self, r: int, c: int) -> float:
        i = r * self.cols + c
        q = int(_view(self._qs, ctypes.c_int8, self.rows * self.cols)[i])
        s = float(_view(self._scales, ctypes.c_float, self.rows * self.cols // 32)[i // 32])
        return q * s


class NativeQ4Matrix(_NativeMatrix):
    """A row-major [rows, cols] matrix in Q4_0 (native.dart:755-868)."""

    format = "q4"

    @classmethod
    def from_gguf_blocks(cls, blocks: np.ndarray, rows: int, cols: int) -> "NativeQ4Matrix":
        """Splits GGUF Q4_0 blocks (a little-endian half scale, then 16 nibble
        bytes) into nibbles and scales without requantizing (native.dart:766-790)."""
        blocks = np.asarray(blocks, dtype=np.uint8)
        if rows <= 0 or cols <= 0 or cols % 32 != 0 or blocks.size != rows * cols // 32 * 18:
            raise ArgumentError(f"invalid Q4_0 blocks for {rows} x {cols}")
        qs = NativeKernels.allocate(rows * cols // 2)
        try:
            scales = NativeKernels.allocate(rows * cols // 32 * 2)
        except BaseException:
            _lib.lib().lab_free(qs)
            raise
        b = blocks.reshape(-1, 18)
        _view(scales, ctypes.c_uint8, rows * cols // 32 * 2)[:] = b[:, :2].reshape(-1)
        _view(qs, ctypes.c_uint8, rows * cols // 2)[:] = b[:, 2:].reshape(-1)
        return cls(rows, cols, qs, scales)

    @classmethod
    def quantize(cls, w, rows: int, cols: int) -> "NativeQ4Matrix":
        if cols % 32 != 0:
            raise ArgumentError(f"Q4 needs cols to be a multiple of 32, got {cols}")
        w = np.ascontiguousarray(w, dtype=np.float32)
        qs = NativeKernels.allocate(rows * cols // 2)
        scales = NativeKernels.allocate(rows * cols // 32 * 2)
        _lib.lib().lab_quantize_q4(w.ctypes.data, qs, scales, rows, cols)
        _check_call("Q4 quantization")
        return cls(rows, cols, qs, scales)

    @classmethod
    def from_pointers(cls, rows: int, cols: int, qs: int, scales: int) -> "NativeQ4Matrix":
        return cls(rows, cols, qs, scales, owned=False)

    @property
    def qs_bytes(self) -> np.ndarray:
        return _view(self._qs, ctypes.c_uint8, self.rows * self.cols // 2)

    @property
    def scale_bytes(self) -> np.ndarray:
        return _view(self._scales, ctypes.c_uint8, self.rows * self.cols // 32 * 2)

    def weight_at(self, r: int, c: int) -> float:
        i = r * self.cols + c
        block, k = i // 32, i % 32
        byte = int(_view(self._qs, ctypes.c_uint8, self.rows * self.cols // 2)[block * 16 + k % 16])
        q = byte & 15 if k < 16 else byte >> 4
        return half_to_double(int(_view(self._scales, ctypes.c_uint16, self.rows * self.cols // 32)[block])) * (q - 8)

"""TEST INFRASTRUCTURE ONLY - the CPU checker of the quantized linear path.

ctypes wrappers over two CPU libraries built by ``oracle/Makefile``:

* ``liboracle.so`` - this repository's scalar C restatement of dianoia's
  ``src/c/lab_native.c`` kernels (``oracle/lab_oracle.c``);
* ``_ref/libref_lab.so`` - the reference's own ``lab_native.c`` compiled
  unmodified (present only where it was built; it is not committed).

plus seeded generators for the inputs the parity tests and the benchmark use.
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
and reference legs may import this module, and only as the checker: the
product path (``dianoia_b200``) never calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_lab.so")

BLOCK = 32

_i64 = ctypes.c_int64
_p = ctypes.c_void_p


def build(ref: bool = True) -> None:
    """Runs the Makefile (the reference target only if its source exists)."""
    subprocess.run(["make", "-s", "-C", HERE, "all" if ref else "oracle"], check=True)


def _ptr(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


class _Lib:
    def __init__(self, path: str):
        self.path = path
        self.lib = ctypes.CDLL(path)


class Oracle(_Lib):
    """The C restatement (liboracle.so)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build(ref=False)
        super().__init__(path)
        L = self.lib
        L.orc_half_to_float.argtypes = [ctypes.c_uint16]
        L.orc_half_to_float.restype = ctypes.c_float
        L.orc_float_to_half.argtypes = [ctypes.c_float]
        L.orc_float_to_half.restype = ctypes.c_uint16
        for name in ("orc_quantize_q8", "orc_quantize_q4"):
            getattr(L, name).argtypes = [_p, _p, _p, _i64, _i64]
            getattr(L, name).restype = None
        for name in ("orc_gemm_q8", "orc_gemm_q4"):
            getattr(L, name).argtypes = [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64]
            getattr(L, name).restype = None
        L.orc_block_dots.argtypes = [ctypes.c_int, _p, _p, _p, _i64, _i64, _i64]
        L.orc_block_dots.restype = None
        L.orc_reference_f64.argtypes = [ctypes.c_int, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _p]
        L.orc_reference_f64.restype = None
        L.orc_rms_norm.argtypes = [_p, _p, _p, _i64, _i64, ctypes.c_double, _i64]
        L.orc_rms_norm.restype = None
        L.orc_swiglu.argtypes = [_p, _p, _i64]
        L.orc_swiglu.restype = None
        L.orc_head_norm_rope.argtypes = [_p, _i64, _p, _p, _i64, _i64, _i64, _i64, ctypes.c_double]
        L.orc_head_norm_rope.restype = None
        L.orc_attention.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p]
        L.orc_attention.restype = None
        L.orc_conv.argtypes = [_p, _p, _p, _p, _i64, _i64, _i64, _p]
        L.orc_conv.restype = None
        L.orc_steer.argtypes = [_p, _p, _i64, _i64, _i64, ctypes.c_double]
        L.orc_steer.restype = None

    def half_to_float(self, h: int) -> float:
        return self.lib.orc_half_to_float(h)

    def float_to_half(self, f: float) -> int:
        return self.lib.orc_float_to_half(f)

    def quantize_q8(self, w: np.ndarray, rows: int, cols: int):
        w = np.ascontiguousarray(w, dtype=np.float32)
        qs = np.zeros(rows * cols, np.int8)
        sc = np.zeros(rows * (cols // BLOCK), np.float32)
        self.lib.orc_quantize_q8(_ptr(w), _ptr(qs), _ptr(sc), rows, cols)
        return qs, sc

    def quantize_q4(self, w: np.ndarray, rows: int, cols: int):
        w = np.ascontiguousarray(w, dtype=np.float32)
        qs = np.zeros(rows * cols // 2, np.uint8)
        sc = np.zeros(rows * (cols // BLOCK), np.uint16)
        self.lib.orc_quantize_q4(_ptr(w), _ptr(qs), _ptr(sc), rows, cols)
        return qs, sc

    def gemm(self, fmt: str, qs, scales, xs, rows: int, cols: int, n: int, mode: int = 1):
        """Returns (ys, xq, xsc) as lab_gemm_q8 / lab_gemm_q4 would leave them."""
        xs = np.ascontiguousarray(xs, dtype=np.float32)
        ys = np.zeros(n * rows, np.float32)
        xq = np.zeros(n * cols, np.int8)
        xsc = np.zeros(n * (cols // BLOCK), np.float32)
        fn = self.lib.orc_gemm_q4 if fmt == "q4" else self.lib.orc_gemm_q8
        fn(_ptr(qs), _ptr(scales), _ptr(xs), _ptr(xq), _ptr(xsc), _ptr(ys), rows, cols, n, mode)
        return ys, xq, xsc

    def block_dots(self, fmt: str, qs, xq, rows: int, cols: int, n: int) -> np.ndarray:
        dots = np.zeros(n * rows * (cols // BLOCK), np.int32)
        self.lib.orc_block_dots(1 if fmt == "q4" else 0, _ptr(qs), _ptr(xq), _ptr(dots),
                                rows, cols, n)
        return dots

    def reference_f64(self, fmt: str, qs, scales, xs, rows: int, cols: int, n: int, mode: int = 1):
        xs = np.ascontiguousarray(xs, dtype=np.float32)
        ref = np.zeros(n * rows, np.float64)
        mag = np.zeros(n * rows, np.float64)
        self.lib.orc_reference_f64(1 if fmt == "q4" else 0, _ptr(qs), _ptr(scales), _ptr(xs),
                                   rows, cols, n, mode, _ptr(ref), _ptr(mag))
        return ref, mag


    def rms_norm(self, x, w, rows: int, cols: int, eps: float, out=None) -> np.ndarray:
        """RMSNorm of the CPU path; with `out` given, added into a copy of it."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        o = np.zeros(rows * cols, np.float32) if out is None else np.array(out, np.float32)
        self.lib.orc_rms_norm(_ptr(x), _ptr(w), _ptr(o), rows, cols, eps, 0 if out is None else 1)
        return o

    def swiglu(self, g, u) -> np.ndarray:
        """silu(g) * u of the CPU feed-forward, as a new array."""
        h = np.array(g, np.float32)
        u = np.ascontiguousarray(u, dtype=np.float32)
        self.lib.orc_swiglu(_ptr(h), _ptr(u), h.size)
        return h


    def head_norm_rope(self, x, x_stride, w, rope, rope_stride, heads, hd, n, eps) -> np.ndarray:
        """Per-head RMSNorm + RoPE of the CPU path, on a copy of x."""
        y = np.array(x, np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        rope = np.ascontiguousarray(rope, dtype=np.float32)
        self.lib.orc_head_norm_rope(_ptr(y), x_stride, _ptr(w), _ptr(rope), rope_stride, heads, hd, n, eps)
        return y

    def attention(self, q, keys, values, gate, position, n, heads, kv_heads, hd, window) -> np.ndarray:
        """The CPU path's attention in double; out [n, heads * hd]."""
        arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, keys, values)]
        g = None if gate is None else np.ascontiguousarray(gate, dtype=np.float32)
        out = np.zeros(n * heads * hd, np.float32)
        scores = np.zeros(position + n, np.float64)
        self.lib.orc_attention(_ptr(arrs[0]), _ptr(arrs[1]), _ptr(arrs[2]), _ptr(g), _ptr(out),
                               position, n, heads, kv_heads, hd, window, _ptr(scores))
        return out

    def conv(self, bcx, weight, history, width, k, n):
        """The gated short conv; returns (y, updated history)."""
        bcx = np.ascontiguousarray(bcx, dtype=np.float32)
        weight = np.ascontiguousarray(weight, dtype=np.float32)
        hist = np.array(history, np.float32)
        y = np.zeros(n * width, np.float32)
        z = np.zeros(max(n * width, 1), np.float32)
        self.lib.orc_conv(_ptr(bcx), _ptr(weight), _ptr(hist), _ptr(y), width, k, n, _ptr(z))
        return y, hist

    def steer(self, x, v, rows, cols, mode, scale) -> np.ndarray:
        y = np.array(x, np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        self.lib.orc_steer(_ptr(y), _ptr(v), rows, cols, mode, scale)
        return y


class Reference(_Lib):
    """The reference's lab_native.c, compiled here (oracle/_ref/libref_lab.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built (oracle/Makefile 'ref' target)")
        super().__init__(path)
        L = self.lib
        L.lab_quantize_q8.argtypes = [_p, _p, _p, _i64, _i64]
        L.lab_quantize_q4.argtypes = [_p, _p, _p, _i64, _i64]
        for name in ("lab_gemm_q8", "lab_gemm_q4"):
            getattr(L, name).argtypes = [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64]
            getattr(L, name).restype = None
        L.lab_quantize_q8.restype = None
        L.lab_quantize_q4.restype = None
        L.lab_attention.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64]
        L.lab_attention.restype = None

    def quantize_q8(self, w, rows, cols):
        w = np.ascontiguousarray(w, dtype=np.float32)
        qs = np.zeros(rows * cols, np.int8)
        sc = np.zeros(rows * (cols // BLOCK), np.float32)
        self.lib.lab_quantize_q8(_ptr(w), _ptr(qs), _ptr(sc), rows, cols)
        return qs, sc

    def quantize_q4(self, w, rows, cols):
        w = np.ascontiguousarray(w, dtype=np.float32)
        qs = np.zeros(rows * cols // 2, np.uint8)
        sc = np.zeros(rows * (cols // BLOCK), np.uint16)
        self.lib.lab_quantize_q4(_ptr(w), _ptr(qs), _ptr(sc), rows, cols)
        return qs, sc

    def attention(self, q, keys, values, gate, position, n, heads, kv_heads, hd, window, threads=1):
        """The reference's own C attention (lab_native.c:703-740, f32 and expf)."""
        arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, keys, values)]
        g = None if gate is None else np.ascontiguousarray(gate, dtype=np.float32)
        out = np.zeros(n * heads * hd, np.float32)
        self.lib.lab_attention(_ptr(arrs[0]), _ptr(arrs[1]), _ptr(arrs[2]), _ptr(g), _ptr(out), n,
                               position, heads, kv_heads, hd, window, threads)
        return out

    def gemm(self, fmt, qs, scales, xs, rows, cols, n, mode=1, threads=1,
             out=None):
        xs = np.ascontiguousarray(xs, dtype=np.float32)
        if out is None:
            out = (np.zeros(n * rows, np.float32), np.zeros(n * cols, np.int8),
                   np.zeros(n * (cols // BLOCK) + 1, np.float32))
        ys, xq, xsc = out
        fn = self.lib.lab_gemm_q4 if fmt == "q4" else self.lib.lab_gemm_q8
        fn(_ptr(qs), _ptr(scales), _ptr(xs), _ptr(xq), _ptr(xsc), _ptr(ys), rows, cols, n,
           threads, mode)
        return ys, xq, xsc[: n * (cols // BLOCK)]


# ----------------------------------------------------------------- inputs
#
# Seeded synthetic inputs with the shapes and value distributions of the
# benchmark configurations (numpy default_rng; no dataset is involved).

def q4_weights(rng: np.random.Generator, rows: int, cols: int,
               scale_lo: float = 0.002, scale_hi: float = 0.02):
    """Q4_0 weights: nibbles U{0..15} (value q - 8), fp16 scales U[lo, hi]."""
    nib = rng.integers(0, 16, size=(rows * cols // BLOCK, BLOCK), dtype=np.uint8)
    qs = (nib[:, :16] | (nib[:, 16:] << 4)).astype(np.uint8).reshape(-1)
    sc = rng.uniform(scale_lo, scale_hi, size=rows * (cols // BLOCK)).astype(np.float16)
    return qs, sc.view(np.uint16)


def q8_weights(rng: np.random.Generator, rows: int, cols: int,
               scale_lo: float = 0.001, scale_hi: float = 0.01):
    """Q8_0 weights: int8 U[-127, 127], fp16 scales U[lo, hi] widened exactly to f32."""
    qs = rng.integers(-127, 128, size=rows * cols, dtype=np.int8)
    sc = rng.uniform(scale_lo, scale_hi, size=rows * (cols // BLOCK)).astype(np.float16)
    return qs, sc.astype(np.float32)


def activations(rng: np.random.Generator, n: int, cols: int) -> np.ndarray:
    """f32 activations N(0, 1), [n, cols] flattened."""
    return rng.standard_normal(n * cols, dtype=np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """f32 -> the nearest bfloat16 (ties to even), returned as f32 (exact)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def pad_cols(x: np.ndarray, rows: int, cols: int, padded: int) -> np.ndarray:
    """[rows, cols] -> [rows, padded] with zeros after each row (padded >= cols)."""
    out = np.zeros((rows, padded), np.float32)
    out[:, :cols] = np.asarray(x, np.float32).reshape(rows, cols)
    return out.reshape(-1)


def vision_weights_f32(rng: np.random.Generator, rows: int, cols: int, padded: int = 0) -> np.ndarray:
    """Config 5's float weights before quantization: bf16 N(0, 0.02) widened to
    f32, each row zero-padded to `padded` columns (K = 4304 is not a multiple
    of the 32-element block; a zero block adds exactly 0 to every dot product
    and leaves the real values' quantization unchanged). The caller quantizes
    them with lab_quantize_q8, as the configuration specifies."""
    w = bf16_round(rng.normal(0.0, 0.02, size=rows * cols).astype(np.float32))
    return pad_cols(w, rows, cols, padded) if padded and padded != cols else w


def max_rel_err(ys: np.ndarray, ref: np.ndarray, mag: np.ndarray) -> float:
    """max |y - ref| / sum|w x| (native_kernels_test.dart:160-176); 0/0 counts as 0."""
    err = np.abs(ys.astype(np.float64) - ref)
    with np.errstate(invalid="ignore", divide="ignore"):
        rel = np.where(mag > 0, err / np.where(mag > 0, mag, 1.0), np.where(err > 0, np.inf, 0.0))
    return float(rel.max()) if rel.size else 0.0

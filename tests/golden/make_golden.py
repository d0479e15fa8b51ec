"""Generates the golden fixtures of the quantized linear path from the
reference itself: dianoia's src/c/lab_native.c compiled unmodified into
oracle/_ref/libref_lab.so (oracle/Makefile).

Run from the repository root, where the reference sources are present:

    python tests/golden/make_golden.py

Each case is one .npz holding the seeded inputs (numpy default_rng; the Dart
tests' math.Random streams cannot be reproduced outside Dart, so the shapes
and distributions follow the Dart tests while the values are numpy's) and
the reference's outputs: ys for mode 0 and mode 1, and the quantized
activations xq / xsc that mode 1 leaves in its scratch.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as orc  # noqa: E402


def linear_case(ref, name, fmt, rows, cols, n, seed, weights="quantize"):
    rng = np.random.default_rng(seed)
    if weights == "quantize":
        # native_kernels_test.dart:33-45 / gpu_linear_test.dart:15-17: weights
        # U(-0.5, 0.5) (gpu_linear: U(-1, 1)) quantized by the reference.
        w = rng.uniform(-0.5, 0.5, rows * cols).astype(np.float32)
        qs, sc = ref.quantize_q4(w, rows, cols) if fmt == "q4" else ref.quantize_q8(w, rows, cols)
        xs = rng.uniform(-1.0, 1.0, n * cols).astype(np.float32)
    else:
        # Benchmark-config distributions (2, 4).
        qs, sc = orc.q4_weights(rng, rows, cols) if fmt == "q4" else orc.q8_weights(rng, rows, cols)
        xs = orc.activations(rng, n, cols)
    ys0, _, _ = ref.gemm(fmt, qs, sc, xs, rows, cols, n, mode=0, threads=4)
    ys1, xq, xsc = ref.gemm(fmt, qs, sc, xs, rows, cols, n, mode=1, threads=4)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), kind="linear", fmt=fmt, rows=rows,
                        cols=cols, n=n, seed=seed, qs=qs, scales=sc, xs=xs, ys_mode0=ys0,
                        ys_mode1=ys1, xq=xq, xsc=xsc)


def special_values(rng, rows, cols):
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    x[0, :32] = 0.0
    x[0, 32:64] = -0.0
    x[1, 5], x[1, 40], x[1, 70] = np.nan, np.inf, -np.inf
    x[2, :32] = 1e-40
    x[2, 32:64] = rng.standard_normal(32).astype(np.float32) * np.float32(1e-39)
    x[3, :32] = 1e38
    x[3, 32:64] = -3e38
    x[4, :32] = np.float32(127.0) * (np.arange(32, dtype=np.float32) - 16) / 16
    x[5, :] = 0.5
    x[6, 1] = np.float32(2e-45)
    x[7, :] = -x[7, :]
    x[7, 3] = x[7, 9] = -4.0  # ties in magnitude with different signs
    x[7, 4] = 4.0
    return x.reshape(-1)


def quantize_case(ref, name, seed):
    rng = np.random.default_rng(seed)
    rows, cols = 8, 32 * 12
    x = special_values(rng, rows, cols)
    xq, xsc = ref.quantize_q8(x, rows, cols)
    q4, s4 = ref.quantize_q4(x, rows, cols)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), kind="quantize", rows=rows, cols=cols,
                        seed=seed, x=x, xq=xq, xsc=xsc, q4=q4, s4=s4)


CASES = [
    # native_kernels_test.dart: rows 37, cols 2048, n 6 (seed 11) and n 3 (seed 23)
    ("nk_q8_n6", "q8", 37, 2048, 6, 11, "quantize"),
    ("nk_q4_n6", "q4", 37, 2048, 6, 11, "quantize"),
    ("nk_q8_n3", "q8", 37, 2048, 3, 23, "quantize"),
    ("nk_q4_n3", "q4", 37, 2048, 3, 23, "quantize"),
    # gpu_linear_test.dart:27-31: shapes that do not divide the GEMM tiles
    ("gl_q4_64x64_n1", "q4", 64, 64, 1, 5, "quantize"),
    ("gl_q4_70x96_n13", "q4", 70, 96, 13, 5, "quantize"),
    ("gl_q8_36x64_n9", "q8", 36, 64, 9, 5, "quantize"),
    ("gl_q8_128x128_n40", "q8", 128, 128, 40, 5, "quantize"),
    # bin/dianoia.dart _nativeQ8Check shapes
    ("st_q8_20x7680_n5", "q8", 20, 7680, 5, 3, "quantize"),
    # benchmark-config distributions at reduced row counts
    ("c1_q4_256x2048_n1", "q4", 256, 2048, 1, 0, "config"),
    ("c2_q8_32x6144_n1", "q8", 32, 6144, 1, 0, "config"),
    ("c4_q4_64x2048_n40", "q4", 64, 2048, 40, 0, "config"),
    # ragged: cols not a multiple of 32 (the reference ignores the tail)
    ("rg_q8_5x100_n3", "q8", 5, 100, 3, 7, "quantize"),
    ("rg_q4_4x72_n2", "q4", 4, 72, 2, 7, "quantize"),
]


def main():
    ref = orc.Reference()
    for case in CASES:
        linear_case(ref, *case)
    quantize_case(ref, "quant_special", 1)
    print("wrote", len(CASES) + 1, "fixtures to", HERE)


if __name__ == "__main__":
    main()

"""The oracle (oracle/lab_oracle.c) against the reference's own outputs.

Pins the C restatement before anything is checked against it: bit-exact
against the committed fixtures made by dianoia's compiled lab_native.c
(tests/golden/make_golden.py), against that library itself on fresh seeded
inputs where it is built, and within the Dart tests' 1e-5 bound of a
double-precision sum (native_kernels_test.dart:146-180).
"""
import numpy as np
import pytest

from conftest import golden_names, load_golden
from oracle import oracle as orc


def bits(a):
    return np.asarray(a).view(np.uint32 if np.asarray(a).dtype == np.float32 else np.uint8)


@pytest.mark.parametrize("name", golden_names("linear"))
@pytest.mark.parametrize("mode", [0, 1])
def test_oracle_matches_golden(oracle, name, mode):
    g = load_golden(name)
    fmt, rows, cols, n = str(g["fmt"]), int(g["rows"]), int(g["cols"]), int(g["n"])
    ys, xq, xsc = oracle.gemm(fmt, g["qs"], g["scales"], g["xs"], rows, cols, n, mode)
    assert np.array_equal(ys.view(np.uint32), g[f"ys_mode{mode}"].view(np.uint32))
    if mode == 1:
        assert np.array_equal(xq, g["xq"])
        assert np.array_equal(xsc.view(np.uint32), g["xsc"].view(np.uint32))


@pytest.mark.parametrize("name", golden_names("linear"))
def test_golden_within_dart_tolerance(oracle, name):
    g = load_golden(name)
    fmt, rows, cols, n = str(g["fmt"]), int(g["rows"]), int(g["cols"]), int(g["n"])
    for mode in (0, 1):
        ref, mag = oracle.reference_f64(fmt, g["qs"], g["scales"], g["xs"], rows, cols, n, mode)
        assert orc.max_rel_err(g[f"ys_mode{mode}"], ref, mag) < 1e-5


def test_quantizers_match_golden_special_values(oracle):
    g = load_golden("quant_special")
    rows, cols = int(g["rows"]), int(g["cols"])
    xq, xsc = oracle.quantize_q8(g["x"], rows, cols)
    assert np.array_equal(xq, g["xq"])
    assert np.array_equal(xsc.view(np.uint32), g["xsc"].view(np.uint32))
    q4, s4 = oracle.quantize_q4(g["x"], rows, cols)
    assert np.array_equal(q4, g["q4"])
    assert np.array_equal(s4, g["s4"])


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("shape", [(37, 2048, 6), (70, 96, 13), (9, 1152, 3), (5, 4320, 2),
                                   (3, 100, 4), (1, 32, 1)])
def test_oracle_matches_reference_library(oracle, reference, fmt, shape):
    rows, cols, n = shape
    rng = np.random.default_rng(rows * 1000 + cols + n)
    w = rng.uniform(-0.5, 0.5, rows * cols).astype(np.float32)
    qa = oracle.quantize_q4(w, rows, cols) if fmt == "q4" else oracle.quantize_q8(w, rows, cols)
    qb = reference.quantize_q4(w, rows, cols) if fmt == "q4" else reference.quantize_q8(w, rows, cols)
    for a, b in zip(qa, qb):
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8))
    xs = rng.standard_normal(n * cols).astype(np.float32)
    for mode in (0, 1):
        ya, xqa, xsa = oracle.gemm(fmt, qa[0], qa[1], xs, rows, cols, n, mode)
        yb, xqb, xsb = reference.gemm(fmt, qa[0], qa[1], xs, rows, cols, n, mode, threads=3)
        assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))
        if mode == 1:
            assert np.array_equal(xqa, xqb) and np.array_equal(xsa.view(np.uint32), xsb.view(np.uint32))


def test_half_conversions_match_numpy(oracle):
    allh = np.arange(65536, dtype=np.uint16)
    f = np.array([oracle.half_to_float(int(h)) for h in allh[::7]], np.float32)
    ref = allh[::7].view(np.float16).astype(np.float32)
    ok = ~np.isnan(ref)
    assert np.array_equal(f[ok].view(np.uint32), ref[ok].view(np.uint32))
    assert np.isnan(f[~ok]).all()
    rng = np.random.default_rng(3)
    vals = np.concatenate([rng.standard_normal(2000).astype(np.float32) * s
                           for s in (1e-8, 1e-5, 1.0, 1e4)] +
                          [np.array([0.0, -0.0, 65504, 65519, 65520, 2.0 ** -25, 2.0 ** -24,
                                     3 * 2.0 ** -26, 2.0 ** -14, np.inf, -np.inf], np.float32)])
    h = np.array([oracle.float_to_half(float(v)) for v in vals], np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(h, vals.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("fmt", ["q8", "q4"])
def test_block_dots_restate_numpy(oracle, fmt):
    rng = np.random.default_rng(9)
    rows, cols, n = 7, 256, 3
    qs, _ = orc.q4_weights(rng, rows, cols) if fmt == "q4" else orc.q8_weights(rng, rows, cols)
    xq = rng.integers(-127, 128, n * cols, dtype=np.int8)
    dots = oracle.block_dots(fmt, qs, xq, rows, cols, n).reshape(n, rows, cols // 32)
    if fmt == "q4":
        b = qs.reshape(rows, cols // 32, 16)
        w = np.concatenate([(b & 15), (b >> 4)], axis=2).astype(np.int64) - 8
    else:
        w = qs.reshape(rows, cols // 32, 32).astype(np.int64)
    x = xq.reshape(n, cols // 32, 32).astype(np.int64)
    want = np.einsum("rbk,tbk->trb", w, x)
    assert np.array_equal(dots, want)

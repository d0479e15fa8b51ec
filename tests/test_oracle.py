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


# ------------------------------------------------------------ neighbours
#
# RMSNorm and SwiGLU live in dianoia's Dart code (lib/src/ops.dart:12-31,
# lib/src/shard.dart:456-460), which cannot run here. The C restatement is
# pinned against a second, independent restatement in Python, whose float is
# the same IEEE double as Dart's and whose math.exp is the same C library
# exp, with f32 stores through numpy's round-to-nearest conversion; and
# against a few answers worked by hand.

def _f32(v):
    return float(np.float32(v))


def _py_rms_norm(x, w, eps):
    s = 0.0
    for v in x:
        s += float(v) * float(v)
    r = 1 / __import__("math").sqrt(s / len(x) + eps)
    return np.array([_f32(float(wj) * _f32(float(xj) * r)) for xj, wj in zip(x, w)], np.float32)


def _py_swiglu(g, u):
    import math
    out = []
    for gj, uj in zip(g, u):
        gd = float(gj)
        try:
            e = math.exp(-gd)
        except OverflowError:  # Python raises where C and Dart give infinity
            e = math.inf
        out.append(_f32(_f32(gd / (1 + e)) * float(uj)))
    return np.array(out, np.float32)


@pytest.mark.parametrize("rows,cols,eps", [(1, 2048, 1e-6), (3, 1000, 1e-5), (2, 7, 0.0)])
def test_rms_norm_restatements_agree(oracle, rows, cols, eps):
    rng = np.random.default_rng(rows * 1000 + cols)
    x = (rng.standard_normal(rows * cols) * 3).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    got = oracle.rms_norm(x, w, rows, cols, eps)
    want = np.concatenate([_py_rms_norm(x[t * cols:(t + 1) * cols], w, eps) for t in range(rows)])
    assert np.array_equal(bits(got), bits(want))
    prev = rng.standard_normal(rows * cols).astype(np.float32)
    acc = oracle.rms_norm(x, w, rows, cols, eps, out=prev)
    assert np.array_equal(bits(acc), bits((prev + want).astype(np.float32)))


def test_rms_norm_known_answers(oracle):
    # [3, 4]: mean square 12.5, r = 1 / sqrt(12.5); unit weights.
    got = oracle.rms_norm(np.array([3, 4], np.float32), np.ones(2, np.float32), 1, 2, 0.0)
    r = 1 / np.sqrt(np.float64(12.5))
    assert got.tolist() == [np.float32(3 * r), np.float32(4 * r)]
    # All zeros with eps 1e-6: r = 1000 exactly in double, outputs stay 0.
    z = oracle.rms_norm(np.zeros(32, np.float32), np.full(32, 2, np.float32), 1, 32, 1e-6)
    assert not z.any()
    # A constant row c normalises to sign(c) * 1 / sqrt(1 + eps / c^2) * weight.
    c = oracle.rms_norm(np.full(64, -2, np.float32), np.full(64, 0.5, np.float32), 1, 64, 0.0)
    assert np.all(c == np.float32(-0.5))


def test_swiglu_restatements_agree(oracle):
    rng = np.random.default_rng(77)
    g = (rng.standard_normal(4096) * 4).astype(np.float32)
    g[:6] = [0.0, -0.0, 90.0, -90.0, 1e-30, -800.0]
    u = rng.standard_normal(4096).astype(np.float32)
    got = oracle.swiglu(g, u)
    assert np.array_equal(bits(got), bits(_py_swiglu(g, u)))
    assert got[0] == 0 and got[2] == np.float32(90.0) * u[2] and got[5] == 0


# ------------------------------------------------------------ the layer's other ops

@pytest.mark.parametrize("heads,kv,hd,pos,n,window,gated", [
    (16, 8, 128, 50, 3, 0, True), (16, 8, 128, 40, 1, 16, False), (4, 4, 64, 0, 5, 0, True),
    (8, 2, 128, 300, 2, 64, True)])
def test_attention_restatement_against_the_reference_c(oracle, reference, heads, kv, hd, pos, n, window, gated):
    """orc_attention (shard.dart's double arithmetic) against the reference's
    own lab_attention (lab_native.c:588-740, f32 with expf), compiled here:
    within f32 rounding of the outputs."""
    rng = np.random.default_rng(heads + pos + n)
    q = rng.standard_normal(n * heads * hd).astype(np.float32)
    k = rng.standard_normal((pos + n) * kv * hd).astype(np.float32)
    v = rng.standard_normal((pos + n) * kv * hd).astype(np.float32)
    g = rng.standard_normal(n * heads).astype(np.float32) if gated else None
    a = oracle.attention(q, k, v, g, pos, n, heads, kv, hd, window)
    b = reference.attention(q, k, v, g, pos, n, heads, kv, hd, window)
    assert np.abs(a - b).max() <= 1e-5 * max(1.0, np.abs(b).max())


def test_conv_steer_and_head_norm_restatements(oracle):
    """orc_conv, orc_steer and orc_head_norm_rope against restatements in
    Python (Dart's double is Python's float; f32 stores through numpy)."""
    import math
    rng = np.random.default_rng(12)
    f = lambda v: float(np.float32(v))
    width, k, n = 5, 3, 4
    bcx = rng.standard_normal(n * 3 * width).astype(np.float32)
    w = rng.standard_normal(width * k).astype(np.float32)
    hist = rng.standard_normal((k - 1) * width).astype(np.float32)
    y, h2 = oracle.conv(bcx, w, hist, width, k, n)
    z = [[f(float(bcx[t * 3 * width + c]) * float(bcx[t * 3 * width + 2 * width + c])) for c in range(width)]
         for t in range(n)]
    for t in range(n):
        for c in range(width):
            acc = 0.0
            for s in range(k):
                src = t - s
                zz = z[src][c] if src >= 0 else float(hist[(k - 1 + src) * width + c])
                acc += float(w[c * k + k - 1 - s]) * zz
            assert y[t * width + c] == np.float32(float(bcx[t * 3 * width + width + c]) * acc)
    assert np.array_equal(h2, np.array(z[-(k - 1):], np.float32).ravel())

    x = rng.standard_normal(3 * 16).astype(np.float32)
    v = rng.standard_normal(16).astype(np.float32)
    got = oracle.steer(x, v, 3, 16, 1, 0.75)
    for t in range(3):
        dot = 0.0
        for j in range(16):
            dot += float(x[t * 16 + j]) * float(v[j])
        c = 0.75 * dot
        want = [f(float(x[t * 16 + j]) - c * float(v[j])) for j in range(16)]
        assert got[t * 16:(t + 1) * 16].tolist() == want
    assert np.array_equal(oracle.steer(x, v, 3, 16, 0, 1.0), x + np.tile(v, 3))

    heads, hd = 2, 8
    xs = rng.standard_normal(heads * hd).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    rope = rng.uniform(-1, 1, hd).astype(np.float32)
    got = oracle.head_norm_rope(xs, heads * hd, nw, rope, hd, heads, hd, 1, 1e-6)
    for hh in range(heads):
        seg = _py_rms_norm(xs[hh * hd:(hh + 1) * hd], nw, 1e-6)
        for j in range(hd // 2):
            x1, x2, c, s = float(seg[j]), float(seg[j + hd // 2]), float(rope[j]), float(rope[hd // 2 + j])
            assert got[hh * hd + j] == np.float32(x1 * c - x2 * s)
            assert got[hh * hd + j + hd // 2] == np.float32(x2 * c + x1 * s)


def test_conv_history_carries_across_short_chunks(oracle):
    """orc_conv on chunks shorter than the kernel (n < k - 1, the history
    shift of shard.dart:509-516) gives the same outputs and history as the
    whole sequence in one chunk."""
    rng = np.random.default_rng(14)
    width, k, total = 6, 4, 7
    bcx = rng.standard_normal(total * 3 * width).astype(np.float32)
    w = rng.standard_normal(width * k).astype(np.float32)
    hist0 = rng.standard_normal((k - 1) * width).astype(np.float32)
    y_all, h_all = oracle.conv(bcx, w, hist0, width, k, total)
    hist, ys = hist0, []
    for t0, n in ((0, 1), (1, 2), (3, 1), (4, 3)):
        y, hist = oracle.conv(bcx[t0 * 3 * width:(t0 + n) * 3 * width], w, hist, width, k, n)
        ys.append(y)
    assert np.array_equal(np.concatenate(ys), y_all)
    assert np.array_equal(hist, h_all)

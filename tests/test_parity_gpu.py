"""CUDA path against the oracle, through the C-ABI (GPU only).

The GEMV and generic paths must equal the reference bit for bit (f32 outputs
included); the tensor-core GEMM must give bit-exact quantized activations and
f32 outputs within the reference's 1e-5 relative bound
(native_kernels_test.dart:146-180). Fixtures come from the reference library
itself; larger shapes are checked against the oracle's C restatement, which
tests/test_oracle.py pins to the reference.
"""
import numpy as np
import pytest

from conftest import golden_names, load_golden
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TOL = 1e-5  # max |y - ref| / sum |w x|, the reference's own bound


def host_gemm(L, fmt, qs, sc, xs, rows, cols, n, mode):
    ys = np.full(n * rows, np.nan, np.float32)
    xq = np.zeros(n * cols, np.int8)
    xsc = np.zeros(n * (cols // 32) + 1, np.float32)
    fn = L.lab_gemm_q4 if fmt == "q4" else L.lab_gemm_q8
    fn(qs.ctypes.data, sc.ctypes.data, xs.ctypes.data, xq.ctypes.data, xsc.ctypes.data,
       ys.ctypes.data, rows, cols, n, 4, mode)
    assert L.dn_last_error() == 0
    return ys, xq, xsc[: n * (cols // 32)]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def dev_linear(L, fmt, qs, sc, xs, rows, cols, n, mode=1, path=-1, ldy=None, flags=0):
    """dn_linear on device tensors; returns (ys [n, ldy], xq, xsc) as numpy."""
    ldy = rows if ldy is None else ldy
    ys = torch.full((n * ldy,), float("nan"), dtype=torch.float32, device="cuda")
    xq = torch.zeros(n * cols, dtype=torch.int8, device="cuda")
    xsc = torch.zeros(n * (cols // 32) + 1, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = L.dn_linear(1 if fmt == "q4" else 0, qs.data_ptr(), sc.data_ptr(), xs.data_ptr(),
                     xq.data_ptr(), xsc.data_ptr(), ys.data_ptr(), rows, cols, n, ldy, mode,
                     path, flags, st)
    torch.cuda.synchronize()
    assert rc == 0, L.dn_error_string(rc)
    assert L.dn_device_status(1) == 0
    return ys.cpu().numpy(), xq.cpu().numpy(), xsc.cpu().numpy()[: n * (cols // 32)]


def same_bits(a, b):
    return np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


def weights(fmt, rng, rows, cols):
    return orc.q4_weights(rng, rows, cols) if fmt == "q4" else orc.q8_weights(rng, rows, cols)


# ----------------------------------------------------------------- fixtures


@pytest.mark.parametrize("name", golden_names("linear"))
@pytest.mark.parametrize("mode", [0, 1])
def test_golden_through_lab_gemm(cuda_lib, name, mode):
    g = load_golden(name)
    fmt, rows, cols, n = str(g["fmt"]), int(g["rows"]), int(g["cols"]), int(g["n"])
    ys, xq, xsc = host_gemm(cuda_lib, fmt, g["qs"], g["scales"], g["xs"], rows, cols, n, mode)
    want = g[f"ys_mode{mode}"]
    path = cuda_lib.dn_linear_path(1 if fmt == "q4" else 0, None, None, None, None, rows, cols, n,
                                   mode)
    if mode == 1:
        assert np.array_equal(xq, g["xq"]) and same_bits(xsc, g["xsc"])
    if path == 1:  # tensor-core GEMM: tolerance, not bits
        ref, mag = orc.Oracle().reference_f64(fmt, g["qs"], g["scales"], g["xs"], rows, cols, n, mode)
        assert orc.max_rel_err(ys, ref, mag) < TOL
    else:
        assert same_bits(ys, want)


def test_quantizers_on_special_values(cuda_lib):
    g = load_golden("quant_special")
    rows, cols = int(g["rows"]), int(g["cols"])
    x = g["x"]
    xq = np.zeros(rows * cols, np.int8)
    xsc = np.zeros(rows * cols // 32, np.float32)
    cuda_lib.lab_quantize_q8(x.ctypes.data, xq.ctypes.data, xsc.ctypes.data, rows, cols)
    assert np.array_equal(xq, g["xq"]) and same_bits(xsc, g["xsc"])
    q4 = np.zeros(rows * cols // 2, np.uint8)
    s4 = np.zeros(rows * cols // 32, np.uint16)
    cuda_lib.lab_quantize_q4(x.ctypes.data, q4.ctypes.data, s4.ctypes.data, rows, cols)
    assert np.array_equal(q4, g["q4"]) and np.array_equal(s4, g["s4"])
    assert cuda_lib.dn_last_error() == 0


# ------------------------------------------------------- configuration shapes

CONFIG_SHAPES = [
    ("q4", 6144, 2048),   # config 1: Qwen3-1.7B MLP up, Q4_0
    ("q8", 2048, 2048),   # config 2: q / o
    ("q8", 1024, 2048),   # config 2: k / v
    ("q8", 6144, 2048),   # config 2: gate / up
    ("q8", 2048, 6144),   # config 2: down
    ("q4", 2048, 6144),   # config 4: down, Q4_0
    ("q8", 3456, 1152),   # config 5: qkv
    ("q8", 1152, 4320),   # config 5: fc2, K zero-padded from 4304
    ("q4", 4304, 1152),   # config 5 fc1 shape in Q4 (K blocks not 16-byte aligned as fp16)
]


@pytest.mark.parametrize("fmt,rows,cols", CONFIG_SHAPES)
@pytest.mark.parametrize("n", [1, 3, 8])
def test_config_shapes_bit_exact(cuda_lib, oracle, fmt, rows, cols, n):
    rng = np.random.default_rng(rows + cols + n)
    qs, sc = weights(fmt, rng, rows, cols)
    xs = orc.activations(rng, n, cols)
    want, wq, wsc = oracle.gemm(fmt, qs, sc, xs, rows, cols, n, 1)
    ys, xq, xsc = dev_linear(cuda_lib, fmt, dev(qs), dev(sc), dev(xs), rows, cols, n, path=0)
    assert np.array_equal(xq, wq) and same_bits(xsc, wsc)
    assert same_bits(ys, want)


@pytest.mark.parametrize("fmt", ["q8", "q4"])
def test_lm_head_bit_exact(cuda_lib, oracle, fmt):
    rows, cols = 151936, 2048
    rng = np.random.default_rng(151936)
    qs, sc = weights(fmt, rng, rows, cols)
    xs = orc.activations(rng, 1, cols)
    want, _, _ = oracle.gemm(fmt, qs, sc, xs, rows, cols, 1, 1)
    ys, _, _ = dev_linear(cuda_lib, fmt, dev(qs), dev(sc), dev(xs), rows, cols, 1)
    assert same_bits(ys, want)


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("rows", [1, 7, 8, 9, 37, 100, 1000, 4097])
@pytest.mark.parametrize("n", [1, 2, 5, 11])
def test_ragged_rows_and_tokens(cuda_lib, oracle, fmt, rows, n):
    cols = 544  # 17 blocks: a partial last stage for both formats
    rng = np.random.default_rng(rows * 31 + n)
    qs, sc = weights(fmt, rng, rows, cols)
    xs = orc.activations(rng, n, cols)
    want, _, _ = oracle.gemm(fmt, qs, sc, xs, rows, cols, n, 1)
    ys, _, _ = dev_linear(cuda_lib, fmt, dev(qs), dev(sc), dev(xs), rows, cols, n, path=0)
    assert same_bits(ys, want)


def test_strided_output_and_pdl(cuda_lib, oracle):
    rows, cols, n, ldy = 300, 1024, 3, 1000
    rng = np.random.default_rng(5)
    qs, sc = weights("q8", rng, rows, cols)
    xs = orc.activations(rng, n, cols)
    want, _, _ = oracle.gemm("q8", qs, sc, xs, rows, cols, n, 1)
    ys, _, _ = dev_linear(cuda_lib, "q8", dev(qs), dev(sc), dev(xs), rows, cols, n, ldy=ldy,
                          flags=1)
    ys = ys.reshape(n, ldy)
    assert same_bits(ys[:, :rows].reshape(-1), want)
    assert np.isnan(ys[:, rows:]).all()  # nothing written past the rows


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("mode", [0, 1])
def test_generic_path_unaligned(cuda_lib, oracle, fmt, mode):
    rows, cols, n = 45, 640, 3
    rng = np.random.default_rng(77)
    qs, sc = weights(fmt, rng, rows, cols)
    xs = orc.activations(rng, n, cols)
    want, wq, wsc = oracle.gemm(fmt, qs, sc, xs, rows, cols, n, mode)
    raw = torch.zeros(qs.nbytes + 16, dtype=torch.uint8, device="cuda")
    raw[1: 1 + qs.nbytes] = dev(qs.view(np.uint8))
    qs_odd = raw[1:]  # 1-byte misaligned: the GEMV's bulk copies cannot take it
    assert cuda_lib.dn_linear_path(1 if fmt == "q4" else 0, qs_odd.data_ptr(), None, None, None,
                                   rows, cols, n, mode) == 2
    ys, xq, xsc = dev_linear(cuda_lib, fmt, qs_odd, dev(sc), dev(xs), rows, cols, n, mode=mode)
    assert same_bits(ys, want)
    if mode == 1:
        assert np.array_equal(xq, wq) and same_bits(xsc, wsc)


def test_zero_and_degenerate_shapes(cuda_lib):
    L = cuda_lib
    xs = np.ones(64, np.float32)
    ys = np.full(4, np.nan, np.float32)
    xq = np.zeros(64, np.int8)
    xsc = np.zeros(4, np.float32)
    w = np.zeros(4 * 16, np.int8)
    s = np.zeros(4, np.float32)
    # cols < 32: no blocks, every output is +0 as in the reference
    L.lab_gemm_q8(w.ctypes.data, s.ctypes.data, xs.ctypes.data, xq.ctypes.data, xsc.ctypes.data,
                  ys.ctypes.data, 4, 16, 1, 1, 1)
    assert L.dn_last_error() == 0 and (ys == 0).all() and not np.signbit(ys).any()
    # n = 0 and rows = 0 do nothing and report nothing
    L.lab_gemm_q8(w.ctypes.data, s.ctypes.data, xs.ctypes.data, xq.ctypes.data, xsc.ctypes.data,
                  ys.ctypes.data, 4, 32, 0, 1, 1)
    L.lab_gemm_q8(w.ctypes.data, s.ctypes.data, xs.ctypes.data, xq.ctypes.data, xsc.ctypes.data,
                  ys.ctypes.data, 0, 32, 2, 1, 1)
    assert L.dn_last_error() == 0
    assert xq[:64].any()  # rows = 0 still quantizes, like lab_gemm_q8
    # bad arguments are reported, not run
    assert L.dn_linear(0, None, None, None, None, None, None, 4, 32, 1, 2, 1, -1, 0, None) == -1
    assert L.dn_linear(7, None, None, None, None, None, None, 4, 32, 1, 4, 1, -1, 0, None) == -1


def test_native_matrix_mirror(cuda_lib, oracle):
    from dianoia_b200 import NativeKernels, NativeQ4Matrix, NativeQ8Matrix, StateError
    NativeKernels.load(None, threads=2)
    rng = np.random.default_rng(11)
    rows, cols, n = 37, 2048, 6
    w = rng.uniform(-0.5, 0.5, rows * cols).astype(np.float32)
    xs = rng.uniform(-1, 1, n * cols).astype(np.float32)
    for cls, fmt in ((NativeQ8Matrix, "q8"), (NativeQ4Matrix, "q4")):
        m = cls.quantize(w, rows, cols)
        qs = np.array(m.qs_bytes)
        sc = np.array(m.scale_bytes).view(np.uint16 if fmt == "q4" else np.float32)
        wq, ws = oracle.quantize_q4(w, rows, cols) if fmt == "q4" else oracle.quantize_q8(w, rows, cols)
        assert np.array_equal(qs, wq.view(np.uint8)) and np.array_equal(sc.view(np.uint8), ws.view(np.uint8))
        for int8 in (True, False):
            ys = np.zeros(n * rows, np.float32)
            m.apply(xs, ys, n, int8_inputs=int8)
            want, _, _ = oracle.gemm(fmt, wq, ws, xs, rows, cols, n, 1 if int8 else 0)
            assert same_bits(ys, want)
        if fmt == "q8":
            assert m.weight_at(3, 100) == float(wq[3 * cols + 100]) * float(ws[(3 * cols + 100) // 32])
        m.free()
        m.free()  # a second free is a no-op
        with pytest.raises(StateError):
            m.apply(xs, np.zeros(n * rows, np.float32), n)


def test_repeat_calls_identical(cuda_lib):
    rng = np.random.default_rng(2)
    rows, cols = 4096, 2048
    qs, sc = weights("q4", rng, rows, cols)
    xs = orc.activations(rng, 1, cols)
    a = host_gemm(cuda_lib, "q4", qs, sc, xs, rows, cols, 1, 1)[0]
    b = host_gemm(cuda_lib, "q4", qs, sc, xs, rows, cols, 1, 1)[0]
    assert same_bits(a, b)


# ------------------------------------------------- quantized-activation chain


def qa_pack(xq, xsc, n, cols):
    """QA blocks (32 int8 + f32 scale per block) from separate xq / xsc."""
    blocks = cols // 32
    out = np.zeros((n, blocks, 36), np.uint8)
    out[:, :, :32] = xq.reshape(n, blocks, 32).view(np.uint8)
    out[:, :, 32:] = xsc.reshape(n, blocks, 1).view(np.uint8).reshape(n, blocks, 4)
    return out.reshape(-1)


# (Shapes with few row tiles, whole or partial chunks of K, and a partial last tile.)
@pytest.mark.parametrize("fmt,rows,cols", [("q8", 4096, 2048), ("q4", 6144, 2048),
                                           ("q8", 2048, 6144), ("q8", 1152, 4320),
                                           ("q4", 96, 1152), ("q8", 2048, 2048),
                                           ("q4", 1024, 4096), ("q8", 2000, 1024)])
@pytest.mark.parametrize("n", [1, 4])
def test_qa_linear_matches_lab_gemm(cuda_lib, oracle, fmt, rows, cols, n):
    L = cuda_lib
    rng = np.random.default_rng(rows ^ cols ^ n)
    qs, sc = weights(fmt, rng, rows, cols)
    xs = orc.activations(rng, n, cols)
    want, wq, wsc = oracle.gemm(fmt, qs, sc, xs, rows, cols, n, 1)
    st = torch.cuda.current_stream().cuda_stream
    xs_d = dev(xs)
    xa = torch.zeros(n * (cols // 32) * 36, dtype=torch.uint8, device="cuda")
    assert L.dn_quantize_qa(xs_d.data_ptr(), xa.data_ptr(), n, cols, cols // 32 * 36, st) == 0
    ys = torch.full((n * rows,), float("nan"), device="cuda")
    ya = torch.zeros(n * (rows // 32) * 36, dtype=torch.uint8, device="cuda")
    qs_d, sc_d = dev(qs), dev(sc)
    rc = L.dn_linear_qa(1 if fmt == "q4" else 0, qs_d.data_ptr(), sc_d.data_ptr(), xa.data_ptr(),
                        cols // 32 * 36, ys.data_ptr(), rows, ya.data_ptr(), rows // 32 * 36,
                        rows, cols, n, 1, st)
    torch.cuda.synchronize()
    assert rc == 0 and L.dn_device_status(1) == 0
    assert np.array_equal(xa.cpu().numpy(), qa_pack(wq, wsc, n, cols))
    assert same_bits(ys.cpu().numpy(), want)
    full = rows // 32 * 32  # QA output exists for whole 32-row tiles only
    yq, ysc = oracle.quantize_q8(np.ascontiguousarray(want.reshape(n, rows)[:, :full]).ravel(), n, full)
    assert np.array_equal(ya.cpu().numpy(), qa_pack(yq, ysc, n, full))


def test_qa_chain_of_projections(cuda_lib, oracle):
    """qkv -> o -> gate/up -> down as in the benchmark, against per-call oracle products."""
    L = cuda_lib
    rng = np.random.default_rng(42)
    shapes = [("qkv", 4096, 2048), ("o", 2048, 2048), ("gu", 12288, 2048), ("down", 2048, 6144)]
    mats = {name: weights("q8", rng, r, c) for name, r, c in shapes}
    x0 = orc.activations(rng, 1, 2048)
    st = torch.cuda.current_stream().cuda_stream
    xa = torch.zeros(2048 // 32 * 36, dtype=torch.uint8, device="cuda")
    assert L.dn_quantize_qa(dev(x0).data_ptr(), xa.data_ptr(), 1, 2048, 2048 // 32 * 36, st) == 0
    x_host = x0
    keep = []
    for name, r, c in shapes:
        qs, sc = mats[name]
        want, _, _ = oracle.gemm("q8", qs, sc, x_host, r, c, 1, 1)
        ys = torch.zeros(r, device="cuda")
        ya = torch.zeros(r // 32 * 36, dtype=torch.uint8, device="cuda")
        qd, sd = dev(qs), dev(sc)
        keep += [qd, sd, ys, ya]
        assert L.dn_linear_qa(0, qd.data_ptr(), sd.data_ptr(), xa.data_ptr(), c // 32 * 36,
                              ys.data_ptr(), r, ya.data_ptr(), r // 32 * 36, r, c, 1, 1, st) == 0
        torch.cuda.synchronize()
        assert same_bits(ys.cpu().numpy(), want), name
        nxt = {"qkv": 2048, "o": 2048, "gu": 6144, "down": 2048}[name]
        x_host = want[:nxt].copy()
        xa = ya  # the prefix of the QA output feeds the next product
    assert L.dn_device_status(1) == 0


# ---------------------------------------------------------- tensor-core GEMM

TC_SHAPES = [
    ("q8", 6144, 2048, 512),   # config 4 gate/up shape, Q8
    ("q4", 6144, 2048, 512),   # config 4: gate/up, Q4_0
    ("q4", 2048, 6144, 512),   # config 4: down, Q4_0
    ("q8", 4304, 1152, 256),   # config 5: fc1 (rows not a multiple of the 128-row tile)
    ("q8", 1152, 4320, 100),   # config 5: fc2, K padded to 4320 (135 blocks), ragged tokens
    ("q8", 3456, 1152, 64),    # config 5: qkv, lm_head-sweep-sized M
    ("q4", 70, 96, 40),        # gpu_linear_test shape: a single partial tile
    ("q8", 128, 128, 16),      # the GEMV/GEMM crossover
]


@pytest.mark.parametrize("fmt,rows,cols,n", TC_SHAPES)
def test_tensor_core_gemm_within_tolerance(cuda_lib, oracle, fmt, rows, cols, n):
    rng = np.random.default_rng(rows * 7 + cols + n)
    qs, sc = weights(fmt, rng, rows, cols)
    xs = orc.activations(rng, n, cols)
    _, wq, wsc = oracle.gemm(fmt, qs[: 32 * (cols // 2 if fmt == "q4" else cols)], sc[: 32 * (cols // 32)],
                             xs, 32, cols, n, 1)
    ys, xq, xsc = dev_linear(cuda_lib, fmt, dev(qs), dev(sc), dev(xs), rows, cols, n, path=1)
    assert np.array_equal(xq, wq) and same_bits(xsc, wsc)  # activations: bit-exact
    ref, mag = oracle.reference_f64(fmt, qs, sc, xs, rows, cols, n, 1)
    err = orc.max_rel_err(ys, ref, mag)
    assert err < TOL, f"max relative error {err:.3e}"


# The narrow-tile kernel (n <= 32: 16-token tiles up to 16 tokens, 32-token
# tiles above): ragged rows and token counts, both formats, tiles across more
# than one wave so the persistent CTAs walk several tiles and the rings run on
# across tile boundaries; and K whose block count the kernel's scale boxes
# cannot take (Q8: not a multiple of 4), which falls back to the wide kernel.
NARROW_CASES = [("q8", 33000, 2048, 5), ("q8", 4097, 1024, 9), ("q8", 1000, 512, 16), ("q8", 20000, 1024, 17),
                ("q8", 3000, 2048, 31), ("q8", 700, 544, 12), ("q4", 9000, 2048, 7), ("q4", 4100, 1024, 24)]


@pytest.mark.parametrize("fmt,rows,cols,n", NARROW_CASES)
def test_narrow_tiles_within_tolerance(cuda_lib, oracle, fmt, rows, cols, n):
    rng = np.random.default_rng(rows * 3 + cols + n)
    qs, sc = weights(fmt, rng, rows, cols)
    xs = orc.activations(rng, n, cols)
    ys, _, _ = dev_linear(cuda_lib, fmt, dev(qs), dev(sc), dev(xs), rows, cols, n, path=1)
    assert not np.isnan(ys).any()
    ref, mag = oracle.reference_f64(fmt, qs, sc, xs, rows, cols, n, 1)
    err = orc.max_rel_err(ys, ref, mag)
    assert err < TOL, f"max relative error {err:.3e}"


def test_narrow_crossover_by_rows(cuda_lib):
    """The tensor-core GEMM takes the lm_head from 5 tokens on (its narrow
    tiles stream faster than the n-token GEMV there), other shapes from 16."""
    assert cuda_lib.dn_linear_path(0, None, None, None, None, 151936, 2048, 4, 1) == 0
    assert cuda_lib.dn_linear_path(0, None, None, None, None, 151936, 2048, 5, 1) == 1
    assert cuda_lib.dn_linear_path(0, None, None, None, None, 6144, 2048, 8, 1) == 0
    assert cuda_lib.dn_linear_path(0, None, None, None, None, 6144, 2048, 16, 1) == 1


def test_auto_path_uses_tensor_cores_for_prefill(cuda_lib):
    assert cuda_lib.dn_linear_path(0, None, None, None, None, 6144, 2048, 512, 1) == 1
    assert cuda_lib.dn_linear_path(1, None, None, None, None, 6144, 2048, 1, 1) == 0


# ------------------------------------------------ int32 block dots on tensor cores


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("rows,cols,n", [(300, 32, 80), (128, 32, 16), (257, 128, 200)])
def test_tensor_core_int32_block_dots(cuda_lib, oracle, fmt, rows, cols, n):
    """The tcgen05 path's int32 block dots, bit for bit (lab_native.c:456-466,
    987-1002). With unit weight scales and integer activations in which every
    block holds a +-127, the activation quantize is exact (scale 1, inv 1), so
    each output is the float of its row's block dots: one block dot for
    cols = 32, and for cols = 128 a sum of four that stays below 2^24."""
    rng = np.random.default_rng(rows * 3 + cols + n)
    qs, _ = weights(fmt, rng, rows, cols)
    blocks = cols // 32
    sc = (np.full(rows * blocks, 0x3C00, np.uint16) if fmt == "q4"   # fp16 1.0
          else np.ones(rows * blocks, np.float32))
    xi = rng.integers(-127, 128, size=(n, cols)).astype(np.float32)
    pos = rng.integers(0, 32, size=(n, blocks))
    sign = rng.choice(np.array([-127.0, 127.0], np.float32), size=(n, blocks))
    for b in range(blocks):
        xi[np.arange(n), b * 32 + pos[:, b]] = sign[:, b]
    xs = xi.reshape(-1)
    ys, xq, xsc = dev_linear(cuda_lib, fmt, dev(qs), dev(sc), dev(xs), rows, cols, n, path=1)
    assert (xsc == 1.0).all() and np.array_equal(xq, xi.astype(np.int8).reshape(-1))
    dots = oracle.block_dots(fmt, qs, xq, rows, cols, n).reshape(n, rows, blocks)
    want = dots.astype(np.int64).sum(axis=2)
    assert np.abs(want).max() < 2 ** 24
    assert same_bits(ys, want.astype(np.float32).reshape(-1))


# ------------------------------------------------------- config 5 at full size

VISION = [("qkv", 3456, 1152, 1152), ("o", 1152, 1152, 1152), ("fc1", 4304, 1152, 1152),
          ("fc2", 1152, 4304, 4320)]


@pytest.mark.parametrize("name,rows,cols,padded", VISION)
def test_config5_vision_m1024(cuda_lib, oracle, name, rows, cols, padded):
    """Config 5 as stated: 1024 image tokens; weights bf16 N(0, 0.02) quantized
    to Q8_0 by lab_quantize_q8 (fc2's K zero-padded from 4304 to 4320 in both
    operands); activations N(0, 1). The library's weight quantize equals the
    oracle's bit for bit, so do the quantized activations, and the tensor-core
    outputs are within the reference's bound."""
    L = cuda_lib
    n = 1024
    rng = np.random.default_rng(5000 + rows + cols)
    w = orc.vision_weights_f32(rng, rows, cols, padded)
    qs, sc = oracle.quantize_q8(w, rows, padded)
    gq = np.zeros(rows * padded, np.int8)
    gs = np.zeros(rows * padded // 32, np.float32)
    L.lab_quantize_q8(w.ctypes.data, gq.ctypes.data, gs.ctypes.data, rows, padded)
    assert L.dn_last_error() == 0
    assert np.array_equal(gq, qs) and same_bits(gs, sc)
    xs = orc.pad_cols(orc.activations(rng, n, cols), n, cols, padded)
    assert L.dn_linear_path(0, None, None, None, None, rows, padded, n, 1) == 1
    ys, xq, xsc = dev_linear(L, "q8", dev(qs), dev(sc), dev(xs), rows, padded, n)
    wq, wsc = oracle.quantize_q8(xs, n, padded)
    assert np.array_equal(xq, wq) and same_bits(xsc, wsc)
    ref, mag = oracle.reference_f64("q8", qs, sc, xs, rows, padded, n, 1)
    err = orc.max_rel_err(ys, ref, mag)
    assert err < TOL, f"{name}: max relative error {err:.3e}"


# ------------------------------------------------------- lm_head M sweep, full size

LM_ROWS, LM_COLS, LM_MAX_M = 151936, 2048, 64


@pytest.fixture(scope="module")
def lm_head_q8(oracle):
    """The tied Q8_0 lm_head and 64 tokens, with the oracle's bit-exact outputs
    for the first 8 tokens and the double-precision check for all 64 (a row's
    result does not depend on how many tokens share the call)."""
    rng = np.random.default_rng(151936 * 64)
    qs, sc = orc.q8_weights(rng, LM_ROWS, LM_COLS)
    xs = orc.activations(rng, LM_MAX_M, LM_COLS)
    bits, _, _ = oracle.gemm("q8", qs, sc, xs[: 8 * LM_COLS], LM_ROWS, LM_COLS, 8, 1)
    ref, mag = oracle.reference_f64("q8", qs, sc, xs, LM_ROWS, LM_COLS, LM_MAX_M, 1)
    return dict(qs=dev(qs), sc=dev(sc), xs=xs, bits=bits, ref=ref, mag=mag)


@pytest.mark.parametrize("m", [1, 2, 4, 8, 16, 32, 64])
def test_lm_head_m_sweep(cuda_lib, lm_head_q8, m):
    """Config 5's lm_head M sweep on the whole 151936 x 2048 matrix: the GEMV
    (small M) bit for bit, the tensor-core GEMM (from the crossover on) within
    the bound."""
    h = lm_head_q8
    path = cuda_lib.dn_linear_path(0, None, None, None, None, LM_ROWS, LM_COLS, m, 1)
    ys, _, _ = dev_linear(cuda_lib, "q8", h["qs"], h["sc"], dev(h["xs"][: m * LM_COLS]),
                          LM_ROWS, LM_COLS, m)
    if path == 0:
        assert same_bits(ys, h["bits"][: m * LM_ROWS])
    else:
        assert path == 1
        err = orc.max_rel_err(ys, h["ref"][: m * LM_ROWS], h["mag"][: m * LM_ROWS])
        assert err < TOL, f"M={m}: max relative error {err:.3e}"

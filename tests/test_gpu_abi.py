"""The lab_gpu_* C-ABI and the GpuLinear mirror, after dianoia's
test/gpu_linear_test.dart: the same shapes (rows and token counts that do not
fill the tiles), growing buffers, errors and buffer accounting. The products
use the reference's integer path (inputs quantized to Q8_0 per block), so
they are checked against the reference's own lab_gemm in mode 1: bit for bit
on the decode GEMV, within the 1e-5 row-scale bound on the tensor-core GEMM."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def values(rng, count):
    return (rng.random(count, dtype=np.float64) * 2 - 1).astype(np.float32)


@pytest.fixture(scope="module")
def gpu(cuda_lib):
    from dianoia_b200 import NativeKernels
    from dianoia_b200.gpu import GpuLinear
    NativeKernels.load(None, threads=4)
    g = GpuLinear.start()
    assert g is not None
    yield g
    g.dispose()


def check(oracle, fmt, m, xs, got, n):
    rows, cols = m.rows, m.cols
    qs = np.array(m.qs_bytes)
    sc = np.array(m.scale_bytes).view(np.uint16 if fmt == "q4" else np.float32)
    want, _, _ = oracle.gemm(fmt, qs, sc, xs, rows, cols, n, 1)
    if n < 16:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    else:
        ref, mag = oracle.reference_f64(fmt, qs, sc, xs, rows, cols, n)
        assert orc.max_rel_err(got, ref, mag) <= 1e-5


@pytest.mark.parametrize("fmt,rows,cols,n", [("q4", 64, 64, 1), ("q4", 70, 96, 13),
                                             ("q8", 36, 64, 9), ("q8", 128, 128, 40)])
def test_matches_cpu_kernels(gpu, oracle, fmt, rows, cols, n):
    from dianoia_b200 import NativeQ4Matrix, NativeQ8Matrix
    rng = np.random.default_rng(5 + rows)
    w = values(rng, rows * cols)
    m = (NativeQ4Matrix if fmt == "q4" else NativeQ8Matrix).quantize(w, rows, cols)
    try:
        gpu.upload("m", m)
        xs = values(rng, n * cols)
        got = np.full(n * rows, np.nan, np.float32)
        gpu.apply("m", xs, got, n)
        check(oracle, fmt, m, xs, got, n)
    finally:
        m.free()


def test_grows_buffers_and_keeps_earlier_matrices(gpu, oracle):
    from dianoia_b200 import NativeQ4Matrix
    rng = np.random.default_rng(9)
    small = NativeQ4Matrix.quantize(values(rng, 32 * 32), 32, 32)
    large = NativeQ4Matrix.quantize(values(rng, 64 * 256), 64, 256)
    try:
        gpu.upload("small", small)
        gpu.upload("large", large)
        for name, m, n in [("small", small, 3), ("large", large, 50), ("small", small, 7)]:
            xs = values(rng, n * m.cols)
            got = np.full(n * m.rows, np.nan, np.float32)
            gpu.apply(name, xs, got, n)
            check(oracle, "q4", m, xs, got, n)
    finally:
        small.free()
        large.free()


def test_rejects_unknown_matrices_and_short_lists(gpu):
    from dianoia_b200 import ArgumentError, NativeQ4Matrix
    m = NativeQ4Matrix.quantize(values(np.random.default_rng(1), 32 * 32), 32, 32)
    try:
        gpu.upload("m", m)
        with pytest.raises(ArgumentError):
            gpu.apply("missing", np.zeros(32, np.float32), np.zeros(32, np.float32), 1)
        with pytest.raises(ArgumentError):
            gpu.apply("m", np.zeros(32, np.float32), np.zeros(32, np.float32), 2)
    finally:
        m.free()


def test_frees_its_buffers_once_and_then_refuses_work(gpu):
    from dianoia_b200 import NativeQ8Matrix, StateError
    from dianoia_b200.gpu import GpuLinear, live_buffers
    rng = np.random.default_rng(2)
    live = live_buffers()
    other = GpuLinear.start()
    m = NativeQ8Matrix.quantize(values(rng, 32 * 32), 32, 32)
    try:
        other.upload("m", m)
        other.apply("m", values(rng, 32), np.zeros(32, np.float32), 1)
        assert live_buffers() == live + 3
        other.dispose()
        other.dispose()
        assert live_buffers() == live
        with pytest.raises(StateError):
            other.apply("m", values(rng, 32), np.zeros(32, np.float32), 1)
    finally:
        m.free()


def test_chained_command_buffer_and_replay(cuda_lib, oracle):
    """Two products in one command buffer, the second reading the first's
    output inside the same buffer; committed twice with new host inputs (the
    second commit replays the captured graph); then a product whose ranges
    do not fit its buffers makes the commit fail."""
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    rng = np.random.default_rng(3)
    r1, c1, r2 = 256, 512, 96
    q1, s1 = orc.q8_weights(rng, r1, c1)
    q2, s2 = orc.q8_weights(rng, r2, r1)

    def weights(qs, sc):
        raw = np.concatenate([qs.view(np.uint8), sc.view(np.uint8)])
        h = L.lab_gpu_wrap(raw.ctypes.data, raw.size)
        assert h >= 0
        raw[:] = 0  # wrap copied: the source may change or go
        return h, qs.size

    w1, at1 = weights(q1, s1)
    w2, at2 = weights(q2, s2)
    act = L.lab_gpu_buffer(4 * (c1 + r1 + r2))
    assert act >= 0
    view = np.ctypeslib.as_array((ctypes.c_float * (c1 + r1 + r2)).from_address(L.lab_gpu_contents(act)))
    try:
        for _ in range(2):
            x = orc.activations(rng, 1, c1)
            view[:c1] = x
            view[c1:] = np.nan
            L.lab_gpu_begin()
            L.lab_gpu_enc_matmul_q8(w1, 0, at1, act, 0, act, 4 * c1, r1, c1, 1)
            L.lab_gpu_enc_matmul_q8(w2, 0, at2, act, 4 * c1, act, 4 * (c1 + r1), r2, r1, 1)
            assert L.lab_gpu_commit(1) == 1
            assert L.lab_gpu_last_ms() > 0
            y1, _, _ = oracle.gemm("q8", q1, s1, x, r1, c1, 1, 1)
            y2, _, _ = oracle.gemm("q8", q2, s2, y1, r2, r1, 1, 1)
            assert np.array_equal(view[c1:c1 + r1].view(np.uint32), y1.view(np.uint32))
            assert np.array_equal(view[c1 + r1:].view(np.uint32), y2.view(np.uint32))
        L.lab_gpu_begin()
        # r1 outputs from float c1 + r1 on run past the buffer's c1 + r1 + r2 floats
        L.lab_gpu_enc_matmul_q8(w1, 0, at1, act, 0, act, 4 * (c1 + r1), r1, c1, 1)
        assert L.lab_gpu_commit(1) == 0
        L.lab_gpu_begin()
        L.lab_gpu_enc_matmul_q8(w1, 0, at1, act, 0, act, 4 * c1, r1, c1, 1)
        assert L.lab_gpu_commit(0) == 1 and L.lab_gpu_wait() == 1
    finally:
        for h in (w1, w2, act):
            L.lab_gpu_release(h)
    assert L.lab_gpu_contents(act) is None


def test_batch_encode_equals_single_calls(cuda_lib, oracle):
    """dn_gpu_enc_batch records the same command buffer as the equivalent
    lab_gpu_enc_matmul_* calls: a Q8 product feeding a Q4 product, bit for
    bit against the reference's kernels; a row whose ranges do not fit makes
    the commit fail, as a single call would."""
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    rng = np.random.default_rng(11)
    r1, c1, r2 = 128, 256, 64
    q1, s1 = orc.q8_weights(rng, r1, c1)
    q2, s2 = orc.q4_weights(rng, r2, r1)

    def weights(qs, sc):
        raw = np.concatenate([qs.view(np.uint8), sc.view(np.uint8)])
        h = L.lab_gpu_wrap(raw.ctypes.data, raw.size)
        assert h >= 0
        return h, qs.size

    w1, at1 = weights(q1, s1)
    w2, at2 = weights(q2, s2)
    act = L.lab_gpu_buffer(4 * (c1 + r1 + r2))
    assert act >= 0
    view = np.ctypeslib.as_array((ctypes.c_float * (c1 + r1 + r2)).from_address(L.lab_gpu_contents(act)))
    table = np.array([[0, w1, 0, at1, act, 0, act, 4 * c1, r1, c1, 1],
                      [1, w2, 0, at2, act, 4 * c1, act, 4 * (c1 + r1), r2, r1, 1]], np.int64)
    try:
        for _ in range(2):
            x = orc.activations(rng, 1, c1)
            view[:c1] = x
            view[c1:] = np.nan
            L.lab_gpu_begin()
            L.dn_gpu_enc_batch(table.ctypes.data, 2)
            assert L.lab_gpu_commit(1) == 1
            y1, _, _ = oracle.gemm("q8", q1, s1, x, r1, c1, 1, 1)
            y2, _, _ = oracle.gemm("q4", q2, s2, y1, r2, r1, 1, 1)
            assert np.array_equal(view[c1:c1 + r1].view(np.uint32), y1.view(np.uint32))
            assert np.array_equal(view[c1 + r1:].view(np.uint32), y2.view(np.uint32))
        bad = table.copy()
        bad[1, 7] = 4 * (c1 + r1 + 1)  # r2 outputs from here run past the buffer
        L.lab_gpu_begin()
        L.dn_gpu_enc_batch(bad.ctypes.data, 2)
        assert L.lab_gpu_commit(1) == 0
    finally:
        for h in (w1, w2, act):
            L.lab_gpu_release(h)


def test_links_for_slices_and_shared_host_inputs(cuda_lib, oracle):
    """One token through products that the command buffer links by QA blocks:
    P2 reads a 32-value-aligned slice of P1's output, P3 reads the same host
    input as P1 (quantized once for both), P4 reads a slice that is not
    32-aligned (no link: it quantizes its f32 input itself). All bit for bit
    against the reference's kernels on the same f32 values."""
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    rng = np.random.default_rng(17)
    c1, r1, r3 = 256, 192, 96
    q1, s1 = orc.q8_weights(rng, r1, c1)
    q2, s2 = orc.q8_weights(rng, 64, 96)      # reads P1's outputs 32 .. 127
    q3, s3 = orc.q4_weights(rng, r3, c1)      # reads the host input, as P1
    q4, s4 = orc.q8_weights(rng, 32, 64)      # reads P1's outputs 40 .. 103

    def weights(qs, sc):
        raw = np.concatenate([qs.view(np.uint8), sc.view(np.uint8)])
        h = L.lab_gpu_wrap(raw.ctypes.data, raw.size)
        assert h >= 0
        return h, qs.size

    hs = [weights(q, s) for q, s in [(q1, s1), (q2, s2), (q3, s3), (q4, s4)]]
    floats = c1 + r1 + 64 + r3 + 32
    act = L.lab_gpu_buffer(4 * floats)
    assert act >= 0
    view = np.ctypeslib.as_array((ctypes.c_float * floats).from_address(L.lab_gpu_contents(act)))
    y1_at, y2_at, y3_at, y4_at = c1, c1 + r1, c1 + r1 + 64, c1 + r1 + 64 + r3
    table = np.array([
        [0, hs[0][0], 0, hs[0][1], act, 0, act, 4 * y1_at, r1, c1, 1],
        [0, hs[1][0], 0, hs[1][1], act, 4 * (y1_at + 32), act, 4 * y2_at, 64, 96, 1],
        [1, hs[2][0], 0, hs[2][1], act, 0, act, 4 * y3_at, r3, c1, 1],
        [0, hs[3][0], 0, hs[3][1], act, 4 * (y1_at + 40), act, 4 * y4_at, 32, 64, 1]], np.int64)
    try:
        for _ in range(2):
            x = orc.activations(rng, 1, c1)
            view[:c1] = x
            view[c1:] = np.nan
            L.lab_gpu_begin()
            L.dn_gpu_enc_batch(table.ctypes.data, len(table))
            assert L.lab_gpu_commit(1) == 1
            y1, _, _ = oracle.gemm("q8", q1, s1, x, r1, c1, 1, 1)
            y2, _, _ = oracle.gemm("q8", q2, s2, y1[32:128], 64, 96, 1, 1)
            y3, _, _ = oracle.gemm("q4", q3, s3, x, r3, c1, 1, 1)
            y4, _, _ = oracle.gemm("q8", q4, s4, y1[40:104], 32, 64, 1, 1)
            for got, want in [(view[y1_at:y1_at + r1], y1), (view[y2_at:y2_at + 64], y2),
                              (view[y3_at:y3_at + r3], y3), (view[y4_at:y4_at + 32], y4)]:
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    finally:
        for h, _ in hs:
            L.lab_gpu_release(h)
        L.lab_gpu_release(act)


def test_device_queries_and_knobs(cuda_lib):
    """The layer's device queries and tuning knobs (lab_vulkan.c:507-718):
    name, sizes, no thermal state; the Vulkan-only modes report unavailable."""
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    name = ctypes.create_string_buffer(256)
    L.lab_gpu_device_name(name, 256)
    assert b"B200" in name.value
    assert L.lab_gpu_max_buffer_length() > 100 * 2**30
    assert L.lab_gpu_recommended_working_set() == L.lab_gpu_max_buffer_length()
    assert L.lab_gpu_max_shared_memory() == 16384 * 4 + 128  # the attention's keys, as the reference reports
    assert L.lab_gpu_thermal_state() == -1
    assert L.lab_gpu_physical_memory() > 2**30
    assert L.lab_gpu_set_q8_group(64) == 0 and L.lab_gpu_set_q8_vector(1) == 0
    assert L.lab_gpu_register_q8_head(0, 0, 128, 128, 0) == 0


def test_generic_decode_rows_and_dispatch_profile(cuda_lib, oracle):
    """lab_gpu_set_decode_rows(0) runs the same products on the generic
    kernel (same bits); with profiling on, lab_gpu_profile reports each kind's
    launches and time per commit in the reference's kind order, and starts
    over after each call."""
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    rng = np.random.default_rng(47)
    r1, c1 = 256, 512
    q1, s1 = orc.q8_weights(rng, r1, c1)
    q2, s2 = orc.q4_weights(rng, 96, r1)
    raw = [np.concatenate([q.view(np.uint8), s.view(np.uint8)]) for q, s in [(q1, s1), (q2, s2)]]
    w = [L.lab_gpu_wrap(r.ctypes.data, r.size) for r in raw]
    act = L.lab_gpu_buffer(4 * (c1 + r1 + 96))
    view = np.ctypeslib.as_array((ctypes.c_float * (c1 + r1 + 96)).from_address(L.lab_gpu_contents(act)))
    kinds = 18
    ms = np.zeros(kinds, np.float64)
    counts = np.zeros(kinds, np.int64)
    try:
        L.lab_gpu_set_profiling(1)
        assert L.lab_gpu_profile(ms.ctypes.data, counts.ctypes.data, kinds) == kinds  # start over
        results = []
        for rows_knob in (-1, 0, -1):
            L.lab_gpu_set_decode_rows(rows_knob)
            x = orc.activations(np.random.default_rng(5), 1, c1)
            view[:c1] = x
            L.lab_gpu_begin()
            L.lab_gpu_enc_matmul_q8(w[0], 0, q1.size, act, 0, act, 4 * c1, r1, c1, 1)
            L.lab_gpu_enc_matmul_q4(w[1], 0, q2.size, act, 4 * c1, act, 4 * (c1 + r1), 96, r1, 1)
            assert L.lab_gpu_commit(1) == 1
            results.append(view[c1:].copy())
        y1, _, _ = oracle.gemm("q8", q1, s1, x, r1, c1, 1, 1)
        y2, _, _ = oracle.gemm("q4", q2, s2, y1, 96, r1, 1, 1)
        for got in results:
            assert np.array_equal(got.view(np.uint32), np.concatenate([y1, y2]).view(np.uint32))
        assert L.lab_gpu_profile(ms.ctypes.data, counts.ctypes.data, kinds) == kinds
        # 3 commits x one Q8 and one Q4 product; the first and last quantize x0 once
        assert counts[13] == 3 and counts[14] == 3 and counts[10] == 2
        assert counts.sum() == 8 and (ms[counts > 0] > 0).all() and (ms[counts == 0] == 0).all()
        L.lab_gpu_profile(ms.ctypes.data, counts.ctypes.data, kinds)
        assert counts.sum() == 0
    finally:
        L.lab_gpu_set_profiling(0)
        L.lab_gpu_set_decode_rows(-1)
        for h in w + [act]:
            L.lab_gpu_release(h)

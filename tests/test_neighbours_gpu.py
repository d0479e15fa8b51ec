"""RMSNorm and SwiGLU on the device, and fused with the quantized products
of the decode path, against dianoia's CPU arithmetic (lib/src/ops.dart:12-31,
lib/src/shard.dart:456-460, restated in oracle/lab_oracle.c).

* dn_rms_norm / dn_swiglu: f32 outputs bit for bit, and their QA outputs
  (the fused quantize) bit for bit against lab_quantize_q8 of those outputs;
  ragged sizes, accumulate, special values.
* The GPU layer (lab_gpu_enc_rms_norm / lab_gpu_enc_swiglu between
  lab_gpu_enc_matmul_* products): one feed-forward block as dianoia's
  GpuForward encodes it (gpu.dart:1180-1188: norm, gate, up, SwiGLU, down,
  and the residual: a post-norm added into it, or a plain add), where the
  norm runs in the prologue of the gate product, gate and up run as one dual
  GEMV with the SwiGLU in its epilogue for one token (for more tokens, up
  takes QA blocks from gate and runs the SwiGLU in its epilogue) and the
  plain add runs in the down product's epilogue.
  Every intermediate the host reads back, and the final product, bit for
  bit against the CPU path on the same inputs; also with the gate and up
  products swapped, with the SwiGLU kept apart from them, and with every
  fusion off (dn_gpu_set_fusion(0)).
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def qa_blocks(oracle, vals, rows, cols):
    qs, sc = oracle.quantize_q8(vals, rows, cols)
    blocks = rows * cols // 32
    out = np.zeros((blocks, 36), np.uint8)
    out[:, :32] = qs.view(np.uint8).reshape(blocks, 32)
    out[:, 32:] = sc.view(np.uint8).reshape(blocks, 4)
    return out


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("rows,cols,acc", [(1, 2048, 0), (4, 2048, 1), (33, 64, 0), (3, 1000, 0),
                                           (2, 4096, 1), (1, 7, 1)])
def test_rms_norm_matches_cpu_path(cuda_lib, oracle, rows, cols, acc):
    L = cuda_lib
    rng = np.random.default_rng(rows * 31 + cols + acc)
    x = (rng.standard_normal(rows * cols) * 2).astype(np.float32)
    x[:3] = [0.0, -0.0, 1e-30]
    w = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    prev = rng.standard_normal(rows * cols).astype(np.float32)
    eps = 1e-6
    want = oracle.rms_norm(x, w, rows, cols, eps, out=prev if acc else None)
    xd, wd = dev(x), dev(w)
    out = dev(prev if acc else np.full(rows * cols, np.nan, np.float32))
    with_qa = cols % 32 == 0
    stride = cols // 32 * 36 + 8  # a row stride wider than the row's blocks
    qa = torch.full((max(rows * stride, 1),), 0xEE, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = L.dn_rms_norm(xd.data_ptr(), wd.data_ptr(), out.data_ptr(), qa.data_ptr() if with_qa else None,
                       stride, rows, cols, eps, acc, 1, st)
    torch.cuda.synchronize()
    assert rc == 0 and L.dn_device_status(1) == 0
    got = out.cpu().numpy()
    assert np.array_equal(bits(got), bits(want))
    if with_qa:
        q = qa.cpu().numpy().reshape(rows, stride)
        assert np.array_equal(q[:, :cols // 32 * 36].reshape(-1, 36), qa_blocks(oracle, want, rows, cols))
        assert (q[:, cols // 32 * 36:] == 0xEE).all()


@pytest.mark.parametrize("count", [6144, 4 * 6144, 33, 1000])
def test_swiglu_matches_cpu_path(cuda_lib, oracle, count):
    L = cuda_lib
    rng = np.random.default_rng(count)
    g = (rng.standard_normal(count) * 4).astype(np.float32)
    g[:6] = [0.0, -0.0, 90.0, -90.0, 1e-30, -800.0][: min(6, count)]
    u = rng.standard_normal(count).astype(np.float32)
    want = oracle.swiglu(g, u)
    gd, ud = dev(g), dev(u)
    with_qa = count % 32 == 0
    qa = torch.full((max(count // 32 * 36, 1),), 0xEE, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = L.dn_swiglu(gd.data_ptr(), ud.data_ptr(), qa.data_ptr() if with_qa else None, count, 0, st)
    torch.cuda.synchronize()
    assert rc == 0 and L.dn_device_status(1) == 0
    assert np.array_equal(bits(gd.cpu().numpy()), bits(want))
    if with_qa:
        assert np.array_equal(qa.cpu().numpy().reshape(-1, 36), qa_blocks(oracle, want, 1, count))


def test_device_entry_points_reject_bad_arguments(cuda_lib):
    L = cuda_lib
    buf = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    st = torch.cuda.current_stream().cuda_stream
    assert L.dn_rms_norm(p + 2, p, p, None, 0, 1, 32, 1e-6, 0, 0, st) == -1      # x not 4-byte aligned
    assert L.dn_rms_norm(p, p, p, p, 36, 1, 40, 1e-6, 0, 0, st) == -1           # QA needs cols % 32 == 0
    assert L.dn_rms_norm(p, p, p, p, 32, 1, 64, 1e-6, 0, 0, st) == -1           # QA row stride too short
    assert L.dn_rms_norm(p, p, p, None, 0, -1, 64, 1e-6, 0, 0, st) == -1
    assert L.dn_swiglu(p, p + 1, None, 8, 0, st) == -1                           # u not aligned
    assert L.dn_swiglu(p, p, p, 40, 0, st) == -1                                 # QA needs count % 32 == 0
    assert L.dn_swiglu(None, None, None, 0, 0, st) == 0                          # nothing to do


# ------------------------------------------------------------------ GPU layer

class Layer:
    """Buffers and weights of one feed-forward block in the GPU layer."""

    def __init__(self, L, rng, h, f, n, out_rows, fmt):
        self.L, self.h, self.f, self.n, self.fmt = L, h, f, n, fmt
        gen = orc.q4_weights if fmt == "q4" else orc.q8_weights
        self.wg, self.wu = gen(rng, f, h), gen(rng, f, h)
        self.wd, self.wo = gen(rng, h, f), gen(rng, out_rows, h)
        self.out_rows = out_rows
        self.norm1 = (1 + 0.1 * rng.standard_normal(h)).astype(np.float32)
        self.norm2 = (1 + 0.1 * rng.standard_normal(h)).astype(np.float32)
        self.handles = []
        self.mats = {k: self._wrap_matrix(getattr(self, k)) for k in ("wg", "wu", "wd", "wo")}
        small = np.concatenate([self.norm1, self.norm2])
        self.small = self._wrap(small.view(np.uint8))
        # activations: x (residual) [n, h], a [n, h], g, u [n, f], m [n, h], y [n, out_rows]
        self.layout = {}
        at = 0
        for name, size in [("x", n * h), ("a", n * h), ("g", n * f), ("u", n * f), ("m", n * h),
                           ("y", n * out_rows)]:
            self.layout[name] = (at, size)
            at += size
        self.floats = at
        self.acts = {}
        for name in ("x", "a", "g", "u", "m", "y"):
            hd = L.lab_gpu_buffer(4 * self.layout[name][1])
            assert hd >= 0
            self.handles.append(hd)
            self.acts[name] = hd

    def _wrap(self, raw):
        h = self.L.lab_gpu_wrap(raw.ctypes.data, raw.size)
        assert h >= 0
        self.handles.append(h)
        return h

    def _wrap_matrix(self, m):
        qs, sc = m
        return self._wrap(np.concatenate([qs.view(np.uint8), sc.view(np.uint8)])), qs.size

    def view(self, name):
        size = self.layout[name][1]
        addr = self.L.lab_gpu_contents(self.acts[name])
        return np.ctypeslib.as_array((ctypes.c_float * size).from_address(addr))

    def rows(self, order="gate_up", apart=False, residual="norm", eps=1e-6):
        """The command buffer as dn_gpu_enc_batch rows."""
        q = 1 if self.fmt == "q4" else 0
        A, h, f, n = self.acts, self.h, self.f, self.n
        eps_bits = int(np.array([eps], np.float64).view(np.int64)[0])

        def mm(key, x, y, rows, cols):
            w, at = self.mats[key]
            return [q, w, 0, at, A[x], 0, A[y], 0, rows, cols, n]

        gate, up = mm("wg", "a", "g", f, h), mm("wu", "a", "u", f, h)
        t = [[2, A["x"], 0, self.small, 0, A["a"], 0, n, h, eps_bits, 0]]
        t += [gate, up] if order == "gate_up" else [up, gate]
        if apart:  # something between the pair and the SwiGLU: no epilogue fusion
            t.append(mm("wo", "a", "y", self.out_rows, h))
        t.append([3, A["g"], A["u"], n * f, 0, 0, 0, 0, 0, 0, 0])
        t.append(mm("wd", "g", "m", h, f))
        if residual == "norm":  # a sandwich post-norm added into the residual stream
            t.append([2, A["m"], 0, self.small, 4 * h, A["x"], 0, n, h, eps_bits, 1])
        else:  # a plain residual add (runs in the down product's epilogue)
            t.append([4, A["m"], 0, A["x"], 0, n * h, 0, 0, 0, 0, 0])
        t.append(mm("wo", "x", "y", self.out_rows, h))
        return np.array(t, np.int64)

    def expected(self, oracle, x, residual="norm", eps=1e-6):
        fmt, h, f, n = self.fmt, self.h, self.f, self.n
        a = oracle.rms_norm(x, self.norm1, n, h, eps)
        g, _, _ = oracle.gemm(fmt, *self.wg, a, f, h, n, 1)
        u, _, _ = oracle.gemm(fmt, *self.wu, a, f, h, n, 1)
        hh = oracle.swiglu(g, u)
        m, _, _ = oracle.gemm(fmt, *self.wd, hh, h, f, n, 1)
        if residual == "norm":
            x2 = oracle.rms_norm(m, self.norm2, n, h, eps, out=x)
        else:
            x2 = (x + m).astype(np.float32)  # one f32 add per value
        y, _, _ = oracle.gemm(fmt, *self.wo, x2, self.out_rows, h, n, 1)
        return {"a": a, "g": hh, "u": u, "m": m, "x": x2, "y": y}

    def release(self):
        for hd in self.handles:
            self.L.lab_gpu_release(hd)


@pytest.mark.parametrize("fmt,h,f,n,order,apart,residual", [
    ("q8", 256, 512, 1, "gate_up", False, "norm"),
    ("q4", 256, 512, 1, "up_gate", False, "add"),
    ("q8", 256, 512, 3, "gate_up", False, "add"),
    ("q4", 256, 512, 5, "up_gate", False, "norm"),
    ("q8", 256, 512, 1, "gate_up", True, "add"),
    ("q4", 2048, 6144, 1, "gate_up", False, "add"),
    ("q8", 2048, 6144, 1, "up_gate", False, "norm"),
])
def test_feed_forward_block_matches_cpu_path(cuda_lib, oracle, fmt, h, f, n, order, apart, residual):
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    rng = np.random.default_rng(h + f + n + (order == "up_gate") + 2 * apart)
    layer = Layer(L, rng, h, f, n, 96, fmt)
    try:
        table = layer.rows(order, apart, residual)
        # Steps 0 and 1 run fused (step 1 replays the captured graph); step 2
        # runs every op alone on f32 inputs (dn_gpu_set_fusion(0)).
        for step in range(3):
            L.dn_gpu_set_fusion(0 if step == 2 else 1)
            x = orc.activations(rng, n, h)
            layer.view("x")[:] = x
            for name in ("a", "g", "u", "m", "y"):
                layer.view(name)[:] = np.nan
            L.lab_gpu_begin()
            if step != 1:
                L.dn_gpu_enc_batch(table.ctypes.data, len(table))
            else:  # the same command buffer through the reference's single calls
                for r in table:
                    r = [int(v) for v in r]
                    if r[0] in (0, 1):
                        (L.lab_gpu_enc_matmul_q4 if r[0] == 1 else L.lab_gpu_enc_matmul_q8)(*r[1:])
                    elif r[0] == 2:
                        eps = float(np.array([r[9]], np.int64).view(np.float64)[0])
                        L.lab_gpu_enc_rms_norm(*r[1:9], eps, r[10])
                    elif r[0] == 3:
                        L.lab_gpu_enc_swiglu(*r[1:4])
                    else:
                        L.lab_gpu_enc_add(*r[1:6])
            assert L.lab_gpu_commit(1) == 1
            want = layer.expected(oracle, x, residual)
            for name in ("a", "g", "u", "m", "x", "y"):
                got = layer.view(name)
                assert np.array_equal(bits(got), bits(want[name])), f"{name} differs at step {step}"
    finally:
        L.dn_gpu_set_fusion(1)
        layer.release()


def test_bad_neighbour_arguments_fail_the_commit(cuda_lib):
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    a = L.lab_gpu_buffer(4 * 256)
    w = L.lab_gpu_buffer(4 * 64)
    try:
        for record in (
            lambda: L.lab_gpu_enc_rms_norm(a, 2, w, 0, a, 0, 1, 64, 1e-6, 0),      # unaligned offset
            lambda: L.lab_gpu_enc_rms_norm(a, 0, w, 4, a, 0, 1, 64, 1e-6, 0),      # weights run past w
            lambda: L.lab_gpu_enc_rms_norm(a, 0, w, 0, a, 0, 5, 64, 1e-6, 0),      # rows run past a
            lambda: L.lab_gpu_enc_swiglu(a, w, 65),                                # u is 64 floats
            lambda: L.lab_gpu_enc_swiglu(a, 12345, 8),                             # no such buffer
            lambda: L.lab_gpu_enc_add(a, 0, w, 4, 64),                             # dst runs past w
            lambda: L.lab_gpu_enc_add(a, 6, w, 0, 8),                              # unaligned offset
        ):
            L.lab_gpu_begin()
            record()
            assert L.lab_gpu_commit(1) == 0
        L.lab_gpu_begin()
        L.lab_gpu_enc_rms_norm(a, 0, w, 0, a, 0, 4, 64, 1e-6, 0)
        L.lab_gpu_enc_swiglu(a, w, 64)
        L.lab_gpu_enc_add(w, 0, a, 4, 64)
        assert L.lab_gpu_commit(1) == 1
    finally:
        L.lab_gpu_release(a)
        L.lab_gpu_release(w)


def test_norm_read_in_part_keeps_its_own_kernel(cuda_lib, oracle):
    """A norm whose output one product reads whole and another only in part
    (a 32-aligned slice) is not folded into the products' prologues: it runs
    as its own kernel and hands QA blocks to both. A second norm read whole by
    one product is folded into it. All bit for bit against the CPU path, fused
    and unfused."""
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    rng = np.random.default_rng(23)
    h, r1, r2 = 256, 96, 64
    q1, s1 = orc.q8_weights(rng, r1, h)
    q2, s2 = orc.q4_weights(rng, r2, 128)      # reads values 64 .. 191 of the norm's output
    q3, s3 = orc.q8_weights(rng, r1, h)
    nw = (1 + 0.1 * rng.standard_normal(2 * h)).astype(np.float32)

    def wrap(raw):
        hd = L.lab_gpu_wrap(raw.ctypes.data, raw.size)
        assert hd >= 0
        return hd

    hs = [wrap(np.concatenate([q.view(np.uint8), s.view(np.uint8)])) for q, s in [(q1, s1), (q2, s2), (q3, s3)]]
    small = wrap(nw.view(np.uint8))
    floats = 2 * h + r1 + r2 + h + r1
    act = L.lab_gpu_buffer(4 * floats)
    assert act >= 0
    view = np.ctypeslib.as_array((ctypes.c_float * floats).from_address(L.lab_gpu_contents(act)))
    a_at, y1_at, y2_at, b_at, y3_at = h, 2 * h, 2 * h + r1, 2 * h + r1 + r2, 3 * h + r1 + r2
    eps = 1e-5
    try:
        for fuse in (1, 0):
            L.dn_gpu_set_fusion(fuse)
            x = orc.activations(rng, 1, h)
            view[:h] = x
            view[h:] = np.nan
            L.lab_gpu_begin()
            L.lab_gpu_enc_rms_norm(act, 0, small, 0, act, 4 * a_at, 1, h, eps, 0)
            L.lab_gpu_enc_matmul_q8(hs[0], 0, q1.size, act, 4 * a_at, act, 4 * y1_at, r1, h, 1)
            L.lab_gpu_enc_matmul_q4(hs[1], 0, q2.size, act, 4 * (a_at + 64), act, 4 * y2_at, r2, 128, 1)
            L.lab_gpu_enc_rms_norm(act, 0, small, 4 * h, act, 4 * b_at, 1, h, eps, 0)
            L.lab_gpu_enc_matmul_q8(hs[2], 0, q3.size, act, 4 * b_at, act, 4 * y3_at, r1, h, 1)
            assert L.lab_gpu_commit(1) == 1
            a = oracle.rms_norm(x, nw[:h], 1, h, eps)
            b = oracle.rms_norm(x, nw[h:], 1, h, eps)
            y1, _, _ = oracle.gemm("q8", q1, s1, a, r1, h, 1, 1)
            y2, _, _ = oracle.gemm("q4", q2, s2, a[64:192], r2, 128, 1, 1)
            y3, _, _ = oracle.gemm("q8", q3, s3, b, r1, h, 1, 1)
            for at, want in [(a_at, a), (y1_at, y1), (y2_at, y2), (b_at, b), (y3_at, y3)]:
                assert np.array_equal(bits(view[at:at + want.size]), bits(want)), (fuse, at)
    finally:
        L.dn_gpu_set_fusion(1)
        for hd in hs + [small, act]:
            L.lab_gpu_release(hd)


def test_prefill_block_with_neighbours_on_the_tensor_core_path(cuda_lib, oracle):
    """n = 20 tokens: the products take the tensor-core GEMM, so nothing is
    fused and the norm, SwiGLU and add run as their own kernels. The norm
    output bit for bit; each product within the reference's 1e-5 row-scale
    bound of a double-precision sum on the inputs the GPU gave it; the
    residual add exact; fused and unfused plans identical."""
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    h, f, n = 256, 512, 20
    rng = np.random.default_rng(41)
    layer = Layer(L, rng, h, f, n, 96, "q8")
    try:
        table = layer.rows("gate_up", False, "add")
        outs = []
        x = orc.activations(rng, n, h)
        for fuse in (1, 0):
            L.dn_gpu_set_fusion(fuse)
            layer.view("x")[:] = x
            L.lab_gpu_begin()
            L.dn_gpu_enc_batch(table.ctypes.data, len(table))
            assert L.lab_gpu_commit(1) == 1
            outs.append({k: layer.view(k).copy() for k in ("a", "g", "u", "m", "x", "y")})
        for k in outs[0]:
            assert np.array_equal(bits(outs[0][k]), bits(outs[1][k])), k
        got = outs[0]
        a = oracle.rms_norm(x, layer.norm1, n, h, 1e-6)
        assert np.array_equal(bits(got["a"]), bits(a))
        ref, mag = oracle.reference_f64("q8", *layer.wu, got["a"], f, h, n)
        assert orc.max_rel_err(got["u"], ref, mag) <= 1e-5
        ref, mag = oracle.reference_f64("q8", *layer.wd, got["g"], h, f, n)
        assert orc.max_rel_err(got["m"], ref, mag) <= 1e-5
        assert np.array_equal(bits(got["x"]), bits((x + got["m"]).astype(np.float32)))
        ref, mag = oracle.reference_f64("q8", *layer.wo, got["x"], 96, h, n)
        assert orc.max_rel_err(got["y"], ref, mag) <= 1e-5
    finally:
        L.dn_gpu_set_fusion(1)
        layer.release()


@pytest.mark.parametrize("fmt", ["q8", "q4"])
def test_grouped_products_of_one_input(cuda_lib, oracle, fmt):
    """GpuForward's q, k and v (gpu.dart:1151-1160), and a fourth product,
    from one RMSNorm: consecutive one-token products of the same input run as
    one grouped launch (the norm in its prologue), each into its own buffer
    or cache row, heights that leave a partial last tile included; then a
    product reads one of their outputs. Bit for bit against the CPU path,
    with the fusions on and off."""
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    rng = np.random.default_rng(33 + (fmt == "q4"))
    h = 256
    shapes = [96, 64, 64, 40]         # q, k, v, a gate with a partial tile
    gen = orc.q4_weights if fmt == "q4" else orc.q8_weights
    mats = [gen(rng, r, h) for r in shapes]
    wo = gen(rng, 32, 96)             # reads q's outputs
    nw = (1 + 0.1 * rng.standard_normal(h)).astype(np.float32)
    hs = []

    def wrap(raw):
        hd = L.lab_gpu_wrap(raw.ctypes.data, raw.size)
        assert hd >= 0
        hs.append(hd)
        return hd

    def buf(floats):
        hd = L.lab_gpu_buffer(4 * floats)
        assert hd >= 0
        hs.append(hd)
        return hd

    def view(hd, floats):
        return np.ctypeslib.as_array((ctypes.c_float * floats).from_address(L.lab_gpu_contents(hd)))

    try:
        wh = [wrap(np.concatenate([q.view(np.uint8), s.view(np.uint8)])) for q, s in mats]
        who = wrap(np.concatenate([wo[0].view(np.uint8), wo[1].view(np.uint8)]))
        small = wrap(nw.view(np.uint8))
        x, a, q, cache, g, o = buf(h), buf(h), buf(96), buf(4 * 64 * 2), buf(40), buf(32)
        ops = [(wh[0], q, 0), (wh[1], cache, 4 * 64 * 2), (wh[2], cache, 4 * 64 * 5), (wh[3], g, 0)]
        xs = orc.activations(rng, 1, h)
        results = []
        for fuse in (1, 0):
            L.dn_gpu_set_fusion(fuse)
            view(x, h)[:] = xs
            for hd, n in ((a, h), (q, 96), (cache, 512), (g, 40), (o, 32)):
                view(hd, n)[:] = np.nan
            L.lab_gpu_begin()
            L.lab_gpu_enc_rms_norm(x, 0, small, 0, a, 0, 1, h, 1e-6, 0)
            enc = L.lab_gpu_enc_matmul_q4 if fmt == "q4" else L.lab_gpu_enc_matmul_q8
            for (w, y, y_off), (qs, _), rows in zip(ops, mats, shapes):
                enc(w, 0, qs.size, a, 0, y, y_off, rows, h, 1)
            enc(who, 0, wo[0].size, q, 0, o, 0, 32, 96, 1)
            assert L.lab_gpu_commit(1) == 1
            results.append([view(hd, n).copy() for hd, n in ((a, h), (q, 96), (cache, 512), (g, 40), (o, 32))])
        an = oracle.rms_norm(xs, nw, 1, h, 1e-6)
        ys = [oracle.gemm(fmt, qs, sc, an, rows, h, 1, 1)[0] for (qs, sc), rows in zip(mats, shapes)]
        yo, _, _ = oracle.gemm(fmt, wo[0], wo[1], ys[0], 32, 96, 1, 1)
        for got in results:
            assert np.array_equal(bits(got[0]), bits(an))
            assert np.array_equal(bits(got[1]), bits(ys[0]))
            assert np.array_equal(bits(got[2][128:192]), bits(ys[1]))
            assert np.array_equal(bits(got[2][320:384]), bits(ys[2]))
            assert np.isnan(got[2][:128]).all() and np.isnan(got[2][192:320]).all()
            assert np.array_equal(bits(got[3]), bits(ys[3]))
            assert np.array_equal(bits(got[4]), bits(yo))
    finally:
        L.dn_gpu_set_fusion(1)
        for hd in hs:
            L.lab_gpu_release(hd)

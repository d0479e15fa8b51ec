"""The decode stack (dn_stack_*): a token's one-token Q8_0 products run by one
persistent kernel, every product's rows split over all SMs. Op for op the
outputs must equal lab_gemm_q8 (mode 1, n = 1) on the f32 output the op
reads - the reference's bits - on every run, replayed from a CUDA graph too,
at small shapes and at config 3's own (lab_native.c:553-579)."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

INPUT_OF = {"qkv": None, "o": "qkv", "gu": "o", "down": "gu", "head": "down"}


def make_stack(rng, layers, hidden, inter, head, q_rows=None):
    """qkv -> o -> gate/up -> down per layer, then a head; every qkv reads x0
    (as bench.py's stack does), o reads the first `hidden` qkv rows and down
    the first `inter` gate/up rows."""
    shapes = []
    for _ in range(layers):
        shapes += [("qkv", q_rows or 2 * hidden, hidden), ("o", hidden, hidden), ("gu", 2 * inter, hidden),
                   ("down", hidden, inter)]
    shapes.append(("head", head, hidden))
    x0 = orc.activations(rng, 1, hidden)
    mats = [(name, r, c, *orc.q8_weights(rng, r, c)) for name, r, c in shapes]
    return x0, mats


def oracle_outputs(oracle, x0, mats):
    ref, outs = [], {}
    for name, r, c, qs, sc in mats:
        src = INPUT_OF[name]
        x = x0 if src is None else outs[src][:c]
        y, _, _ = oracle.gemm("q8", qs, sc, x, r, c, 1, 1)
        outs[name] = y
        ref.append(y)
    return ref


class Stack:
    """Device buffers and the dn_stack handle of make_stack's ops."""

    def __init__(self, L, x0, mats):
        from dianoia_b200 import _lib
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        self.L = L
        self.x0 = dev(x0)
        self.keep, self.ys = [], []
        ops, last = [], {}
        for i, (name, r, c, qs, sc) in enumerate(mats):
            q, s = dev(qs), dev(sc)
            y = torch.full((r,), float("nan"), device="cuda")
            self.keep += [q, s]
            src = INPUT_OF[name]
            if src is not None:
                x, dep = last[src][0], last[src][1]
            else:
                # Later layers' qkv read x0 after the previous layer's down (an
                # ordering edge, as the norm between them would impose).
                x, dep = self.x0, (last["down"][1] if "down" in last else -1)
            ops.append(_lib.StackOp(q.data_ptr(), s.data_ptr(), x.data_ptr(), y.data_ptr(), r, c, dep))
            self.ys.append(y)
            last[name] = (y, i)
        arr = (_lib.StackOp * len(ops))(*ops)
        self.handle = ctypes.c_void_p()
        rc = L.dn_stack_create(_lib.DN_Q8, arr, len(ops), ctypes.byref(self.handle))
        assert rc == 0, rc

    def run(self, stream):
        return self.L.dn_stack_run(self.handle, 1, stream)

    def close(self):
        self.L.dn_stack_destroy(self.handle)


def check(stack, mats, ref, tag):
    for (name, *_), y, want in zip(mats, stack.ys, ref):
        got = y.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (tag, name)


@pytest.mark.parametrize("hidden,inter,head,layers", [(512, 1536, 4096, 2), (1024, 3072, 6000, 1)])
def test_stack_matches_reference_small(cuda_lib, oracle, hidden, inter, head, layers):
    L = cuda_lib
    rng = np.random.default_rng(hidden + layers)
    x0, mats = make_stack(rng, layers, hidden, inter, head)
    ref = oracle_outputs(oracle, x0, mats)
    st = Stack(L, x0, mats)
    stream = torch.cuda.current_stream().cuda_stream
    try:
        for run in range(3):
            for y in st.ys:
                y.fill_(float("nan"))
            assert st.run(stream) == 0
            torch.cuda.synchronize()
            assert L.dn_device_status(1) == 0
            check(st, mats, ref, f"run {run}")
        # Replayed from a CUDA graph: the counters carry over from run to run.
        s2 = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s2):
            with torch.cuda.graph(g, stream=s2):
                assert st.run(torch.cuda.current_stream().cuda_stream) == 0
        for rep in range(3):
            for y in st.ys:
                y.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            assert L.dn_device_status(1) == 0
            check(st, mats, ref, f"graph {rep}")
        del g
    finally:
        st.close()


def test_stack_config3_shapes(cuda_lib, oracle):
    """One Qwen3-1.7B-shaped layer (qkv 4096x2048, o 2048x2048, gate/up
    12288x2048, down 2048x6144) and the 151936-row lm_head: 14-, 28- and
    32-row tiles, 1024- and 512-byte stages, 33 tiles per SM."""
    L = cuda_lib
    rng = np.random.default_rng(11)
    x0, mats = make_stack(rng, 1, 2048, 6144, 151936, q_rows=4096)
    ref = oracle_outputs(oracle, x0, mats)
    st = Stack(L, x0, mats)
    stream = torch.cuda.current_stream().cuda_stream
    try:
        for run in range(2):
            for y in st.ys:
                y.fill_(float("nan"))
            assert st.run(stream) == 0
            torch.cuda.synchronize()
            assert L.dn_device_status(1) == 0
            check(st, mats, ref, f"run {run}")
    finally:
        st.close()


def test_stack_special_inputs(cuda_lib, oracle):
    """Inputs with zero blocks, ties, huge and denormal values quantize as
    lab_quantize_q8 does inside the kernel."""
    L = cuda_lib
    rng = np.random.default_rng(5)
    x0, mats = make_stack(rng, 1, 512, 512, 1000)
    x0[:32] = 0.0
    x0[32:64] = np.float32(1e-40)
    x0[64:96] = np.linspace(-3.5, 3.5, 32, dtype=np.float32)
    x0[96:128] = np.float32(1e20) * np.sign(rng.standard_normal(32)).astype(np.float32)
    ref = oracle_outputs(oracle, x0, mats)
    st = Stack(L, x0, mats)
    try:
        assert st.run(torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert L.dn_device_status(1) == 0
        check(st, mats, ref, "special")
    finally:
        st.close()


def test_stack_rejects_bad_tables(cuda_lib):
    from dianoia_b200 import _lib
    L = cuda_lib
    q = torch.zeros(64 * 512, dtype=torch.int8, device="cuda")
    s = torch.zeros(64 * 16, dtype=torch.float32, device="cuda")
    x = torch.zeros(512, device="cuda")
    y0, y1 = torch.zeros(64, device="cuda"), torch.zeros(64, device="cuda")
    h = ctypes.c_void_p()

    def create(fmt, *ops):
        arr = (_lib.StackOp * len(ops))(*ops)
        rc = L.dn_stack_create(fmt, arr, len(ops), ctypes.byref(h))
        if rc == 0:
            L.dn_stack_destroy(h)
        return rc

    op = lambda y, dep, cols=512, xx=x: _lib.StackOp(q.data_ptr(), s.data_ptr(), xx.data_ptr(), y.data_ptr(),
                                                      64, cols, dep)
    assert create(_lib.DN_Q8, op(y0, -1), op(y1, 0)) == 0
    assert create(_lib.DN_Q4, op(y0, -1)) == _lib.DN_ERR_UNSUPPORTED
    assert create(_lib.DN_Q8, op(y0, 1), op(y1, 0)) == _lib.DN_ERR_ARGS          # dep must point back
    assert create(_lib.DN_Q8, op(y0, -1), op(y0, 0)) == _lib.DN_ERR_ARGS         # two ops, one output
    assert create(_lib.DN_Q8, op(y0, -1, cols=480)) == _lib.DN_ERR_ARGS          # cols % 512
    # An op reading another's output without a dep edge to it.
    other = torch.zeros(64, device="cuda")
    x_in_y0 = torch.zeros(512, device="cuda")
    writes = _lib.StackOp(q.data_ptr(), s.data_ptr(), x.data_ptr(), x_in_y0.data_ptr(), 64, 512, -1)
    reads = _lib.StackOp(q.data_ptr(), s.data_ptr(), x_in_y0.data_ptr(), other.data_ptr(), 64, 512, -1)
    assert create(_lib.DN_Q8, writes, reads) == _lib.DN_ERR_ARGS
    reads.dep = 0
    assert create(_lib.DN_Q8, writes, reads) == 0

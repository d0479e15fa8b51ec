"""The lm_head's all-gather fused into the product (dn_linear_qa_allgather,
dn_peer_wait), on one GPU: the ranks' row slices run one after another, each
storing its rows into every rank's copy of the output and counting its tiles
in every rank's counter; the waits then find their counts complete. Every
copy must equal the reference's whole output bit for bit - a row does not
depend on the split (lab_native.c:550-552) - on two steps in a row (the
counters only grow). No kernel here waits on another that runs at the same
time: each wait is queued after the products it counts."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("fmt,rows,cols,world", [("q8", 151936 // 16, 2048, 2), ("q8", 1000, 1152, 3),
                                                 ("q4", 4096, 2048, 4)])
def test_fused_allgather_matches_whole_product(cuda_lib, oracle, fmt, rows, cols, world):
    from dianoia_b200 import _lib
    L = cuda_lib
    rng = np.random.default_rng(rows + world)
    qs, sc = orc.q4_weights(rng, rows, cols) if fmt == "q4" else orc.q8_weights(rng, rows, cols)
    x = orc.activations(rng, 1, cols)
    want, _, _ = oracle.gemm(fmt, qs, sc, x, rows, cols, 1, 1)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    st = torch.cuda.current_stream().cuda_stream
    xa = torch.zeros(cols // 32 * 36, dtype=torch.uint8, device="cuda")
    assert L.dn_quantize_qa(dev(x).data_ptr(), xa.data_ptr(), 1, cols, cols // 32 * 36, st) == 0
    outs = [torch.full((rows,), float("nan"), device="cuda") for _ in range(world)]
    counters = torch.zeros(world, dtype=torch.int32, device="cuda")
    expects = torch.zeros(world, dtype=torch.int32, device="cuda")
    ys = (ctypes.c_void_p * world)(*[o.data_ptr() for o in outs])
    cnts = (ctypes.c_void_p * world)(*[counters.data_ptr() + 4 * p for p in range(world)])
    wb = cols // 2 if fmt == "q4" else cols
    spans = [(rows * p // world, rows * (p + 1) // world) for p in range(world)]
    slices = [(dev(qs[r0 * wb:r1 * wb]), dev(sc[r0 * (cols // 32):r1 * (cols // 32)])) for r0, r1 in spans]
    tiles = sum(-(-(r1 - r0) // 32) for r0, r1 in spans)
    f = _lib.DN_Q4 if fmt == "q4" else _lib.DN_Q8
    for step in range(2):
        for o in outs:
            o.fill_(float("nan"))
        for (r0, r1), (q, s) in zip(spans, slices):
            assert L.dn_linear_qa_allgather(f, q.data_ptr(), s.data_ptr(), xa.data_ptr(), r1 - r0, cols, r0,
                                            ys, cnts, world, 0, st) == 0
        for p in range(world):
            assert L.dn_peer_wait(counters.data_ptr() + 4 * p, expects.data_ptr() + 4 * p, tiles, st) == 0
        torch.cuda.synchronize()
        assert L.dn_device_status(1) == 0
        assert counters.cpu().tolist() == [tiles * (step + 1)] * world
        assert expects.cpu().tolist() == [tiles * (step + 1)] * world
        for o in outs:
            assert np.array_equal(o.cpu().numpy().view(np.uint32), want.view(np.uint32)), step


def test_allgather_arguments(cuda_lib):
    from dianoia_b200 import _lib
    L = cuda_lib
    ys = (ctypes.c_void_p * 1)(None)
    assert L.dn_linear_qa_allgather(_lib.DN_Q8, None, None, None, 32, 64, 0, None, None, 1, 0, None) == \
        _lib.DN_ERR_ARGS
    assert L.dn_linear_qa_allgather(_lib.DN_Q8, None, None, None, 32, 64, 0, ys, ys, 9, 0, None) == \
        _lib.DN_ERR_ARGS
    assert L.dn_peer_wait(None, None, 1, None) == _lib.DN_ERR_ARGS


@pytest.mark.parametrize("fmt,rows,cols,n,world", [("q8", 1000, 1152, 100, 3), ("q4", 4096, 2048, 64, 2),
                                                   ("q8", 3456, 1152, 1024, 4), ("q8", 5000, 2048, 16, 3),
                                                   ("q4", 4096, 2048, 32, 2)])
def test_gemm_allgather_matches_whole_product(cuda_lib, oracle, fmt, rows, cols, n, world):
    """The tensor-core GEMM with the all-gather fused into its epilogue
    (dn_linear_allgather), the ranks' row slices run one after another on one
    GPU: every rank's copy of Y[n, rows] must equal dn_linear's tensor-core
    product of the whole matrix value for value (a row's result does not
    depend on the split), on two steps in a row, and lie within the
    reference's 1e-5 bound of the row's absolute-sum scale."""
    from dianoia_b200 import _lib
    L = cuda_lib
    rng = np.random.default_rng(rows + n + world)
    qs, sc = orc.q4_weights(rng, rows, cols) if fmt == "q4" else orc.q8_weights(rng, rows, cols)
    x = orc.activations(rng, n, cols)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    st = torch.cuda.current_stream().cuda_stream
    f = _lib.DN_Q4 if fmt == "q4" else _lib.DN_Q8
    xd = dev(x)
    xq = torch.zeros(n * cols, dtype=torch.int8, device="cuda")
    xsc = torch.zeros(n * (cols // 32) + 4, device="cuda")
    whole = torch.full((n * rows,), float("nan"), device="cuda")
    assert L.dn_linear_path(f, dev(qs).data_ptr(), dev(sc).data_ptr(), xd.data_ptr(), xq.data_ptr(),
                            rows, cols, n, 1) == 1  # the tensor-core path
    assert L.dn_linear(f, dev(qs).data_ptr(), dev(sc).data_ptr(), xd.data_ptr(), xq.data_ptr(), xsc.data_ptr(),
                       whole.data_ptr(), rows, cols, n, rows, 1, -1, 0, st) == 0
    torch.cuda.synchronize()
    want = whole.cpu().numpy()
    ref, mag = oracle.reference_f64(fmt, qs, sc, x, rows, cols, n, 1)
    assert orc.max_rel_err(want, ref, mag) < 1e-5
    outs = [torch.full((n * rows,), float("nan"), device="cuda") for _ in range(world)]
    counters = torch.zeros(world, dtype=torch.int32, device="cuda")
    expects = torch.zeros(world, dtype=torch.int32, device="cuda")
    ys = (ctypes.c_void_p * world)(*[o.data_ptr() for o in outs])
    cnts = (ctypes.c_void_p * world)(*[counters.data_ptr() + 4 * p for p in range(world)])
    wb = cols // 2 if fmt == "q4" else cols
    spans = [(rows * p // world, rows * (p + 1) // world) for p in range(world)]
    slices = [(dev(qs[r0 * wb:r1 * wb]), dev(sc[r0 * (cols // 32):r1 * (cols // 32)])) for r0, r1 in spans]
    tiles = world  # one count per rank's product
    for step in range(2):
        for o in outs:
            o.fill_(float("nan"))
        for (r0, r1), (q, s) in zip(spans, slices):
            assert L.dn_linear_allgather(f, q.data_ptr(), s.data_ptr(), xd.data_ptr(), xq.data_ptr(),
                                         xsc.data_ptr(), r1 - r0, cols, n, r0, rows, ys, cnts, world, st) == 0
        for p in range(world):
            assert L.dn_peer_wait(counters.data_ptr() + 4 * p, expects.data_ptr() + 4 * p, tiles, st) == 0
        torch.cuda.synchronize()
        assert L.dn_device_status(1) == 0
        assert counters.cpu().tolist() == [tiles * (step + 1)] * world
        for o in outs:
            assert np.array_equal(o.cpu().numpy().view(np.uint32), want.view(np.uint32)), step


def test_gemm_allgather_arguments(cuda_lib):
    from dianoia_b200 import _lib
    L = cuda_lib
    ys = (ctypes.c_void_p * 1)(None)
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    args = lambda **k: dict(dict(f=_lib.DN_Q8, rows=128, n=64, row0=0, total=128, world=1), **k)
    def call(f, rows, n, row0, total, world):
        return L.dn_linear_allgather(f, p, p, p, p, p, rows, 64, n, row0, total, ys, ys, world, None)
    assert call(**args(total=100)) == _lib.DN_ERR_ARGS        # rows past the whole matrix
    assert call(**args(world=9)) == _lib.DN_ERR_ARGS          # more ranks than supported
    assert call(**args(f=2)) == _lib.DN_ERR_ARGS              # no such format
    assert call(**args(row0=-1)) == _lib.DN_ERR_ARGS

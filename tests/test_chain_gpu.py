"""The decode chain (dn_chain_*): a token's projections in one persistent
kernel must give, op for op, exactly what separate products give - the
reference's outputs bit for bit - on every run, including runs replayed from
a CUDA graph (the kernel resets its own completion counters)."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def build_layers(fmt, rng, layers, hidden=512, inter=1536, head=4096):
    """qkv -> o -> gate/up -> down per layer, then a head; every layer's qkv
    reads x0 (as bench.py's stack). Returns op list and reference outputs."""
    from dianoia_b200 import _lib
    shapes = []
    for _ in range(layers):
        shapes += [("qkv", 2 * hidden, hidden), ("o", hidden, hidden), ("gu", 2 * inter, hidden),
                   ("down", hidden, inter)]
    shapes.append(("head", head, hidden))
    x0 = orc.activations(rng, 1, hidden)
    mats = []
    for name, r, c in shapes:
        qs, sc = orc.q4_weights(rng, r, c) if fmt == "q4" else orc.q8_weights(rng, r, c)
        mats.append((name, r, c, qs, sc))
    return shapes, x0, mats


@pytest.mark.parametrize("fmt", ["q8", "q4"])
def test_chain_matches_separate_products(cuda_lib, oracle, fmt):
    from dianoia_b200 import _lib
    L = cuda_lib
    rng = np.random.default_rng(3 if fmt == "q8" else 4)
    shapes, x0, mats = build_layers(fmt, rng, layers=2)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    # Oracle: each op on the f32 output of the op it reads.
    inputs_of = {"qkv": None, "o": "qkv", "gu": "o", "down": "gu", "head": "down"}
    ref, outs = [], {}
    for name, r, c, qs, sc in mats:
        src = inputs_of[name]
        x = x0 if src is None else outs[src][:c]
        y, _, _ = oracle.gemm(fmt, qs, sc, x, r, c, 1, 1)
        outs[name] = y
        ref.append(y)
    # Device buffers and the op table.
    xa0 = torch.zeros(x0.size // 32 * 36, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.dn_quantize_qa(dev(x0).data_ptr(), xa0.data_ptr(), 1, x0.size, x0.size // 32 * 36, st) == 0
    keep, ops, ys, last = [], [], [], {}
    for i, (name, r, c, qs, sc) in enumerate(mats):
        q, s = dev(qs), dev(sc)
        y = torch.full((r,), float("nan"), device="cuda")
        ya = torch.zeros(r // 32 * 36, dtype=torch.uint8, device="cuda") if name != "head" else None
        keep += [q, s, y] + ([ya] if ya is not None else [])
        src = inputs_of[name]
        if src is not None:
            xa, dep = last[src]
        else:
            # Layer 2's qkv reads x0 but starts after layer 1's down (an
            # ordering edge, as the norm between them would impose).
            xa, dep = xa0, (last["down"][1] if "down" in last else -1)
        ops.append(_lib.ChainOp(q.data_ptr(), s.data_ptr(), xa.data_ptr(), y.data_ptr(),
                                None if ya is None else ya.data_ptr(), r, c, dep))
        ys.append(y)
        if ya is not None:
            last[name] = (ya, i)
    arr = (_lib.ChainOp * len(ops))(*ops)
    handle = ctypes.c_void_p()
    assert L.dn_chain_create(1 if fmt == "q4" else 0, arr, len(ops), ctypes.byref(handle)) == 0
    try:
        for run in range(3):
            for y in ys:
                y.fill_(float("nan"))
            assert L.dn_chain_run(handle, 1, st) == 0
            torch.cuda.synchronize()
            assert L.dn_device_status(1) == 0
            for (name, *_), y, want in zip(mats, ys, ref):
                got = y.cpu().numpy()
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (run, name)
        # Replayed from a CUDA graph.
        s2 = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s2):
            with torch.cuda.graph(g, stream=s2):
                assert L.dn_chain_run(handle, 1, torch.cuda.current_stream().cuda_stream) == 0
        for _ in range(2):
            for y in ys:
                y.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            assert L.dn_device_status(1) == 0
            assert np.array_equal(ys[-1].cpu().numpy().view(np.uint32), ref[-1].view(np.uint32))
        del g
    finally:
        L.dn_chain_destroy(handle)


def test_chain_rejects_bad_tables(cuda_lib):
    from dianoia_b200 import _lib
    L = cuda_lib
    q = torch.zeros(64 * 64, dtype=torch.int8, device="cuda")
    s = torch.zeros(64 * 2, dtype=torch.float32, device="cuda")
    xa = torch.zeros(64 // 32 * 36, dtype=torch.uint8, device="cuda")
    y = torch.zeros(64, device="cuda")
    ya = torch.zeros(64 // 32 * 36, dtype=torch.uint8, device="cuda")
    handle = ctypes.c_void_p()
    y1 = torch.zeros(64, device="cuda")
    # dep must point backwards
    bad = (_lib.ChainOp * 2)(_lib.ChainOp(q.data_ptr(), s.data_ptr(), xa.data_ptr(), y.data_ptr(), None, 64, 64, 1),
                             _lib.ChainOp(q.data_ptr(), s.data_ptr(), xa.data_ptr(), y1.data_ptr(), None, 64, 64, 0))
    assert L.dn_chain_create(0, bad, 2, ctypes.byref(handle)) == _lib.DN_ERR_ARGS
    # An ordering edge: op 1 reads a prepared input, after op 0.
    order = (_lib.ChainOp * 2)(_lib.ChainOp(q.data_ptr(), s.data_ptr(), xa.data_ptr(), y.data_ptr(), None, 64, 64, -1),
                               _lib.ChainOp(q.data_ptr(), s.data_ptr(), xa.data_ptr(), y1.data_ptr(), None, 64, 64, 0))
    assert L.dn_chain_create(0, order, 2, ctypes.byref(handle)) == 0
    assert L.dn_chain_destroy(handle) == 0
    fwd = (_lib.ChainOp * 1)(_lib.ChainOp(q.data_ptr(), s.data_ptr(), xa.data_ptr(), y.data_ptr(), ya.data_ptr(), 64, 64, 0))
    assert L.dn_chain_create(0, fwd, 1, ctypes.byref(handle)) == _lib.DN_ERR_ARGS
    odd = (_lib.ChainOp * 1)(_lib.ChainOp(q.data_ptr(), s.data_ptr(), xa.data_ptr(), y.data_ptr(), ya.data_ptr(), 48, 64, -1))
    assert L.dn_chain_create(0, odd, 1, ctypes.byref(handle)) == _lib.DN_ERR_ARGS
    # An input that is not inside the producer's QA output.
    ya2 = torch.zeros(64 // 32 * 36, dtype=torch.uint8, device="cuda")
    y2 = torch.zeros(64, device="cuda")
    off = (_lib.ChainOp * 2)(_lib.ChainOp(q.data_ptr(), s.data_ptr(), xa.data_ptr(), None, ya.data_ptr(), 64, 64, -1),
                             _lib.ChainOp(q.data_ptr(), s.data_ptr(), ya.data_ptr() + 4, y2.data_ptr(), None, 64, 64, 0))
    assert L.dn_chain_create(0, off, 2, ctypes.byref(handle)) == _lib.DN_ERR_ARGS
    # Two ops writing one buffer (layers reusing it) would race.
    reuse = (_lib.ChainOp * 2)(_lib.ChainOp(q.data_ptr(), s.data_ptr(), xa.data_ptr(), None, ya.data_ptr(), 64, 64, -1),
                               _lib.ChainOp(q.data_ptr(), s.data_ptr(), xa.data_ptr(), None, ya.data_ptr(), 64, 64, -1))
    assert L.dn_chain_create(0, reuse, 2, ctypes.byref(handle)) == _lib.DN_ERR_ARGS
    # An output over an independent op's input.
    war = (_lib.ChainOp * 2)(_lib.ChainOp(q.data_ptr(), s.data_ptr(), ya2.data_ptr(), None, ya.data_ptr(), 64, 64, -1),
                             _lib.ChainOp(q.data_ptr(), s.data_ptr(), xa.data_ptr(), None, ya2.data_ptr(), 64, 64, -1))
    assert L.dn_chain_create(0, war, 2, ctypes.byref(handle)) == _lib.DN_ERR_ARGS
    # The same two ops with separate buffers and a dep edge are fine.
    ok = (_lib.ChainOp * 2)(_lib.ChainOp(q.data_ptr(), s.data_ptr(), xa.data_ptr(), None, ya.data_ptr(), 64, 64, -1),
                            _lib.ChainOp(q.data_ptr(), s.data_ptr(), ya.data_ptr(), y2.data_ptr(), ya2.data_ptr(), 64, 64, 0))
    assert L.dn_chain_create(0, ok, 2, ctypes.byref(handle)) == 0
    assert L.dn_chain_destroy(handle) == 0


@pytest.mark.parametrize("fmt", ["q8", "q4"])
def test_chain_ragged_shapes(cuda_lib, oracle, fmt):
    """Partial last stages (cols 1152: 36 blocks), scales too narrow for TMA
    (Q4_0 rows of 72 scale bytes), a partial last tile (1000 rows, f32 only)
    and an input read from the middle of a producer's QA output."""
    from dianoia_b200 import _lib
    L = cuda_lib
    rng = np.random.default_rng(11 if fmt == "q8" else 12)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    # (rows, cols, input: None = x0 | (op, first block), keep QA output)
    spec = [(4096, 1152, None, True),      # 0
            (1000, 1152, None, False),     # 1: f32 only, partial tile
            (960, 2048, (0, 32), True),    # 2: reads blocks 32..95 of op 0's output
            (352, 960, (2, 0), False)]     # 3
    x0 = orc.activations(rng, 1, 1152)
    outs, ref, mats = {}, [], []
    for i, (r, c, src, _) in enumerate(spec):
        qs, sc = orc.q4_weights(rng, r, c) if fmt == "q4" else orc.q8_weights(rng, r, c)
        x = x0 if src is None else outs[src[0]][src[1] * 32:src[1] * 32 + c]
        y, _, _ = oracle.gemm(fmt, qs, sc, x, r, c, 1, 1)
        outs[i] = y
        ref.append(y)
        mats.append((qs, sc))
    st = torch.cuda.current_stream().cuda_stream
    xa0 = torch.zeros(1152 // 32 * 36, dtype=torch.uint8, device="cuda")
    assert L.dn_quantize_qa(dev(x0).data_ptr(), xa0.data_ptr(), 1, 1152, 1152 // 32 * 36, st) == 0
    keep, ops, ys, yas = [], [], [], {}
    for i, ((r, c, src, qa_out), (qs, sc)) in enumerate(zip(spec, mats)):
        q, s = dev(qs), dev(sc)
        y = torch.full((r,), float("nan"), device="cuda")
        ya = torch.zeros(r // 32 * 36, dtype=torch.uint8, device="cuda") if qa_out else None
        keep += [q, s, y, ya]
        yas[i] = ya
        if src is None:
            xa, dep = xa0.data_ptr(), -1
        else:
            xa, dep = yas[src[0]].data_ptr() + src[1] * 36, src[0]
        ops.append(_lib.ChainOp(q.data_ptr(), s.data_ptr(), xa, y.data_ptr(),
                                None if ya is None else ya.data_ptr(), r, c, dep))
        ys.append(y)
    arr = (_lib.ChainOp * len(ops))(*ops)
    handle = ctypes.c_void_p()
    assert L.dn_chain_create(1 if fmt == "q4" else 0, arr, len(ops), ctypes.byref(handle)) == 0
    try:
        for run in range(2):
            for y in ys:
                y.fill_(float("nan"))
            assert L.dn_chain_run(handle, 0, st) == 0
            torch.cuda.synchronize()
            assert L.dn_device_status(1) == 0
            for i, (y, want) in enumerate(zip(ys, ref)):
                assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32)), (run, i)
    finally:
        L.dn_chain_destroy(handle)

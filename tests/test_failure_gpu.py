"""Failure detection on one GPU, without a fault.

A sharded decode chain (dn_chain_create_sharded) waits on a counter that the
other ranks add to over NVLink. Run as rank 0 of 2 on one GPU, with a plain
buffer standing in for rank 1's region, the counter never reaches its target:
the bounded wait must run out (after a limit shortened with
dn_set_wait_limit_ns), the kernel must return, and the status word must carry
the peer-timeout bit (the reference's GPU layer reports such a failure as
lab_gpu_commit() == 0, lab_vulkan.c:737-757). After dn_chain_reset the host
plays rank 1 - it writes rank 1's QA block of the first op and its count into
rank 0's region, as rank 1's tile would have over NVLink - and the next run
must complete and equal the reference bit for bit."""
import ctypes
import time

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

PEER_TIMEOUT = 2  # status bit of a wait on another GPU's count that ran out


def qa_blocks(xq, xsc):
    """QA layout (32 int8 + f32 scale per 32 values) of quantized values."""
    blocks = xsc.size
    out = np.zeros((blocks, 36), np.uint8)
    out[:, :32] = xq.reshape(blocks, 32).view(np.uint8)
    out[:, 32:] = xsc.reshape(blocks, 1).view(np.uint8).reshape(blocks, 4)
    return out.reshape(-1)


def test_peer_wait_times_out_and_chain_recovers(cuda_lib, oracle):
    from dianoia_b200 import _lib
    L = cuda_lib
    rows, cols = 64, 64  # two 32-row tiles per op: rank 0 owns tile 0, rank 1 tile 1
    rng = np.random.default_rng(21)
    q0, s0 = orc.q8_weights(rng, rows, cols)
    q1, s1 = orc.q8_weights(rng, rows, cols)
    x0 = orc.activations(rng, 1, cols)
    y0, _, _ = oracle.gemm("q8", q0, s0, x0, rows, cols, 1, 1)
    y1, _, _ = oracle.gemm("q8", q1, s1, y0, rows, cols, 1, 1)
    yq, ysc = oracle.quantize_q8(y0, 1, rows)
    qa_y0 = qa_blocks(yq, ysc)  # op 0's whole QA output: rank 0's block, then rank 1's

    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    st = torch.cuda.current_stream().cuda_stream
    # Rank 0's row slices of both ops (rows 0..31).
    w0, sc0 = dev(q0[: 32 * cols]), dev(s0[: 32 * cols // 32])
    w1, sc1 = dev(q1[: 32 * cols]), dev(s1[: 32 * cols // 32])
    xa0 = torch.zeros(cols // 32 * 36, dtype=torch.uint8, device="cuda")
    assert L.dn_quantize_qa(dev(x0).data_ptr(), xa0.data_ptr(), 1, cols, cols // 32 * 36, st) == 0
    # The region: op 0's QA output (72 bytes) at 0, the counters (nops + 2
    # ints) at 128. Rank 1's stand-in region has the same layout.
    region = torch.zeros(256, dtype=torch.uint8, device="cuda")
    peer = torch.zeros(256, dtype=torch.uint8, device="cuda")
    counters = region[128:144].view(torch.int32)
    ys0 = torch.full((rows,), float("nan"), device="cuda")
    ys1 = torch.full((rows,), float("nan"), device="cuda")
    ops = (_lib.ChainOp * 2)(
        _lib.ChainOp(w0.data_ptr(), sc0.data_ptr(), xa0.data_ptr(), ys0.data_ptr(), region.data_ptr(),
                     32, cols, -1),
        _lib.ChainOp(w1.data_ptr(), sc1.data_ptr(), region.data_ptr(), ys1.data_ptr(), None, 32, cols, 0))
    bases = (ctypes.c_void_p * 2)(region.data_ptr(), peer.data_ptr())
    handle = ctypes.c_void_p()
    assert L.dn_chain_create_sharded(_lib.DN_Q8, ops, (ctypes.c_int64 * 2)(0, 0),
                                     (ctypes.c_int64 * 2)(rows, rows), 2, 0, 2, bases, 256,
                                     counters.data_ptr(), ctypes.byref(handle)) == 0
    L.dn_device_status(1)
    assert L.dn_set_wait_limit_ns(10_000_000) == 0  # 10 ms
    try:
        # Run 1: rank 1 never counts in, so op 1 waits for a count that never comes.
        t0 = time.perf_counter()
        assert L.dn_chain_run(handle, 0, st) == 0
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        status = L.dn_device_status(1)
        assert status & PEER_TIMEOUT, f"status {status}"
        assert elapsed < 1.0, f"the kernel took {elapsed:.3f} s to give up"
        # Rank 0's own tile of op 0 completed before the wait.
        assert np.array_equal(ys0[:32].cpu().numpy().view(np.uint32), y0[:32].view(np.uint32))
        assert np.array_equal(region[:36].cpu().numpy(), qa_y0[:36])

        # Recovery: clear the counters and run index, then deliver what rank 1
        # would have - its QA block of op 0 and one count - and run again.
        assert L.dn_chain_reset(handle, st) == 0
        torch.cuda.synchronize()
        region[36:72] = dev(qa_y0[36:72])
        counters[0] = 1
        ys1.fill_(float("nan"))
        torch.cuda.synchronize()
        assert L.dn_chain_run(handle, 0, st) == 0
        torch.cuda.synchronize()
        assert L.dn_device_status(1) == 0
        assert np.array_equal(ys1[:32].cpu().numpy().view(np.uint32), y1[:32].view(np.uint32))
        assert np.isnan(ys1[32:].cpu().numpy()).all()  # rank 1's rows are not rank 0's to write
    finally:
        assert L.dn_set_wait_limit_ns(0) == 0
        L.dn_chain_destroy(handle)


def test_wait_limit_arguments(cuda_lib):
    from dianoia_b200 import _lib
    assert cuda_lib.dn_set_wait_limit_ns(-1) == _lib.DN_ERR_ARGS
    assert cuda_lib.dn_set_wait_limit_ns(0) == 0

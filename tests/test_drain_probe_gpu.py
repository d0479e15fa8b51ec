"""The GEMM's drain ceiling probe (dn_drain_probe): the per-block drain step
of the tensor-core GEMM alone, one CTA per SM. Its argument checks, and one
run whose every drain lane returns the sum the step must produce: each D slot
holds the seed 0x4B400000 (block dot 0), so every product adds exactly 0."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def test_drain_probe_runs_and_sums_zero(cuda_lib):
    from dianoia_b200 import _lib
    L = cuda_lib
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    threads = 576  # the probe's block: 18 warps
    out = torch.full((sms * threads,), float("nan"), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.dn_drain_probe(sms, 20, out.data_ptr(), st) == 0
    torch.cuda.synchronize()
    assert L.dn_device_status(1) == 0
    o = out.cpu().numpy().reshape(sms, threads)
    # Warps 2-17 are the drain warps: their sums are 0 (dots of 0 times any
    # scale); the other warps write nothing.
    assert np.array_equal(o[:, 64:576], np.zeros((sms, 512), np.float32))
    assert np.isnan(o[:, :64]).all()
    assert L.dn_drain_probe(0, 20, out.data_ptr(), st) == _lib.DN_ERR_ARGS
    assert L.dn_drain_probe(sms, 0, out.data_ptr(), st) == _lib.DN_ERR_ARGS
    assert L.dn_drain_probe(sms, 20, None, st) == _lib.DN_ERR_ARGS

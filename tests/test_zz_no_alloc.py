"""dn_linear_noalloc (scratch in the library's fixed device array, no
allocation) against dn_linear with caller-provided scratch: the same kernels,
so the results agree bit for bit, on two calls in a row, on the GEMV path
(n = 1) and the tensor-core path (n = 64), with the fixed array's status word
read back through dn_linear_noalloc_status. Collected last, and must also
pass alone in a fresh process."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("n", [1, 64])
def test_noalloc_matches_dn_linear(cuda_lib, oracle, fmt, n):
    from dianoia_b200 import _lib
    L = cuda_lib
    rows, cols = 640, 2048
    rng = np.random.default_rng(100 + n + (7 if fmt == "q4" else 0))
    qs, sc = orc.q4_weights(rng, rows, cols) if fmt == "q4" else orc.q8_weights(rng, rows, cols)
    x = orc.activations(rng, n, cols)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    q, s, xs = dev(qs), dev(sc), dev(x)
    f = _lib.DN_Q4 if fmt == "q4" else _lib.DN_Q8
    st = torch.cuda.current_stream().cuda_stream
    want = torch.full((n, rows), float("nan"), device="cuda")
    xq = torch.empty(n * cols, dtype=torch.int8, device="cuda")
    xsc = torch.empty(n * cols // 32, dtype=torch.float32, device="cuda")
    assert L.dn_linear(f, q.data_ptr(), s.data_ptr(), xs.data_ptr(), xq.data_ptr(), xsc.data_ptr(),
                       want.data_ptr(), rows, cols, n, rows, 1, _lib.DN_PATH_AUTO, 0, st) == 0
    for call in range(2):
        got = torch.full((n, rows), float("nan"), device="cuda")
        assert L.dn_linear_noalloc(f, q.data_ptr(), s.data_ptr(), xs.data_ptr(), got.data_ptr(),
                                   rows, cols, n, rows, 0, st) == 0
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int32), want.view(torch.int32)), call
        # Every bounded wait of the call completed (the fixed array's status word).
        assert L.dn_linear_noalloc_status(1) == 0
    # And against the reference's own algorithm: bit-exact on the GEMV path,
    # within the 1e-5 bound of the row's absolute-sum scale on the GEMM path.
    ref, _, _ = oracle.gemm(fmt, qs, sc, x, rows, cols, n, 1)
    got_np = got.cpu().numpy().reshape(-1)
    if n == 1:
        assert np.array_equal(got_np.view(np.uint32), ref.view(np.uint32))
    else:
        ref64, mag = oracle.reference_f64(fmt, qs, sc, x, rows, cols, n)
        assert orc.max_rel_err(got_np, ref64, mag) <= 1e-5


def test_noalloc_rejects_oversize(cuda_lib):
    from dianoia_b200 import _lib
    L = cuda_lib
    st = torch.cuda.current_stream().cuda_stream
    dummy = torch.zeros(1024, device="cuda")
    # 8 Mi activations is the limit: 4097 tokens x 2048 columns is over it.
    assert L.dn_linear_noalloc(_lib.DN_Q8, dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
                               dummy.data_ptr(), 32, 2048, 4097, 32, 0, st) == _lib.DN_ERR_TOO_LARGE
    assert L.dn_linear_noalloc(9, dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
                               dummy.data_ptr(), 32, 2048, 1, 32, 0, st) == _lib.DN_ERR_ARGS

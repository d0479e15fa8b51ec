"""A Q8 cache file on the GPU: the whole file read straight into device
memory (dn_gpu_wrap_file) or copied from its mapping (lab_gpu_wrap, as
dianoia's GpuForward._wrapWeights does, gpu.dart:942-979), then products
recorded at the matrices' file offsets. Results bit for bit against the
reference's kernels on the same matrices, and equal between the two wraps."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


class Split:
    def __init__(self, fmt, qs, sc, rows, cols):
        self.format, self.rows, self.cols = fmt, rows, cols
        self.qs, self.sc = qs, sc
        self.qs_bytes, self.scale_bytes = qs.view(np.uint8), sc.view(np.uint8)


def test_products_on_a_wrapped_cache(cuda_lib, oracle, tmp_path):
    from dianoia_b200.q8_cache import Q8Cache
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    rng = np.random.default_rng(31)
    shapes = {"q": ("q8", 256, 512), "gate": ("q4", 192, 512), "head": ("q8", 1000, 256)}
    mats = {}
    for name, (fmt, rows, cols) in shapes.items():
        gen = orc.q4_weights if fmt == "q4" else orc.q8_weights
        mats[name] = Split(fmt, *gen(rng, rows, cols), rows, cols)
    path = str(tmp_path / "stack.q8cache")
    Q8Cache.write(path, "key", mats)
    cache = Q8Cache.open(path, "key")
    assert cache is not None
    handles = []
    try:
        on_file = cache.wrap_on_gpu()
        handles.append(on_file)
        assert L.lab_gpu_contents(on_file) is None
        mapped = L.lab_gpu_wrap(cache.file.address, cache.file.length)
        assert mapped >= 0
        handles.append(mapped)
        floats = 512 + 1000
        act = L.lab_gpu_buffer(4 * floats)
        handles.append(act)
        view = np.ctypeslib.as_array((ctypes.c_float * floats).from_address(L.lab_gpu_contents(act)))
        for name, m in mats.items():
            o = cache.offsets(name, m.rows, m.cols)
            x = orc.activations(rng, 1, m.cols)
            want, _, _ = oracle.gemm(m.format, m.qs, m.sc, x, m.rows, m.cols, 1, 1)
            for w in (on_file, mapped):
                view[:m.cols] = x
                view[512:] = np.nan
                L.lab_gpu_begin()
                enc = L.lab_gpu_enc_matmul_q4 if m.format == "q4" else L.lab_gpu_enc_matmul_q8
                enc(w, o["qs"], o["scales"], act, 0, act, 4 * 512, m.rows, m.cols, 1)
                assert L.lab_gpu_commit(1) == 1
                got = view[512:512 + m.rows]
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (name, w)
    finally:
        for h in handles:
            L.lab_gpu_release(h)
        cache.close()


def test_wrap_file_rejects_what_it_cannot_read(cuda_lib, tmp_path):
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    p = tmp_path / "f"
    p.write_bytes(bytes(range(256)) * 4)
    assert L.dn_gpu_wrap_file(str(tmp_path / "absent").encode(), 0, 16) == -1
    assert L.dn_gpu_wrap_file(str(p).encode(), 0, 1025) == -1      # longer than the file
    assert L.dn_gpu_wrap_file(str(p).encode(), 1000, 32) == -1     # runs past the end
    assert L.dn_gpu_wrap_file(str(p).encode(), -1, 16) == -1
    live = L.lab_gpu_live_buffers()
    h = L.dn_gpu_wrap_file(str(p).encode(), 16, 1008)
    assert h >= 0 and L.lab_gpu_live_buffers() == live + 1
    L.lab_gpu_release(h)
    assert L.lab_gpu_live_buffers() == live


def test_a_file_read_by_several_threads(cuda_lib, oracle, tmp_path):
    """A 168 MB matrix file, read as two slices on two host threads (slices
    are at least 64 MiB): the product on the wrapped file equals the
    reference's kernels bit for bit."""
    L = cuda_lib
    assert L.lab_gpu_init() == 1
    rng = np.random.default_rng(43)
    rows, cols = 20480, 8192
    qs, sc = orc.q8_weights(rng, rows, cols)
    path = tmp_path / "big.bin"
    with open(path, "wb") as f:
        f.write(bytes(4096))            # a header the offsets skip
        f.write(qs.tobytes())
        f.write(sc.tobytes())
    size = path.stat().st_size
    assert size > 2 * (64 << 20)
    h = L.dn_gpu_wrap_file(str(path).encode(), 0, size)
    act = L.lab_gpu_buffer(4 * (cols + rows))
    try:
        assert h >= 0 and act >= 0
        view = np.ctypeslib.as_array((ctypes.c_float * (cols + rows)).from_address(L.lab_gpu_contents(act)))
        x = orc.activations(rng, 1, cols)
        view[:cols] = x
        L.lab_gpu_begin()
        L.lab_gpu_enc_matmul_q8(h, 4096, 4096 + qs.size, act, 0, act, 4 * cols, rows, cols, 1)
        assert L.lab_gpu_commit(1) == 1
        want, _, _ = oracle.gemm("q8", qs, sc, x, rows, cols, 1, 1)
        assert np.array_equal(view[cols:].view(np.uint32), want.view(np.uint32))
    finally:
        for hd in (h, act):
            if hd >= 0:
                L.lab_gpu_release(hd)

"""The C-ABI library without a GPU: it loads, exports every function the
header declares, and refuses work cleanly when no device is present.

The host-side mirror (dianoia_b200.native) keeps the reference's argument
checks and error types (native.dart:634-636, 718-721, 840-843).
"""
import ctypes
import os

import numpy as np
import pytest

import dianoia_b200
from dianoia_b200 import _lib
from dianoia_b200 import native as nat


@pytest.fixture(scope="module")
def L():
    if not os.path.exists(dianoia_b200.LIB_PATH):
        from dianoia_b200 import build
        build.build()
    return dianoia_b200.lib()


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def test_header_declares_the_reference_symbols():
    names = _lib.header_functions()
    for sym in ("lab_alloc", "lab_free", "lab_cpu_supported", "lab_quantize_q8", "lab_quantize_q4",
                "lab_gemm_q8", "lab_gemm_q4", "lab_gemv_q8",
                # the GPU layer's product ABI (gpu.dart:36-312)
                "lab_gpu_init", "lab_gpu_buffer", "lab_gpu_readback_buffer", "lab_gpu_wrap",
                "lab_gpu_wrap_copies", "lab_gpu_contents", "lab_gpu_release", "lab_gpu_live_buffers",
                "lab_gpu_begin", "lab_gpu_commit", "lab_gpu_wait", "lab_gpu_last_ms",
                "lab_gpu_enc_matmul_q8", "lab_gpu_enc_matmul_q4",
                # the GPU layer's neighbours, queries, knobs and profiling (gpu.dart:36-312)
                "lab_gpu_enc_rms_norm", "lab_gpu_enc_swiglu", "lab_gpu_enc_add",
                "lab_gpu_device_name", "lab_gpu_max_buffer_length", "lab_gpu_max_shared_memory",
                "lab_gpu_recommended_working_set", "lab_gpu_thermal_state", "lab_gpu_physical_memory",
                "lab_gpu_set_decode_rows", "lab_gpu_set_q8_group", "lab_gpu_set_q8_vector",
                "lab_gpu_register_q8_head", "lab_gpu_set_profiling", "lab_gpu_profile",
                # host helpers of the same asset (native.dart:218-240)
                "lab_map_file", "lab_unmap_file", "lab_evict_file", "lab_phys_footprint"):
        assert sym in names


def test_library_exports_every_declared_symbol(L):
    names = _lib.header_functions()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures and header disagree"


def test_library_does_not_link_torch():
    import subprocess
    out = subprocess.run(["ldd", dianoia_b200.LIB_PATH], capture_output=True, text=True).stdout
    assert "torch" not in out and "c10" not in out


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device behaviour")
def test_no_device_behaviour(L):
    assert L.lab_cpu_supported() == 0
    assert not L.lab_alloc(64)
    assert L.dn_linear(0, None, None, None, None, None, None, 1, 32, 1, 1, 1, -1, 0, None) == _lib.DN_ERR_NO_DEVICE
    L.dn_last_error()
    ys = np.zeros(4, np.float32)
    L.lab_gemm_q8(None, None, None, None, None, ys.ctypes.data, 4, 32, 1, 1, 1)
    assert L.dn_last_error() == _lib.DN_ERR_NO_DEVICE
    assert L.dn_last_error() == _lib.DN_OK  # cleared by reading
    with pytest.raises(nat.StateError):
        nat.NativeKernels.load(None)
    with pytest.raises(nat.StateError):
        nat.NativeKernels.instance()
    # The GPU layer does not start; its functions refuse work without crashing.
    assert L.lab_gpu_init() == 0
    assert L.lab_gpu_buffer(64) == -1
    assert L.lab_gpu_contents(0) is None
    assert L.lab_gpu_live_buffers() == 0
    L.lab_gpu_begin()
    L.lab_gpu_enc_matmul_q8(0, 0, 0, 0, 0, 0, 0, 32, 32, 1)
    assert L.lab_gpu_commit(1) == 0
    assert L.lab_gpu_wrap_copies() == 1
    from dianoia_b200.gpu import GpuLinear
    assert GpuLinear.start() is None


def test_error_strings(L):
    assert L.dn_error_string(0) == b"ok"
    assert L.dn_error_string(-5).startswith(b"size")


def test_argument_errors_come_first():
    with pytest.raises(nat.ArgumentError):
        nat.NativeQ8Matrix.quantize(np.zeros(48, np.float32), 1, 48)
    with pytest.raises(nat.ArgumentError):
        nat.NativeQ4Matrix.quantize(np.zeros(40, np.float32), 1, 40)
    with pytest.raises(nat.ArgumentError):
        nat.NativeQ4Matrix.from_gguf_blocks(np.zeros(17, np.uint8), 1, 32)


def test_half_to_double_matches_numpy():
    allh = np.arange(65536, dtype=np.uint16)
    want = allh.view(np.float16).astype(np.float64)
    got = np.array([nat.half_to_double(int(h)) for h in allh])
    ok = ~np.isnan(want)
    assert np.array_equal(got[ok], want[ok])
    assert np.isnan(got[~ok]).all()


def test_file_mapping_helpers(L, tmp_path):
    """lab_map_file / lab_unmap_file / lab_evict_file as dianoia's MappedFile
    uses them (native.dart:268-306): the bytes of the file, still readable
    after an eviction; NULL for a missing or empty file."""
    data = np.random.default_rng(1).integers(0, 256, 3 * 4096 + 17, dtype=np.uint8)
    path = tmp_path / "f.bin"
    path.write_bytes(data.tobytes())
    size = ctypes.c_int64(0)
    p = L.lab_map_file(str(path).encode(), ctypes.byref(size))
    assert p and size.value == data.size
    view = np.ctypeslib.as_array((ctypes.c_uint8 * data.size).from_address(p))
    assert np.array_equal(view, data)
    L.lab_evict_file(p, size.value)
    assert np.array_equal(view, data)
    del view
    L.lab_unmap_file(p, size.value)
    assert not L.lab_map_file(str(tmp_path / "absent").encode(), ctypes.byref(size))
    (tmp_path / "empty").write_bytes(b"")
    assert not L.lab_map_file(str(tmp_path / "empty").encode(), ctypes.byref(size))
    assert L.lab_phys_footprint() > 0

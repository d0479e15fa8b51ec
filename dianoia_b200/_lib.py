"""Loads libdianoia_b200.so (the CUDA kernels behind the C-ABI) with ctypes.

There is no fallback: if the library is missing, importing the product path
fails loudly. Build it with ``python dianoia_b200/build.py`` (or
``__graft_entry__.build()``).
"""
from __future__ import annotations

import ctypes
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libdianoia_b200.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "dianoia_b200.h")

_i64 = ctypes.c_int64
_p = ctypes.c_void_p

# Every exported function with its ctypes signature (restype, argtypes).
SIGNATURES = {
    "lab_alloc": (_p, [_i64]),
    "lab_free": (None, [_p]),
    "lab_cpu_supported": (_i64, []),
    "lab_quantize_q8": (None, [_p, _p, _p, _i64, _i64]),
    "lab_quantize_q4": (None, [_p, _p, _p, _i64, _i64]),
    "lab_gemm_q8": (None, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64]),
    "lab_gemm_q4": (None, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64]),
    "lab_gemv_q8": (None, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64]),
    "lab_map_file": (_p, [ctypes.c_char_p, _p]),
    "lab_unmap_file": (None, [_p, _i64]),
    "lab_evict_file": (None, [_p, _i64]),
    "lab_phys_footprint": (_i64, []),
    "lab_gpu_init": (_i64, []),
    "lab_gpu_device_name": (None, [ctypes.c_char_p, _i64]),
    "lab_gpu_max_buffer_length": (_i64, []),
    "lab_gpu_max_shared_memory": (_i64, []),
    "lab_gpu_recommended_working_set": (_i64, []),
    "lab_gpu_thermal_state": (_i64, []),
    "lab_gpu_physical_memory": (_i64, []),
    "lab_gpu_set_decode_rows": (None, [_i64]),
    "lab_gpu_set_q8_group": (_i64, [_i64]),
    "lab_gpu_set_q8_vector": (_i64, [_i64]),
    "lab_gpu_register_q8_head": (_i64, [_i64] * 5),
    "lab_gpu_set_profiling": (None, [_i64]),
    "lab_gpu_profile": (_i64, [_p, _p, _i64]),
    "lab_gpu_buffer": (_i64, [_i64]),
    "lab_gpu_readback_buffer": (_i64, [_i64]),
    "lab_gpu_wrap": (_i64, [_p, _i64]),
    "lab_gpu_wrap_copies": (_i64, []),
    "lab_gpu_contents": (_p, [_i64]),
    "lab_gpu_release": (None, [_i64]),
    "lab_gpu_live_buffers": (_i64, []),
    "lab_gpu_begin": (None, []),
    "lab_gpu_commit": (_i64, [_i64]),
    "lab_gpu_wait": (_i64, []),
    "lab_gpu_last_ms": (ctypes.c_double, []),
    "lab_gpu_enc_matmul_q8": (None, [_i64] * 10),
    "lab_gpu_enc_matmul_q4": (None, [_i64] * 10),
    "lab_gpu_enc_rms_norm": (None, [_i64] * 8 + [ctypes.c_double, _i64]),
    "lab_gpu_enc_swiglu": (None, [_i64] * 3),
    "lab_gpu_enc_add": (None, [_i64] * 5),
    "lab_gpu_enc_copy": (None, [_i64] * 5),
    "lab_gpu_enc_steer": (None, [_i64] * 7 + [ctypes.c_double]),
    "lab_gpu_enc_head_norm_rope": (None, [_i64] * 11 + [ctypes.c_double]),
    "lab_gpu_enc_conv": (None, [_i64] * 8),
    "lab_gpu_enc_attention": (None, [_i64] * 11),
    "dn_gpu_enc_batch": (None, [_p, _i64]),
    "dn_gpu_set_fusion": (None, [_i64]),
    "dn_gpu_wrap_file": (_i64, [ctypes.c_char_p, _i64, _i64]),
    "dn_gpu_device_buffer": (_i64, [_i64]),
    "dn_linear": (_i64, [_i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p]),
    "dn_linear_path": (_i64, [_i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64]),
    "dn_quantize_q8": (_i64, [_p, _p, _p, _i64, _i64, _p]),
    "dn_gguf_split": (_i64, [_i64, _p, _i64, _p, _p, _p]),
    "dn_gguf_linear_qa": (_i64, [_i64, _p, _p, _p, _i64, _i64, _i64, _p]),
    "dn_quantize_q4": (_i64, [_p, _p, _p, _i64, _i64, _p]),
    "dn_quantize_qa": (_i64, [_p, _p, _i64, _i64, _i64, _p]),
    "dn_rms_norm": (_i64, [_p, _p, _p, _p, _i64, _i64, _i64, ctypes.c_double, _i64, _i64, _p]),
    "dn_swiglu": (_i64, [_p, _p, _p, _i64, _i64, _p]),
    "dn_linear_qa": (_i64, [_i64, _p, _p, _p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p]),
    "dn_linear_allgather": (_i64, [_i64, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _i64, _p]),
    "dn_linear_qa_allgather": (_i64, [_i64, _p, _p, _p, _i64, _i64, _i64, _p, _p, _i64, _i64, _p]),
    "dn_peer_wait": (_i64, [_p, _p, _i64, _p]),
    "dn_drain_probe": (_i64, [_i64, _i64, _p, _p]),
    "dn_chain_create": (_i64, [_i64, _p, _i64, _p]),
    "dn_chain_create_sharded": (_i64, [_i64, _p, _p, _p, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "dn_peer_alloc": (_i64, [_i64, _p, _p]),
    "dn_peer_open": (_i64, [_p, _p]),
    "dn_peer_close": (_i64, [_p]),
    "dn_peer_free": (_i64, [_p]),
    "dn_chain_run": (_i64, [_p, _i64, _p]),
    "dn_chain_reset": (_i64, [_p, _p]),
    "dn_chain_destroy": (_i64, [_p]),
    "dn_stack_create": (_i64, [_i64, _p, _i64, _p]),
    "dn_stack_run": (_i64, [_p, _i64, _p]),
    "dn_stack_reset": (_i64, [_p, _p]),
    "dn_stack_destroy": (_i64, [_p]),
    "dn_linear_noalloc": (_i64, [_i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p]),
    "dn_linear_noalloc_status": (_i64, [_i64]),
    "dn_set_wait_limit_ns": (_i64, [_i64]),
    "dn_last_error": (_i64, []),
    "dn_device_status": (_i64, [_i64]),
    "dn_error_string": (ctypes.c_char_p, [_i64]),
}

# Status codes (include/dianoia_b200.h).
DN_OK, DN_ERR_ARGS, DN_ERR_CUDA, DN_ERR_NO_DEVICE, DN_ERR_UNSUPPORTED, DN_ERR_TOO_LARGE = 0, -1, -2, -3, -4, -5
DN_Q8, DN_Q4 = 0, 1
DN_PATH_AUTO, DN_PATH_GEMV, DN_PATH_TC, DN_PATH_GENERIC = -1, 0, 1, 2
DN_FLAG_PDL = 1
(DN_BATCH_Q8, DN_BATCH_Q4, DN_BATCH_RMS_NORM, DN_BATCH_SWIGLU, DN_BATCH_ADD, DN_BATCH_COPY, DN_BATCH_STEER,
 DN_BATCH_HEAD_NORM_ROPE, DN_BATCH_CONV, DN_BATCH_ATTENTION) = range(10)
QA_BYTES = 36  # QA activation block: 32 int8 + f32 scale
DN_PEER_HANDLE_BYTES = 64


class ChainOp(ctypes.Structure):
    """dn_chain_op (include/dianoia_b200.h)."""
    _fields_ = [("qs", _p), ("scales", _p), ("xa", _p), ("ys", _p), ("ya", _p),
                ("rows", _i64), ("cols", _i64), ("dep", _i64)]


class StackOp(ctypes.Structure):
    """dn_stack_op (include/dianoia_b200.h)."""
    _fields_ = [("qs", _p), ("scales", _p), ("x", _p), ("y", _p),
                ("rows", _i64), ("cols", _i64), ("dep", _i64)]

_lib = None


class LibraryMissing(ImportError):
    pass


def lib() -> ctypes.CDLL:
    """The loaded library, with argument types set; raises if it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LibraryMissing(
                f"{LIB_PATH} is not built; run `python dianoia_b200/build.py` (nvcc, sm_100a)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def header_functions(path: str = HEADER) -> list[str]:
    """Names of the functions include/dianoia_b200.h declares."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:lab|dn)_\w+)\s*\(", text)))


def check(code: int, what: str = "dianoia_b200") -> None:
    if code != DN_OK:
        msg = lib().dn_error_string(code).decode()
        raise RuntimeError(f"{what}: {msg} ({code})")

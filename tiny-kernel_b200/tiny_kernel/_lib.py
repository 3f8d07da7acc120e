"""ctypes binding of libtkcuda (include/tk_cuda.h).

Loads the in-tree ``lib/libtkcuda.so`` built by the package Makefile.  There is no
fallback: if the library is missing, every call raises, so a GPU run can never pass on
a CPU or library stand-in.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get(
    "TK_LIB_PATH", os.path.join(os.path.dirname(_HERE), "lib", "libtkcuda.so"))

TK_OK = 0
TK_ERR_ARG = -1
TK_ERR_CUDA = -2
TK_ERR_NCCL = -3
TK_ERR_TIMEOUT = -4
TK_ERR_UNSUPPORTED = -5
TK_ERR_NOMEM = -6

TK_MEM_DEVICE = 0
TK_MEM_SHARED = 1
TK_MEM_HOST = 2

TK_FFN_RESIDUAL = 1
TK_FFN_HOST_IO = 2
TK_TP_UNIQUE_ID_BYTES = 128
TK_Q4_0_REFERENCE_ORDER = 0
TK_Q4_0_GGML_ORDER = 1

vp = C.c_void_p
u32 = C.c_uint32
f32 = C.c_float
i32 = C.c_int


class Int4MatrixC(C.Structure):
    """tk_int4_matrix: device pointers of one packed INT4 matrix."""
    _fields_ = [("w_packed", vp), ("scales", vp), ("zeros", vp)]


# name -> (restype, argtypes); the exported surface of include/tk_cuda.h
SIGNATURES = {
    "tk_abi_version": (i32, []),
    "tk_last_error_string": (C.c_char_p, []),
    "tk_status_string": (C.c_char_p, [i32]),
    "tk_device_create": (i32, [i32, C.POINTER(vp)]),
    "tk_device_destroy": (None, [vp]),
    "tk_device_name": (C.c_char_p, [vp]),
    "tk_device_sm_count": (i32, [vp]),
    "tk_device_launch_count": (C.c_uint64, [vp]),
    "tk_device_stream": (vp, [vp]),
    "tk_device_synchronize": (i32, [vp]),
    "tk_device_check_error": (i32, [vp]),
    "tk_buffer_alloc": (i32, [vp, C.c_size_t, i32, C.POINTER(vp)]),
    "tk_buffer_free": (i32, [vp, vp]),
    "tk_buffer_upload": (i32, [vp, vp, vp, C.c_size_t]),
    "tk_buffer_download": (i32, [vp, vp, vp, C.c_size_t]),
    "tk_buffer_upload_async": (i32, [vp, vp, vp, C.c_size_t, vp]),
    "tk_buffer_download_async": (i32, [vp, vp, vp, C.c_size_t, vp]),
    "tk_qmatmul_int4": (i32, [vp, vp, vp, vp, vp, vp, u32, u32, u32, u32]),
    "tk_qmatmul_int4_async": (i32, [vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, vp]),
    "tk_qmatmul_int4_path": (i32, [u32, u32, u32, u32]),
    "tk_int4_ffn_path": (i32, [u32, u32, u32, u32]),
    "tk_qmatmul_int4_noalloc": (i32, [vp, vp, vp, vp, vp, u32, u32, u32, u32, vp]),
    "tk_rmsnorm": (i32, [vp, vp, vp, vp, u32, u32, f32]),
    "tk_rmsnorm_async": (i32, [vp, vp, vp, vp, u32, u32, f32, vp]),
    "tk_fused_rmsnorm_rope": (i32, [vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, f32]),
    "tk_fused_rmsnorm_rope_async": (i32, [vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, f32, vp]),
    "tk_silu_mul": (i32, [vp, vp, vp, vp, u32]),
    "tk_silu_mul_async": (i32, [vp, vp, vp, vp, u32, vp]),
    "tk_int4_ffn": (i32, [vp, vp, vp, C.POINTER(Int4MatrixC), C.POINTER(Int4MatrixC),
                          C.POINTER(Int4MatrixC), vp, vp, u32, u32, u32, u32, f32, u32]),
    "tk_int4_ffn_async": (i32, [vp, vp, vp, C.POINTER(Int4MatrixC), C.POINTER(Int4MatrixC),
                                C.POINTER(Int4MatrixC), vp, vp, u32, u32, u32, u32, f32, u32,
                                vp]),
    "tk_dequant_int4": (i32, [vp, vp, vp, vp, vp, u32, u32, u32]),
    "tk_matvec": (i32, [vp, vp, vp, vp, u32, u32]),
    "tk_matvec_async": (i32, [vp, vp, vp, vp, u32, u32, vp]),
    "tk_matvec_dual": (i32, [vp, vp, vp, vp, vp, vp, u32, u32]),
    "tk_matvec_dual_async": (i32, [vp, vp, vp, vp, vp, vp, u32, u32, vp]),
    "tk_repack_q4_0": (i32, [vp, vp, vp, vp, vp, u32, u32, i32]),
    "tk_paged_attention": (i32, [vp, vp, vp, vp, vp, vp, vp, u32, u32, u32, u32]),
    "tk_paged_attention_async": (i32, [vp, vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, vp]),
    "tk_argmax": (i32, [vp, vp, u32, vp]),
    "tk_argmax_async": (i32, [vp, vp, u32, vp, vp]),
    "tk_softmax_sample": (i32, [vp, vp, vp, vp, u32, f32, f32]),
    "tk_softmax_sample_async": (i32, [vp, vp, vp, vp, u32, f32, f32, vp]),
    "tk_tp_unique_id": (i32, [vp]),
    "tk_tp_create": (i32, [vp, i32, i32, vp, C.POINTER(vp)]),
    "tk_tp_destroy": (None, [vp]),
    "tk_tp_allreduce_sum_f32": (i32, [vp, vp, C.c_size_t, vp]),
    "tk_tp_uses_p2p": (i32, [vp]),
    "tk_int4_ffn_tp_exchange": (i32, [vp, u32, u32, u32, u32]),
    "tk_int4_ffn_tp": (i32, [vp, vp, vp, C.POINTER(Int4MatrixC), C.POINTER(Int4MatrixC),
                             C.POINTER(Int4MatrixC), vp, u32, u32, u32, u32, f32, u32]),
    "tk_int4_ffn_tp_async": (i32, [vp, vp, vp, C.POINTER(Int4MatrixC), C.POINTER(Int4MatrixC),
                                   C.POINTER(Int4MatrixC), vp, u32, u32, u32, u32, f32, u32,
                                   vp]),
    "tk_device_trace_enable": (i32, [vp, i32]),
    "tk_device_trace_read": (i32, [vp, vp, C.c_size_t, C.POINTER(C.c_size_t)]),
}


class TKError(RuntimeError):
    """A negative status returned by libtkcuda."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


_lib = None


def bundled_nccl() -> str | None:
    """The libnccl.so.2 of the ``nvidia-nccl`` wheel that torch links against, if installed.

    The tensor-parallel entry points load NCCL at their first call; a process holds one
    libnccl.so.2, so loading an older system copy before ``import torch`` would leave torch's
    newer NCCL symbols unresolved.  Pointing TK_NCCL_LIB at the wheel's copy keeps both on one.
    """
    import importlib.util

    try:
        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        return None
    for root in (spec.submodule_search_locations or []) if spec else []:
        path = os.path.join(root, "lib", "libnccl.so.2")
        if os.path.exists(path):
            return path
    return None


def lib() -> C.CDLL:
    """The loaded library (raises OSError if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"libtkcuda is not built: {LIB_PATH} (run `make -C tiny-kernel_b200`)")
        if not os.environ.get("TK_NCCL_LIB"):
            nccl = bundled_nccl()
            if nccl:
                os.environ["TK_NCCL_LIB"] = nccl
        handle = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int) -> None:
    if status != TK_OK:
        msg = lib().tk_last_error_string()
        raise TKError(status, msg.decode() if msg else "libtkcuda error")

"""ctypes binding of oracle/lib/libtkcpu.so, the multithreaded CPU transcription of the
reference shaders (cpu_baseline.cpp).  Test / benchmark infrastructure only: it is the
timed CPU baseline and an f32 cross-check, never part of the product path."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libtkcpu.so")
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is not built (make -C oracle)")
        L = C.CDLL(LIB_PATH)
        p, i, f = C.c_void_p, C.c_int, C.c_float
        L.tkcpu_default_threads.restype = i
        L.tkcpu_qmatmul_int4.argtypes = [p, p, p, p, p, i, i, i, i, i]
        L.tkcpu_qmatmul_int4.restype = i
        L.tkcpu_rmsnorm.argtypes = [p, p, p, i, i, f]
        L.tkcpu_silu_mul.argtypes = [p, p, p, i]
        L.tkcpu_int4_ffn.argtypes = [p, p, p, p, p, p, p, p, p, p, p, p, i, i, i, i, f, i, p, i]
        L.tkcpu_int4_ffn.restype = i
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def default_threads() -> int:
    return lib().tkcpu_default_threads()


def qmatmul_int4(x, M, threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, M.K)
    out = np.empty((x.shape[0], M.N), dtype=np.float32)
    rc = lib().tkcpu_qmatmul_int4(_p(x), _p(M.w), _p(M.s), _p(M.z), _p(out), x.shape[0], M.K,
                                  M.N, M.gs, threads)
    if rc:
        raise ValueError("invalid shape")
    return out


class FFNRunner:
    """Holds contiguous host copies + scratch so repeated calls time only the math."""

    def __init__(self, W, m: int, eps: float = 1e-5, residual: bool = False, threads: int = 0):
        self.W, self.m, self.eps, self.residual = W, m, eps, residual
        self.threads = threads
        self.scratch = np.empty(m * (W.hidden + 3 * W.inter), dtype=np.float32)
        self.out = np.empty((m, W.hidden), dtype=np.float32)

    def __call__(self, x) -> np.ndarray:
        W = self.W
        x = np.ascontiguousarray(x, dtype=np.float32)
        rc = lib().tkcpu_int4_ffn(
            _p(x), _p(W.norm_w), _p(W.gate.w), _p(W.gate.s), _p(W.gate.z), _p(W.up.w),
            _p(W.up.s), _p(W.up.z), _p(W.down.w), _p(W.down.s), _p(W.down.z), _p(self.out),
            self.m, W.hidden, W.inter, W.gs, self.eps, int(self.residual), _p(self.scratch),
            self.threads)
        if rc:
            raise ValueError("invalid shape")
        return self.out

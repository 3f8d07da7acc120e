"""CPU checks of the C-ABI boundary: the library loads without a GPU and exports every
entry point include/tk_cuda.h declares; calls that need no device behave."""
import ctypes as C
import os
import re

import pytest

from tiny_kernel import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "tk_cuda.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tk_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_symbols()
    for must in ("tk_qmatmul_int4", "tk_int4_ffn", "tk_rmsnorm", "tk_fused_rmsnorm_rope",
                 "tk_silu_mul", "tk_device_create", "tk_buffer_alloc", "tk_dequant_int4"):
        assert must in names


def test_library_exports_every_declared_symbol():
    L = C.CDLL(_lib.LIB_PATH)
    missing = [n for n in declared_symbols() if not hasattr(L, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_calls_without_gpu():
    L = _lib.lib()
    assert L.tk_abi_version() == 1
    assert L.tk_status_string(_lib.TK_ERR_TIMEOUT) == b"device-side wait timed out"
    assert L.tk_qmatmul_int4_path(1, 4096, 14336, 64) == 3   # the decode kernel (1-4 rows)
    assert L.tk_qmatmul_int4_path(3, 4096, 14336, 64) == 3   # its four-row instantiation
    assert L.tk_qmatmul_int4_path(1, 4800, 14336, 48) == 0
    assert L.tk_qmatmul_int4_path(1, 4096, 14335, 64) == -1
    assert L.tk_qmatmul_int4_path(1, 100, 64, 8) == -1
    assert L.tk_qmatmul_int4_path(16, 4096, 14336, 64) == 2
    assert L.tk_qmatmul_int4_path(16, 4096, 14464, 64) == 3   # 14464 % 256 != 0: 4-row decodes
    assert L.tk_qmatmul_int4_path(15, 4096, 14336, 64) == 2   # the GEMM from 5 rows
    assert L.tk_qmatmul_int4_path(5, 4096, 14336, 64) == 2
    assert L.tk_int4_ffn_path(1, 4096, 14336, 64) == 3
    assert L.tk_int4_ffn_path(2, 8192, 28672, 64) == 3
    assert L.tk_int4_ffn_path(4, 4096, 14336, 64) == 3
    assert L.tk_int4_ffn_path(16, 4096, 14336, 64) == 2
    assert L.tk_int4_ffn_path(16, 4800, 9600, 48) == 0


def test_null_arguments_rejected():
    L = _lib.lib()
    assert L.tk_device_create(0, None) == _lib.TK_ERR_ARG
    assert L.tk_qmatmul_int4(None, None, None, None, None, None, 1, 64, 32, 8) == _lib.TK_ERR_ARG
    assert b"NULL" in L.tk_last_error_string()


def test_tp_group_id_and_argument_checks():
    """tk_tp_*: the group id comes from NCCL (loaded at first use, no GPU needed for the id);
    malformed calls are refused before any NCCL or CUDA work."""
    import ctypes as C

    from tiny_kernel import tp
    L = _lib.lib()
    a, b = tp.unique_id(), tp.unique_id()
    assert len(a) == _lib.TK_TP_UNIQUE_ID_BYTES and a != b
    idbuf = (C.c_uint8 * _lib.TK_TP_UNIQUE_ID_BYTES).from_buffer_copy(a)
    h = C.c_void_p()
    assert L.tk_tp_create(None, 2, 0, idbuf, C.byref(h)) == _lib.TK_ERR_ARG
    assert L.tk_tp_unique_id(None) == _lib.TK_ERR_ARG
    assert L.tk_int4_ffn_tp(None, None, None, None, None, None, None, 1, 128, 128, 64, 1e-5, 0) \
        == _lib.TK_ERR_ARG
    assert L.tk_tp_allreduce_sum_f32(None, None, 0, None) == _lib.TK_ERR_ARG
    L.tk_tp_destroy(None)  # no-op


def test_tp_id_before_torch_import_keeps_torch_loadable():
    """NCCL loaded by the tensor-parallel entry points before ``import torch`` is the copy torch
    links against, so torch still imports (an older system libnccl.so.2 loaded first would leave
    torch's libtorch_cuda.so with unresolved NCCL symbols)."""
    import subprocess
    import sys

    pkg = os.path.dirname(os.path.dirname(os.path.abspath(_lib.__file__)))
    code = ("import sys; sys.path.insert(0, %r)\n"
            "from tiny_kernel import tp\n"
            "assert len(tp.unique_id()) == 128\n"
            "import torch\n"
            "print('ok', torch.__version__)\n") % pkg
    env = {k: v for k, v in os.environ.items() if k != "TK_NCCL_LIB"}
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env,
                       timeout=600)
    assert r.returncode == 0 and r.stdout.startswith("ok"), r.stderr[-2000:]


def test_zig_shims_call_only_exported_symbols():
    """The Zig kernel API files (tiny-kernel_b200/zig, not compiled here: no Zig toolchain) call
    only entry points that include/tk_cuda.h declares and libtkcuda exports, and keep the
    reference's struct names and forward() methods."""
    import re
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    zdir = os.path.join(root, "tiny-kernel_b200", "zig", "src")
    header = open(os.path.join(root, "include", "tk_cuda.h")).read()
    L = _lib.lib()
    called = set()
    text = ""
    for dirpath, _, files in os.walk(zdir):
        for f in files:
            if f.endswith(".zig"):
                t = open(os.path.join(dirpath, f)).read()
                text += t
                called |= set(re.findall(r"\bc\.(tk_[a-z0-9_]+)\(", t))
    assert len(called) >= 12
    for name in sorted(called):
        assert re.search(rf"\b{name}\s*\(", header), name
        assert hasattr(L, name), name
    for struct in ("QMatMulInt4", "RMSNorm", "FusedRMSNormRoPE", "FusedSiluMul", "Matvec",
                   "MatvecDual", "FusedInt4FFN"):
        assert re.search(rf"pub const {struct} = struct", text), struct

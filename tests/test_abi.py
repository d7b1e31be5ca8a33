"""C ABI checks that need no GPU: the library loads, exports every function
include/*.h declares, and rejects bad arguments with status codes (never an
abort) before touching a device."""
import ctypes
import glob
import os
import re
import subprocess

import pytest

import macrograd_b200 as mg
from macrograd_b200 import _lib
from macrograd_b200._lib import i32_array

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"\b(mg_[a-z0-9_]+)\s*\(", text):
            if not m.group(1).endswith("_fn"):
                names.add(m.group(1))
    return names


def test_library_builds_and_loads():
    lib = mg.load(build_if_missing=True)
    assert b"sm_100a" in lib.mg_version()


def test_every_declared_symbol_is_exported():
    mg.load(build_if_missing=True)
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.lib_path()], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    declared = declared_functions()
    assert declared, "no declarations parsed"
    missing = declared - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    assert declared == set(_lib.SIGNATURES), "ctypes binding out of sync with the header"


def test_kernels_are_built_for_sm100a_only():
    """The build compiles every kernel for sm_100a and nothing else."""
    from macrograd_b200 import build

    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_desc_init_defaults():
    lib = mg.load()
    d = _lib.GemmDesc()
    lib.mg_gemm_desc_init(ctypes.byref(d), 5, 6, 7, 1, 0)
    assert (d.M, d.N, d.K, d.lda, d.ldb, d.ldc) == (5, 6, 7, 5, 6, 6)
    assert d.alpha == 1.0 and d.beta == 0.0 and d.mode == _lib.MG_MODE_DEFAULT


@pytest.mark.parametrize("args,fragment", [
    (([2, 3], [2, 4], [5, 3], 2, 0, 0), "incompatible inner"),
    (([2, 3], [2, 4], [4, 3], 1, 0, 0), "rank 1"),
    (([3, 2, 3], [2, 2, 4], [3, 4, 3], 3, 0, 0), "not broadcastable"),
    (([2, 9], [2, 4], [4, 3], 2, 0, 0), "out shape"),
])
def test_seam_shape_errors_return_status(args, fragment):
    lib = mg.load()
    o, a, b, rank, ta, tb = args
    rc = lib.mg_matmul(None, None, None, i32_array(o), i32_array(a), i32_array(b), rank, ta, tb, None)
    assert rc == _lib.MG_ERR_INVALID
    assert fragment in lib.mg_last_error().decode()


def test_gemm_descriptor_errors_return_status():
    lib = mg.load()
    d = _lib.GemmDesc()
    lib.mg_gemm_desc_init(ctypes.byref(d), 4, 300, 8, 0, 0)
    d.epilogue = _lib.MG_EPI_SOFTMAX
    assert lib.mg_gemm(ctypes.byref(d), None, None, None, None, None) == _lib.MG_ERR_UNSUPPORTED
    d.epilogue = _lib.MG_EPI_CAUSAL
    assert lib.mg_gemm(ctypes.byref(d), None, None, None, None, None) == _lib.MG_ERR_INVALID
    d.epilogue = 0
    d.lda = 3
    assert lib.mg_gemm(ctypes.byref(d), None, None, None, None, None) == _lib.MG_ERR_INVALID
    assert "leading dimension" in lib.mg_last_error().decode()
    assert lib.mg_gemm(None, None, None, None, None, None) == _lib.MG_ERR_INVALID


def test_empty_problem_is_a_no_op_without_device():
    lib = mg.load()
    d = _lib.GemmDesc()
    lib.mg_gemm_desc_init(ctypes.byref(d), 0, 7, 5, 0, 0)
    assert lib.mg_gemm(ctypes.byref(d), None, None, None, None, None) == _lib.MG_OK


def test_mode_switch():
    lib = mg.load()
    old = lib.mg_get_mode()
    assert lib.mg_set_mode(_lib.MG_MODE_TF32) == _lib.MG_OK
    assert lib.mg_get_mode() == _lib.MG_MODE_TF32
    assert lib.mg_set_mode(7) == _lib.MG_ERR_INVALID
    lib.mg_set_mode(old)
    assert lib.mg_get_mode() == old


def test_no_device_reports_cuda_error_not_abort():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    lib = mg.load()
    d = _lib.GemmDesc()
    lib.mg_gemm_desc_init(ctypes.byref(d), 4, 4, 4, 0, 0)
    buf = (ctypes.c_float * 16)()
    rc = lib.mg_gemm(ctypes.byref(d), buf, buf, buf, None, None)
    assert rc in (_lib.MG_ERR_CUDA, _lib.MG_ERR_UNSUPPORTED)


def test_softmax_backward_entry_errors_return_status():
    """mg_matmul_softmax_backward: P is required, its epilogue cannot be
    requested through mg_gemm (no P there), N <= 256, shapes as mg_matmul."""
    lib = mg.load()
    P = (ctypes.c_float * 16)()
    o, a, b = i32_array([4, 4]), i32_array([4, 8]), i32_array([4, 8])
    assert lib.mg_matmul_softmax_backward(None, None, None, None, o, a, b, 2, 0, 1, 1.0, None) == \
        _lib.MG_ERR_INVALID
    assert "P is NULL" in lib.mg_last_error().decode()
    bad = i32_array([4, 5])
    assert lib.mg_matmul_softmax_backward(None, None, None, P, bad, a, b, 2, 0, 1, 1.0, None) == \
        _lib.MG_ERR_INVALID
    d = _lib.GemmDesc()
    lib.mg_gemm_desc_init(ctypes.byref(d), 4, 4, 8, 0, 1)
    d.epilogue = 8                      # the internal softmax-backward flag
    buf = (ctypes.c_float * 64)()
    assert lib.mg_gemm(ctypes.byref(d), buf, buf, buf, None, None) == _lib.MG_ERR_INVALID
    lib.mg_gemm_desc_init(ctypes.byref(d), 4, 300, 8, 0, 1)
    d.epilogue = 8
    assert lib.mg_gemm(ctypes.byref(d), buf, buf, buf, None, None) == _lib.MG_ERR_INVALID


def _needed(path):
    out = subprocess.run(["readelf", "-d", path], capture_output=True, text=True, check=True).stdout
    return re.findall(r"\(NEEDED\)\s+Shared library: \[([^\]]+)\]", out)


def test_no_cublas_in_the_product_libraries():
    """No cuBLAS on the product path: neither the GEMM library nor the drop-in
    build of the reference (whose renamed cuBLASLt bodies are never called and
    resolve to shim/cublaslt_absent.c) needs a cuBLAS library at load time."""
    mg.load(build_if_missing=True)
    libs = [_lib.lib_path()]
    seam = os.path.join(ROOT, "macrograd_b200", "shim", "_build", "libmacrograd_seam.so")
    if os.path.exists(seam):
        libs.append(seam)
    for path in libs:
        needed = _needed(path)
        assert not [n for n in needed if "cublas" in n.lower()], f"{os.path.basename(path)} needs {needed}"
    if len(libs) == 2:
        assert any("mg_gemm" in n for n in _needed(seam)), "the drop-in build must link libmg_gemm.so"

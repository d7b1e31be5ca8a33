"""Drop-in check: the REFERENCE's own Tensor API on "cuda", with
kernel_ops::matmul / matmul_bias replaced by the seam
(macrograd_b200/shim/kernel_ops_matmul.inc), reaches the sm_100a kernels and
agrees with the oracle -- forward and the reference autograd backward.

Needs macrograd_b200/shim/_build/libmacrograd_seam.so, built from the
reference sources by `make -C macrograd_b200/shim` (build() does this where the
reference is present; the built library travels with the repository).
"""
import ctypes
import os

import numpy as np
import pytest

import oracle_bridge as ob

torch = pytest.importorskip("torch")
import macrograd_b200 as mg  # noqa: E402

pytestmark = pytest.mark.gpu

SEAM = os.path.join(ob.ROOT, "macrograd_b200", "shim", "_build", "libmacrograd_seam.so")
_P = ctypes.c_void_p
_I32P = ctypes.POINTER(ctypes.c_int32)


def _i32(v):
    v = [int(x) for x in v]
    return (ctypes.c_int32 * max(1, len(v)))(*v)


def _ptr(a):
    return a.ctypes.data_as(_P) if a is not None else None


@pytest.fixture(scope="module")
def seam():
    if not os.path.exists(SEAM):
        pytest.skip("seam library not built (needs the reference sources at build time)")
    mg.load()                       # the seam resolves libmg_gemm.so to this same copy
    lib = ctypes.CDLL(SEAM)
    lib.seam_matmul.argtypes = [_P, _P, _P, _P, _I32P, ctypes.c_int32, _I32P, ctypes.c_int32, _I32P,
                                ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
    lib.seam_matmul_backward.argtypes = [_P, _P, _P, _P, _P, _P, _P, _I32P, ctypes.c_int32, _I32P,
                                         ctypes.c_int32, _I32P, ctypes.c_int32, _I32P, ctypes.c_int32,
                                         ctypes.c_int32, ctypes.c_int32]
    return lib


def seam_matmul(lib, A, B, ta=False, tb=False, bias=None):
    out = np.empty(ob.oracle_matmul(A, B, ta, tb, bias).shape, np.float32)
    lib.seam_matmul(_ptr(out), _ptr(A), _ptr(B), _ptr(bias), _i32(A.shape), A.ndim, _i32(B.shape), B.ndim,
                    _i32(bias.shape) if bias is not None else None, bias.ndim if bias is not None else 0,
                    int(ta), int(tb))
    return out


@pytest.mark.parametrize("sa,sb,ta,tb,bias_shape", [
    ((8, 256, 384), (384, 384), False, False, None),          # config 1 forward
    ((512, 384), (1536, 384), False, True, (1536,)),          # config 2 layer, fewer rows
    ((2, 3, 256, 64), (2, 3, 256, 64), False, True, (256, 256)),   # score product + mask bias
    ((3, 33, 20), (1, 33, 44), True, False, None),
    ((5, 7), (7,), False, False, None),
])
def test_reference_api_forward_through_seam(seam, sa, sb, ta, tb, bias_shape):
    A = ob.seeded_uniform(sa, 11)
    B = ob.seeded_uniform(sb, 12)
    bias = ob.seeded_uniform(bias_shape, 13) if bias_shape else None
    n0 = mg.load().mg_launch_count()
    got = seam_matmul(seam, A, B, ta, tb, bias)
    assert mg.load().mg_launch_count() > n0, "the reference's matmul did not reach the sm_100a library"
    ref = ob.oracle_matmul(A, B, ta, tb, bias)
    assert ob.frob_rel_err(got, ref) <= 1e-5


def test_reference_autograd_backward_through_seam(seam):
    """Config 1 through the reference's own autograd on "cuda": A[8,256,384] @
    W[384,384], dC = ones; dA and the batch-reduced dW as the reference computes
    them (its `+=` broadcast reduction runs in the reference's own kernels)."""
    A = ob.seeded_uniform((8, 256, 384), 1)
    W = ob.seeded_uniform((384, 384), 1001)
    dC = np.ones((8, 256, 384), np.float32)
    dA = np.empty_like(A)
    dW = np.empty_like(W)
    n0 = mg.load().mg_launch_count()
    seam.seam_matmul_backward(_ptr(dA), _ptr(dW), None, _ptr(A), _ptr(W), None, _ptr(dC), _i32(A.shape), 3,
                              _i32(W.shape), 2, None, 0, _i32(dC.shape), 3, 0, 0)
    assert mg.load().mg_launch_count() >= n0 + 3   # forward + dA + dW GEMMs
    rA, rW, _ = ob.oracle_matmul_backward(A, W, dC)
    assert ob.frob_rel_err(dA, rA) <= 1e-5
    assert ob.frob_rel_err(dW, rW) <= 1e-5

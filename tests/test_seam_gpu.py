"""Drop-in check: the REFERENCE's own Tensor API on "cuda", with
kernel_ops::matmul / matmul_bias replaced by the seam
(macrograd_b200/shim/kernel_ops_matmul.inc), reaches the sm_100a kernels and
agrees with the oracle -- forward and the reference autograd backward.

Two builds, both from the reference sources by `make -C macrograd_b200/shim`
(build() does this where the reference is present; the built libraries
travel with the repository): libmacrograd_seam.so, the reference's code as it
is, and libmacrograd_seam_fused.so, the opt-in build whose tensor_ops.cpp is
patched (shim/fuse_tensor_ops.py) so that MatMulOp / MatMulBiasOp's gradient
`+=` is one accumulating GEMM (mg_matmul_accumulate), the bias gradient the
library's reduction (mg_sum_into), and Functional::matmul's output is
allocated without MemPool's zero fill. Every test runs on both.
"""
import ctypes
import os

import numpy as np
import pytest

import oracle_bridge as ob

torch = pytest.importorskip("torch")
import macrograd_b200 as mg  # noqa: E402

pytestmark = pytest.mark.gpu

BUILD = os.path.join(ob.ROOT, "macrograd_b200", "shim", "_build")
SEAMS = {"default": os.path.join(BUILD, "libmacrograd_seam.so"),
         "fused": os.path.join(BUILD, "libmacrograd_seam_fused.so")}
_P = ctypes.c_void_p
_I32P = ctypes.POINTER(ctypes.c_int32)


def _i32(v):
    v = [int(x) for x in v]
    return (ctypes.c_int32 * max(1, len(v)))(*v)


def _ptr(a):
    return a.ctypes.data_as(_P) if a is not None else None


@pytest.fixture(scope="module", params=sorted(SEAMS))
def seam(request):
    path = SEAMS[request.param]
    if not os.path.exists(path):
        pytest.skip(f"{os.path.basename(path)} not built (needs the reference sources at build time)")
    mg.load()                       # the seam resolves libmg_gemm.so to this same copy
    lib = ctypes.CDLL(path)
    lib.seam_shared_operand_backward.argtypes = [_P] * 6 + [_I32P, _I32P, _I32P, ctypes.c_int32]
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


def test_gradient_accumulates_into_a_nonzero_gradient(seam):
    """A feeds two products: its gradient receives dC1 W1^T, then dC2 W2^T is
    added to it (`internal_gradient() +=`, in the fused build a beta = 1 GEMM
    into the non-zero gradient)."""
    A = ob.seeded_uniform((4, 96, 80), 21)
    W1 = ob.seeded_uniform((80, 72), 22)
    W2 = ob.seeded_uniform((80, 72), 23)
    dC1 = ob.seeded_normal((4, 96, 72), 24)
    dC2 = ob.seeded_normal((4, 96, 72), 25)
    dA = np.empty_like(A)
    W1e, W2e = W1.reshape(1, 80, 72), W2.reshape(1, 80, 72)
    seam.seam_shared_operand_backward(_ptr(dA), _ptr(A), _ptr(W1e), _ptr(W2e), _ptr(dC1), _ptr(dC2),
                                      _i32(A.shape), _i32(W1e.shape), _i32(dC1.shape), 3)
    r1, _, _ = ob.oracle_matmul_backward(A, W1e, dC1)
    r2, _, _ = ob.oracle_matmul_backward(A, W2e, dC2)
    assert ob.frob_rel_err(dA, r1 + r2) <= 1e-5


@pytest.mark.parametrize("sa,sb,tb,bias_shape", [
    ((6, 64, 96), (96, 80), False, (80,)),       # batched input, 2-D weight, row bias
    ((300, 96), (160, 96), True, (1, 160)),      # linear layer, W stored [out, in]
])
def test_reference_bias_backward_through_seam(seam, sa, sb, tb, bias_shape):
    """MatMulBiasOp::_backward through the reference autograd: the weight's
    gradient summed over the batch and the bias gradient (dC summed to the
    bias shape) against the oracle."""
    A = ob.seeded_uniform(sa, 31)
    B = ob.seeded_uniform(sb, 32)
    bias = ob.seeded_uniform(bias_shape, 33)
    C = ob.oracle_matmul(A, B, False, tb, bias)
    dC = ob.seeded_normal(C.shape, 34)
    dA, dB, db = np.empty_like(A), np.empty_like(B), np.empty_like(bias)
    seam.seam_matmul_backward(_ptr(dA), _ptr(dB), _ptr(db), _ptr(A), _ptr(B), _ptr(bias), _ptr(dC),
                              _i32(A.shape), A.ndim, _i32(B.shape), B.ndim, _i32(bias.shape), bias.ndim,
                              _i32(dC.shape), dC.ndim, 0, int(tb))
    rA, rB, rb = ob.oracle_matmul_backward(A, B, dC, False, tb, bias.shape)
    assert ob.frob_rel_err(dA, rA) <= 1e-5
    assert ob.frob_rel_err(dB, rB) <= 1e-5
    assert ob.frob_rel_err(db, rb) <= 1e-5

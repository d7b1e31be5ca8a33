"""Test-side bridge to the oracle (oracle/liboracle.so, and the reference build
oracle/_ref/libmgref.so when present). Test infrastructure only.

The helpers take numpy float32 arrays with the shapes a user passes to
Functional::matmul and apply the same rank equalisation
(tensor_ops.cpp:4547-4579) before calling the C restatement.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
ORACLE_LIB = os.path.join(ORACLE_DIR, "liboracle.so")
REF_LIB = os.path.join(ORACLE_DIR, "_ref", "libmgref.so")

_P = ctypes.c_void_p
_I32P = ctypes.POINTER(ctypes.c_int32)
_oracle = None
_ref = None


def _i32(v):
    v = [int(x) for x in v]
    return (ctypes.c_int32 * max(1, len(v)))(*v)


def _ptr(a):
    return a.ctypes.data_as(_P) if a is not None else None


def oracle():
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_LIB):
            subprocess.run(["make", "-s", "-C", ORACLE_DIR, "liboracle.so"], check=True)
        lib = ctypes.CDLL(ORACLE_LIB)
        lib.oracle_matmul.restype = ctypes.c_int
        lib.oracle_matmul.argtypes = [_P, _P, _P, _P, _I32P, _I32P, _I32P, _I32P, ctypes.c_int32,
                                      ctypes.c_int32, ctypes.c_int32]
        lib.oracle_softmax_rows.argtypes = [_P, _P, ctypes.c_int64, ctypes.c_int64]
        lib.oracle_causal_mask.argtypes = [_P, ctypes.c_int32]
        lib.oracle_reduce_to.argtypes = [_P, _P, _I32P, _I32P, ctypes.c_int32]
        lib.oracle_rng_set_seed.argtypes = [ctypes.c_uint64]
        lib.oracle_rng_uniform.argtypes = [_P, ctypes.c_int64, ctypes.c_float, ctypes.c_float]
        lib.oracle_rng_normal.argtypes = [_P, ctypes.c_int64, ctypes.c_float, ctypes.c_float]
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def ref():
    """The reference's own CPU code (oracle/_ref/libmgref.so); None if not built."""
    global _ref
    if _ref is None and ref_available():
        lib = ctypes.CDLL(REF_LIB)
        lib.ref_matmul.restype = ctypes.c_int
        lib.ref_matmul.argtypes = [_P, ctypes.POINTER(ctypes.c_int64), _P, _P, _P, _I32P, ctypes.c_int32,
                                   _I32P, ctypes.c_int32, _I32P, ctypes.c_int32, ctypes.c_int32,
                                   ctypes.c_int32]
        lib.ref_matmul_backward.restype = ctypes.c_int
        lib.ref_matmul_backward.argtypes = [_P, _P, _P, _P, _P, _P, _P, _I32P, ctypes.c_int32, _I32P,
                                            ctypes.c_int32, _I32P, ctypes.c_int32, _I32P,
                                            ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
        lib.ref_softmax_lastdim.argtypes = [_P, _P, ctypes.c_int64, ctypes.c_int64]
        lib.ref_softmax_backward.restype = ctypes.c_int
        lib.ref_softmax_backward.argtypes = [_P, _P, _P, _P, ctypes.c_int64, ctypes.c_int64]
        lib.ref_causal_mask.argtypes = [_P, ctypes.c_int32]
        lib.ref_init_uniform.argtypes = [_P, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float, ctypes.c_float]
        lib.ref_init_normal.argtypes = [_P, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float, ctypes.c_float]
        lib.ref_matmul_rows_mp.restype = ctypes.c_int
        lib.ref_matmul_rows_mp.argtypes = [_P, _P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                           ctypes.c_int32]
        _ref = lib
    return _ref


# ------------------------------------------------------------------ inputs
def seeded_uniform(shape, seed, lo=-1.0, hi=1.0):
    """Random::set_seed(seed) + Initialization::uniform(t, lo, hi) on a CPU tensor."""
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, np.float32)
    lib = oracle()
    lib.oracle_rng_set_seed(seed)
    lib.oracle_rng_uniform(_ptr(out), n, lo, hi)
    return out.reshape(shape)


def seeded_normal(shape, seed, mean=0.0, std=1.0):
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, np.float32)
    lib = oracle()
    lib.oracle_rng_set_seed(seed)
    lib.oracle_rng_normal(_ptr(out), n, mean, std)
    return out.reshape(shape)


def seeded_stream(seed):
    """Consecutive fills from one seeded stream (set_seed once, then several
    Initialization calls), returned as a callable(kind, shape, a, b)."""
    lib = oracle()
    lib.oracle_rng_set_seed(seed)

    def fill(kind, shape, a=-1.0, b=1.0):
        n = int(np.prod(shape))
        out = np.empty(n, np.float32)
        if kind == "uniform":
            lib.oracle_rng_uniform(_ptr(out), n, a, b)
        else:
            lib.oracle_rng_normal(_ptr(out), n, a, b)
        return out.reshape(shape)

    return fill


# ------------------------------------------------------------------ matmul
def equalize(a_shape, b_shape, transA, transB):
    a, b = list(a_shape), list(b_shape)
    a1, b1 = len(a) == 1, len(b) == 1
    if a1:
        a = [1] + a
    if b1:
        b = b + [1]
    while len(a) > len(b):
        b = [1] + b
    while len(b) > len(a):
        a = [1] + a
    out = [max(x, y) for x, y in zip(a[:-2], b[:-2])]
    out += [a[-1] if transA else a[-2], b[-2] if transB else b[-1]]
    return a, b, out, a1, b1


def oracle_matmul(A, B, transA=False, transB=False, bias=None):
    """Functional::matmul on "cpu" (C restatement), any shapes it accepts."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    a, b, o, a1, b1 = equalize(A.shape, B.shape, transA, transB)
    out = np.empty(o, np.float32)
    bs = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, np.float32)
        bs = [1] * (len(o) - bias.ndim) + list(bias.shape)
    rc = oracle().oracle_matmul(_ptr(out), _ptr(A), _ptr(B), _ptr(bias), _i32(o), _i32(a), _i32(b),
                                _i32(bs) if bs else None, len(o), int(transA), int(transB))
    if rc != 0:
        raise ValueError(f"oracle_matmul rejected the shapes (code {rc})")
    if a1:
        out = out.squeeze(-2)
    if b1:
        out = out.squeeze(-1)
    return out


def oracle_reduce_to(src, dst_shape):
    """src summed over the dims where dst_shape is 1, like `grad += tmp`."""
    src = np.ascontiguousarray(src, np.float32)
    dst = np.zeros(dst_shape, np.float32)
    oracle().oracle_reduce_to(_ptr(dst), _ptr(src), _i32(dst_shape), _i32(src.shape), len(dst_shape))
    return dst


def oracle_matmul_backward(A, B, dC, transA=False, transB=False, bias_shape=None):
    """The GEMMs of MatMulOp::_backward (tensor_ops.cpp:4504-4517) through the
    oracle, with the `+=` reduction of a broadcast operand's gradient."""
    a, b, o, _, _ = equalize(A.shape, B.shape, transA, transB)
    Av, Bv, dCv = A.reshape(a), B.reshape(b), dC.reshape(o)
    if transA:
        tA = oracle_matmul(Bv, dCv, transB, True)
    else:
        tA = oracle_matmul(dCv, Bv, False, not transB)
    if transB:
        tB = oracle_matmul(dCv, Av, True, transA)
    else:
        tB = oracle_matmul(Av, dCv, not transA, False)
    dA = oracle_reduce_to(tA, a).reshape(A.shape)
    dB = oracle_reduce_to(tB, b).reshape(B.shape)
    dbias = None
    if bias_shape is not None:
        bs = [1] * (len(o) - len(bias_shape)) + list(bias_shape)
        dbias = oracle_reduce_to(dCv, bs).reshape(bias_shape)
    return dA, dB, dbias


def oracle_softmax_rows(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    n = x.shape[-1]
    oracle().oracle_softmax_rows(_ptr(out), _ptr(x), x.size // n if n else 0, n)
    return out


def oracle_causal_mask(L):
    out = np.empty((L, L), np.float32)
    oracle().oracle_causal_mask(_ptr(out), L)
    return out


def ref_matmul(A, B, transA=False, transB=False, bias=None):
    """Functional::matmul through the reference's own compiled CPU code."""
    lib = ref()
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    _, _, o, a1, b1 = equalize(A.shape, B.shape, transA, transB)
    if a1:
        o = o[:-2] + [o[-1]]
    if b1:
        o = o[:-1]
    out = np.empty(o if o else [1], np.float32)
    n = ctypes.c_int64()
    if bias is not None:
        bias = np.ascontiguousarray(bias, np.float32)
    lib.ref_matmul(_ptr(out), ctypes.byref(n), _ptr(A), _ptr(B), _ptr(bias), _i32(A.shape), A.ndim,
                   _i32(B.shape), B.ndim, _i32(bias.shape) if bias is not None else None,
                   bias.ndim if bias is not None else 0, int(transA), int(transB))
    assert n.value == out.size
    return out


def ref_matmul_backward(A, B, dC, transA=False, transB=False, bias=None):
    lib = ref()
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    dC = np.ascontiguousarray(dC, np.float32)
    dA = np.empty_like(A)
    dB = np.empty_like(B)
    db = np.empty_like(bias) if bias is not None else None
    lib.ref_matmul_backward(_ptr(dA), _ptr(dB), _ptr(db), _ptr(A), _ptr(B), _ptr(bias), _ptr(dC),
                            _i32(A.shape), A.ndim, _i32(B.shape), B.ndim,
                            _i32(bias.shape) if bias is not None else None,
                            bias.ndim if bias is not None else 0, _i32(dC.shape), dC.ndim,
                            int(transA), int(transB))
    return dA, dB, db


def ref_softmax_rows(x):
    """Tensor::softmax(-1) through the reference's own compiled CPU code."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    n = x.shape[-1]
    ref().ref_softmax_lastdim(_ptr(out), _ptr(x), x.size // n if n else 0, n)
    return out


def ref_softmax_backward(S, G):
    """P = Tensor::softmax(S, -1) and the gradient of sum(P * G) with respect to
    S, through the reference's own autograd (SoftOp::_backward)."""
    S = np.ascontiguousarray(S, np.float32)
    G = np.ascontiguousarray(G, np.float32)
    P = np.empty_like(S)
    dS = np.empty_like(S)
    n = S.shape[-1]
    ref().ref_softmax_backward(_ptr(dS), _ptr(P), _ptr(S), _ptr(G), S.size // n, n)
    return P, dS


# ------------------------------------------------------------------ metrics
def frob_rel_err(x, ref):
    """||x - ref||_F / ||ref||_F in float64 (the Frobenius-normalised error the
    tolerances 1e-5 (3xTF32) and 2e-3 (TF32) are stated in)."""
    x = np.asarray(x, np.float64)
    r = np.asarray(ref, np.float64)
    den = np.linalg.norm(r.ravel())
    num = np.linalg.norm((x - r).ravel())
    return float(num / den) if den > 0 else float(num)


def max_rel_err(x, ref):
    """max |x - ref| / rms(ref): the worst element against the typical magnitude."""
    x = np.asarray(x, np.float64)
    r = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(r * r)) if r.size else 0.0
    m = float(np.max(np.abs(x - r))) if r.size else 0.0
    return m / rms if rms > 0 else m

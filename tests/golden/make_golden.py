"""Generates tests/golden/matmul_golden.npz from the REFERENCE ITSELF.

Run in a container that has the reference sources, after
`make -C oracle ref REF=/path/to/macrograd`
built oracle/_ref/libmgref.so from them:

    python tests/golden/make_golden.py

Every output in the fixture comes from the reference's own compiled CPU code
(Functional::matmul, its autograd backward, Tensor::softmax and its
backward, Functional::causal_mask, Random + Initialization), called through
oracle/ref_driver.cpp. Inputs come from the reference's CPU random stream. The
fixture is small (a few tens of KB) and is what pins the oracle restatement
and the GPU kernels where the reference cannot be built (the GPU box).
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import oracle_bridge as ob  # noqa: E402

# (name, A shape, B shape, bias shape or None, transA, transB, seed)
FORWARD = [
    ("bcast_b", (2, 3, 5, 7), (7, 6), None, False, False, 11),
    ("trans_a", (4, 9, 5), (4, 9, 3), None, True, False, 12),
    ("trans_b", (6, 33), (17, 33), None, False, True, 13),
    ("trans_ab", (2, 1, 8, 10), (1, 3, 12, 8), None, True, True, 14),
    ("bias_row", (20, 16), (24, 16), (24,), False, True, 15),
    ("bias_full", (2, 2, 8, 4), (2, 2, 8, 4), (8, 8), False, True, 16),
    ("bias_col", (3, 7, 5), (5, 9), (7, 1), False, False, 17),
    ("gemv", (5, 7), (7,), None, False, False, 18),
    ("vecmat", (7,), (7, 3), None, False, False, 19),
    ("k65", (4, 65), (65, 3), None, False, False, 20),
    ("blocked_k", (70, 130), (130, 66), None, False, False, 21),
]

# (name, A shape, B shape, bias shape or None, transA, transB, dC kind, seed)
BACKWARD = [
    ("cfg1_small", (3, 16, 12), (12, 10), None, False, False, "ones", 31),
    ("linear_bias", (12, 8), (6, 8), (6,), False, True, "normal", 32),
    ("attn_like", (2, 3, 8, 4), (2, 3, 8, 4), None, False, True, "normal", 33),
    ("trans_a_bwd", (2, 9, 5), (2, 9, 3), None, True, False, "normal", 34),
    ("bias_full_bwd", (2, 2, 8, 4), (2, 2, 8, 4), (8, 8), False, True, "normal", 35),
    ("bias_col_bwd", (3, 7, 5), (5, 9), (7, 1), False, False, "normal", 36),
]


def main():
    if not ob.ref_available():
        raise SystemExit("oracle/_ref/libmgref.so is missing: run `make -C oracle ref` first")
    ref = ob.ref()
    out = {}

    def uniform(n, seed):
        buf = np.empty(n, np.float32)
        ref.ref_init_uniform(buf.ctypes.data_as(ctypes.c_void_p), n, seed, -1.0, 1.0)
        return buf

    def normal(n, seed):
        buf = np.empty(n, np.float32)
        ref.ref_init_normal(buf.ctypes.data_as(ctypes.c_void_p), n, seed, 0.0, 1.0)
        return buf

    out["rng_uniform_seed7"] = uniform(257, 7)
    out["rng_normal_seed7"] = normal(257, 7)

    for name, sa, sb, sbias, ta, tb, seed in FORWARD:
        A = uniform(int(np.prod(sa)), seed).reshape(sa)
        B = uniform(int(np.prod(sb)), seed + 1000).reshape(sb)
        bias = uniform(int(np.prod(sbias)), seed + 2000).reshape(sbias) if sbias else None
        if name == "bias_full":
            mask = np.empty((8, 8), np.float32)
            ref.ref_causal_mask(mask.ctypes.data_as(ctypes.c_void_p), 8)
            bias = mask
        C = ob.ref_matmul(A, B, ta, tb, bias)
        out[f"fwd/{name}/A"] = A
        out[f"fwd/{name}/B"] = B
        if bias is not None:
            out[f"fwd/{name}/bias"] = bias
        out[f"fwd/{name}/C"] = C
        out[f"fwd/{name}/flags"] = np.array([int(ta), int(tb)], np.int32)

    for name, sa, sb, sbias, ta, tb, kind, seed in BACKWARD:
        A = uniform(int(np.prod(sa)), seed).reshape(sa)
        B = uniform(int(np.prod(sb)), seed + 1000).reshape(sb)
        bias = uniform(int(np.prod(sbias)), seed + 2000).reshape(sbias) if sbias else None
        C = ob.ref_matmul(A, B, ta, tb, bias)
        dC = np.ones_like(C) if kind == "ones" else normal(C.size, seed + 3000).reshape(C.shape)
        dA, dB, db = ob.ref_matmul_backward(A, B, dC, ta, tb, bias)
        for k, v in (("A", A), ("B", B), ("C", C), ("dC", dC), ("dA", dA), ("dB", dB)):
            out[f"bwd/{name}/{k}"] = v
        if bias is not None:
            out[f"bwd/{name}/bias"] = bias
            out[f"bwd/{name}/dbias"] = db
        out[f"bwd/{name}/flags"] = np.array([int(ta), int(tb)], np.int32)

    # causal mask + row softmax of a scaled, masked score block (config-3 shape, small)
    L = 9
    mask = np.empty((L, L), np.float32)
    ref.ref_causal_mask(mask.ctypes.data_as(ctypes.c_void_p), L)
    Q = normal(2 * L * 4, 41).reshape(2, L, 4)
    K = normal(2 * L * 4, 42).reshape(2, L, 4)
    S = ob.ref_matmul(Q * np.float32(0.5), K, False, True, mask)
    P = np.empty_like(S)
    ref.ref_softmax_lastdim(P.ctypes.data_as(ctypes.c_void_p), S.ctypes.data_as(ctypes.c_void_p),
                            S.size // L, L)
    out["attn/mask"] = mask
    out["attn/Q"] = Q
    out["attn/K"] = K
    out["attn/S"] = S
    out["attn/P"] = P

    # the softmax derivative through the reference's autograd (SoftOp::_backward)
    # on that masked block, for a seeded upstream gradient
    G = normal(S.size, 43).reshape(S.shape)
    P2, dS = ob.ref_softmax_backward(S, G)
    assert np.array_equal(P2, P)
    out["softmax_bwd/G"] = G
    out["softmax_bwd/dS"] = dS

    path = os.path.join(HERE, "matmul_golden.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes,", len(out), "arrays")


if __name__ == "__main__":
    main()

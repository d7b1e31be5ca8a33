"""Gradient accumulation as the library runs it: every `grad += matmul(...)`
of MatMulOp / MatMulBiasOp::_backward (tensor_ops.cpp:4504-4517, :4723-4737)
is ONE GEMM (mg_matmul_accumulate) -- the `+=` broadcast reduction of a
broadcast operand's gradient (tensor_ops.cpp:3345-3451) summed inside the
kernel's K loop, beta = 1 into an existing gradient -- and the bias gradient
`bias.grad += out.grad` is the library's own deterministic reduction
(mg_sum_into). Checked against the oracle's restatement of the reference's
GEMMs followed by its `+=` reduction (oracle_matmul_backward,
oracle_reduce_to), in both modes, with the tolerance of test_gemm_gpu.py.
"""
import numpy as np
import pytest

import oracle_bridge as ob

torch = pytest.importorskip("torch")
import macrograd_b200 as mg  # noqa: E402
from macrograd_b200 import _lib, functional as F  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = {_lib.MG_MODE_TF32X3: 1e-5, _lib.MG_MODE_TF32: 2e-3}
MODES = [_lib.MG_MODE_TF32X3, _lib.MG_MODE_TF32]


@pytest.fixture(autouse=True)
def _mode_guard():
    lib = mg.load()
    old = lib.mg_get_mode()
    yield
    lib.mg_set_mode(old)


def cuda(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def close(x, ref, mode, what):
    assert x.shape == ref.shape, f"{what}: {x.shape} vs {ref.shape}"
    assert np.all(np.isfinite(x)), what
    e = ob.frob_rel_err(x, ref)
    assert e <= TOL[mode], f"{what}: frobenius rel err {e:.3e} > {TOL[mode]:.0e}"


# (A storage shape, B storage shape, transA, transB): forms whose gradients
# reduce over broadcast leading dims (the weight of a batched product, mixed
# 4-D broadcasts), K not a multiple of 32 inside each reduction step, all
# four transpose combinations, and a reduction long enough for the K split.
CASES = [
    ((8, 256, 384), (384, 384), False, False),      # config 1: dW summed over the batch of 8
    ((8, 256, 384), (384, 384), False, True),       # the same with W stored [N, K]
    ((6, 70, 33), (70, 50), True, False),           # A stored [K, M], K = 70 per step
    ((5, 40, 33), (1, 20, 40), True, True),
    ((2, 1, 40, 33), (1, 3, 33, 20), False, False),  # dA sums over dim 1, dB over dim 0
    ((3, 1, 45, 64), (3, 4, 96, 64), False, True),
    ((64, 100, 96), (96, 80), False, False),        # 64 steps x 4 K-blocks on one tile: K split
    ((96, 80), (4, 7, 80, 24), False, False),       # A broadcast over two dims
]


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("sa,sb,ta,tb", CASES)
def test_gradient_gemms_reduce_in_the_kernel(mode, sa, sb, ta, tb):
    assert mg.load().mg_set_mode(mode) == 0
    A = ob.seeded_uniform(sa, 700)
    B = ob.seeded_uniform(sb, 701)
    _, _, o, _, _ = F.equalize(sa, sb, ta, tb)
    dC = ob.seeded_normal(tuple(o), 702)
    n0 = mg.load().mg_launch_count()
    dA, dB, _ = F.matmul_backward(cuda(A), cuda(B), cuda(dC), ta, tb)
    torch.cuda.synchronize()
    # one GEMM launch per gradient, whatever the broadcast (no temporary, no
    # reduction pass) -- plus a re-layout copy for an operand whose rows are
    # not a multiple of 16 bytes (TMA's rule)
    if all(s[-1] % 4 == 0 for s in (sa, sb, o)):
        assert mg.load().mg_launch_count() - n0 == 2
    rA, rB, _ = ob.oracle_matmul_backward(A, B, dC, ta, tb)
    close(host(dA), rA, mode, "dA")
    close(host(dB), rB, mode, "dB")


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("sa,sb,ta,tb", [CASES[0], CASES[2], CASES[4], CASES[6]])
def test_gradient_gemms_accumulate_with_beta_one(mode, sa, sb, ta, tb):
    """grad_a / grad_b given: the GEMM adds into them (the reference's `+=`
    into internal_gradient()), including across a K split."""
    assert mg.load().mg_set_mode(mode) == 0
    A = ob.seeded_uniform(sa, 710)
    B = ob.seeded_uniform(sb, 711)
    _, _, o, _, _ = F.equalize(sa, sb, ta, tb)
    dC = ob.seeded_normal(tuple(o), 712)
    prevA = ob.seeded_normal(sa, 713)
    prevB = ob.seeded_normal(sb, 714)
    gA, gB = cuda(prevA), cuda(prevB)
    rA, rB = F.matmul_backward(cuda(A), cuda(B), cuda(dC), ta, tb, grad_a=gA, grad_b=gB)[:2]
    assert rA.data_ptr() == gA.data_ptr() and rB.data_ptr() == gB.data_ptr()
    oA, oB, _ = ob.oracle_matmul_backward(A, B, dC, ta, tb)
    close(host(gA), prevA + oA, mode, "grad_a += dA")
    close(host(gB), prevB + oB, mode, "grad_b += dB")


@pytest.mark.parametrize("mode", MODES)
def test_two_dimensional_weight_accumulates_with_beta_one(mode):
    """A linear layer's 2-D weight and input: dX += dY W and dW += dY^T X
    (tensor_ops.cpp:4504-4517 with transB), each one beta = 1 GEMM, and the
    bias gradient += the column sums of dY."""
    assert mg.load().mg_set_mode(mode) == 0
    X = ob.seeded_uniform((1000, 96), 720)
    W = ob.seeded_uniform((160, 96), 721)
    b = ob.seeded_uniform((160,), 722)
    dY = ob.seeded_normal((1000, 160), 723)
    pX, pW, pb = ob.seeded_normal((1000, 96), 724), ob.seeded_normal((160, 96), 725), ob.seeded_normal((160,), 726)
    gX, gW, gb = cuda(pX), cuda(pW), cuda(pb)
    F.matmul_backward(cuda(X), cuda(W), cuda(dY), False, True, True, (160,), grad_a=gX, grad_b=gW, grad_bias=gb)
    rX, rW, rb = ob.oracle_matmul_backward(X, W, dY, False, True, (160,))
    close(host(gX), pX + rX, mode, "dX")
    close(host(gW), pW + rW, mode, "dW")
    close(host(gb), pb + rb, _lib.MG_MODE_TF32X3, "dbias")


# (src shape, dst shape): the bias-gradient forms (row bias over a batch of
# rows, a mask bias over batch and heads), inner and interleaved reductions,
# widths that do / do not allow float4 columns, and a plain copy.
SUMS = [
    ((16384, 1536), (1, 1536)),
    ((64, 256, 384), (1, 1, 384)),
    ((4, 6, 256, 256), (1, 1, 256, 256)),
    ((1000, 65), (1, 65)),
    ((30, 40), (30, 1)),
    ((2, 3, 4, 5), (2, 1, 4, 1)),
    ((7, 1, 9), (1, 1, 9)),
    ((3, 5), (3, 5)),
    ((50000,), (1,)),
]


@pytest.mark.parametrize("beta", [0.0, 1.0])
@pytest.mark.parametrize("src_shape,dst_shape", SUMS)
def test_sum_into_matches_the_reference_reduction(src_shape, dst_shape, beta):
    """A sum's fp32 rounding depends on its order, and the reference's order
    (one running sum) differs from a parallel one; both are held to the same
    bound against the exact (float64) sum: per output, 1e-6 of the summed
    magnitudes (sum of |x|) -- a sum of n terms in any order is within
    about n * 2^-24 of them, and n here is at most 50000."""
    src = ob.seeded_normal(src_shape, 730)
    prev = ob.seeded_normal(dst_shape, 731)
    g = cuda(prev) if beta else None
    got = host(F.sum_into(cuda(src), dst_shape, g)).astype(np.float64)
    dims = tuple(i for i, (a, b) in enumerate(zip(src_shape, dst_shape)) if a != b)
    exact = src.astype(np.float64).sum(axis=dims, keepdims=True) + (prev if beta else 0.0)
    mass = np.abs(src.astype(np.float64)).sum(axis=dims, keepdims=True) + (np.abs(prev) if beta else 0.0)
    oracle = ob.oracle_reduce_to(src, list(dst_shape)).astype(np.float64) + (prev if beta else 0.0)
    for name, x in (("library", got), ("oracle", oracle)):
        worst = float(np.max(np.abs(x - exact) / np.maximum(mass, 1e-30)))
        assert worst <= 1e-6, f"{name} {src_shape}->{dst_shape}: error {worst:.2e} of the summed magnitudes"
    # deterministic: the same call gives the same bits
    again = host(F.sum_into(cuda(src), dst_shape, cuda(prev) if beta else None)).astype(np.float64)
    assert np.array_equal(got, again)


def test_no_wait_timed_out():
    import ctypes

    detail = ctypes.c_int32(0)
    st = mg.load().mg_device_status(ctypes.byref(detail), 0)
    assert st == 0, f"device status {st}, wait site {detail.value}"

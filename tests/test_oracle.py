"""The oracle pinned: C restatement vs the reference's golden outputs (and vs
the reference build itself when present), and the README known-answer test."""
import numpy as np
import pytest

import oracle_bridge as ob

GOLDEN = np.load(__import__("os").path.join(ob.ROOT, "tests", "golden", "matmul_golden.npz"))


def _cases(prefix):
    return sorted({k.split("/")[1] for k in GOLDEN.files if k.startswith(prefix + "/")})


def test_rng_restatement_matches_reference_stream():
    assert np.array_equal(ob.seeded_uniform((257,), 7), GOLDEN["rng_uniform_seed7"])
    assert np.array_equal(ob.seeded_normal((257,), 7), GOLDEN["rng_normal_seed7"])


@pytest.mark.parametrize("name", _cases("fwd"))
def test_oracle_forward_bit_exact_vs_golden(name):
    g = lambda k: GOLDEN[f"fwd/{name}/{k}"]
    ta, tb = (bool(x) for x in g("flags"))
    bias = GOLDEN[f"fwd/{name}/bias"] if f"fwd/{name}/bias" in GOLDEN.files else None
    C = ob.oracle_matmul(g("A"), g("B"), ta, tb, bias)
    assert C.shape == g("C").shape
    assert np.array_equal(C, g("C")), f"max diff {np.abs(C - g('C')).max()}"


@pytest.mark.parametrize("name", _cases("bwd"))
def test_oracle_backward_bit_exact_vs_golden(name):
    g = lambda k: GOLDEN[f"bwd/{name}/{k}"]
    ta, tb = (bool(x) for x in g("flags"))
    has_bias = f"bwd/{name}/bias" in GOLDEN.files
    bias = g("bias") if has_bias else None
    assert np.array_equal(ob.oracle_matmul(g("A"), g("B"), ta, tb, bias), g("C"))
    dA, dB, db = ob.oracle_matmul_backward(g("A"), g("B"), g("dC"), ta, tb,
                                           bias.shape if has_bias else None)
    assert np.array_equal(dA, g("dA"))
    assert np.array_equal(dB, g("dB"))
    if has_bias:
        assert np.array_equal(db, g("dbias"))


def test_oracle_mask_and_softmax_vs_golden():
    L = GOLDEN["attn/mask"].shape[0]
    assert np.array_equal(ob.oracle_causal_mask(L), GOLDEN["attn/mask"])
    S = ob.oracle_matmul(GOLDEN["attn/Q"] * np.float32(0.5), GOLDEN["attn/K"], False, True,
                         GOLDEN["attn/mask"])
    assert np.array_equal(S, GOLDEN["attn/S"])
    assert np.array_equal(ob.oracle_softmax_rows(S), GOLDEN["attn/P"])


def _softmax_backward_expr(P, G):
    """The expected values the fused softmax-backward epilogue is tested
    against: P * (G - rowsum(P * G)) in float64."""
    P64, G64 = P.astype(np.float64), G.astype(np.float64)
    return P64 * (G64 - (P64 * G64).sum(-1, keepdims=True))


def test_softmax_backward_expression_is_the_references_vs_golden():
    """On the reference's own softmax derivative (SoftOp::_backward through its
    autograd, golden) the float64 expression agrees to fp32 rounding, and the
    masked (-inf) scores get exactly zero gradient in both."""
    S, P = GOLDEN["attn/S"], GOLDEN["attn/P"]
    dS = GOLDEN["softmax_bwd/dS"]
    expr = _softmax_backward_expr(P, GOLDEN["softmax_bwd/G"])
    assert ob.frob_rel_err(expr.astype(np.float32), dS) <= 1e-6
    masked = np.isneginf(S)
    assert masked.any() and np.all(dS[masked] == 0) and np.all(expr[masked] == 0)


@pytest.mark.skipif(not ob.ref_available(), reason="reference build oracle/_ref not present")
def test_softmax_backward_expression_is_the_references_vs_reference_build():
    S = ob.seeded_normal((3, 40, 256), 44, 0.0, 2.0)
    S[..., 200:] = np.where(ob.seeded_uniform((3, 40, 56), 45) > 0, -np.inf, S[..., 200:])
    G = ob.seeded_normal((3, 40, 256), 46)
    P, dS = ob.ref_softmax_backward(S, G)
    assert ob.frob_rel_err(_softmax_backward_expr(P, G).astype(np.float32), dS) <= 1e-6


# README.md:166-235: least squares A x = y by gradient descent through
# Functional::matmul (GEMV: B is 1-D) and mean_squared_error; printed losses
# and final parameters / gradients to 4 decimals.
README_DATA = np.array([[+0.2, +1.0, +0.2, -2.0],
                        [+0.5, -1.1, +1.4, +2.0],
                        [+0.2, -1.4, +0.7, -2.0],
                        [+3.0, +1.0, -2.1, -1.2]], np.float32)
README_TARGET = np.array([+1.3, -2.5, +0.2, -0.1], np.float32)
README_LOSSES = [1.9975, 0.6437, 0.3287, 0.1824, 0.1077, 0.0668, 0.0432, 0.0292, 0.0207, 0.0153]
README_FINAL_PARAMS = [-0.5934, +0.4394, -0.2778, -0.5795]
README_FINAL_GRAD = [+0.1446, -0.0588, +0.1176, -0.0043]


def readme_least_squares(matmul, matmul_grad_b):
    """The README loop with the two GEMMs supplied by the caller; the MSE and
    its gradient restated in float32 as tensor_ops.cpp:5099-5106, 5154-5162."""
    params = np.zeros(4, np.float32)
    losses = []
    grad = None
    for _ in range(10):
        preds = matmul(README_DATA, params)                      # [4,4] @ [4] -> [4]
        d = (preds - README_TARGET).astype(np.float32)
        loss = np.float32(0)
        for v in d:
            loss = np.float32(loss + v * v)
        loss = np.float32(loss / np.float32(4))
        deriv = (d * np.float32(1.0 * (2.0 / 4))).astype(np.float32)  # internal_multiply(grad=1, 2/n)
        grad = matmul_grad_b(README_DATA, deriv)                  # dB = A^T dC
        params = (params + np.float32(-0.1) * grad).astype(np.float32)
        losses.append(float(loss))
    return losses, params, grad


def test_readme_known_answer_through_oracle():
    losses, params, grad = readme_least_squares(
        lambda A, x: ob.oracle_matmul(A, x),
        lambda A, dC: ob.oracle_matmul(A, dC.reshape(4, 1), True, False).reshape(4))
    assert np.allclose(losses, README_LOSSES, atol=5e-5)
    assert np.allclose(params, README_FINAL_PARAMS, atol=5e-5)
    assert np.allclose(grad, README_FINAL_GRAD, atol=5e-5)


@pytest.mark.skipif(not ob.ref_available(), reason="reference build oracle/_ref not present")
@pytest.mark.parametrize("shape", [((3, 70, 130), (130, 65), 0, 0), ((2, 1, 33, 17), (1, 4, 17, 9), 0, 0),
                                   ((5, 40, 30), (5, 50, 30), 0, 1), ((40, 30), (40, 50), 1, 0),
                                   ((2, 64, 129), (2, 65, 64), 1, 1)])
def test_oracle_bit_exact_vs_reference_build(shape):
    sa, sb, ta, tb = shape
    A = ob.seeded_uniform(sa, 5)
    B = ob.seeded_uniform(sb, 6)
    assert np.array_equal(ob.oracle_matmul(A, B, ta, tb), ob.ref_matmul(A, B, ta, tb))


@pytest.mark.skipif(not ob.ref_available(), reason="reference build oracle/_ref not present")
def test_reference_row_sliced_processes_equal_one_call():
    A = ob.seeded_uniform((37, 50), 8)
    B = ob.seeded_uniform((50, 21), 9)
    C = np.empty((37, 21), np.float32)
    rc = ob.ref().ref_matmul_rows_mp(ob._ptr(C), ob._ptr(A), ob._ptr(B), 37, 21, 50, 4)
    assert rc == 0
    assert np.array_equal(C, ob.ref_matmul(A, B))

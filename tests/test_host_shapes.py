"""Host mirror of Functional::matmul's shape logic (no GPU needed)."""
import pytest

from macrograd_b200 import functional as F
from macrograd_b200._lib import MacrogradError


@pytest.mark.parametrize("a,b,ta,tb,out", [
    ((8, 256, 384), (384, 384), False, False, [8, 256, 384]),
    ((16384, 384), (1536, 384), False, True, [16384, 1536]),
    ((64, 6, 256, 64), (64, 6, 256, 64), False, True, [64, 6, 256, 256]),
    ((4, 4), (4,), False, False, [4, 1]),
    ((7,), (7, 3), False, False, [1, 3]),
    ((2, 1, 8, 10), (1, 3, 12, 8), True, True, [2, 3, 10, 12]),
])
def test_equalize_matches_reference_rules(a, b, ta, tb, out):
    _, _, o, _, _ = F.equalize(a, b, ta, tb)
    assert o == out


@pytest.mark.parametrize("a,b,ta,tb", [((3, 4), (5, 6), False, False), ((4,), (4, 3), True, False),
                                       ((2, 3, 4), (3, 4, 5), False, False)])
def test_equalize_rejects_like_reference(a, b, ta, tb):
    with pytest.raises(MacrogradError):
        F.equalize(a, b, ta, tb)


def test_bias_equalize():
    assert F.equalize_bias((1536,), [16384, 1536]) == [1, 1536]
    assert F.equalize_bias((256, 256), [64, 6, 256, 256]) == [1, 1, 256, 256]
    with pytest.raises(MacrogradError):
        F.equalize_bias((3,), [4, 5])


def test_accumulate_and_sum_into_refuse_bad_shapes_before_any_device_call():
    """mg_matmul_accumulate (the gradient GEMM with its `+=` reduction) and
    mg_sum_into (the bias gradient's reduction) check their shapes like the
    reference's `+=` (a dim equal to the product's, or 1) and return
    MG_ERR_INVALID -- no abort, no device touched (this runs without a GPU)."""
    import ctypes

    from macrograd_b200 import _lib
    from macrograd_b200._lib import i32_array

    lib = _lib.load(build_if_missing=True)
    null = ctypes.c_void_p(0)
    acc = lib.mg_matmul_accumulate
    # product [8, 384, 384] of A^T[8,384,256] . dC[8,256,384]: out may be [8,..] or [1,..], not [2,..]
    assert acc(null, null, null, i32_array([2, 384, 384]), i32_array([8, 256, 384]), i32_array([8, 256, 384]),
               3, 1, 0, ctypes.c_float(1.0), null) == _lib.MG_ERR_INVALID
    assert b"or 1" in lib.mg_last_error()
    assert acc(null, null, null, i32_array([1, 384, 384]), i32_array([8, 256, 384]), i32_array([8, 256, 384]),
               3, 1, 0, ctypes.c_float(0.5), null) == _lib.MG_ERR_INVALID   # beta 0 or 1 only
    assert acc(null, null, null, i32_array([1, 384, 300]), i32_array([8, 256, 384]), i32_array([8, 256, 384]),
               3, 1, 0, ctypes.c_float(1.0), null) == _lib.MG_ERR_INVALID   # wrong N
    s = lib.mg_sum_into
    assert s(null, null, i32_array([1, 3]), i32_array([4, 5]), 2, ctypes.c_float(0.0), null) == _lib.MG_ERR_INVALID
    assert s(null, null, i32_array([1, 5]), i32_array([4, 5]), 2, ctypes.c_float(2.0), null) == _lib.MG_ERR_INVALID
    assert s(null, null, i32_array([1, 5]), i32_array([4, 5]), 0, ctypes.c_float(0.0), null) == _lib.MG_ERR_INVALID
    assert s(null, null, i32_array([1, 5]), i32_array([4, 5]), 2, ctypes.c_float(0.0), null) == _lib.MG_ERR_INVALID
    assert b"NULL" in lib.mg_last_error()


def test_view_layout_reads_strides_of_head_split_views():
    """functional.matmul_view maps torch views onto the descriptor: which of the
    last two dims is contiguous decides the transpose flag and the row pitch,
    the leading strides become batch strides (no copy of the head split)."""
    import torch

    from macrograd_b200 import functional as F

    B, L, H, d = 2, 5, 3, 4
    E = H * d
    heads = torch.zeros(B, L, E).view(B, L, H, d).transpose(1, 2)   # [B, H, L, d]
    assert F.view_layout(heads.shape, heads.stride()) == (0, E, [L * E, d])
    kt = heads.transpose(-1, -2)
    assert F.view_layout(kt.shape, kt.stride()) == (1, E, [L * E, d])
    bad = torch.zeros(4, 6, 8)[:, ::2, ::2]
    with pytest.raises(F.MacrogradError):
        F.view_layout(bad.shape, bad.stride())


def test_scatter_matmul_rejects_operands_it_cannot_describe():
    """The row-sharded GEMM passes raw pointers with a contiguous row-major
    descriptor, so anything else is refused before the library is called."""
    import types

    import torch

    from macrograd_b200.sharded import scatter_matmul

    peers = types.SimpleNamespace(full=torch.zeros(8, 6), array=None, ptrs=[])
    A, B = torch.zeros(4, 5), torch.zeros(5, 6)
    with pytest.raises(ValueError, match="CUDA tensor"):
        scatter_matmul(A, B, peers, 0)                       # host tensors
    with pytest.raises(ValueError, match="contiguous"):
        scatter_matmul(torch.zeros(5, 4).t(), B, peers, 0)   # a transposed view
    with pytest.raises(ValueError, match="float32"):
        scatter_matmul(A.double(), B, peers, 0)


def test_calls_take_one_device():
    """Every entry point runs on the one device all its tensors (and the
    stream) are on; mixed devices are refused."""
    import types

    import torch

    a = torch.zeros(2)
    assert F._one_device(a, None, a) == torch.device("cpu")
    with pytest.raises(MacrogradError, match="different devices"):
        F._one_device(a, torch.zeros(2, device="meta"))
    with pytest.raises(MacrogradError, match="different devices"):
        F._one_device(a, stream=types.SimpleNamespace(device=torch.device("cuda", 0)))


# (A shape, B shape, transA, transB, bias shape or None): shape errors of
# Functional::matmul and its bias form
ERROR_CASES = [
    ((3, 4), (5, 6), False, False, None),
    ((5,), (4, 3), False, False, None),
    ((4,), (4, 3), True, False, None),
    ((2, 3), (3,), False, True, None),
    ((2, 3, 4), (3, 4, 5), False, False, None),
    ((4, 3), (3, 5), False, False, (7,)),
    ((2, 4, 3), (3, 5), False, False, (3, 4, 5)),
    ((4, 3), (3, 5), False, False, (2, 3, 4, 5)),
]


def _our_message(a, b, ta, tb, bias):
    try:
        _, _, out, _, _ = F.equalize(a, b, ta, tb)
        if bias is not None:
            F.equalize_bias(bias, out)
    except MacrogradError as e:
        return str(e).split(": ", 1)[1]
    return None


@pytest.mark.parametrize("case", ERROR_CASES)
def test_shape_errors_carry_the_references_messages(case):
    """The reference prints its MACROGRAD_CHECK message and aborts; run it in a
    child process and compare the message with the one raised here."""
    import os
    import subprocess
    import sys

    import oracle_bridge as ob

    if not ob.ref_available():
        pytest.skip("reference build oracle/_ref not present")
    a, b, ta, tb, bias = case
    bias_src = "None" if bias is None else f"np.zeros({bias}, np.float32)"
    code = ("import numpy as np, oracle_bridge as ob\n"
            f"ob.ref_matmul(np.zeros({a}, np.float32), np.zeros({b}, np.float32), {ta}, {tb}, {bias_src})\n")
    here = os.path.dirname(os.path.abspath(__file__))
    run = subprocess.run([sys.executable, "-c", code], cwd=here, capture_output=True, text=True, timeout=120)
    assert run.returncode != 0, "the reference accepted the shapes"
    text = run.stdout + run.stderr
    assert "Message: " in text, text
    ref_message = text.split("Message: ", 1)[1].strip()
    assert _our_message(a, b, ta, tb, bias) == ref_message

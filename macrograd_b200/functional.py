"""Host-side mirror of Macrograd's matmul API over the sm_100a library.

Mirrors, for torch CUDA tensors (torch provides device memory and streams;
every GEMM and every gradient reduction runs in libmg_gemm.so -- no torch
arithmetic on the path):
  matmul(mat0, mat1, transA, transB)            Functional::matmul
      macrograd/source/tensor_ops.cpp:4482-4694
  matmul(mat0, mat1, bias, transA, transB)      Functional::matmul with bias
      macrograd/source/tensor_ops.cpp:4700-4949
  matmul_backward(...)                          MatMulOp / MatMulBiasOp::_backward
      macrograd/source/tensor_ops.cpp:4504-4517, 4723-4737, each gradient
      GEMM accumulating straight into its gradient (mg_matmul_accumulate),
      the bias gradient summed by mg_sum_into (the `+=` of
      tensor_ops.cpp:3345-3451)
  attention_scores(...)                         matmul(Q/sqrt(d), K, mask, false, true)
      followed by softmax(-1), mini_shakespeare/include/transformer.h:233-234
  matmul_view(...)                              the same product on strided views (the
      attention head split/merge read and written in place)
  attention_softmax_backward(...)               dP = dO V^T and the softmax derivative
      (tensor_ops.cpp:2056-2059) in one kernel

Shape rules, error conditions and messages follow the reference; the GEMM
itself always runs in libmg_gemm.so (mg_matmul / mg_matmul_bias / mg_gemm).
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Sequence, Tuple

import torch

from . import _lib
from ._lib import MacrogradError, check, i32_array


# ------------------------------------------------------------------ shapes
def _shape_str(shape: Sequence[int]) -> str:
    """A shape as the reference prints it (Shape::str): "(3, 4)", "(5)"."""
    return "(" + ", ".join(str(int(x)) for x in shape) + ")"


def equalize(a_shape: Sequence[int], b_shape: Sequence[int], transA: bool, transB: bool):
    """Rank-equalised storage shapes and the output shape, with the reference's
    checks and their messages (tensor_ops.cpp:4521-4579). Returns (A, B, out,
    a_was_1d, b_was_1d)."""
    a, b = list(a_shape), list(b_shape)
    if len(a) == 0:
        raise MacrogradError(_lib.MG_ERR_INVALID,
                             "Trying to matrix multiply two tensors while the first tensor is empty.")
    if len(b) == 0:
        raise MacrogradError(_lib.MG_ERR_INVALID,
                             "Trying to matrix multiply two tensors while the second tensor is empty.")
    for flag, t, name in ((transA, a, "transA"), (transB, b, "transB")):
        if flag and len(t) < 2:
            raise MacrogradError(_lib.MG_ERR_INVALID,
                                 "Addint a transposition to a single dimensional tensor for a matmul call is not "
                                 "allowed.\n"
                                 f"Make sure your tensor has at least 2 dimensions if you set '{name}' as true.")
    a_was_1d, b_was_1d = len(a) == 1, len(b) == 1
    if a_was_1d:
        a = [1] + a
    if b_was_1d:
        b = b + [1]
    while len(a) > len(b):
        b = [1] + b
    while len(b) > len(a):
        a = [1] + a
    ka = a[-2] if transA else a[-1]
    kb = b[-1] if transB else b[-2]
    if ka != kb:
        raise MacrogradError(_lib.MG_ERR_INVALID,
                             "Incompatible dimensions found inside a matmul() call.\n"
                             "Please make sure your tensors follow proper matrix multiplication logic "
                             "(...,M,K) @ (...,K,N) = (...,M,N).\n"
                             f"Matrix0 shape: {_shape_str(a_shape)} | Matrix1 shape: {_shape_str(b_shape)}")
    for i in range(len(a) - 2):
        if not (a[i] == b[i] or a[i] == 1 or b[i] == 1):
            raise MacrogradError(_lib.MG_ERR_INVALID,
                                 "Trying to matrix multiply two tensors with incompatible shapes.\n"
                                 "Make sure leading shapes are compatible, meaning they have the same sizes or one "
                                 "of them is unitary for broadcasting.\n"
                                 f"Found shapes | Unsqueezed Matrix0: {_shape_str(a)} | "
                                 f"Unsqueezed Matrix1: {_shape_str(b)}")
    out = [max(x, y) for x, y in zip(a[:-2], b[:-2])]
    out += [a[-1] if transA else a[-2], b[-2] if transB else b[-1]]
    return a, b, out, a_was_1d, b_was_1d


def equalize_bias(bias_shape: Sequence[int], out_shape: Sequence[int]):
    """Bias rank-equalised to the output, with the reference's checks and
    messages (tensor_ops.cpp:4784-4785, 4807-4818)."""
    bs = list(bias_shape)
    if len(bs) > len(out_shape):
        raise MacrogradError(_lib.MG_ERR_INVALID,
                             "Trying to add a bias to a matmul tensor with more dimensions than the matmul output.\n"
                             "Make sure the bias is broadcastable to the matmul output, bias dimensionality must "
                             "be less or equal.\n"
                             f"Found shapes | Matmul output: {_shape_str(out_shape)} | Bias: {_shape_str(bs)}")
    while len(bs) < len(out_shape):
        bs = [1] + bs
    for o, x in zip(out_shape, bs):
        if not (o == x or x == 1):
            raise MacrogradError(_lib.MG_ERR_INVALID,
                                 "Trying to add a bias to a matmul tensor with incompatible shapes.\n"
                                 "Make sure leading shapes are compatible, meaning they have the same sizes or the "
                                 "bias one is unitary for broadcasting.\n"
                                 f"Found shapes | Matmul output: {_shape_str(out_shape)} | "
                                 f"Unsqueezed bias: {_shape_str(bs)}")
    return bs


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream_handle(t: torch.Tensor, stream: Optional[torch.cuda.Stream]):
    s = stream if stream is not None else torch.cuda.current_stream(t.device)
    return ctypes.c_void_p(s.cuda_stream)


def _one_device(*tensors, stream: Optional[torch.cuda.Stream] = None) -> torch.device:
    """The one CUDA device all given tensors (None skipped) and the stream are
    on: the library runs each call on the current device, so a call is made
    under this one."""
    devs = {t.device for t in tensors if t is not None}
    if stream is not None:
        devs.add(torch.device(stream.device))
    if len(devs) != 1:
        raise MacrogradError(_lib.MG_ERR_INVALID,
                             "operands (and stream) are on different devices: " + ", ".join(sorted(map(str, devs))))
    return next(iter(devs))


def _check_operand(t: torch.Tensor, name: str):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise MacrogradError(_lib.MG_ERR_INVALID, f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32:
        raise MacrogradError(_lib.MG_ERR_INVALID, f"{name} must be float32")
    if not t.is_contiguous():
        raise MacrogradError(_lib.MG_ERR_INVALID, f"{name} must be contiguous (Macrograd tensors always are)")


# ------------------------------------------------------------------ forward
def matmul(mat0: torch.Tensor, mat1: torch.Tensor, bias: Optional[torch.Tensor] = None,
           transA: bool = False, transB: bool = False, out: Optional[torch.Tensor] = None,
           stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Functional::matmul(mat0, mat1[, bias], transA, transB) on CUDA tensors."""
    lib = _lib.load()
    _check_operand(mat0, "mat0")
    _check_operand(mat1, "mat1")
    if bias is not None:
        _check_operand(bias, "bias")
    if out is not None:
        _check_operand(out, "out")
    dev = _one_device(mat0, mat1, bias, out, stream=stream)
    a, b, oshape, a1d, b1d = equalize(mat0.shape, mat1.shape, transA, transB)
    if out is None:
        out = torch.empty(oshape, device=dev, dtype=torch.float32)
    elif list(out.shape) != oshape:
        raise MacrogradError(_lib.MG_ERR_INVALID, f"out must be a contiguous tensor of shape {oshape}")
    rank = len(oshape)
    st = _stream_handle(mat0, stream)
    with torch.cuda.device(dev):
        if bias is None:
            check(lib.mg_matmul(_ptr(out), _ptr(mat0), _ptr(mat1), i32_array(oshape), i32_array(a),
                                i32_array(b), rank, int(transA), int(transB), st))
        else:
            bs = equalize_bias(bias.shape, oshape)
            check(lib.mg_matmul_bias(_ptr(out), _ptr(mat0), _ptr(mat1), _ptr(bias), i32_array(oshape),
                                     i32_array(a), i32_array(b), i32_array(bs), rank, int(transA),
                                     int(transB), st))
    if a1d:
        out = out.squeeze(-2)
    if b1d:
        out = out.squeeze(-1)
    return out


def attention_scores(q: torch.Tensor, k: torch.Tensor, scale: float, causal: bool = True,
                     mask: Optional[torch.Tensor] = None,
                     stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """P = softmax(scale * q @ k^T (+ mask) (+ causal -inf), dim=-1), one kernel.

    The reference computes this as Functional::matmul(Q / sqrt(d), K, mask,
    false, true) then Tensor::softmax(-1) (transformer.h:233-234); dividing Q by
    a power of two and scaling the product by the same power are bit-identical."""
    lib = _lib.load()
    _check_operand(q, "q")
    _check_operand(k, "k")
    if mask is not None:
        _check_operand(mask, "mask")
    dev = _one_device(q, k, mask, stream=stream)
    a, b, oshape, _, _ = equalize(q.shape, k.shape, False, True)
    out = torch.empty(oshape, device=dev, dtype=torch.float32)
    bs = equalize_bias(mask.shape, oshape) if mask is not None else None
    with torch.cuda.device(dev):
        check(lib.mg_matmul_softmax(_ptr(out), _ptr(q), _ptr(k), _ptr(mask), i32_array(oshape),
                                    i32_array(a), i32_array(b), i32_array(bs) if bs else None,
                                    len(oshape), 0, 1, ctypes.c_float(scale), int(causal),
                                    _stream_handle(q, stream)))
    return out


def attention_softmax_backward(dO: torch.Tensor, v: torch.Tensor, p: torch.Tensor, alpha: float = 1.0,
                               stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """dS = P * (G - rowsum(P * G)) with G = alpha * dO @ v^T, one kernel: the
    attention backward's dP = dO V^T (the GEMM MatMulOp::_backward issues for
    O = P V, tensor_ops.cpp:4504-4517) and the softmax derivative
    SoftOp::_backward applies to it (tensor_ops.cpp:2056-2059), which the
    reference runs as separate passes over the [.., L, L] scores."""
    lib = _lib.load()
    _check_operand(dO, "dO")
    _check_operand(v, "v")
    _check_operand(p, "p")
    dev = _one_device(dO, v, p, stream=stream)
    a, b, oshape, _, _ = equalize(dO.shape, v.shape, False, True)
    if list(p.shape) != oshape:
        raise MacrogradError(_lib.MG_ERR_INVALID, f"p must have the product's shape {oshape}")
    out = torch.empty(oshape, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        check(lib.mg_matmul_softmax_backward(_ptr(out), _ptr(dO), _ptr(v), _ptr(p), i32_array(oshape),
                                             i32_array(a), i32_array(b), len(oshape), 0, 1, ctypes.c_float(alpha),
                                             _stream_handle(dO, stream)))
    return out


# ------------------------------------------------------------------ strided views
def view_layout(shape: Sequence[int], strides: Sequence[int], name: str = "operand"):
    """(trans, ld, batch strides) of a view whose logical last two dims are
    [rows, cols] with one of the two at unit stride: trans = 0 when the
    columns are contiguous (ld = row stride), 1 when the rows are (ld =
    column stride, i.e. stored transposed)."""
    if len(shape) < 2:
        raise MacrogradError(_lib.MG_ERR_INVALID, f"{name} must have at least 2 dims")
    r, c = shape[-2], shape[-1]
    sr, sc = strides[-2], strides[-1]
    if sc == 1 or c == 1:
        return 0, max(sr, c, 1), list(strides[:-2])
    if sr == 1 or r == 1:
        return 1, max(sc, r, 1), list(strides[:-2])
    raise MacrogradError(_lib.MG_ERR_UNSUPPORTED,
                         f"{name}: one of the last two dims must have unit stride (strides {tuple(strides)})")


def _view_operand(t: torch.Tensor, name: str):
    if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.float32:
        raise MacrogradError(_lib.MG_ERR_INVALID, f"{name} must be a float32 CUDA tensor")
    return view_layout(list(t.shape), list(t.stride()), name)


def matmul_view(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None,
                bias: Optional[torch.Tensor] = None, alpha: float = 1.0,
                stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """out[..., M, N] = alpha * a[..., M, K] @ b[..., K, N] (+ bias) on strided
    views, read and written in place -- no transposed or head-split copy.

    For the multi-head attention of mini_shakespeare/include/transformer.h
    (226-228, 244), which materialises `Q.view(B, L, H, d).transpose(1, 2)`
    and its inverse with Tensor::transpose copies (tensor_ops.cpp:469-576):
    here the head split is just strides of the GEMM operands and output
    (row pitch E, batch strides L*E and d). Leading dims broadcast as in
    Functional::matmul (size 1 or stride 0); one of each operand's last two
    dims must have unit stride. Operands whose strides TMA cannot read
    (not multiples of 16 bytes) are re-laid out by the library first."""
    lib = _lib.load()
    ta, lda, sa = _view_operand(a, "a")
    tb, ldb, sb = _view_operand(b, "b")
    M, K = a.shape[-2], a.shape[-1]
    if b.shape[-2] != K:
        raise MacrogradError(_lib.MG_ERR_INVALID,
                             "Incompatible dimensions found inside a matmul() call.\n"
                             "Please make sure your tensors follow proper matrix multiplication logic "
                             "(...,M,K) @ (...,K,N) = (...,M,N).\n"
                             f"Matrix0 shape: {_shape_str(a.shape)} | Matrix1 shape: {_shape_str(b.shape)}")
    N = b.shape[-1]
    nb = max(a.dim(), b.dim()) - 2
    ash = [1] * (nb - (a.dim() - 2)) + list(a.shape[:-2])
    bsh = [1] * (nb - (b.dim() - 2)) + list(b.shape[:-2])
    sa = [0] * (nb - len(sa)) + sa
    sb = [0] * (nb - len(sb)) + sb
    batch = []
    for i in range(nb):
        if not (ash[i] == bsh[i] or ash[i] == 1 or bsh[i] == 1):
            raise MacrogradError(_lib.MG_ERR_INVALID,
                                 "Trying to matrix multiply two tensors with incompatible shapes.\n"
                                 "Make sure leading shapes are compatible, meaning they have the same sizes or one "
                                 "of them is unitary for broadcasting.\n"
                                 f"Found shapes | Unsqueezed Matrix0: {_shape_str(ash + [M, K])} | "
                                 f"Unsqueezed Matrix1: {_shape_str(bsh + [K, N])}")
        batch.append(max(ash[i], bsh[i]))
    if nb > _lib.MG_MAX_BATCH_DIMS:
        raise MacrogradError(_lib.MG_ERR_UNSUPPORTED, f"more than {_lib.MG_MAX_BATCH_DIMS} leading dims")
    oshape = batch + [M, N]
    if out is not None and (not out.is_cuda or out.dtype != torch.float32):
        raise MacrogradError(_lib.MG_ERR_INVALID, "out must be a float32 CUDA tensor")
    if bias is not None:
        _check_operand(bias, "bias")
    dev = _one_device(a, b, out, bias, stream=stream)
    if out is None:
        out = torch.empty(oshape, device=dev, dtype=torch.float32)
    if list(out.shape) != oshape or out.stride(-1) != 1:
        raise MacrogradError(_lib.MG_ERR_INVALID, f"out must have shape {oshape} and unit column stride")
    d = _lib.GemmDesc()
    lib.mg_gemm_desc_init(ctypes.byref(d), M, N, K, ta, tb)
    d.lda, d.ldb, d.ldc = lda, ldb, max(out.stride(-2), N)
    d.batch_rank = nb
    for i in range(nb):
        d.batch[i] = batch[i]
        d.a_batch_stride[i] = 0 if ash[i] == 1 else sa[i]
        d.b_batch_stride[i] = 0 if bsh[i] == 1 else sb[i]
        d.c_batch_stride[i] = out.stride(i)
    d.alpha = alpha
    if bias is not None:
        bs = equalize_bias(bias.shape, oshape)
        d.epilogue = _lib.MG_EPI_BIAS
        # contiguous bias broadcast to out: element strides, 0 where broadcast
        strides = [0] * len(bs)
        acc = 1
        for i in range(len(bs) - 1, -1, -1):
            strides[i] = 0 if bs[i] == 1 else acc
            acc *= bs[i]
        d.bias_rs, d.bias_cs = strides[-2], strides[-1]
        for i in range(nb):
            d.bias_batch_stride[i] = strides[i]
    with torch.cuda.device(dev):
        check(lib.mg_gemm(ctypes.byref(d), _ptr(out), _ptr(a), _ptr(b), _ptr(bias), _stream_handle(a, stream)))
    return out


# ------------------------------------------------------------------ backward
def _grad_gemm(X: torch.Tensor, Y: torch.Tensor, tX: bool, tY: bool, target_shape,
               accumulate: Optional[torch.Tensor], stream) -> torch.Tensor:
    """`grad += matmul(X, Y, tX, tY)` of MatMulOp::_backward
    (tensor_ops.cpp:4504-4517) as ONE library call (mg_matmul_accumulate):
    the product is summed over the leading dims where target_shape (the
    rank-equalised shape of the operand whose gradient this is) is 1 -- the
    reference's `+=` broadcast reduction, tensor_ops.cpp:3345-3451 -- inside
    the GEMM's K loop, and added to `accumulate` (beta = 1) when given, else
    written to a new tensor."""
    lib = _lib.load()
    _check_operand(X, "gradient operand")
    _check_operand(Y, "gradient operand")
    if accumulate is not None:
        _check_operand(accumulate, "gradient accumulator")
    dev = _one_device(X, Y, accumulate, stream=stream)
    xs, ys = list(X.shape), list(Y.shape)
    dst = accumulate if accumulate is not None else torch.empty(list(target_shape), device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        check(lib.mg_matmul_accumulate(_ptr(dst), _ptr(X), _ptr(Y), i32_array(target_shape), i32_array(xs),
                                       i32_array(ys), len(xs), int(tX), int(tY),
                                       ctypes.c_float(1.0 if accumulate is not None else 0.0),
                                       _stream_handle(X, stream)))
    return dst


def sum_into(src: torch.Tensor, dst_shape: Sequence[int], accumulate: Optional[torch.Tensor] = None,
             stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """`dst += src` where dst broadcasts to src (the reference's `+=`,
    tensor_ops.cpp:3345-3451, squeeze direction): src summed over the dims
    where dst_shape (rank-equalised to src) is 1, added to `accumulate` when
    given, else written to a new tensor. One library call (mg_sum_into)."""
    lib = _lib.load()
    _check_operand(src, "src")
    if accumulate is not None:
        _check_operand(accumulate, "accumulator")
    dev = _one_device(src, accumulate, stream=stream)
    ss = list(src.shape)
    ds = [1] * (len(ss) - len(dst_shape)) + list(dst_shape)
    if len(ds) != len(ss):
        raise MacrogradError(_lib.MG_ERR_INVALID, f"dst shape {list(dst_shape)} has more dims than src {ss}")
    dst = accumulate if accumulate is not None else torch.empty(ds, device=dev, dtype=torch.float32)
    if accumulate is not None and accumulate.numel() != math.prod(ds):
        raise MacrogradError(_lib.MG_ERR_INVALID, f"accumulator has {accumulate.numel()} elements, dst shape {ds}")
    with torch.cuda.device(dev):
        check(lib.mg_sum_into(_ptr(dst), _ptr(src), i32_array(ds), i32_array(ss), len(ss),
                              ctypes.c_float(1.0 if accumulate is not None else 0.0), _stream_handle(src, stream)))
    return dst


def matmul_backward(A: torch.Tensor, B: torch.Tensor, dC: torch.Tensor, transA: bool = False,
                    transB: bool = False, has_bias: bool = False,
                    bias_shape: Optional[Sequence[int]] = None,
                    need_a: bool = True, need_b: bool = True,
                    grad_a: Optional[torch.Tensor] = None, grad_b: Optional[torch.Tensor] = None,
                    grad_bias: Optional[torch.Tensor] = None,
                    stream: Optional[torch.cuda.Stream] = None
                    ) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor], Optional[torch.Tensor]]:
    """Gradients of C = op(A) op(B) (+ bias) for an upstream dC, exactly the GEMMs
    MatMulOp::_backward issues (tensor_ops.cpp:4504-4517):
        dA = transA ? matmul(B, dC, transB, true) : matmul(dC, B, false, !transB)
        dB = transB ? matmul(dC, A, true, transA) : matmul(A, dC, !transA, false)
    with A and B rank-equalised as the forward left them, each reduced to its
    operand's shape like `internal_gradient() += ...` inside the same GEMM (a
    gradient whose operand was broadcast over the batch -- a weight -- sums
    the batch in the GEMM's K loop: no batched temporary, no separate
    reduction), and dbias = dC summed to the bias shape (MatMulBiasOp,
    tensor_ops.cpp:4736) by the library's reduction. grad_a / grad_b /
    grad_bias, when given, are accumulated into (beta = 1, the `+=`) instead of
    freshly allocated."""
    for name, g in (("grad_a", grad_a), ("grad_b", grad_b), ("grad_bias", grad_bias)):
        if g is not None:
            _check_operand(g, name)   # reshaped below as a view: the accumulation lands in it
    a, b, oshape, _, _ = equalize(A.shape, B.shape, transA, transB)
    Av = A.reshape(a)
    Bv = B.reshape(b)
    dCv = dC.reshape(oshape)
    dA = dB = dbias = None
    if need_a:
        if transA:
            dA = _grad_gemm(Bv, dCv, transB, True, a, grad_a.reshape(a) if grad_a is not None else None, stream)
        else:
            dA = _grad_gemm(dCv, Bv, False, not transB, a, grad_a.reshape(a) if grad_a is not None else None, stream)
        dA = dA.reshape(A.shape)
    if need_b:
        if transB:
            dB = _grad_gemm(dCv, Av, True, transA, b, grad_b.reshape(b) if grad_b is not None else None, stream)
        else:
            dB = _grad_gemm(Av, dCv, not transA, False, b, grad_b.reshape(b) if grad_b is not None else None, stream)
        dB = dB.reshape(B.shape)
    if has_bias:
        bs = equalize_bias(bias_shape, oshape)
        if not dCv.is_contiguous():
            dCv = dCv.contiguous()
        dbias = sum_into(dCv, bs, grad_bias.reshape(bs) if grad_bias is not None else None, stream=stream)
        dbias = dbias.reshape(bias_shape)
    return dA, dB, dbias

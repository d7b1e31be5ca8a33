// seam_fused.h -- forced into the fused build's patched tensor_ops.cpp
// (fuse_tensor_ops.py): the three calls its patched lines make, defined in
// seam_fused.cpp.
#pragma once

class Tensor;

// Skip (true) or restore (false) MemPool's zero fill of the blocks allocated
// on this host thread in between: brackets Functional::matmul's output.
void mg_seam_skip_zero_fill(bool on);

// grad += Functional::matmul(X, Y, tX, tY), the gradient accumulation of
// MatMulOp / MatMulBiasOp::_backward, as one accumulating GEMM where it can be
// done in place -- exactly where `grad += ...` itself works in place -- and
// as the original expression otherwise.
void mg_seam_accumulate_matmul(Tensor& grad, const Tensor& X, const Tensor& Y, bool tX, bool tY);

// grad += src where grad broadcasts to src (MatMulBiasOp's bias gradient),
// by the library's reduction where it can be done in place.
void mg_seam_accumulate_sum(Tensor& grad, const Tensor& src);

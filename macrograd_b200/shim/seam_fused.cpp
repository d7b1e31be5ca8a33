// seam_fused.cpp -- Tensor-level half of the opt-in fused drop-in build: the
// calls that fuse_tensor_ops.py puts in place of MatMulOp / MatMulBiasOp's
// `grad += ...` lines (tensor_ops.cpp:4508-4515, :4727-4736). Each keeps the
// reference's meaning: `Tensor::operator+=` (tensor_ops.cpp:3345-3451) adds
// in place only when the tensor has no gradient of its own and no other
// instance shares its data, otherwise it builds a new tensor; the fused path
// is taken in exactly the in-place case, on "cuda", and the original
// expression runs in every other.
#include "macrograd.h"
#include "seam_fused.h"

// device-side halves (kernel_ops_fused.inc, in the backend's translation unit)
void mg_seam_matmul_accumulate(void* grad, const void* X, const void* Y, const Shape& g, const Shape& x,
                               const Shape& y, bool tX, bool tY);
void mg_seam_sum_into(void* dst, const void* src, const Shape& d, const Shape& s);

namespace {

bool in_place(const Tensor& grad) { return grad.is_gpu() && !grad.has_grad() && grad.instances() == 1; }

}  // namespace

void mg_seam_accumulate_matmul(Tensor& grad, const Tensor& X, const Tensor& Y, bool tX, bool tY)
{
    // MatMulOp keeps its operands rank-equalised, so the gradient (of such an
    // operand) and both factors have one rank; anything else takes the
    // original path
    if (in_place(grad) && X.is_gpu() && Y.is_gpu() && X.dim() == Y.dim() && grad.dim() == X.dim() &&
        X.dim() >= 2) {
        mg_seam_matmul_accumulate(grad.internal_data(), X.internal_data(), Y.internal_data(), grad.shape(),
                                  X.shape(), Y.shape(), tX, tY);
        return;
    }
    grad += Functional::matmul(X, Y, tX, tY);
}

void mg_seam_accumulate_sum(Tensor& grad, const Tensor& src)
{
    if (in_place(grad) && src.is_gpu() && grad.dim() == src.dim()) {
        mg_seam_sum_into(grad.internal_data(), src.internal_data(), grad.shape(), src.shape());
        return;
    }
    grad += src;
}

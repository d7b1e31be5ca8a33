// seam_driver.cpp -- C entry points over the REFERENCE's Tensor API running on
// "cuda", with kernel_ops::matmul / matmul_bias replaced by the seam in
// kernel_ops_matmul.inc (see Makefile in this directory).
//
// Used by the drop-in tests: the reference's own Functional::matmul and its
// autograd backward, called exactly as a Macrograd user would, must reach the
// sm_100a kernels and agree with the oracle.
#include <cstdint>
#include <cstring>
#include <vector>

#include "macrograd.h"

namespace {

Shape make_shape(const int32_t* s, int32_t rank)
{
    std::vector<int> v(s, s + rank);
    return Shape(unsigned(rank), v.data());
}

Tensor to_cuda(const float* data, const int32_t* s, int32_t rank, bool grad)
{
    Tensor host(make_shape(s, rank), "cpu", false);
    size_t n = 1;
    for (int32_t i = 0; i < rank; i++) n *= size_t(s[i]);
    std::memcpy(host.internal_data(), data, n * sizeof(float));
    return host.to("cuda", grad);
}

void to_host(const Tensor& t, float* out)
{
    Tensor h = t.to("cpu");
    std::memcpy(out, h.internal_data(), size_t(h.numel()) * sizeof(float));
}

}  // namespace

extern "C" {

// out = Functional::matmul(A, B[, bias], transA, transB) with "cuda" tensors.
int seam_matmul(float* out, const float* A, const float* B, const float* bias,
                const int32_t* A_shape, int32_t A_rank, const int32_t* B_shape, int32_t B_rank,
                const int32_t* bias_shape, int32_t bias_rank, int32_t transA, int32_t transB)
{
    Tensor a = to_cuda(A, A_shape, A_rank, false);
    Tensor b = to_cuda(B, B_shape, B_rank, false);
    Tensor c = bias ? Functional::matmul(a, b, to_cuda(bias, bias_shape, bias_rank, false),
                                         transA != 0, transB != 0)
                    : Functional::matmul(a, b, transA != 0, transB != 0);
    to_host(c, out);
    return 0;
}

// Forward + the reference autograd on "cuda" with upstream gradient dC:
// loss = sum(C * dC), so MatMulOp / MatMulBiasOp::_backward run with C's
// gradient equal to dC, through Functional::matmul and the seam again.
int seam_matmul_backward(float* dA, float* dB, float* dbias, const float* A, const float* B,
                         const float* bias, const float* dC, const int32_t* A_shape, int32_t A_rank,
                         const int32_t* B_shape, int32_t B_rank, const int32_t* bias_shape,
                         int32_t bias_rank, const int32_t* C_shape, int32_t C_rank, int32_t transA,
                         int32_t transB)
{
    Tensor a = to_cuda(A, A_shape, A_rank, true);
    Tensor b = to_cuda(B, B_shape, B_rank, true);
    Tensor bi;
    if (bias) bi = to_cuda(bias, bias_shape, bias_rank, true);
    Tensor c = bias ? Functional::matmul(a, b, bi, transA != 0, transB != 0)
                    : Functional::matmul(a, b, transA != 0, transB != 0);
    Tensor g = to_cuda(dC, C_shape, C_rank, false);
    Tensor loss = (c * g).flatten().sum(0);
    loss.backward();
    to_host(a.gradient(), dA);
    to_host(b.gradient(), dB);
    if (bias && dbias) to_host(bi.gradient(), dbias);
    return 0;
}

void seam_synchronize(void) { Cuda::synchronize(); }

}  // extern "C"

// seam_driver.cpp -- C entry points over the REFERENCE's Tensor API running on
// "cuda", with kernel_ops::matmul / matmul_bias replaced by the seam in
// kernel_ops_matmul.inc (see Makefile in this directory).
//
// Used by the drop-in tests: the reference's own Functional::matmul and its
// autograd backward, called exactly as a Macrograd user would, must reach the
// sm_100a kernels and agree with the oracle.
#include <chrono>
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

// A used by two products: loss = sum(A W1 * dC1) + sum(A W2 * dC2), so the
// reference autograd accumulates A's gradient twice -- the second time into a
// gradient that already holds the first product's share.
int seam_shared_operand_backward(float* dA, const float* A, const float* W1, const float* W2, const float* dC1,
                                 const float* dC2, const int32_t* A_shape, const int32_t* W_shape,
                                 const int32_t* C_shape, int32_t rank)
{
    Tensor a = to_cuda(A, A_shape, rank, true);
    Tensor w1 = to_cuda(W1, W_shape, rank, false);
    Tensor w2 = to_cuda(W2, W_shape, rank, false);
    Tensor g1 = to_cuda(dC1, C_shape, rank, false);
    Tensor g2 = to_cuda(dC2, C_shape, rank, false);
    Tensor loss = (Functional::matmul(a, w1) * g1).flatten().sum(0) + (Functional::matmul(a, w2) * g2).flatten().sum(0);
    loss.backward();
    to_host(a.gradient(), dA);
    return 0;
}

// Milliseconds per Functional::matmul of two n x n "cuda" tensors through the
// reference's API (output allocation included), over `iters` calls after
// `warmup`, host-timed around a device synchronisation.
double seam_time_matmul(int32_t n, int32_t warmup, int32_t iters)
{
    const int32_t s[2] = {n, n};
    Tensor a(make_shape(s, 2), "cuda", false);
    Tensor b(make_shape(s, 2), "cuda", false);
    for (int32_t i = 0; i < warmup; ++i) Tensor c = Functional::matmul(a, b);
    Cuda::synchronize();
    const auto t0 = std::chrono::steady_clock::now();
    for (int32_t i = 0; i < iters; ++i) Tensor c = Functional::matmul(a, b);
    Cuda::synchronize();
    const auto t1 = std::chrono::steady_clock::now();
    return std::chrono::duration<double, std::milli>(t1 - t0).count() / (iters > 0 ? iters : 1);
}

void seam_synchronize(void) { Cuda::synchronize(); }

}  // extern "C"

/*
 * mg_oracle.h -- CPU restatement of Macrograd's matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the oracle that the tests, the smoke check
 * and the CPU-baseline leg of the benchmark use to CHECK the CUDA library. It is
 * never the thing measured on the GPU and never part of the product path.
 *
 * Every function restates the reference's CPU branch (file:line in the
 * reference tree, MiquelNasarre/macrograd):
 *   oracle_matmul        macrograd/source/tensor_ops.cpp:4597-4682  (no bias)
 *                        macrograd/source/tensor_ops.cpp:4837-4937  (bias)
 *   oracle_softmax_rows  macrograd/source/tensor_ops.cpp:2093-2112  (last dim)
 *   oracle_causal_mask   macrograd/source/tensor_ops.cpp:5479-5488
 *   oracle_reduce_to     macrograd/source/tensor_ops.cpp:3393-3446  (the `+=`
 *                        broadcast reduction a gradient goes through)
 *   oracle_rng_*         macrograd/source/tensor_ops.cpp:5500-5521, 5533-5536,
 *                        5660-5699 (splitmix64 seed stream, Random::set_seed,
 *                        Initialization::uniform / normal on the CPU)
 *
 * Shapes are rank-equalised exactly like Functional::matmul leaves them
 * (tensor_ops.cpp:4547-4557, 4770-4783): every shape has `rank` entries,
 * leading dims equal or 1. Storage is contiguous row-major fp32.
 *
 * Build flags are pinned (-O3 -ffp-contract=off, no -march) so that the sum
 * `c_row[j] += a * b` is a separate multiply and add, as in the reference's
 * CMake Release build on x86-64 without FMA.
 */
#ifndef MG_ORACLE_H
#define MG_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* C[...,M,N] = op(A) @ op(B) (+ bias). `out` is overwritten (the reference
 * writes into a zero-filled tensor; this function zero-fills first).
 * bias / bias_shape may be NULL for the no-bias form. Returns 0 on success,
 * nonzero on a shape error (same checks as tensor_ops.cpp:4559-4572, 4807-4818). */
int oracle_matmul(float* out, const float* A, const float* B, const float* bias,
                  const int32_t* out_shape, const int32_t* A_shape,
                  const int32_t* B_shape, const int32_t* bias_shape,
                  int32_t rank, int32_t transA, int32_t transB);

/* Row softmax over the last dimension of a [rows, n] block, in place semantics
 * of Tensor::softmax(-1): max (first element, strict >), expf(x - max), sum in
 * order, divide. */
void oracle_softmax_rows(float* out, const float* in, int64_t rows, int64_t n);

/* [L, L] mask: -inf strictly above the diagonal, 0 elsewhere. */
void oracle_causal_mask(float* out, int32_t L);

/* dst[dst_shape] += src[src_shape] with src reduced over the dims where dst has
 * size 1 (Tensor::operator+= on CPU with `t1.sum(i, true)`), both rank `rank`. */
void oracle_reduce_to(float* dst, const float* src, const int32_t* dst_shape,
                      const int32_t* src_shape, int32_t rank);

/* The reference's CPU random stream: one global splitmix64 state (seed 42 at
 * load), Random::set_seed replaces it. The fill functions consume the stream
 * exactly like Initialization::uniform / normal on a CPU tensor of n elements. */
void oracle_rng_set_seed(uint64_t seed);
void oracle_rng_uniform(float* out, int64_t n, float lo, float hi);
void oracle_rng_normal(float* out, int64_t n, float mean, float stddev);

#ifdef __cplusplus
}
#endif

#endif /* MG_ORACLE_H */

/*
 * mg_oracle.c -- CPU restatement of Macrograd's matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA library, never the thing
 * measured or shipped. See mg_oracle.h for the reference file:line each
 * function follows. Compile with -O3 -ffp-contract=off (no -march) so the
 * multiply and the add of `c_row[j] += a * b` stay separate roundings.
 */
#include "mg_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* Contiguous row-major strides of a shape (tensor.cpp:647-650). */
static void contiguous_strides(const int32_t* shape, int32_t rank, int64_t* stride)
{
    stride[rank - 1] = 1;
    for (int32_t i = rank - 2; i >= 0; i--)
        stride[i] = stride[i + 1] * (int64_t)shape[i + 1];
}

/* The blocked i/j/k triple loop of tensor_ops.cpp:4626-4664 (64-wide blocks,
 * k strictly in order per output element). When `bias` is given the block of C
 * is first seeded with the bias, as tensor_ops.cpp:4885-4893 does. */
static void block_gemm(float* C, const float* A, const float* B, const float* bias,
                       int64_t bm_stride, int64_t bn_stride, uint32_t M, uint32_t N,
                       uint32_t K, uint32_t A_cols, uint32_t B_cols, int transA, int transB)
{
    for (uint32_t i0 = 0; i0 < M; i0 += 64) {
        const uint32_t i1 = (i0 + 64 < M) ? (i0 + 64) : M;
        for (uint32_t j0 = 0; j0 < N; j0 += 64) {
            const uint32_t j1 = (j0 + 64 < N) ? (j0 + 64) : N;
            if (bias) {
                for (uint32_t i = i0; i < i1; ++i) {
                    float* c_row = C + (int64_t)i * N;
                    const float* bias_row = bias + (int64_t)i * bm_stride;
                    for (uint32_t j = j0; j < j1; ++j)
                        c_row[j] = bias_row[(int64_t)j * bn_stride];
                }
            }
            for (uint32_t k0 = 0; k0 < K; k0 += 64) {
                const uint32_t k1 = (k0 + 64 < K) ? (k0 + 64) : K;
                for (uint32_t i = i0; i < i1; ++i) {
                    float* c_row = C + (int64_t)i * N;
                    for (uint32_t k = k0; k < k1; ++k) {
                        const float a = transA ? A[(int64_t)k * A_cols + i]
                                               : A[(int64_t)i * A_cols + k];
                        for (uint32_t j = j0; j < j1; ++j) {
                            const float b = transB ? B[(int64_t)j * B_cols + k]
                                                   : B[(int64_t)k * B_cols + j];
                            c_row[j] += a * b;
                        }
                    }
                }
            }
        }
    }
}

int oracle_matmul(float* out, const float* A, const float* B, const float* bias,
                  const int32_t* out_shape, const int32_t* A_shape,
                  const int32_t* B_shape, const int32_t* bias_shape,
                  int32_t rank, int32_t transA, int32_t transB)
{
    if (rank < 2 || rank > 16) return 1;
    /* K agreement and broadcastable leading dims (tensor_ops.cpp:4559-4572). */
    const int32_t Ka = transA ? A_shape[rank - 2] : A_shape[rank - 1];
    const int32_t Kb = transB ? B_shape[rank - 1] : B_shape[rank - 2];
    if (Ka != Kb) return 2;
    for (int32_t i = 0; i < rank - 2; i++) {
        if (!(A_shape[i] == B_shape[i] || A_shape[i] == 1 || B_shape[i] == 1)) return 3;
        const int32_t o = A_shape[i] > B_shape[i] ? A_shape[i] : B_shape[i];
        if (out_shape[i] != o) return 4;
    }
    const uint32_t M = (uint32_t)out_shape[rank - 2];
    const uint32_t N = (uint32_t)out_shape[rank - 1];
    const uint32_t K = (uint32_t)Ka;
    if ((int32_t)M != (transA ? A_shape[rank - 1] : A_shape[rank - 2])) return 5;
    if ((int32_t)N != (transB ? B_shape[rank - 2] : B_shape[rank - 1])) return 5;
    if (bias) {
        for (int32_t i = 0; i < rank; i++)
            if (!(bias_shape[i] == out_shape[i] || bias_shape[i] == 1)) return 6;
    }

    int64_t so[16], sa[16], sb[16], sbias[16];
    contiguous_strides(out_shape, rank, so);
    contiguous_strides(A_shape, rank, sa);
    contiguous_strides(B_shape, rank, sb);
    if (bias) contiguous_strides(bias_shape, rank, sbias);

    int64_t numel = 1;
    for (int32_t i = 0; i < rank; i++) numel *= out_shape[i];
    memset(out, 0, (size_t)numel * sizeof(float));
    if (numel == 0) return 0;

    /* Bias strides on the last two dims: 0 where the bias dim is 1
     * (tensor_ops.cpp:4840-4841). */
    const int64_t bm_stride = bias ? (bias_shape[rank - 2] == 1 ? 0 : sbias[rank - 2]) : 0;
    const int64_t bn_stride = bias ? (bias_shape[rank - 1] == 1 ? 0 : sbias[rank - 1]) : 0;

    /* Odometer over the leading dims (tensor_ops.cpp:4600-4681). A size-1 dim
     * contributes no offset (stride-0 broadcast). */
    const int32_t nb = rank - 2;
    int64_t nbatch = 1;
    for (int32_t d = 0; d < nb; d++) nbatch *= out_shape[d];
    int32_t idx[16] = {0};
    for (int64_t b = 0; b < nbatch; b++) {
        int64_t o_off = 0, a_off = 0, b_off = 0, bias_off = 0;
        for (int32_t d = 0; d < nb; d++) {
            if (out_shape[d] != 1) o_off += idx[d] * so[d];
            if (A_shape[d] != 1) a_off += idx[d] * sa[d];
            if (B_shape[d] != 1) b_off += idx[d] * sb[d];
            if (bias && bias_shape[d] != 1) bias_off += idx[d] * sbias[d];
        }
        block_gemm(out + o_off, A + a_off, B + b_off, bias ? bias + bias_off : NULL,
                   bm_stride, bn_stride, M, N, K, (uint32_t)A_shape[rank - 1],
                   (uint32_t)B_shape[rank - 1], transA, transB);
        for (int32_t d = nb - 1; d >= 0; d--) {
            if (++idx[d] < out_shape[d]) break;
            idx[d] = 0;
        }
    }
    return 0;
}

void oracle_softmax_rows(float* out, const float* in, int64_t rows, int64_t n)
{
    for (int64_t r = 0; r < rows; r++) {
        const float* x = in + r * n;
        float* y = out + r * n;
        if (n <= 0) continue;
        float max = x[0];
        for (int64_t j = 0; j < n; j++)
            if (x[j] > max) max = x[j];
        float sum = 0.f;
        for (int64_t j = 0; j < n; j++) {
            y[j] = expf(x[j] - max);
            sum += y[j];
        }
        for (int64_t j = 0; j < n; j++) y[j] /= sum;
    }
}

void oracle_causal_mask(float* out, int32_t L)
{
    const float neg_inf = -INFINITY;
    memset(out, 0, (size_t)L * (size_t)L * sizeof(float));
    for (int32_t i = 0; i < L; ++i)
        for (int32_t j = i + 1; j < L; ++j) out[(int64_t)i * L + j] = neg_inf;
}

/* Sum `src` over one dim (keepdim), sequentially from 0 (tensor_ops.cpp:1714-1727). */
static void sum_dim(float* dst, const float* src, const int32_t* shape, int32_t rank, int32_t dim)
{
    int64_t post = 1, prev = 1;
    for (int32_t i = dim + 1; i < rank; i++) post *= shape[i];
    for (int32_t i = 0; i < dim; i++) prev *= shape[i];
    const int64_t size = shape[dim];
    for (int64_t p = 0; p < prev; p++)
        for (int64_t q = 0; q < post; q++) {
            float acc = 0.f;
            int64_t s = p * size * post + q;
            for (int64_t c = 0; c < size; c++, s += post) acc += src[s];
            dst[p * post + q] = acc;
        }
}

void oracle_reduce_to(float* dst, const float* src, const int32_t* dst_shape,
                      const int32_t* src_shape, int32_t rank)
{
    /* Reduce src over every dim where dst is 1 and src is not, in increasing dim
     * order (tensor_ops.cpp:3394-3398), then add elementwise with broadcast of
     * the remaining unit dims of src. */
    int32_t cur_shape[16] = {0};
    if (rank < 0 || rank > 16) return;
    int64_t n = 1;
    for (int32_t i = 0; i < rank; i++) { cur_shape[i] = src_shape[i]; n *= src_shape[i]; }
    float* cur = (float*)malloc((size_t)(n > 0 ? n : 1) * sizeof(float));
    memcpy(cur, src, (size_t)n * sizeof(float));
    for (int32_t d = 0; d < rank; d++) {
        if (dst_shape[d] == 1 && cur_shape[d] != 1) {
            int64_t m = n / cur_shape[d];
            float* nxt = (float*)malloc((size_t)(m > 0 ? m : 1) * sizeof(float));
            sum_dim(nxt, cur, cur_shape, rank, d);
            free(cur);
            cur = nxt;
            n = m;
            cur_shape[d] = 1;
        }
    }
    int64_t sd[16], sc[16];
    contiguous_strides(dst_shape, rank, sd);
    contiguous_strides(cur_shape, rank, sc);
    int64_t total = 1;
    for (int32_t i = 0; i < rank; i++) total *= dst_shape[i];
    int32_t idx[16] = {0};
    for (int64_t e = 0; e < total; e++) {
        int64_t off = 0;
        for (int32_t d = 0; d < rank; d++)
            if (cur_shape[d] != 1) off += idx[d] * sc[d];
        dst[e] += cur[off];
        for (int32_t d = rank - 1; d >= 0; d--) {
            if (++idx[d] < dst_shape[d]) break;
            idx[d] = 0;
        }
    }
    free(cur);
}

/* ---- the reference's CPU random stream (tensor_ops.cpp:5500-5521) ---- */
static uint64_t g_seed = 42ull;

static uint64_t splitmix(void)
{
    g_seed += 0x9E3779B97F4A7C15ull;
    g_seed = (g_seed ^ (g_seed >> 30)) * 0xBF58476D1CE4E5B9ull;
    g_seed = (g_seed ^ (g_seed >> 27)) * 0x94D049BB133111EBull;
    g_seed ^= (g_seed >> 31);
    return g_seed;
}

/* (x >> 8) converted to float, times 2^-56: a value in [0, 1). */
static float random_0_1(void)
{
    return (float)(splitmix() >> 8) * (1.0f / 72057594037927936.0f);
}

void oracle_rng_set_seed(uint64_t seed) { g_seed = seed; }

void oracle_rng_uniform(float* out, int64_t n, float lo, float hi)
{
    for (int64_t i = 0; i < n; i++) out[i] = random_0_1() * (hi - lo) + lo;
}

/* Box-Muller with the constants of tensor_ops.cpp:5515-5521. */
void oracle_rng_normal(float* out, int64_t n, float mean, float stddev)
{
    for (int64_t i = 0; i < n; i++) {
        const float r1 = random_0_1();
        const float r2 = random_0_1();
        const float z = sqrtf(-2.0f * logf(r1)) * cosf(2.0f * 3.1415926535f * r2);
        out[i] = z * stddev + mean;
    }
}

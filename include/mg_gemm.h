/*
 * mg_gemm.h -- C ABI of the B200 (sm_100a) GEMM library that replaces the
 * matmul hot path of Macrograd (MiquelNasarre/macrograd).
 *
 * The reference seam is the pair of device entry points
 *   kernel_ops::matmul       macrograd/include/cuda_backend.h:173
 *                            (body macrograd/kernels/cuda_backend.cu:3548-3759)
 *   kernel_ops::matmul_bias  macrograd/include/cuda_backend.h:174
 *                            (body macrograd/kernels/cuda_backend.cu:3761-4004)
 * called from Functional::matmul (macrograd/source/tensor_ops.cpp:4596, :4836)
 * and, through it, from the MatMulOp / MatMulBiasOp backward
 * (tensor_ops.cpp:4504-4517, :4723-4737). mg_matmul / mg_matmul_bias take the
 * same arguments (Shape objects flattened to int32 arrays) and keep the same
 * preconditions; mg_gemm is the general strided form under both.
 *
 * Plain C: pointers, sizes and status codes only. No call aborts; every
 * failure returns an mg_status and mg_last_error() describes it. All work is
 * enqueued on the caller's stream; no call synchronises the host except
 * mg_device_status() and the set-up calls.
 */
#ifndef MG_GEMM_H
#define MG_GEMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum mg_status {
    MG_OK = 0,
    MG_ERR_INVALID = 1,      /* bad arguments: shapes, ranks, pointers, strides */
    MG_ERR_UNSUPPORTED = 2,  /* valid request the library cannot run (e.g. no sm_100 device) */
    MG_ERR_CUDA = 3,         /* a CUDA runtime / driver call failed */
    MG_ERR_ALLOC = 4,        /* the workspace allocator returned NULL */
    MG_ERR_TIMEOUT = 5,      /* a kernel wait ran out its time limit (device status) */
    MG_ERR_NO_KERNEL = 6     /* the library has no kernel image for this device */
} mg_status;

/* Arithmetic of the tensor-core contraction.
 *   MG_MODE_TF32X3: fp32-accurate. Each fp32 operand x is split into
 *     hi = x with its low 13 mantissa bits cleared and lo = x - hi; the
 *     accumulator receives hi*hi + hi*lo + lo*hi on the TF32 tensor cores.
 *     The default.
 *   MG_MODE_TF32: one TF32 product per term (fast mode, ~1e-3 relative).
 * The reference computes in strict FP32 (CUBLAS_COMPUTE_32F,
 * cuda_backend.cu:3644); TF32X3 is the mode that matches it within 1e-5. */
typedef enum mg_mode {
    MG_MODE_TF32X3 = 0,
    MG_MODE_TF32 = 1,
    MG_MODE_DEFAULT = -1     /* use the library mode (mg_set_mode / MG_GEMM_MODE) */
} mg_mode;

/* Epilogue flags, combined with |. */
enum {
    MG_EPI_BIAS = 1,         /* + bias[m*bias_rs + n*bias_cs] (+ per-batch offset) */
    MG_EPI_CAUSAL = 2,       /* element (m, n) with n > m becomes -inf before softmax */
    MG_EPI_SOFTMAX = 4       /* row softmax over n (requires N <= 256) */
};

#define MG_MAX_BATCH_DIMS 6

/* General strided GEMM, in elements:
 *   C[b][m][n] = alpha * sum_k op(A)[b][m][k] * op(B)[b][k][n]
 *              (+ bias) (+ beta * C[b][m][n])     then optional row softmax.
 * op(A) is A stored [M][K] with row stride lda (trans_a = 0) or stored [K][M]
 * (trans_a = 1); op(B) is B stored [K][N] (trans_b = 0) or [N][K] (trans_b = 1).
 * The batch index b runs over batch[0..batch_rank) (row-major); an operand's
 * stride 0 on a dim broadcasts it there. C's stride 0 on a dim of size > 1
 * makes it a reduction dim: C receives the product summed over it (not with
 * the softmax epilogues; a bias must not vary along it). Operands are fp32
 * device memory. */
typedef struct mg_gemm_desc {
    int32_t M, N, K;
    int32_t trans_a, trans_b;
    int64_t lda, ldb, ldc;
    int32_t batch_rank;
    int32_t batch[MG_MAX_BATCH_DIMS];
    int64_t a_batch_stride[MG_MAX_BATCH_DIMS];
    int64_t b_batch_stride[MG_MAX_BATCH_DIMS];
    int64_t c_batch_stride[MG_MAX_BATCH_DIMS];
    int64_t bias_batch_stride[MG_MAX_BATCH_DIMS];
    int64_t bias_rs, bias_cs;  /* bias row / column strides (0 = broadcast) */
    float alpha;               /* scale on the product (1 for matmul) */
    float beta;                /* 0: overwrite C; 1: accumulate into C */
    int32_t epilogue;          /* MG_EPI_* flags */
    int32_t mode;              /* mg_mode */
} mg_gemm_desc;

/* Fills a descriptor for a plain row-major C[M][N] = op(A) op(B), batch 1. */
void mg_gemm_desc_init(mg_gemm_desc* d, int32_t M, int32_t N, int32_t K,
                       int32_t trans_a, int32_t trans_b);

/* Runs one described GEMM on `stream` (a cudaStream_t; NULL = legacy default). */
mg_status mg_gemm(const mg_gemm_desc* d, float* C, const float* A, const float* B,
                  const float* bias, void* stream);

/* Replaces kernel_ops::matmul (cuda_backend.h:173, cuda_backend.cu:3548).
 * Shapes are the rank-equalised shapes Functional::matmul passes
 * (tensor_ops.cpp:4547-4579): `rank` >= 2 entries each; A_shape and B_shape
 * are the STORAGE shapes (before the transpose flags); leading dims are equal
 * or 1; out_shape = [max(A_i, B_i)..., M, N]. All tensors contiguous fp32.
 * `out` is overwritten (the reference's out is zero-filled and written with
 * beta = 0, cuda_backend.cu:3554-3555). */
mg_status mg_matmul(float* out, const float* A, const float* B,
                    const int32_t* out_shape, const int32_t* A_shape,
                    const int32_t* B_shape, int32_t rank, int32_t trans_a,
                    int32_t trans_b, void* stream);

/* Replaces kernel_ops::matmul_bias (cuda_backend.h:174, cuda_backend.cu:3761).
 * bias_shape is rank-equalised to `rank`; each dim equals out's or is 1
 * (tensor_ops.cpp:4807-4818). Any such bias is fused into the epilogue. */
mg_status mg_matmul_bias(float* out, const float* A, const float* B, const float* bias,
                         const int32_t* out_shape, const int32_t* A_shape,
                         const int32_t* B_shape, const int32_t* bias_shape,
                         int32_t rank, int32_t trans_a, int32_t trans_b, void* stream);

/* Replaces the gradient accumulation of MatMulOp / MatMulBiasOp::_backward
 * (tensor_ops.cpp:4504-4517, :4723-4737):
 *     grad += Functional::matmul(X, Y, tX, tY)
 * which the reference runs as kernel_ops::matmul into a zero-filled
 * temporary followed by kernel_ops::shaped_add (cuda_backend.cu:4496-4592;
 * its squeeze kernel when the gradient's operand was broadcast). Here it is
 * one GEMM: out = beta * out + sum over the broadcast dims of op(A) op(B).
 * Shapes as mg_matmul, except that out_shape may be 1 on a leading dim where
 * max(A_i, B_i) is not: the product is summed over that dim (folded into the
 * kernel's K loop, no temporary). beta is 0 (overwrite) or 1 (accumulate into
 * out, the `+=`). */
mg_status mg_matmul_accumulate(float* out, const float* A, const float* B,
                               const int32_t* out_shape, const int32_t* A_shape,
                               const int32_t* B_shape, int32_t rank, int32_t trans_a,
                               int32_t trans_b, float beta, void* stream);

/* Replaces the squeeze direction of kernel_ops::shaped_add
 * (cuda_backend.cu:4496-4592) behind `tensor += other` when the tensor
 * broadcasts to `other` (tensor_ops.cpp:3393-3446), e.g. the bias gradient of
 * MatMulBiasOp::_backward (`bias.internal_gradient() += out.gradient()`,
 * tensor_ops.cpp:4736):
 *     dst = beta * dst + src summed over the dims where dst_shape is 1.
 * Both shapes have `rank` dims; dst_shape[i] is src_shape[i] or 1; both
 * tensors contiguous fp32. beta is 0 or 1. Deterministic (fixed summation
 * order for given shapes and device). */
mg_status mg_sum_into(float* dst, const float* src, const int32_t* dst_shape,
                      const int32_t* src_shape, int32_t rank, float beta, void* stream);

/* Fused attention-score product: out = softmax_rows(alpha * op(A) op(B) (+ bias)
 * (+ causal mask)), i.e. what the reference's MultiHeadSelfAttention computes
 * with Functional::matmul(Q / sqrt(d), K, mask, false, true) followed by
 * Tensor::softmax(-1) (mini_shakespeare/include/transformer.h:233-234,
 * tensor_ops.cpp:2034-2121). Shapes as mg_matmul_bias; bias may be NULL
 * (bias_shape ignored then). `causal` applies -inf strictly above the diagonal
 * (Functional::causal_mask, tensor_ops.cpp:5468-5492). Requires N <= 256. */
mg_status mg_matmul_softmax(float* out, const float* A, const float* B, const float* bias,
                            const int32_t* out_shape, const int32_t* A_shape,
                            const int32_t* B_shape, const int32_t* bias_shape,
                            int32_t rank, int32_t trans_a, int32_t trans_b,
                            float alpha, int32_t causal, void* stream);

/* Fused softmax backward (no counterpart in the reference, which runs it as
 * a separate pass, tensor_ops.cpp:2056-2059): with G = alpha * op(A) op(B)
 * the upstream gradient of a row softmax whose output is P,
 *     dS = P * (G - rowsum(P * G)),
 * e.g. the attention backward's dP = dO V^T (A = dO, B = V, trans_b = 1)
 * followed by the softmax derivative, in one launch. P has out's shape and is
 * contiguous like out. Shapes as mg_matmul. Requires N <= 256. */
mg_status mg_matmul_softmax_backward(float* dS, const float* A, const float* B, const float* P,
                                     const int32_t* out_shape, const int32_t* A_shape,
                                     const int32_t* B_shape, int32_t rank, int32_t trans_a,
                                     int32_t trans_b, float alpha, void* stream);

/* ---- multi-GPU: row-sharded GEMM with the all-gather fused into it ------
 * No counterpart in the reference (single-GPU only, README.md:538). A job of
 * R ranks (one process per GPU) splits the rows of A (and of C) into R blocks;
 * B is replicated. Each rank runs mg_gemm_scatter_rows on its rows, and every
 * finished tile of them reaches the full C of every rank (peer_C[0..npeers),
 * this rank's own included) at row row0 + m, over NVLink peer mappings -- so
 * the all-gather travels while the tensor cores work, instead of after. By
 * default the epilogue writes the tile into this rank's own C and the
 * kernel's export warps copy it on to the other ranks (MG_GEMM_EXPORT=0: the
 * epilogue stores every rank's copy itself; MG_GEMM_EXPORT=2: the rows are
 * computed in column bands, one launch each, and the copy engines send each
 * finished band while the next one computes; the call returns with `stream`
 * ordered after those copies). The export-warp and copy-engine forms need
 * one of peer_C in this process's own memory. No collective runs inside the
 * kernel; the caller orders steps across ranks (e.g. a small NCCL all-reduce
 * after the GEMM) before reading a C that other ranks write into, or
 * overwriting it again. `d` describes this rank's GEMM (M = its rows);
 * d->ldc is the row stride of the full C buffers, which have rows_full rows;
 * beta must be 0. */
#define MG_MAX_PEERS 8
mg_status mg_gemm_scatter_rows(const mg_gemm_desc* d, const float* A, const float* B,
                               const float* bias, float* const* peer_C, int32_t npeers,
                               int64_t row0, int64_t rows_full, void* stream);

/* CUDA IPC plumbing for peer_C: export a device buffer of this process
 * (a handle plus the buffer's offset inside its allocation), and map a buffer
 * another process exported (valid until mg_ipc_close). */
typedef struct mg_ipc_handle { unsigned char bytes[64]; } mg_ipc_handle;
mg_status mg_ipc_export(const void* dev_ptr, mg_ipc_handle* handle, uint64_t* offset);
mg_status mg_ipc_import(const mg_ipc_handle* handle, uint64_t offset, void** dev_ptr);
mg_status mg_ipc_close(void* dev_ptr);

/* No counterpart in the reference: an allocation-free form of mg_matmul.
 *
 * Some callers cannot let a library allocate device memory during a call:
 * runtimes that plan all device memory ahead of time and own every byte of
 * it, or latency-critical loops that must not touch an allocator. mg_matmul
 * takes scratch memory (through mg_set_allocator's allocator, else the
 * library's own stream-ordered pool) in three cases:
 *   1. an operand whose row pitch is not a multiple of 16 bytes (e.g. rows of
 *      65 floats) is first copied into padded scratch;
 *   2. when the last wave of output tiles would leave SMs idle, it is split
 *      along K, and the partial ranges exchange fp32 partial tiles through
 *      scratch slots with a zeroed counter per slot;
 *   3. only with MG_GEMM_PRESPLIT=1: the 3xTF32 lo planes of both operands.
 * This entry point takes 1 and 2 from a fixed buffer inside the library
 * instead -- a file-scope device array of MG_NOALLOC_SCRATCH_BYTES, which
 * every GPU that loads the library holds until the process exits -- and never
 * does 3. It calls no cudaMalloc / cudaFree and no allocator. Arguments,
 * results and errors are those of mg_matmul.
 *
 * Limits: a call whose re-laid-out operands (case 1) would need more than
 * MG_NOALLOC_SCRATCH_BYTES is rejected with MG_ERR_INVALID before anything
 * runs. When the K-split slots (case 2) do not fit in what case 1 leaves of
 * the buffer, the call runs without the K split: same result within the
 * tolerance, possibly slower than mg_matmul. The buffer is shared by all
 * calls on a device and keeps the previous call's contents (the split
 * counters are cleared on the call's stream before the kernel runs; every
 * other byte a call reads it has written first); calls that overlap on the
 * GPU (several streams, or several host threads) race on it, so serialise
 * them. The first call on each device looks up the buffer's device address;
 * make that first call before any stream capture. The cached address is not
 * valid across cudaDeviceReset. */
#define MG_NOALLOC_SCRATCH_BYTES (16u << 20)
mg_status mg_matmul_noalloc(float* out, const float* A, const float* B,
                            const int32_t* out_shape, const int32_t* A_shape,
                            const int32_t* B_shape, int32_t rank, int32_t trans_a,
                            int32_t trans_b, void* stream);

/* Workspace allocator, stream-ordered like the reference's MemPool
 * (cuda_backend.h:63-79: cudaMallocAsync / cudaFreeAsync on the library
 * stream). The library asks for scratch only on paths that need it: operands
 * whose row stride is not a multiple of 16 bytes are re-laid out there, a
 * K-split last wave exchanges its partial tiles there, and MG_GEMM_PRESPLIT=1
 * keeps the 3xTF32 lo planes there.
 * Passing NULL functions restores the default (cudaMallocAsync on the call's
 * stream). The allocator replaces MemPool::allocate/free for the workspace. */
typedef void* (*mg_alloc_fn)(size_t bytes, void* stream, void* ctx);
typedef void (*mg_free_fn)(void* ptr, void* stream, void* ctx);
void mg_set_allocator(mg_alloc_fn alloc_fn, mg_free_fn free_fn, void* ctx);

/* Library default mode (initially from env MG_GEMM_MODE=3xtf32|tf32, else TF32X3). */
mg_status mg_set_mode(int32_t mode);
int32_t mg_get_mode(void);

/* Message of the last failing call on this host thread ("" if none). */
const char* mg_last_error(void);

/* Reads (and with reset != 0 clears) the device-side status word of the
 * current device: MG_OK, or MG_ERR_TIMEOUT when a kernel's bounded wait ran
 * out (the kernel then skipped its remaining work and exited cleanly).
 * Synchronises the device. `detail` (may be NULL) receives a code naming the
 * wait that gave up. */
mg_status mg_device_status(int32_t* detail, int32_t reset);

/* Number of kernel launches the library has issued in this process
 * (all devices). For accounting in benchmarks. */
uint64_t mg_launch_count(void);

/* Library version string. */
const char* mg_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MG_GEMM_H */

// cuda_backend_seam.cu -- the reference's CUDA backend with the matmul seam.
//
// Compiles the reference's macrograd/kernels/cuda_backend.cu UNMODIFIED, from
// where it lies (include path set by the Makefile), with its two cuBLASLt
// matmul entry points renamed out of the way by the preprocessor, and then
// defines kernel_ops::matmul / matmul_bias from kernel_ops_matmul.inc in the
// same translation unit (so the seam sees `stream`, MemPool and
// MACROGRAD_CHECK exactly as the replaced code did). The renamed cuBLASLt
// functions are dead code: nothing calls them, and the cuBLASLt symbols they
// name resolve to the never-called stand-ins of cublaslt_absent.c, so the
// drop-in library does not link cuBLASLt. kernel_ops_fused.inc adds the
// device-side calls of the opt-in fused build (unused by the default one).
#include <cuda_runtime.h>

// MemPool::allocate zero-fills every block it hands out (cudaMemsetAsync,
// cuda_backend.cu:153). Its calls go through this wrapper, which skips the
// fill only while the fused build's Functional::matmul allocates its output
// (mg_seam_skip_zero_fill, kernel_ops_fused.inc) and otherwise forwards.
namespace mg_seam_zero_fill {
thread_local bool skip = false;
inline cudaError_t memset_async(void* p, int value, size_t bytes, cudaStream_t s)
{
    return skip ? cudaSuccess : cudaMemsetAsync(p, value, bytes, s);
}
}  // namespace mg_seam_zero_fill

#define matmul mg_unused_cublaslt_matmul
#define matmul_bias mg_unused_cublaslt_matmul_bias
#define cudaMemsetAsync mg_seam_zero_fill::memset_async
#include "cuda_backend.cu"
#undef cudaMemsetAsync
#undef matmul
#undef matmul_bias

namespace kernel_ops {
void matmul(void* out_data, const void* A_data, const void* B_data, const Shape& out_shape,
            const Shape& A_shape, const Shape& B_shape, bool transA, bool transB);
void matmul_bias(void* out_data, const void* A_data, const void* B_data, const void* bias,
                 const Shape& out_shape, const Shape& A_shape, const Shape& B_shape,
                 const Shape& bias_shape, bool transA, bool transB);
}  // namespace kernel_ops

#include "kernel_ops_matmul.inc"
#include "kernel_ops_fused.inc"

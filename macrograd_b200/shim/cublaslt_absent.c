/* cublaslt_absent.c -- link-time stand-ins for the cuBLASLt entry points that
 * the reference's renamed (and never called) cuBLASLt matmul bodies still
 * name, so the drop-in build links no cuBLASLt at all.
 *
 * cuda_backend_seam.cu compiles macrograd/kernels/cuda_backend.cu unmodified;
 * its `cublas` class and the two renamed matmul functions (cuda_backend.cu
 * :3450-4004) stay in the object as dead code, and nothing reaches them: every
 * GEMM goes through kernel_ops_matmul.inc into libmg_gemm.so, and the class's
 * handle, preference and workspace are function-local statics built only on
 * a first call that never comes. Each stand-in reports and returns
 * CUBLAS_STATUS_NOT_SUPPORTED (15), which the reference's CUBLAS_CHECK turns
 * into its usual error report, should a future change ever route a call here.
 * Only the symbol names matter to the linker; the stand-ins take no
 * arguments because they never run. */
#include <stdio.h>

#define MG_CUBLASLT_ABSENT(name)                                                           \
    int name(void)                                                                         \
    {                                                                                      \
        fprintf(stderr, "drop-in build: " #name " called, but cuBLASLt is not linked\n"); \
        return 15;                                                                         \
    }

MG_CUBLASLT_ABSENT(cublasLtCreate)
MG_CUBLASLT_ABSENT(cublasLtMatmul)
MG_CUBLASLT_ABSENT(cublasLtMatmulAlgoGetHeuristic)
MG_CUBLASLT_ABSENT(cublasLtMatmulDescCreate)
MG_CUBLASLT_ABSENT(cublasLtMatmulDescDestroy)
MG_CUBLASLT_ABSENT(cublasLtMatmulDescSetAttribute)
MG_CUBLASLT_ABSENT(cublasLtMatmulPreferenceCreate)
MG_CUBLASLT_ABSENT(cublasLtMatmulPreferenceSetAttribute)
MG_CUBLASLT_ABSENT(cublasLtMatrixLayoutCreate)
MG_CUBLASLT_ABSENT(cublasLtMatrixLayoutDestroy)
MG_CUBLASLT_ABSENT(cublasLtMatrixLayoutSetAttribute)

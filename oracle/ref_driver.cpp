// ref_driver.cpp -- a C entry layer over the REFERENCE's own CPU Tensor code.
//
// TEST INFRASTRUCTURE ONLY. Compiled by oracle/Makefile together with the
// reference's unmodified macrograd/source/tensor.cpp and tensor_ops.cpp into
// oracle/_ref/libmgref.so. It lets the tests pin the C restatement
// (mg_oracle.c) against the reference itself, and lets the benchmark's
// reference arm time the reference's own CPU matmul. Nothing here runs on the
// product path.
//
// Every function builds "cpu" Tensors, calls the reference API exactly as a
// user would (Functional::matmul, macrograd.h:219 / :224; autograd through
// Tensor::backward, tensor.cpp:878) and copies the result out.
#include <sys/mman.h>
#include <sys/wait.h>
#include <unistd.h>

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

int64_t numel_of(const int32_t* s, int32_t rank)
{
    int64_t n = 1;
    for (int32_t i = 0; i < rank; i++) n *= s[i];
    return n;
}

Tensor make_tensor(const float* data, const int32_t* s, int32_t rank, bool grad)
{
    Tensor t(make_shape(s, rank), "cpu", grad);
    std::memcpy(t.internal_data(), data, size_t(numel_of(s, rank)) * sizeof(float));
    return t;
}

}  // namespace

extern "C" {

// out = Functional::matmul(A, B[, bias], transA, transB) on CPU tensors.
// The shapes are passed as given to Functional::matmul (any rank it accepts);
// out receives the result's element count, written to *out_numel.
int ref_matmul(float* out, int64_t* out_numel, const float* A, const float* B,
               const float* bias, const int32_t* A_shape, int32_t A_rank,
               const int32_t* B_shape, int32_t B_rank, const int32_t* bias_shape,
               int32_t bias_rank, int32_t transA, int32_t transB)
{
    Tensor a = make_tensor(A, A_shape, A_rank, false);
    Tensor b = make_tensor(B, B_shape, B_rank, false);
    Tensor c = bias ? Functional::matmul(a, b, make_tensor(bias, bias_shape, bias_rank, false),
                                         transA != 0, transB != 0)
                    : Functional::matmul(a, b, transA != 0, transB != 0);
    const int64_t n = int64_t(c.numel());
    if (out) std::memcpy(out, c.internal_data(), size_t(n) * sizeof(float));
    if (out_numel) *out_numel = n;
    return 0;
}

// Forward + backward through the reference autograd with a given upstream
// gradient dC: loss = sum(C * dC), so C's gradient is exactly dC and the
// MatMulOp / MatMulBiasOp backward (tensor_ops.cpp:4504-4517, 4723-4737) runs
// with it, including the `+=` reduction of a broadcast operand's gradient.
int ref_matmul_backward(float* dA, float* dB, float* dbias, const float* A,
                        const float* B, const float* bias, const float* dC,
                        const int32_t* A_shape, int32_t A_rank, const int32_t* B_shape,
                        int32_t B_rank, const int32_t* bias_shape, int32_t bias_rank,
                        const int32_t* C_shape, int32_t C_rank, int32_t transA,
                        int32_t transB)
{
    Tensor a = make_tensor(A, A_shape, A_rank, true);
    Tensor b = make_tensor(B, B_shape, B_rank, true);
    Tensor bi;
    if (bias) bi = make_tensor(bias, bias_shape, bias_rank, true);
    Tensor c = bias ? Functional::matmul(a, b, bi, transA != 0, transB != 0)
                    : Functional::matmul(a, b, transA != 0, transB != 0);
    Tensor g = make_tensor(dC, C_shape, C_rank, false);
    Tensor loss = (c * g).flatten().sum(0);
    loss.backward();
    std::memcpy(dA, a.gradient().internal_data(), size_t(a.numel()) * sizeof(float));
    std::memcpy(dB, b.gradient().internal_data(), size_t(b.numel()) * sizeof(float));
    if (bias && dbias)
        std::memcpy(dbias, bi.gradient().internal_data(), size_t(bi.numel()) * sizeof(float));
    return 0;
}

// Tensor::softmax(-1) on a [rows, n] CPU tensor.
int ref_softmax_lastdim(float* out, const float* in, int64_t rows, int64_t n)
{
    int32_t s[2] = {int32_t(rows), int32_t(n)};
    Tensor t = make_tensor(in, s, 2, false);
    Tensor y = t.softmax(-1);
    std::memcpy(out, y.internal_data(), size_t(rows * n) * sizeof(float));
    return 0;
}

// The softmax derivative through the reference's autograd: P = softmax(S)
// over the last dim of a [rows, n] tensor, loss = sum(P * G), so S's gradient
// is what SoftOp::_backward (tensor_ops.cpp:2056-2059) makes of the upstream G.
int ref_softmax_backward(float* dS, float* P, const float* S, const float* G, int64_t rows, int64_t n)
{
    int32_t s[2] = {int32_t(rows), int32_t(n)};
    Tensor t = make_tensor(S, s, 2, true);
    Tensor y = t.softmax(-1);
    Tensor g = make_tensor(G, s, 2, false);
    Tensor loss = (y * g).flatten().sum(0);
    loss.backward();
    std::memcpy(P, y.internal_data(), size_t(rows * n) * sizeof(float));
    std::memcpy(dS, t.gradient().internal_data(), size_t(rows * n) * sizeof(float));
    return 0;
}

// Functional::causal_mask(L, "cpu").
int ref_causal_mask(float* out, int32_t L)
{
    Tensor m = Functional::causal_mask(unsigned(L), "cpu");
    std::memcpy(out, m.internal_data(), size_t(L) * size_t(L) * sizeof(float));
    return 0;
}

// Random::set_seed + Initialization::uniform / normal on a CPU tensor of n elements.
int ref_init_uniform(float* out, int64_t n, uint64_t seed, float lo, float hi)
{
    Random::set_seed(seed);
    int32_t s[1] = {int32_t(n)};
    Tensor t(make_shape(s, 1), "cpu", false);
    Initialization::uniform(t, lo, hi);
    std::memcpy(out, t.internal_data(), size_t(n) * sizeof(float));
    return 0;
}

int ref_init_normal(float* out, int64_t n, uint64_t seed, float mean, float stddev)
{
    Random::set_seed(seed);
    int32_t s[1] = {int32_t(n)};
    Tensor t(make_shape(s, 1), "cpu", false);
    Initialization::normal(t, mean, stddev);
    std::memcpy(out, t.internal_data(), size_t(n) * sizeof(float));
    return 0;
}

// Row-sliced C = A @ B (2-D, no transposes) over `workers` processes, each
// calling Functional::matmul on its own contiguous block of rows of A. Rows of
// C depend only on the same rows of A, so the result equals one full call; the
// split only spreads the reference's single-threaded CPU loop over cores.
// Processes, not threads: the reference's tensor reference counts are plain
// integers (tensor.cpp:615-621), so threads sharing B would race on them.
// The children share B copy-on-write and write their rows into a shared map.
int ref_matmul_rows_mp(float* C, const float* A, const float* B, int32_t M, int32_t N,
                       int32_t K, int32_t workers)
{
    if (workers < 1) workers = 1;
    if (workers > M) workers = M > 0 ? M : 1;
    const size_t cbytes = size_t(M) * size_t(N) * sizeof(float);
    void* shared = mmap(nullptr, cbytes ? cbytes : 4, PROT_READ | PROT_WRITE,
                        MAP_SHARED | MAP_ANONYMOUS, -1, 0);
    if (shared == MAP_FAILED) return 1;
    int32_t bshape[2] = {K, N};
    Tensor b = make_tensor(B, bshape, 2, false);
    const int32_t per = (M + workers - 1) / workers;
    std::vector<pid_t> kids;
    int rc = 0;
    for (int32_t t = 0; t < workers; t++) {
        const int32_t r0 = t * per;
        const int32_t r1 = (r0 + per < M) ? r0 + per : M;
        if (r0 >= r1) break;
        pid_t pid = fork();
        if (pid == 0) {
            int32_t ashape[2] = {r1 - r0, K};
            Tensor a = make_tensor(A + int64_t(r0) * K, ashape, 2, false);
            Tensor c = Functional::matmul(a, b);
            std::memcpy(static_cast<float*>(shared) + int64_t(r0) * N, c.internal_data(),
                        size_t(r1 - r0) * size_t(N) * sizeof(float));
            _exit(0);
        }
        if (pid < 0) { rc = 2; break; }
        kids.push_back(pid);
    }
    for (pid_t pid : kids) {
        int st = 0;
        if (waitpid(pid, &st, 0) < 0 || !WIFEXITED(st) || WEXITSTATUS(st) != 0) rc = 3;
    }
    if (rc == 0) std::memcpy(C, shared, cbytes);
    munmap(shared, cbytes ? cbytes : 4);
    return rc;
}

}  // extern "C"

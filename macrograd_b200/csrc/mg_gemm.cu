// mg_gemm.cu -- host side and C ABI of the sm_100a GEMM library.
//
// Replaces kernel_ops::matmul / kernel_ops::matmul_bias of Macrograd
// (macrograd/kernels/cuda_backend.cu:3548-4004). Where the reference builds
// cuBLASLt descriptors, a heuristic cache and per-batch pointer arrays
// (cuda_backend.cu:3556-3719), this library maps every operand onto a TMA
// tensor map whose extra dimensions carry the batch (stride-0 dims simply do
// not appear), and launches one persistent tcgen05 kernel per call.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>

#include "mg_gemm.h"
#include "mg_gemm_kernel.cuh"

namespace {

// ---------------------------------------------------------------- state
thread_local std::string g_last_error;
std::atomic<int32_t> g_mode{-2};                 // -2: not read from env yet
std::atomic<uint64_t> g_launches{0};
mg_alloc_fn g_alloc = nullptr;
mg_free_fn g_free = nullptr;
void* g_alloc_ctx = nullptr;
std::mutex g_mu;

__device__ int g_device_status[2];

constexpr int kMaxDevices = 64;

// Fixed scratch of mg_matmul_noalloc (MG_NOALLOC_SCRATCH_BYTES), one copy per
// GPU that loads this library, held until the process exits. In host code this
// name is only a handle for cudaGetSymbolAddress, never a device address. It
// holds the padded copies of operands TMA cannot read in place and, after
// them, the K-split partial slots and their counters.
static __device__ __align__(256) uint8_t g_noalloc_scratch[MG_NOALLOC_SCRATCH_BYTES];
// its device address, per device ordinal (null: not looked up yet; not valid
// across cudaDeviceReset, like the rest of the per-device state)
std::atomic<uint8_t*> g_noalloc_ptr[kMaxDevices];
struct DeviceState {
    std::atomic<bool> ready{false};   // set last, under g_mu (read without it)
    int sm_count = 0;
    int max_smem = 0;
    size_t attr_smem[3][8] = {};      // dynamic smem opted in, per kernel variant [row epilogue][width, pair]
    int max_clusters[3][4] = {};      // resident CTA pairs, per pair-kernel [row epilogue][tile width]
    int* status = nullptr;   // device address of g_device_status
    cudaMemPool_t pool = nullptr;   // the library's own stream-ordered pool (workspace)
    // the copy-engine all-gather: a stream per destination, an event per band
    std::atomic<bool> copy_ready{false};
    cudaStream_t copy_stream[mg::kMaxPeers] = {};
    cudaEvent_t band_done[mg::kMaxBands] = {};
    cudaEvent_t copies_done[mg::kMaxPeers] = {};
};
DeviceState g_dev[kMaxDevices];

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

// Peer buffers mapped by mg_ipc_import: the pointer handed out and the base
// cudaIpcOpenMemHandle returned (needed to unmap).
struct IpcMap {
    void* user = nullptr;
    void* base = nullptr;
    size_t size = 0;            // of the mapped allocation (0: unknown)
};
IpcMap g_ipc_maps[64];

// Whether p lies in a buffer mapped from another process by mg_ipc_import.
bool ipc_imported(const void* p)
{
    std::lock_guard<std::mutex> lk(g_mu);
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    for (const auto& m : g_ipc_maps) {
        if (!m.user) continue;
        const uintptr_t b = reinterpret_cast<uintptr_t>(m.base);
        if (m.size ? (a >= b && a < b + m.size) : p == m.user) return true;
    }
    return false;
}

// NVTX range around a C-ABI entry point, so that profiler timelines show the
// library's calls (header-only NVTX: without an attached tool a range costs a
// check of a function pointer).
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

mg_status fail(mg_status s, const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return s;
}

#define MG_CUDA_TRY(call)                                                                   \
    do {                                                                                    \
        cudaError_t e_ = (call);                                                            \
        if (e_ != cudaSuccess)                                                              \
            return fail(MG_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));      \
    } while (0)

int32_t resolve_default_mode()
{
    int32_t m = g_mode.load();
    if (m != -2) return m;
    int32_t v = MG_MODE_TF32X3;
    if (const char* e = std::getenv("MG_GEMM_MODE")) {
        if (!std::strcmp(e, "tf32") || !std::strcmp(e, "TF32") || !std::strcmp(e, "1xtf32")) v = MG_MODE_TF32;
    }
    int32_t expect = -2;
    g_mode.compare_exchange_strong(expect, v);
    return g_mode.load();
}

template <int BN, bool kPair, int kRow>
constexpr auto kernel_of()
{
    return &mg::mg_gemm_tc_kernel<BN, kPair, kRow>;
}

int bn_slot(int bn) { return bn == 64 ? 0 : (bn == 128 ? 1 : (bn == 224 ? 3 : 2)); }

mg_status device_state(DeviceState** out)
{
    int dev = 0;
    MG_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(MG_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    DeviceState& d = g_dev[dev];
    if (!d.ready.load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!d.ready.load(std::memory_order_relaxed)) {
            cudaDeviceProp prop;
            MG_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
            if (prop.major != 10)
                return fail(MG_ERR_UNSUPPORTED,
                            "device %d is sm_%d%d; this library is built for sm_100a (B200) only",
                            dev, prop.major, prop.minor);
            d.sm_count = prop.multiProcessorCount;
            d.max_smem = (int)prop.sharedMemPerBlockOptin;
            void* sp = nullptr;
            MG_CUDA_TRY(cudaGetSymbolAddress(&sp, g_device_status));
            d.status = static_cast<int*>(sp);
            if (g_encode == nullptr) {
                void* fn = nullptr;
                cudaDriverEntryPointQueryResult q;
                MG_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
                if (q != cudaDriverEntryPointSuccess || fn == nullptr)
                    return fail(MG_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
                g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
            }
            // Workspace (K-split partials, re-laid-out operands) comes from a
            // pool of the library's own that keeps its memory between calls:
            // the device's default pool would hand it back at every
            // synchronisation and re-map it on the next call.
            cudaMemPoolProps pp = {};
            pp.allocType = cudaMemAllocationTypePinned;
            pp.location.type = cudaMemLocationTypeDevice;
            pp.location.id = dev;
            MG_CUDA_TRY(cudaMemPoolCreate(&d.pool, &pp));
            uint64_t keep = ~0ull;
            MG_CUDA_TRY(cudaMemPoolSetAttribute(d.pool, cudaMemPoolAttrReleaseThreshold, &keep));
            d.ready.store(true, std::memory_order_release);
        }
    }
    *out = &d;
    return MG_OK;
}

// Streams and events of the copy-engine all-gather, made on first use.
mg_status copy_engine_state(DeviceState* d)
{
    if (d->copy_ready.load(std::memory_order_acquire)) return MG_OK;
    std::lock_guard<std::mutex> lk(g_mu);
    if (d->copy_ready.load(std::memory_order_relaxed)) return MG_OK;
    for (int q = 0; q < mg::kMaxPeers; ++q) {
        if (!d->copy_stream[q]) MG_CUDA_TRY(cudaStreamCreateWithFlags(&d->copy_stream[q], cudaStreamNonBlocking));
        if (!d->copies_done[q]) MG_CUDA_TRY(cudaEventCreateWithFlags(&d->copies_done[q], cudaEventDisableTiming));
    }
    for (int b = 0; b < mg::kMaxBands; ++b)
        if (!d->band_done[b]) MG_CUDA_TRY(cudaEventCreateWithFlags(&d->band_done[b], cudaEventDisableTiming));
    d->copy_ready.store(true, std::memory_order_release);
    return MG_OK;
}

// ---------------------------------------------------------------- helpers
struct Operand {
    const float* ptr;
    int64_t rows, cols;       // stored matrix (cols contiguous)
    int64_t ld;               // elements between stored rows
    int64_t bs[MG_MAX_BATCH_DIMS];
};

// Mapping of an operand's batch dims onto at most 3 extra tensor-map dims.
struct BatchMap {
    int nmap = 0;
    int64_t extent[3] = {1, 1, 1};
    int64_t stride[3] = {0, 0, 0};   // elements
    int8_t map[MG_MAX_BATCH_DIMS];
    int32_t mult[MG_MAX_BATCH_DIMS];
};

// Innermost batch dim first; stride-0 dims are broadcast and get no map dim;
// a dim whose stride continues the current map dim (stride == map stride *
// extent so far) merges into it (mixed-radix coordinate).
bool build_batch_map(int nbd, const int32_t* bsize, const int64_t* bs, BatchMap* bm)
{
    for (int d = 0; d < MG_MAX_BATCH_DIMS; ++d) { bm->map[d] = -1; bm->mult[d] = 0; }
    bm->nmap = 0;
    for (int d = nbd - 1; d >= 0; --d) {
        if (bs[d] == 0 || bsize[d] == 1) continue;
        const int j = bm->nmap - 1;
        if (j >= 0 && bs[d] == bm->stride[j] * bm->extent[j] &&
            bm->extent[j] * (int64_t)bsize[d] < (1ll << 31)) {
            bm->map[d] = (int8_t)j;
            bm->mult[d] = (int32_t)bm->extent[j];
            bm->extent[j] *= bsize[d];
        } else {
            if (bm->nmap == 3) return false;
            bm->map[d] = (int8_t)bm->nmap;
            bm->mult[d] = 1;
            bm->extent[bm->nmap] = bsize[d];
            bm->stride[bm->nmap] = bs[d];
            bm->nmap++;
        }
    }
    return true;
}

bool tma_compatible(const Operand& x, const BatchMap& bm)
{
    if (reinterpret_cast<uintptr_t>(x.ptr) & 15u) return false;
    if ((x.ld * 4) % 16 != 0) return false;
    for (int j = 0; j < bm.nmap; ++j)
        if ((bm.stride[j] * 4) % 16 != 0) return false;
    if (x.cols >= (1ll << 31) || x.rows >= (1ll << 31)) return false;
    return true;
}

mg_status encode_map(CUtensorMap* map, const Operand& x, const BatchMap& bm, int box_rows_is_k,
                     uint32_t box_outer, bool plain = false)
{
    // dims: {cols (contiguous), rows, batch map dims...}
    cuuint64_t dims[5];
    cuuint64_t strides[4];
    cuuint32_t box[5];
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const int rank = 2 + bm.nmap;
    dims[0] = (cuuint64_t)x.cols;
    dims[1] = (cuuint64_t)x.rows;
    strides[0] = (cuuint64_t)(x.ld * 4);
    for (int j = 0; j < bm.nmap; ++j) {
        dims[2 + j] = (cuuint64_t)bm.extent[j];
        strides[1 + j] = (cuuint64_t)(bm.stride[j] * 4);
        box[2 + j] = 1;
    }
    box[0] = 32;
    box[1] = box_rows_is_k ? 32u : box_outer;
    // K-major boxes: 16-byte-chunk 128B swizzle; MN-major boxes: 32-byte-chunk
    // 128B swizzle (the only MN-major layout the TF32 MMA reads); `plain`: no
    // swizzle, for an A tile that only the split warps read (A in TMEM).
    const CUtensorMapSwizzle sw = plain ? CU_TENSOR_MAP_SWIZZLE_NONE
                                        : (box_rows_is_k ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B);
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank,
                          const_cast<float*>(x.ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MG_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return MG_OK;
}

// ---------------------------------------------------------------- aux kernels
// Copies every distinct batch element of an operand into a dense buffer whose
// rows are padded to a multiple of 4 floats (16 bytes), so a TMA map can read
// it. Used only for operands whose own strides break TMA's 16-byte rules
// (e.g. the vocab-65 logits of the character model: rows of 260 bytes).
struct PadParams {
    const float* src;
    float* dst;
    int64_t rows, cols, src_ld, dst_ld;
    int nd;
    int64_t size[MG_MAX_BATCH_DIMS];
    int64_t sstride[MG_MAX_BATCH_DIMS];
};

__global__ void pad_copy_kernel(PadParams p)
{
    const int64_t row_global = blockIdx.x;   // over nbatch * rows
    const int64_t b = row_global / p.rows;
    const int64_t r = row_global - b * p.rows;
    int64_t rem = b, soff = 0;
    for (int d = p.nd - 1; d >= 0; --d) {
        const int64_t i = rem % p.size[d];
        rem /= p.size[d];
        soff += i * p.sstride[d];
    }
    const float* s = p.src + soff + r * p.src_ld;
    float* o = p.dst + row_global * p.dst_ld;
    for (int64_t c = threadIdx.x; c < p.dst_ld; c += blockDim.x) o[c] = c < p.cols ? s[c] : 0.f;
}

// lo plane of the 3xTF32 split over an operand's storage span: lo = x - hi,
// hi = x with its 13 low mantissa bits cleared (0 for non-finite x). One HBM
// pass (4 bytes read, 4 written per element); the GEMM then loads hi (the raw
// operand) and lo tiles instead of splitting every tile it loads.
__global__ void lo_plane_kernel(const float* __restrict__ x, float* __restrict__ lo, int64_t n)
{
    const int64_t n4 = n / 4;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float4* l4 = reinterpret_cast<float4*>(lo);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 v = x4[i];
        float4 r;
        r.x = __uint_as_float(mg::split_lo(__float_as_uint(v.x)));
        r.y = __uint_as_float(mg::split_lo(__float_as_uint(v.y)));
        r.z = __uint_as_float(mg::split_lo(__float_as_uint(v.z)));
        r.w = __uint_as_float(mg::split_lo(__float_as_uint(v.w)));
        l4[i] = r;
    }
    for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        lo[i] = __uint_as_float(mg::split_lo(__float_as_uint(x[i])));
}

// K == 0: C = bias (+ beta C), or the softmax of the bias / mask alone.
struct FillParams {
    int M, N, nbd;
    int bsize[MG_MAX_BATCH_DIMS];
    float* C;
    int64_t ldc, c_bs[MG_MAX_BATCH_DIMS];
    const float* bias;
    int64_t bias_rs, bias_cs, bias_bs[MG_MAX_BATCH_DIMS];
    float beta;
    int epi;
    int64_t rows_total;
};

__global__ void k0_fill_kernel(FillParams p)
{
    const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= p.rows_total) return;
    int64_t b = row / p.M;
    const int m = (int)(row - b * p.M);
    int64_t coff = 0, boff = 0;
    for (int d = p.nbd - 1; d >= 0; --d) {
        const int64_t i = b % p.bsize[d];
        b /= p.bsize[d];
        coff += i * p.c_bs[d];
        boff += i * p.bias_bs[d];
    }
    float* c = p.C + coff + (int64_t)m * p.ldc;
    const float* bi = p.bias ? p.bias + boff + (int64_t)m * p.bias_rs : nullptr;
    auto val = [&](int n) {
        float v = 0.f;
        if (bi && (p.epi & mg::kEpiBias)) v += bi[(int64_t)n * p.bias_cs];
        if ((p.epi & mg::kEpiCausal) && n > m) v = -INFINITY;
        return v;
    };
    if (p.epi & mg::kEpiSoftmax) {
        float mx = -INFINITY, sum = 0.f;
        for (int n = 0; n < p.N; ++n) mx = fmaxf(mx, val(n));
        for (int n = 0; n < p.N; ++n) sum += expf(val(n) - mx);
        for (int n = 0; n < p.N; ++n) c[n] = expf(val(n) - mx) / sum;
    } else {
        for (int n = 0; n < p.N; ++n) c[n] = val(n) + (p.beta != 0.f ? p.beta * c[n] : 0.f);
    }
}

// dst = beta * dst + src summed over the dims where dst has size 1 and src
// does not: the squeeze direction of the reference's `+=` (its
// kernel_ops::shaped_add, cuda_backend.cu:4496-4592, reached from
// tensor_ops.cpp:3393-3446), e.g. a bias gradient, the output gradient summed
// over its rows. Dims are canonicalised on the host (size-1 dims dropped,
// neighbours of the same kind merged): src is then nk kept dims and nr reduced
// dims, interleaved, contiguous. Deterministic: the reduced range is cut into
// `splits` contiguous parts, each part's partial sums go to part[split][o],
// and sum_parts_kernel adds them in split order.
struct SumParams {
    const float* src;
    float* dst;
    float* part;                // [splits][P] partial sums (splits > 1)
    int64_t P, R;               // output elements; reduced elements per output
    int64_t rchunk;             // reduced elements per split
    int splits;
    int rows;                   // src is [R][P] row-major (the common case)
    int vec;                    // rows && P % 4 == 0 and 16-byte aligned pointers: float4 columns
    float beta;
    int nk, nr;
    int64_t ksize[MG_MAX_BATCH_DIMS + 2], kstride[MG_MAX_BATCH_DIMS + 2];   // kept dims, outer first
    int64_t rsize[MG_MAX_BATCH_DIMS + 2], rstride[MG_MAX_BATCH_DIMS + 2];   // reduced dims, outer first
};

__device__ __forceinline__ int64_t sum_src_offset(const SumParams& p, int64_t o, int64_t r)
{
    int64_t off = 0;
    for (int i = p.nk - 1; i >= 0; --i) {
        off += (o % p.ksize[i]) * p.kstride[i];
        o /= p.ksize[i];
    }
    for (int i = p.nr - 1; i >= 0; --i) {
        off += (r % p.rsize[i]) * p.rstride[i];
        r /= p.rsize[i];
    }
    return off;
}

__global__ void sum_into_kernel(SumParams p)
{
    const int s = blockIdx.y;
    const int64_t r0 = (int64_t)s * p.rchunk;
    const int64_t r1 = min(p.R, r0 + p.rchunk);
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p.vec) {
        // four consecutive outputs per thread, rows read as float4 (coalesced)
        if (t >= p.P / 4) return;
        const float4* src = reinterpret_cast<const float4*>(p.src) + t;
        const int64_t ld = p.P / 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int64_t r = r0; r < r1; ++r) {
            const float4 v = __ldg(src + r * ld);
            acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
        }
        if (p.splits > 1) {
            reinterpret_cast<float4*>(p.part + (int64_t)s * p.P)[t] = acc;
        } else {
            float4* d = reinterpret_cast<float4*>(p.dst) + t;
            if (p.beta != 0.f) {
                const float4 o = *d;
                acc.x += p.beta * o.x, acc.y += p.beta * o.y, acc.z += p.beta * o.z, acc.w += p.beta * o.w;
            }
            *d = acc;
        }
        return;
    }
    if (t >= p.P) return;
    float acc = 0.f;
    if (p.rows) {
        for (int64_t r = r0; r < r1; ++r) acc += __ldg(p.src + r * p.P + t);
    } else {
        for (int64_t r = r0; r < r1; ++r) acc += __ldg(p.src + sum_src_offset(p, t, r));
    }
    if (p.splits > 1) p.part[(int64_t)s * p.P + t] = acc;
    else p.dst[t] = p.beta != 0.f ? acc + p.beta * p.dst[t] : acc;
}

__global__ void sum_parts_kernel(const float* __restrict__ part, float* dst, int64_t P, int splits, float beta)
{
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= P) return;
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) acc += part[(int64_t)s * P + t];
    dst[t] = beta != 0.f ? acc + beta * dst[t] : acc;
}

// ---------------------------------------------------------------- workspace
// Per-call scratch. By default it allocates through the registered allocator
// (or cudaMallocAsync) and frees stream-ordered at the end of the call. Given
// an arena (the no-allocation entry point), it hands out 256-byte aligned
// pieces of that fixed buffer instead and never allocates or frees.
struct Workspace {
    void* stream;
    cudaMemPool_t pool = nullptr;
    void* ptrs[8] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    int n = 0;
    uint8_t* arena = nullptr;
    size_t arena_cap = 0, arena_used = 0;
    ~Workspace()
    {
        if (arena) return;
        for (int i = 0; i < n; ++i) {
            if (g_free) g_free(ptrs[i], stream, g_alloc_ctx);
            else cudaFreeAsync(ptrs[i], (cudaStream_t)stream);
        }
    }
    void* get(size_t bytes)
    {
        if (arena) {
            const size_t at = (arena_used + 255) & ~size_t(255);
            if (at + bytes > arena_cap) return nullptr;
            arena_used = at + bytes;
            return arena + at;
        }
        void* p = nullptr;
        if (g_alloc) p = g_alloc(bytes, stream, g_alloc_ctx);
        else if (cudaMallocFromPoolAsync(&p, bytes, pool, (cudaStream_t)stream) != cudaSuccess) p = nullptr;
        if (p) ptrs[n++] = p;
        return p;
    }
};

// Scratch bytes relayout_operand asks for: the operand's distinct batch
// elements, each rows x (cols rounded up to 4 floats), plus 16 bytes.
size_t relayout_bytes(const Operand& x, int nbd, const int32_t* bsize)
{
    int64_t nbatch = 1;
    for (int d = 0; d < nbd; ++d)
        if (x.bs[d] != 0 && bsize[d] != 1) nbatch *= bsize[d];
    return (size_t)(nbatch * x.rows * ((x.cols + 3) / 4 * 4)) * sizeof(float) + 16;
}

// Re-lays out operand x (stored rows x cols, per-dim batch strides) densely
// with 16-byte row pitch; afterwards its batch strides are dense over its own
// non-broadcast dims.
mg_status relayout_operand(Operand& x, int nbd, const int32_t* bsize, Workspace& ws, cudaStream_t st)
{
    PadParams pp;
    pp.src = x.ptr;
    pp.rows = x.rows;
    pp.cols = x.cols;
    pp.src_ld = x.ld;
    pp.dst_ld = (x.cols + 3) / 4 * 4;
    pp.nd = 0;
    int64_t nbatch = 1;
    int dims[MG_MAX_BATCH_DIMS];
    for (int d = 0; d < nbd; ++d) {
        if (x.bs[d] != 0 && bsize[d] != 1) {
            dims[pp.nd] = d;
            pp.size[pp.nd] = bsize[d];
            pp.sstride[pp.nd] = x.bs[d];
            pp.nd++;
            nbatch *= bsize[d];
        }
    }
    const int64_t mat = pp.rows * pp.dst_ld;
    float* dst = static_cast<float*>(ws.get((size_t)(nbatch * mat) * sizeof(float) + 16));
    if (!dst) return fail(MG_ERR_ALLOC, "workspace allocation of %lld bytes failed",
                          (long long)(nbatch * mat * 4));
    pp.dst = dst;
    if (nbatch * x.rows > 0) {
        if (nbatch * x.rows >= (1ll << 31)) return fail(MG_ERR_UNSUPPORTED, "operand too large to re-lay out");
        pad_copy_kernel<<<(unsigned)(nbatch * x.rows), 128, 0, st>>>(pp);
        MG_CUDA_TRY(cudaGetLastError());
        g_launches++;
    }
    // new dense batch strides over the operand's own dims
    int64_t s = mat;
    for (int i = pp.nd - 1; i >= 0; --i) {
        x.bs[dims[i]] = s;
        s *= pp.size[i];
    }
    x.ptr = dst;
    x.ld = pp.dst_ld;
    return MG_OK;
}

int tuning_int(const char* name, int dflt, int lo, int hi);

// K split of the last partial wave (mg_plan.h): MG_GEMM_SPLIT=0 turns it off,
// MG_GEMM_SPLIT_MIN_KB sets the shortest range in K-blocks: by default 16, or
// 4 for a launch of less than half a wave (e.g. 16 tiles of a batched
// [8, 256, 384] product on 74 SM pairs), whose few tiles would otherwise run
// their whole K one stage after another while most SMs idle.
int plan_split(mg::GemmParams& gp, int units)
{
    const int dflt = 2 * (int64_t)gp.total_tiles <= units ? 4 : 16;
    const int min_kb = tuning_int("MG_GEMM_SPLIT", 1, 0, 1) ? tuning_int("MG_GEMM_SPLIT_MIN_KB", dflt, 1, 1 << 20) : 0;
    return mg::plan_k_split(gp.plan, gp.total_tiles, units, gp.num_kb, min_kb);
}

// Plans the K split for `units` resident CTAs (pairs) and takes its workspace:
// one slot of 2 x 128 x BN floats per partial range (both CTAs of a pair) plus
// a zeroed counter per slot and CTA. Without workspace the launch goes unsplit.
template <int BN>
bool setup_split(mg::GemmParams& gp, int units, Workspace* ws, cudaStream_t st, bool allow)
{
    const int nslots = allow ? plan_split(gp, units) : 0;
    gp.tail_share = 0;
    if (nslots == 0) {
        gp.plan.full_tiles = gp.total_tiles;
        gp.plan.nlev = 0;
        return false;
    }
    const size_t part = (size_t)nslots * 2 * mg::kBM * BN * sizeof(float);
    // fused all-gather: a counter per last-level tile half, for the shared export
    const bool tail = gp.export_peers && gp.npeers > 0 && tuning_int("MG_GEMM_TAIL_SHARE", 1, 0, 1);
    const size_t nflags = (size_t)nslots * 2 + (tail ? (size_t)gp.plan.lev_tiles[gp.plan.nlev - 1] * 2 : 0);
    const size_t flags = nflags * sizeof(unsigned int);
    uint8_t* w = static_cast<uint8_t*>(ws ? ws->get(part + flags) : nullptr);
    if (!w || cudaMemsetAsync(w + part, 0, flags, st) != cudaSuccess) {
        gp.plan.full_tiles = gp.total_tiles;
        gp.plan.nlev = 0;
        return false;
    }
    gp.part_ws = reinterpret_cast<float*>(w);
    gp.part_flag = reinterpret_cast<unsigned int*>(w + part);
    gp.tail_share = tail ? 1 : 0;
    gp.tail_flag = gp.part_flag + (size_t)nslots * 2;
    return true;
}

template <int BN, bool kPair, int kRow>
mg_status launch_tc(DeviceState* dev, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& malo,
                    const CUtensorMap& mblo, const CUtensorMap& mp, const CUtensorMap& mc, mg::GemmParams& gp, const mg::PeerMaps& pm,
                    cudaStream_t st, Workspace* ws, bool allow_split)
{
    using L = mg::Layout<BN, kPair>;
    const int split = gp.split;
    // raw (+ lo) tiles; with A in TMEM only B's lo tile sits beside each stage
    // (b2: inside the stage, right after B)
    const size_t per_stage = (size_t)L::kStageBytes + (split ? (gp.a_tmem ? L::kBBytes : L::kStageBytes) : 0);
    // alignment slack + barriers + the epilogue's store staging (4 KB per warp)
    // (+ the softmax backward's P ring, when two operand stages still fit)
    size_t fixed = 1024 + mg::kSharedStateBytes + (size_t)mg::kEpiWarps * mg::kStageFloatsPerWarp * 4 + 64;
    const size_t ring = (size_t)mg::kPRingSlots * mg::kPSlotBytes;
    if (kRow != mg::kRowSoftmaxBwd || (size_t)dev->max_smem < fixed + ring + 2 * per_stage) gp.p_tma = 0;
    if (gp.p_tma) fixed += ring;
    int stages = (int)((size_t)(dev->max_smem - (int)fixed) / per_stage);
    stages = std::min(stages, mg::kMaxStages);
    if (stages < 2) return fail(MG_ERR_UNSUPPORTED, "not enough shared memory for a 2-stage pipeline");
    // A second staging block per epilogue warp (two TMA stores of C in flight
    // a warp) where it costs no operand stage the K loop can use: stages to
    // spare, or short K (every K-block of a tile resident at once).
    // MG_GEMM_STAGE_BLOCKS=1 / 2 forces one / two where two stages still fit.
    gp.stage_blocks = 1;
    if (kRow != mg::kRowSoftmaxBwd && gp.c_tma) {
        const size_t more = (size_t)mg::kEpiWarps * mg::kStageFloatsPerWarp * 4;
        const int stages2 = std::min((int)((size_t)(dev->max_smem - (int)(fixed + more)) / per_stage), mg::kMaxStages);
        const int want = tuning_int("MG_GEMM_STAGE_BLOCKS", 0, 0, 2);
        if (stages2 >= 2 && (want == 2 || (want == 0 && stages2 >= std::min(stages, gp.num_kb)))) {
            gp.stage_blocks = 2;
            fixed += more;
            stages = stages2;
        }
    }
    gp.stages = stages;
    // A in TMEM (gp.a_tmem, set with the maps): 64 columns a stage after the accumulators
    gp.a_col0 = 0;
    gp.tmem_cols = (int)L::kTmemCols;
    if (gp.a_tmem) {
        // the A tiles' columns fit beside the two accumulators (2 BN wide each with b2)
        // (MG_GEMM_A_TMEM_STAGES caps them)
        const int acc_cols = 2 * BN * (gp.b2 ? 2 : 1);
        stages = std::min(stages, std::min((512 - acc_cols) / 64, tuning_int("MG_GEMM_A_TMEM_STAGES", 8, 2, 8)));
        gp.stages = stages;
        gp.a_col0 = acc_cols;
        gp.tmem_cols = (int)mg::pow2_at_least((uint32_t)(acc_cols + 64 * stages));
    }
    const size_t smem = fixed + per_stage * stages;
    auto k = kernel_of<BN, kPair, kRow>();
    const int slot = bn_slot(BN) + (kPair ? 4 : 0);
    if (dev->attr_smem[kRow][slot] < smem) {
        MG_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        dev->attr_smem[kRow][slot] = smem;
    }
    if (kPair) {
        // one cluster of two CTAs (two SMs) per work unit, persistent over the
        // tiles; as many clusters as can be resident at once
        cudaLaunchConfig_t cfg = {};
        cfg.blockDim = dim3(mg::kThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (dev->max_clusters[kRow][slot - 4] == 0) {
            cfg.gridDim = dim3((unsigned)dev->sm_count, 1, 1);
            int n = 0;
            MG_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, k, &cfg));
            dev->max_clusters[kRow][slot - 4] = std::max(1, std::min(n, dev->sm_count / 2));
        }
        const int resident = dev->max_clusters[kRow][slot - 4];
        const bool split_k = setup_split<BN>(gp, resident, ws, st, allow_split);
        gp.dbuf = (!split_k && gp.num_kb <= gp.chunk_kb && tuning_int("MG_GEMM_DBUF", 1, 0, 1)) ? 1 : 0;
        if (split_k) {
            // the final K-ranges wait for partials from other CTAs of the grid:
            // launch it cooperatively, so every CTA is resident at once
            cudaLaunchAttribute attr2[2] = {attr[0], {}};
            attr2[1].id = cudaLaunchAttributeCooperative;
            attr2[1].val.cooperative = 1;
            cfg.attrs = attr2;
            cfg.numAttrs = 2;
            cfg.gridDim = dim3((unsigned)(2 * resident), 1, 1);
            if (cudaLaunchKernelEx(&cfg, k, ma, mb, malo, mblo, mp, mc, gp, pm) == cudaSuccess) {
                g_launches++;
                return MG_OK;
            }
            (void)cudaGetLastError();   // not launchable cooperatively here: run unsplit
            gp.plan.full_tiles = gp.total_tiles;
            gp.plan.nlev = 0;
            gp.tail_share = 0;
            gp.dbuf = (gp.num_kb <= gp.chunk_kb && tuning_int("MG_GEMM_DBUF", 1, 0, 1)) ? 1 : 0;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
        }
        const int pairs = std::max(1, std::min(gp.total_tiles, resident));
        cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
        MG_CUDA_TRY(cudaLaunchKernelEx(&cfg, k, ma, mb, malo, mblo, mp, mc, gp, pm));
    } else {
        const bool split_k = setup_split<BN>(gp, dev->sm_count, ws, st, allow_split);
        gp.dbuf = (!split_k && gp.num_kb <= gp.chunk_kb && tuning_int("MG_GEMM_DBUF", 1, 0, 1)) ? 1 : 0;
        if (split_k) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)dev->sm_count, 1, 1);
            cfg.blockDim = dim3(mg::kThreads, 1, 1);
            cfg.dynamicSmemBytes = smem;
            cfg.stream = st;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeCooperative;
            attr[0].val.cooperative = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            if (cudaLaunchKernelEx(&cfg, k, ma, mb, malo, mblo, mp, mc, gp, pm) == cudaSuccess) {
                g_launches++;
                return MG_OK;
            }
            (void)cudaGetLastError();
            gp.plan.full_tiles = gp.total_tiles;
            gp.plan.nlev = 0;
            gp.tail_share = 0;
            gp.dbuf = (gp.num_kb <= gp.chunk_kb && tuning_int("MG_GEMM_DBUF", 1, 0, 1)) ? 1 : 0;
        }
        const int grid = std::max(1, std::min(gp.total_tiles, dev->sm_count));
        k<<<grid, mg::kThreads, smem, st>>>(ma, mb, malo, mblo, mp, mc, gp, pm);
        MG_CUDA_TRY(cudaGetLastError());
    }
    g_launches++;
    return MG_OK;
}

// Tuning override from the environment (clamped), else the default.
int tuning_int(const char* name, int dflt, int lo, int hi)
{
    if (const char* e = std::getenv(name)) {
        const int v = std::atoi(e);
        if (v >= lo && v <= hi) return v;
    }
    return dflt;
}

// Elements from an operand's first to its last element, as its tensor map
// addresses them: the storage a same-layout lo plane needs.
int64_t operand_span(const Operand& x, const BatchMap& bm)
{
    int64_t span = (x.rows - 1) * x.ld + x.cols;
    for (int j = 0; j < bm.nmap; ++j) span += (bm.extent[j] - 1) * bm.stride[j];
    return span;
}

// Pre-split pays one HBM pass over both operands and workspace of their size,
// and doubles the bytes each stage loads; in-kernel splitting repeats the
// split once per tile that loads an operand tile. Measured at 8192^3 the
// in-kernel split is faster (189 vs 184 TFLOP/s, median of 3), so pre-split
// is off unless MG_GEMM_PRESPLIT=1 asks for it.
bool want_presplit(double flops, int64_t m_tiles, int64_t n_tiles)
{
    if (const char* e = std::getenv("MG_GEMM_PRESPLIT")) {
        if (e[0] == '1') return flops > 0 && m_tiles > 0 && n_tiles > 0;
    }
    return false;
}

// Pair kernel (two SMs per 256-row tile) when a batch has more than 128 rows;
// MG_GEMM_PAIR=0 / =1 forces the single-SM / pair kernel (tests, tuning).
// Output tile width. Pair tiles may be 224 wide instead of 256 when that
// takes fewer waves over the SM pairs. A K-block costs the pipeline about the
// same time at either width (its hand-offs, not the MMAs, set the pace), so
// only the wave count counts and 256 wins ties.
int choose_bn(const mg_gemm_desc* d, bool pair, int64_t nbatch, int64_t red_steps, const DeviceState* dev)
{
    const int forced = tuning_int("MG_GEMM_BN", 0, 64, 256);
    const bool row_epi = (d->epilogue & (MG_EPI_SOFTMAX | mg::kEpiSoftmaxBwd)) != 0;
    const bool fits = !row_epi || d->N <= forced;   // softmax: one tile per row
    // (the row epilogues are built for widths 64, 128 and 256 only)
    if (fits && (forced == 64 || forced == 128 || forced == 256 || (forced == 224 && pair && !row_epi)))
        return forced;
    const int base = d->N <= 64 ? 64 : (d->N <= 128 ? 128 : 256);
    if (row_epi) return base;
    const int64_t m_tiles = (d->M + (pair ? 2 : 1) * mg::kBM - 1) / ((pair ? 2 : 1) * mg::kBM);
    const int64_t units = std::max(1, pair ? dev->sm_count / 2 : dev->sm_count);
    // Less than a wave of tiles at the base width: narrower tiles put more
    // SMs to work, and may make the K split unnecessary. At these sizes a
    // tile's K loop is paced by its stage hand-offs, not by its width, so the
    // widths compare by the K-blocks of their busiest unit as the split would
    // cut them (plan_k_split: up to 8 ranges a tile, ranges of at least 4
    // K-blocks below half a wave, 16 above), a split's partial-sum exchange
    // (workspace traffic in proportion to the tile) counted as 3 K-blocks per
    // 64 columns. Measured: 2048 x 384 x 384 runs 26.6 us at width 64
    // unsplit, 32.0 us at 256 split three ways; 384 x 384 x (8 x 256) is
    // faster at 64 split six ways than at 256 split eight ways; the linear
    // layer's 1536 x 384 x 16384 weight gradient stays at 256 split six ways.
    auto tiles_at = [&](int bn) { return nbatch * m_tiles * ((d->N + bn - 1) / bn); };
    if (tiles_at(base) < units) {
        const int64_t num_kb = std::max<int64_t>(1, (d->K + mg::kBK - 1) / mg::kBK * red_steps);
        auto busiest = [&](int bn) {
            const int64_t t = tiles_at(bn);
            const int64_t min_kb = 2 * t <= units ? 4 : 16;
            int64_t sp = std::min<int64_t>(std::min<int64_t>(8, units / t), num_kb / min_kb);
            if (sp < 2) sp = 1;
            return (num_kb + sp - 1) / sp + (sp > 1 ? 3 * bn / 64 : 0);
        };
        int best = base;
        for (int bn : {128, 64})
            if (bn < base && tiles_at(bn) <= units && busiest(bn) < busiest(best)) best = bn;
        return best;
    }
    if (!pair || base != 256) return base;
    auto cost = [&](int bn) {
        const int64_t tiles = nbatch * m_tiles * ((d->N + bn - 1) / bn);
        return (tiles + units - 1) / units;   // waves
    };
    return cost(224) < cost(256) ? 224 : 256;
}

// The SM-pair kernel for output matrices of more than 128 rows -- it halves
// the B tile each SM loads and keeps more stages in flight, which large GEMMs
// need -- except for many small matrices (at most 256 rows each, e.g. the
// per-head products of attention) whose single-SM tiles fill at least a wave:
// there the pair's cross-SM hand-off per stage costs more than it saves
// (measured on the attention products: 0.066 vs 0.079 ms for P V). The fused
// softmax backward wider than 128 columns in 3xTF32 stays on pairs, whose
// shared memory has room for its P ring beside two operand stages.
bool use_pair(const mg_gemm_desc* d, int64_t nbatch, int sm_count, int32_t mode)
{
    if (const char* e = std::getenv("MG_GEMM_PAIR")) {
        if (e[0] == '0') return false;
        if (e[0] == '1') return true;
    }
    if (d->M <= mg::kBM) return false;
    if (d->M <= 2 * mg::kBM && nbatch * ((d->M + mg::kBM - 1) / mg::kBM) >= sm_count) {
        const bool wide_bwd = (d->epilogue & mg::kEpiSoftmaxBwd) && d->N > 128 && mode == MG_MODE_TF32X3;
        if (!wide_bwd) return false;
    }
    return true;
}

mg_status validate(const mg_gemm_desc* d, float* C, const float* A, const float* B, const float* bias)
{
    if (!d) return fail(MG_ERR_INVALID, "descriptor is NULL");
    if (d->M < 0 || d->N < 0 || d->K < 0) return fail(MG_ERR_INVALID, "negative M/N/K (%d, %d, %d)", d->M, d->N, d->K);
    if (d->batch_rank < 0 || d->batch_rank > MG_MAX_BATCH_DIMS)
        return fail(MG_ERR_INVALID, "batch_rank %d outside [0, %d]", d->batch_rank, MG_MAX_BATCH_DIMS);
    for (int i = 0; i < d->batch_rank; ++i)
        if (d->batch[i] < 0) return fail(MG_ERR_INVALID, "negative batch size at dim %d", i);
    if (d->mode != MG_MODE_DEFAULT && d->mode != MG_MODE_TF32X3 && d->mode != MG_MODE_TF32)
        return fail(MG_ERR_INVALID, "unknown mode %d", d->mode);
    if (d->epilogue & ~(MG_EPI_BIAS | MG_EPI_CAUSAL | MG_EPI_SOFTMAX | mg::kEpiSoftmaxBwd))
        return fail(MG_ERR_INVALID, "unknown epilogue flags 0x%x", d->epilogue);
    if ((d->epilogue & mg::kEpiSoftmaxBwd) && (d->epilogue != mg::kEpiSoftmaxBwd || d->N > 256 || d->beta != 0.f))
        return fail(MG_ERR_INVALID, "the softmax-backward epilogue stands alone, with N <= 256 and beta 0");
    if ((d->epilogue & MG_EPI_CAUSAL) && !(d->epilogue & MG_EPI_SOFTMAX))
        return fail(MG_ERR_INVALID, "MG_EPI_CAUSAL requires MG_EPI_SOFTMAX");
    if ((d->epilogue & MG_EPI_SOFTMAX) && d->N > 256)
        return fail(MG_ERR_UNSUPPORTED, "softmax epilogue needs N <= 256 (got %d)", d->N);
    if ((d->epilogue & MG_EPI_SOFTMAX) && d->beta != 0.f)
        return fail(MG_ERR_INVALID, "softmax epilogue does not accumulate (beta must be 0)");
    if ((d->epilogue & MG_EPI_BIAS) && !bias) return fail(MG_ERR_INVALID, "MG_EPI_BIAS with NULL bias");
    const int64_t a_cols = d->trans_a ? d->M : d->K;
    const int64_t b_cols = d->trans_b ? d->K : d->N;
    if (d->lda < std::max<int64_t>(1, a_cols) || d->ldb < std::max<int64_t>(1, b_cols) ||
        d->ldc < std::max<int64_t>(1, d->N))
        return fail(MG_ERR_INVALID, "leading dimension smaller than the row length");
    int64_t total = (int64_t)d->M * d->N;
    for (int i = 0; i < d->batch_rank; ++i) total *= d->batch[i];
    if (total > 0) {
        if (!C) return fail(MG_ERR_INVALID, "C is NULL");
        if (d->K > 0 && (!A || !B)) return fail(MG_ERR_INVALID, "A or B is NULL");
    }
    return MG_OK;
}

}  // namespace

// ====================================================================== C ABI
extern "C" {

void mg_gemm_desc_init(mg_gemm_desc* d, int32_t M, int32_t N, int32_t K, int32_t trans_a, int32_t trans_b)
{
    std::memset(d, 0, sizeof(*d));
    d->M = M;
    d->N = N;
    d->K = K;
    d->trans_a = trans_a != 0;
    d->trans_b = trans_b != 0;
    d->lda = std::max<int64_t>(1, trans_a ? M : K);
    d->ldb = std::max<int64_t>(1, trans_b ? K : N);
    d->ldc = std::max<int64_t>(1, N);
    d->alpha = 1.f;
    d->beta = 0.f;
    d->mode = MG_MODE_DEFAULT;
}

// Destinations of a row-sharded GEMM whose rows go to every rank's full C.
struct ScatterSpec {
    int npeers;
    int64_t row0;
    int64_t rows_full;          // rows of every rank's full C
    float* peers[mg::kMaxPeers];
};

// The body of mg_gemm. With arena == nullptr the per-call scratch (operand
// re-layout, K-split slots, pre-split lo planes) is allocated as usual; with
// an arena the re-layout and the split slots come from that fixed buffer (a
// re-layout that does not fit is rejected before anything runs; split slots
// that do not fit leave the launch unsplit) and there is no pre-split.
static mg_status gemm_impl(const mg_gemm_desc* d, float* C, const float* A, const float* B,
                           const float* bias, void* stream, uint8_t* arena, size_t arena_cap,
                           const ScatterSpec* scatter = nullptr, const float* aux = nullptr)
{
    g_last_error.clear();
    mg_status s = validate(d, C, A, B, bias);
    if (s != MG_OK) return s;
    if ((d->epilogue & mg::kEpiSoftmaxBwd) && !aux)
        return fail(MG_ERR_INVALID, "the softmax-backward epilogue needs P (mg_matmul_softmax_backward)");
    cudaStream_t st = (cudaStream_t)stream;
    // Batch dims where C has stride 0 (and size > 1) are reduction dims: C
    // receives the sum of the product over them (the `+=` of a gradient whose
    // operand was broadcast), folded into the kernel's K loop. The others are
    // tiled; nbatch counts their output matrices.
    int64_t nbatch = 1, red_steps = 1, all_batch = 1;
    bool red[MG_MAX_BATCH_DIMS] = {false, false, false, false, false, false};
    for (int i = 0; i < d->batch_rank; ++i) {
        all_batch *= d->batch[i];
        red[i] = d->c_batch_stride[i] == 0 && d->batch[i] > 1;
        if (red[i]) red_steps *= d->batch[i];
        else nbatch *= d->batch[i];
    }
    if (d->M == 0 || d->N == 0 || all_batch == 0) return MG_OK;
    if (red_steps > 1) {
        if (d->epilogue & (MG_EPI_SOFTMAX | mg::kEpiSoftmaxBwd))
            return fail(MG_ERR_INVALID, "a row softmax epilogue cannot reduce over batch dims (C batch stride 0)");
        if (scatter) return fail(MG_ERR_INVALID, "the scattering GEMM cannot reduce over batch dims");
        for (int i = 0; i < d->batch_rank; ++i)
            if (red[i] && (d->epilogue & MG_EPI_BIAS) && d->bias_batch_stride[i] != 0)
                return fail(MG_ERR_INVALID, "bias varies along reduced batch dim %d", i);
    }

    DeviceState* dev = nullptr;
    s = device_state(&dev);
    if (s != MG_OK) return s;

    const int nbd = d->batch_rank;
    const bool has_bias = (d->epilogue & MG_EPI_BIAS) != 0;

    if (d->K == 0) {
        FillParams fp;
        std::memset(&fp, 0, sizeof(fp));
        fp.M = d->M;
        fp.N = d->N;
        fp.nbd = nbd;
        for (int i = 0; i < nbd; ++i) {
            fp.bsize[i] = red[i] ? 1 : d->batch[i];   // a sum over an empty K is 0: C = bias (+ beta C) once
            fp.c_bs[i] = d->c_batch_stride[i];
            fp.bias_bs[i] = d->bias_batch_stride[i];
        }
        fp.C = C;
        fp.ldc = d->ldc;
        fp.bias = has_bias ? bias : nullptr;
        fp.bias_rs = d->bias_rs;
        fp.bias_cs = d->bias_cs;
        fp.beta = d->beta;
        fp.epi = d->epilogue;
        fp.rows_total = nbatch * d->M;
        k0_fill_kernel<<<(unsigned)((fp.rows_total + 127) / 128), 128, 0, st>>>(fp);
        MG_CUDA_TRY(cudaGetLastError());
        g_launches++;
        return MG_OK;
    }

    const int32_t mode = d->mode == MG_MODE_DEFAULT ? resolve_default_mode() : d->mode;

    Operand a{A, d->trans_a ? d->K : d->M, d->trans_a ? d->M : d->K, d->lda, {0}};
    Operand b{B, d->trans_b ? d->N : d->K, d->trans_b ? d->K : d->N, d->ldb, {0}};
    for (int i = 0; i < nbd; ++i) {
        a.bs[i] = d->a_batch_stride[i];
        b.bs[i] = d->b_batch_stride[i];
    }

    Workspace ws;
    ws.stream = stream;
    ws.pool = dev->pool;
    ws.arena = arena;
    ws.arena_cap = arena_cap;
    BatchMap am, bmp;
    const bool a_ok = build_batch_map(nbd, d->batch, a.bs, &am) && tma_compatible(a, am);
    const bool b_ok = build_batch_map(nbd, d->batch, b.bs, &bmp) && tma_compatible(b, bmp);
    if (arena) {
        size_t need = 0;
        if (!a_ok) need = ((need + 255) & ~size_t(255)) + relayout_bytes(a, nbd, d->batch);
        if (!b_ok) need = ((need + 255) & ~size_t(255)) + relayout_bytes(b, nbd, d->batch);
        if (need > arena_cap)
            return fail(MG_ERR_INVALID,
                        "this call needs %zu bytes of scratch to re-lay out its operands; the "
                        "no-allocation entry point has %zu (MG_NOALLOC_SCRATCH_BYTES)",
                        need, arena_cap);
    }
    if (!a_ok) {
        s = relayout_operand(a, nbd, d->batch, ws, st);
        if (s != MG_OK) return s;
        if (!build_batch_map(nbd, d->batch, a.bs, &am) || !tma_compatible(a, am))
            return fail(MG_ERR_UNSUPPORTED, "operand A cannot be mapped for TMA");
    }
    if (!b_ok) {
        s = relayout_operand(b, nbd, d->batch, ws, st);
        if (s != MG_OK) return s;
        if (!build_batch_map(nbd, d->batch, b.bs, &bmp) || !tma_compatible(b, bmp))
            return fail(MG_ERR_UNSUPPORTED, "operand B cannot be mapped for TMA");
    }

    const bool pair = use_pair(d, nbatch, dev->sm_count, mode);
    const int bn = choose_bn(d, pair, nbatch, red_steps, dev);
    const int tile_rows = pair ? 2 * mg::kBM : mg::kBM;   // output rows per tile
    const int b_rows = pair ? bn / 2 : bn;                // B rows (N) one CTA loads

    const int a_mn = d->trans_a ? 1 : 0;   // A stored [K][M]: M contiguous
    const int b_mn = d->trans_b ? 0 : 1;   // B stored [K][N]: N contiguous
    CUtensorMap ma, mb;
    s = encode_map(&ma, a, am, a_mn, mg::kBM);
    if (s != MG_OK) return s;
    s = encode_map(&mb, b, bmp, b_mn, (uint32_t)b_rows);
    if (s != MG_OK) return s;

    // 3xTF32 on large problems: precompute the lo planes once (HBM pass) so the
    // main loop loads hi and lo tiles instead of splitting every tile it loads.
    const int64_t m_tiles_est = (d->M + tile_rows - 1) / tile_rows;
    const int64_t n_tiles_est = (d->N + bn - 1) / bn;
    const bool presplit = mode == MG_MODE_TF32X3 && arena == nullptr &&
                          want_presplit(2.0 * d->M * d->N * d->K * (double)all_batch, m_tiles_est, n_tiles_est);
    // Narrow 3xTF32 tiles (single SM or pair): A's hi and lo tiles go to TMEM (written
    // by the split warps, 64 columns a stage after the accumulators) and the
    // MMAs read A there. Their three MMAs per K-step otherwise each read the
    // whole 128-row A tile from shared memory for only 64-128 output columns,
    // which sets the pace of the K loop. Only the split warps then read A's
    // shared-memory tile, so an MN-major A lands unswizzled (rows of M at
    // 128-byte K steps). MG_GEMM_A_TMEM=0 keeps A in shared memory.
    const bool a_tmem = mode == MG_MODE_TF32X3 && !presplit && bn <= 128 &&
                        tuning_int("MG_GEMM_A_TMEM", 1, 0, 1) && (!pair || tuning_int("MG_GEMM_A_TMEM_PAIR", 1, 0, 1));
    if (a_tmem && a_mn) {
        s = encode_map(&ma, a, am, a_mn, mg::kBM, true);
        if (s != MG_OK) return s;
    }
    CUtensorMap malo = ma, mblo = mb;
    if (presplit) {
        for (int which = 0; which < 2; ++which) {
            Operand x = which ? b : a;
            const BatchMap& bm = which ? bmp : am;
            const int64_t span = operand_span(x, bm);
            float* lo = static_cast<float*>(ws.get((size_t)span * sizeof(float) + 16));
            if (!lo) return fail(MG_ERR_ALLOC, "workspace allocation of %lld bytes failed", (long long)(span * 4));
            const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((span / 4 + 255) / 256, 8ll * dev->sm_count));
            lo_plane_kernel<<<(unsigned)blocks, 256, 0, st>>>(x.ptr, lo, span);
            MG_CUDA_TRY(cudaGetLastError());
            g_launches++;
            x.ptr = lo;
            s = which ? encode_map(&mblo, x, bm, b_mn, (uint32_t)b_rows) : encode_map(&malo, x, bm, a_mn, mg::kBM);
            if (s != MG_OK) return s;
        }
    }

    mg::GemmParams gp;
    std::memset(&gp, 0, sizeof(gp));
    gp.M = d->M;
    gp.N = d->N;
    gp.K = d->K;
    gp.kb_per = (d->K + mg::kBK - 1) / mg::kBK;
    if ((int64_t)gp.kb_per * red_steps >= (1ll << 31))
        return fail(MG_ERR_UNSUPPORTED, "K x reduced batch too large (%lld K-blocks)", (long long)gp.kb_per * red_steps);
    gp.red_steps = (int)red_steps;
    gp.num_kb = gp.kb_per * gp.red_steps;
    gp.m_tiles = (d->M + tile_rows - 1) / tile_rows;
    gp.n_tiles = (d->N + bn - 1) / bn;
    gp.tiles_per_batch = gp.m_tiles * gp.n_tiles;
    const int64_t total = nbatch * gp.tiles_per_batch;
    if (total >= (1ll << 31)) return fail(MG_ERR_UNSUPPORTED, "too many output tiles (%lld)", (long long)total);
    gp.total_tiles = (int)total;
    gp.plan.full_tiles = gp.total_tiles;   // no K split unless launch_tc plans one
    gp.plan.num_kb = gp.num_kb;
    gp.group_m = tuning_int("MG_GEMM_GROUP_M", 16, 1, 1 << 16);
    // any positive value; at least the K-blocks of a tile means no promotion at
    // all (one accumulator over the whole K: within TF32 mode's tolerance, not
    // within 3xTF32's -- the MMA's accumulation truncates)
    gp.chunk_kb = tuning_int("MG_GEMM_CHUNK_KB", mg::kChunkKb, 1, 1 << 20);
    gp.relay_spin = tuning_int("MG_GEMM_RELAY_SPIN", 0, 0, 1);
    gp.split = mode == MG_MODE_TF32X3 ? 1 : 0;
    gp.presplit = presplit ? 1 : 0;
    gp.a_tmem = a_tmem ? 1 : 0;
    // width 64 with A in TMEM and a plain epilogue: B's lo tile right after B's
    // in the stage, so [B hi | B lo] is one operand 128 wide and a K-step is two
    // MMAs (A hi, A lo) instead of three -- each MMA costs about the same time
    // at widths up to 128, so the K loop's MMAs take two thirds of the time.
    // MG_GEMM_B2=0 keeps three MMAs of width 64.
    gp.b2 = (a_tmem && !pair && bn == 64 && (d->epilogue & (MG_EPI_SOFTMAX | mg::kEpiSoftmaxBwd)) == 0 &&
             tuning_int("MG_GEMM_B2", 1, 0, 1)) ? 1 : 0;
    gp.a_mn = a_mn;
    gp.b_mn = b_mn;
    gp.a_rank = 2 + am.nmap;
    gp.b_rank = 2 + bmp.nmap;
    // instruction descriptor: D f32, A/B tf32, majors, N = bn, M = 128 (one SM) or 256 (pair).
    // A read from TMEM (a_tmem) is always K-major there (lane = row, column = K),
    // whatever its layout in memory: the MN-major flag with a TMEM A operand is
    // an illegal instruction.
    gp.idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(a_mn && !a_tmem) << 15) | ((uint32_t)b_mn << 16) |
               ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(tile_rows >> 4) << 24);
    gp.idesc2 = (gp.idesc & ~(0x3Fu << 17)) | ((uint32_t)((2 * bn) >> 3) << 17);   // N = 2 bn (b2)
    gp.nbd = nbd;
    for (int i = 0; i < mg::kMaxBatchDims; ++i) {
        gp.bsize[i] = i < nbd && !red[i] ? d->batch[i] : 1;
        gp.rsize[i] = i < nbd && red[i] ? d->batch[i] : 1;
        gp.a_map[i] = am.map[i];
        gp.b_map[i] = bmp.map[i];
        gp.a_mult[i] = am.mult[i];
        gp.b_mult[i] = bmp.mult[i];
        gp.c_bs[i] = i < nbd ? d->c_batch_stride[i] : 0;
        gp.bias_bs[i] = i < nbd ? d->bias_batch_stride[i] : 0;
    }
    gp.C = C;
    gp.ldc = d->ldc;
    gp.bias = has_bias ? bias : nullptr;
    gp.aux = aux;
    // output blocks by TMA tensor stores where C allows a map (16-byte row
    // pitch and batch strides, aligned base) and is only written (beta 0, no
    // rows to other ranks): the epilogue warps go on while the writes drain
    CUtensorMap mc = ma;
    if (!scatter && d->beta == 0.f && tuning_int("MG_GEMM_C_TMA", 1, 0, 1)) {
        Operand cx{C, d->M, d->N, d->ldc, {0}};
        for (int i = 0; i < nbd; ++i) cx.bs[i] = d->c_batch_stride[i];
        BatchMap cbm;
        if (build_batch_map(nbd, d->batch, cx.bs, &cbm) && tma_compatible(cx, cbm)) {
            s = encode_map(&mc, cx, cbm, 0, 32);
            if (s != MG_OK) return s;
            gp.c_tma = 1;
            gp.c_rank = 2 + cbm.nmap;
            for (int i = 0; i < mg::kMaxBatchDims; ++i) {
                gp.c_map[i] = cbm.map[i];
                gp.c_mult[i] = cbm.mult[i];
            }
        }
    }
    // softmax backward: P (laid out like C) streamed by TMA into the epilogue's
    // ring, where its layout allows a tensor map (16-byte row pitch and batch
    // strides, aligned base); otherwise the epilogue reads it directly
    CUtensorMap mp = ma;
    if (aux && !scatter) {
        Operand px{aux, d->M, d->N, d->ldc, {0}};
        for (int i = 0; i < nbd; ++i) px.bs[i] = d->c_batch_stride[i];
        BatchMap pbm;
        if (build_batch_map(nbd, d->batch, px.bs, &pbm) && tma_compatible(px, pbm) &&
            tuning_int("MG_GEMM_P_TMA", 1, 0, 1)) {
            s = encode_map(&mp, px, pbm, 0, 128);
            if (s != MG_OK) return s;
            gp.p_tma = 1;
            gp.p_rank = 2 + pbm.nmap;
            for (int i = 0; i < mg::kMaxBatchDims; ++i) {
                gp.p_map[i] = pbm.map[i];
                gp.p_mult[i] = pbm.mult[i];
            }
        }
    }
    gp.bias_rs = d->bias_rs;
    gp.bias_cs = d->bias_cs;
    gp.alpha = d->alpha;
    gp.beta = d->beta;
    gp.epi = d->epilogue;
    // causal row softmax: a tile's work grows with its m-tile (the live
    // columns end at the diagonal), and consecutive tiles alternate m-tiles of
    // the same batch; mirrored waves give each CTA both kinds in turn instead
    // of one kind every wave (an even CTA count keeps a tile's parity)
    gp.plan.mirror = ((d->epilogue & mg::kEpiSoftmax) && (d->epilogue & mg::kEpiCausal) &&
                      tuning_int("MG_GEMM_MIRROR", 1, 0, 1)) ? 1 : 0;
    gp.status = dev->status;
    // bounded waits: 4 s, unless shortened (MG_GEMM_WAIT_LIMIT_MS, 1..4000);
    // MG_GEMM_TEST_STALL=1 withholds every CTA's second K-block so that a test
    // can watch a wait run out and the kernel report it (mg_device_status)
    const int limit_ms = (int)(mg::kWaitLimitNs / 1000000ull);
    gp.wait_limit_ns = (uint64_t)tuning_int("MG_GEMM_WAIT_LIMIT_MS", limit_ms, 1, limit_ms) * 1000000ull;
    gp.test_stall = tuning_int("MG_GEMM_TEST_STALL", 0, 0, 1);
    mg::PeerMaps pm;
    std::memset(&pm, 0, sizeof(pm));
    // Export mode (default): the epilogue writes this GPU's own full C and the
    // kernel's export warps copy each finished tile to the other ranks, so the
    // epilogue never waits on NVLink. Needs one destination in this process's
    // own memory (not mapped from another rank).
    int local = -1;
    if (scatter && tuning_int("MG_GEMM_EXPORT", 1, 0, 2) != 0) {   // (a 2 that reached here: export warps)
        for (int q = 0; q < scatter->npeers && local < 0; ++q)
            if (!ipc_imported(scatter->peers[q])) local = q;
    }
    if (scatter && local >= 0) {
        gp.C = scatter->peers[local];
        gp.peer_row0 = scatter->row0;
        gp.export_peers = 1;
        bool vec = d->N % 4 == 0 && d->ldc % 4 == 0;
        for (int i = 0; i < nbd; ++i) vec = vec && d->c_batch_stride[i] % 4 == 0;
        for (int q = 0; q < scatter->npeers; ++q) {
            vec = vec && (reinterpret_cast<uintptr_t>(scatter->peers[q]) & 15u) == 0;
            if (q != local) gp.peers[gp.npeers++] = scatter->peers[q];
        }
        gp.export_vec = vec ? 1 : 0;
        // one export warp: the second one sped the copies up less than it slowed
        // the GEMM (8 x 1024-row shards: 1129 vs 1068 TFLOP/s for the job)
        gp.export_threads = tuning_int("MG_GEMM_EXPORT_WARPS", 1, 1, 2) * 32;
        gp.export_stream = tuning_int("MG_GEMM_EXPORT_STREAM", 0, 0, 1);
    } else if (scatter) {
        gp.npeers = scatter->npeers;
        gp.peer_row0 = scatter->row0;
        for (int q = 0; q < scatter->npeers; ++q) gp.peers[q] = scatter->peers[q];
        // TMA bulk stores need a 2-D C with 16-byte aligned rows in every destination
        bool tma_ok = nbd == 0 && (d->ldc * 4) % 16 == 0 && scatter->rows_full < (1ll << 31);
        for (int q = 0; q < scatter->npeers; ++q)
            tma_ok = tma_ok && (reinterpret_cast<uintptr_t>(scatter->peers[q]) & 15u) == 0;
        if (tma_ok) {
            for (int q = 0; q < scatter->npeers; ++q) {
                cuuint64_t dims[2] = {(cuuint64_t)d->N, (cuuint64_t)scatter->rows_full};
                cuuint64_t strides[1] = {(cuuint64_t)(d->ldc * 4)};
                cuuint32_t box[2] = {32, 32};
                cuuint32_t estr[2] = {1, 1};
                CUresult r = g_encode(&pm.m[q], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, scatter->peers[q], dims, strides,
                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
                if (r != CUDA_SUCCESS) return fail(MG_ERR_CUDA, "tensor map of peer C %d failed (%d)", q, (int)r);
            }
            gp.peer_tma = 1;
        }
    }

    // the row softmax (and its backward) needs whole rows in one tile: no K split there
    const int row = (d->epilogue & MG_EPI_SOFTMAX) ? mg::kRowSoftmax
                    : (d->epilogue & mg::kEpiSoftmaxBwd) ? mg::kRowSoftmaxBwd : mg::kRowNone;
    const bool allow_split = row == mg::kRowNone;
    auto go = [&](auto bn_c, auto pair_c, auto row_c) {
        return launch_tc<decltype(bn_c)::value, decltype(pair_c)::value, decltype(row_c)::value>(
            dev, ma, mb, malo, mblo, mp, mc, gp, pm, st, &ws, allow_split);
    };
    using T = std::true_type;
    using F = std::false_type;
    auto by_width = [&](auto pair_c, auto row_c) -> mg_status {
        switch (bn) {
        case 64: return go(std::integral_constant<int, 64>{}, pair_c, row_c);
        case 128: return go(std::integral_constant<int, 128>{}, pair_c, row_c);
        case 256: return go(std::integral_constant<int, 256>{}, pair_c, row_c);
        default: return fail(MG_ERR_UNSUPPORTED, "no kernel of tile width %d for this epilogue", bn);
        }
    };
    if (row == mg::kRowSoftmax) {
        using R = std::integral_constant<int, mg::kRowSoftmax>;
        return pair ? by_width(T{}, R{}) : by_width(F{}, R{});
    }
    if (row == mg::kRowSoftmaxBwd) {
        using R = std::integral_constant<int, mg::kRowSoftmaxBwd>;
        return pair ? by_width(T{}, R{}) : by_width(F{}, R{});
    }
    using R0 = std::integral_constant<int, mg::kRowNone>;
    if (pair && bn == 224) return go(std::integral_constant<int, 224>{}, T{}, R0{});
    return pair ? by_width(T{}, R0{}) : by_width(F{}, R0{});
}

mg_status mg_gemm(const mg_gemm_desc* d, float* C, const float* A, const float* B, const float* bias,
                  void* stream)
{
    NvtxRange nvtx_range("mg_gemm");
    return gemm_impl(d, C, A, B, bias, stream, nullptr, 0);
}

// Shared by mg_matmul / mg_matmul_bias / mg_matmul_softmax: turns the
// reference's rank-equalised contiguous shapes into a descriptor. Mirrors the
// shape checks of Functional::matmul (tensor_ops.cpp:4559-4572, 4807-4818).
// With `reduce`, out_shape may be 1 on a leading dim where the product is
// not: that dim becomes a reduction dim (C batch stride 0), i.e. out receives
// the product summed over it -- what `out += product` does in the reference
// when out broadcasts to the product (tensor_ops.cpp:3393-3446).
static mg_status seam_desc(mg_gemm_desc* d, const int32_t* out_shape, const int32_t* A_shape,
                           const int32_t* B_shape, const int32_t* bias_shape, int32_t rank,
                           int32_t trans_a, int32_t trans_b, bool reduce = false)
{
    if (!out_shape || !A_shape || !B_shape) return fail(MG_ERR_INVALID, "shape pointer is NULL");
    if (rank < 2) return fail(MG_ERR_INVALID, "rank %d < 2: shapes must be rank-equalised to >= 2", rank);
    if (rank - 2 > MG_MAX_BATCH_DIMS)
        return fail(MG_ERR_UNSUPPORTED, "rank %d has more than %d leading dims", rank, MG_MAX_BATCH_DIMS);
    for (int i = 0; i < rank; ++i)
        if (out_shape[i] < 0 || A_shape[i] < 0 || B_shape[i] < 0 || (bias_shape && bias_shape[i] < 0))
            return fail(MG_ERR_INVALID, "negative dimension at %d", i);
    const int32_t M = trans_a ? A_shape[rank - 1] : A_shape[rank - 2];
    const int32_t K = trans_a ? A_shape[rank - 2] : A_shape[rank - 1];
    const int32_t Kb = trans_b ? B_shape[rank - 1] : B_shape[rank - 2];
    const int32_t N = trans_b ? B_shape[rank - 2] : B_shape[rank - 1];
    if (K != Kb) return fail(MG_ERR_INVALID, "incompatible inner dimensions %d and %d", K, Kb);
    if (out_shape[rank - 2] != M || out_shape[rank - 1] != N)
        return fail(MG_ERR_INVALID, "out shape [.., %d, %d] does not match [.., %d, %d]",
                    out_shape[rank - 2], out_shape[rank - 1], M, N);
    mg_gemm_desc_init(d, M, N, K, trans_a, trans_b);
    d->batch_rank = rank - 2;
    // contiguous element strides of each stored tensor; size-1 dims broadcast
    int64_t sa = (int64_t)A_shape[rank - 2] * A_shape[rank - 1];
    int64_t sb = (int64_t)B_shape[rank - 2] * B_shape[rank - 1];
    int64_t sc = (int64_t)M * N;
    int64_t sbias = bias_shape ? (int64_t)bias_shape[rank - 2] * bias_shape[rank - 1] : 0;
    for (int i = rank - 3; i >= 0; --i) {
        const int j = i;
        if (!(A_shape[i] == B_shape[i] || A_shape[i] == 1 || B_shape[i] == 1))
            return fail(MG_ERR_INVALID, "leading dim %d not broadcastable (%d vs %d)", i, A_shape[i], B_shape[i]);
        const int32_t o = std::max(A_shape[i], B_shape[i]);
        if (out_shape[i] != o && !(reduce && out_shape[i] == 1))
            return fail(MG_ERR_INVALID, "out leading dim %d is %d, expected %d%s", i, out_shape[i], o,
                        reduce ? " or 1" : "");
        d->batch[j] = o;
        d->a_batch_stride[j] = A_shape[i] == 1 ? 0 : sa;
        d->b_batch_stride[j] = B_shape[i] == 1 ? 0 : sb;
        d->c_batch_stride[j] = out_shape[i] == 1 ? 0 : sc;
        sa *= A_shape[i];
        sb *= B_shape[i];
        sc *= out_shape[i];
        if (bias_shape) {
            if (!(bias_shape[i] == o || bias_shape[i] == 1))
                return fail(MG_ERR_INVALID, "bias dim %d is %d, not %d or 1", i, bias_shape[i], o);
            d->bias_batch_stride[j] = bias_shape[i] == 1 ? 0 : sbias;
            sbias *= bias_shape[i];
        }
    }
    if (bias_shape) {
        if (!(bias_shape[rank - 2] == M || bias_shape[rank - 2] == 1) ||
            !(bias_shape[rank - 1] == N || bias_shape[rank - 1] == 1))
            return fail(MG_ERR_INVALID, "bias [.., %d, %d] does not broadcast to [.., %d, %d]",
                        bias_shape[rank - 2], bias_shape[rank - 1], M, N);
        d->bias_rs = bias_shape[rank - 2] == 1 ? 0 : bias_shape[rank - 1];
        d->bias_cs = bias_shape[rank - 1] == 1 ? 0 : 1;
    }
    return MG_OK;
}

mg_status mg_matmul(float* out, const float* A, const float* B, const int32_t* out_shape,
                    const int32_t* A_shape, const int32_t* B_shape, int32_t rank, int32_t trans_a,
                    int32_t trans_b, void* stream)
{
    NvtxRange nvtx_range("mg_matmul");
    g_last_error.clear();
    mg_gemm_desc d;
    mg_status s = seam_desc(&d, out_shape, A_shape, B_shape, nullptr, rank, trans_a, trans_b);
    if (s != MG_OK) return s;
    return mg_gemm(&d, out, A, B, nullptr, stream);
}

mg_status mg_matmul_bias(float* out, const float* A, const float* B, const float* bias,
                         const int32_t* out_shape, const int32_t* A_shape, const int32_t* B_shape,
                         const int32_t* bias_shape, int32_t rank, int32_t trans_a, int32_t trans_b,
                         void* stream)
{
    NvtxRange nvtx_range("mg_matmul_bias");
    g_last_error.clear();
    if (!bias_shape) return fail(MG_ERR_INVALID, "bias_shape is NULL");
    mg_gemm_desc d;
    mg_status s = seam_desc(&d, out_shape, A_shape, B_shape, bias_shape, rank, trans_a, trans_b);
    if (s != MG_OK) return s;
    d.epilogue = MG_EPI_BIAS;
    return mg_gemm(&d, out, A, B, bias, stream);
}

mg_status mg_matmul_accumulate(float* out, const float* A, const float* B, const int32_t* out_shape,
                               const int32_t* A_shape, const int32_t* B_shape, int32_t rank, int32_t trans_a,
                               int32_t trans_b, float beta, void* stream)
{
    NvtxRange nvtx_range("mg_matmul_accumulate");
    g_last_error.clear();
    if (beta != 0.f && beta != 1.f) return fail(MG_ERR_INVALID, "beta must be 0 or 1 (got %g)", (double)beta);
    mg_gemm_desc d;
    mg_status s = seam_desc(&d, out_shape, A_shape, B_shape, nullptr, rank, trans_a, trans_b, true);
    if (s != MG_OK) return s;
    d.beta = beta;
    return mg_gemm(&d, out, A, B, nullptr, stream);
}

mg_status mg_sum_into(float* dst, const float* src, const int32_t* dst_shape, const int32_t* src_shape,
                      int32_t rank, float beta, void* stream)
{
    NvtxRange nvtx_range("mg_sum_into");
    g_last_error.clear();
    if (!dst_shape || !src_shape) return fail(MG_ERR_INVALID, "shape pointer is NULL");
    if (rank < 1 || rank > MG_MAX_BATCH_DIMS + 2)
        return fail(MG_ERR_INVALID, "rank %d outside [1, %d]", rank, MG_MAX_BATCH_DIMS + 2);
    if (beta != 0.f && beta != 1.f) return fail(MG_ERR_INVALID, "beta must be 0 or 1 (got %g)", (double)beta);
    int64_t P = 1, R = 1, total = 1;
    for (int i = 0; i < rank; ++i) {
        if (dst_shape[i] < 0 || src_shape[i] < 0) return fail(MG_ERR_INVALID, "negative dimension at %d", i);
        if (dst_shape[i] != src_shape[i] && dst_shape[i] != 1)
            return fail(MG_ERR_INVALID, "dst dim %d is %d: it must be src's (%d) or 1", i, dst_shape[i],
                        src_shape[i]);
        P *= dst_shape[i];
        total *= src_shape[i];
    }
    if (P == 0) return MG_OK;
    if (!dst) return fail(MG_ERR_INVALID, "dst is NULL");
    if (total > 0 && !src) return fail(MG_ERR_INVALID, "src is NULL");
    R = total / P;
    SumParams sp;
    std::memset(&sp, 0, sizeof(sp));
    // canonical dims of src (contiguous row-major): drop size-1 dims, merge
    // neighbours of the same kind (kept: dst has the dim; reduced: dst has 1)
    int kind[MG_MAX_BATCH_DIMS + 2];
    int64_t size[MG_MAX_BATCH_DIMS + 2], stride[MG_MAX_BATCH_DIMS + 2];
    int n = 0;
    int64_t st = 1;
    for (int i = rank - 1; i >= 0; --i) {
        const int64_t sz = src_shape[i];
        if (sz != 1) {
            const int k = dst_shape[i] == 1 ? 1 : 0;
            if (n > 0 && kind[n - 1] == k && stride[n - 1] * size[n - 1] == st) {
                size[n - 1] *= sz;
            } else {
                kind[n] = k;
                size[n] = sz;
                stride[n] = st;
                ++n;
            }
        }
        st *= sz;
    }
    // outer first
    for (int i = n - 1; i >= 0; --i) {
        if (kind[i]) {
            sp.rsize[sp.nr] = size[i];
            sp.rstride[sp.nr++] = stride[i];
        } else {
            sp.ksize[sp.nk] = size[i];
            sp.kstride[sp.nk++] = stride[i];
        }
    }
    sp.src = src;
    sp.dst = dst;
    sp.P = P;
    sp.R = R;
    sp.beta = beta;
    // [R][P]: one reduced dim outside one kept dim (or either alone)
    sp.rows = (sp.nr <= 1 && sp.nk <= 1 && (n < 2 || kind[n - 1] == 1)) ? 1 : 0;
    sp.vec = sp.rows && P % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0 &&
             (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
    DeviceState* dev = nullptr;
    mg_status s = device_state(&dev);
    if (s != MG_OK) return s;
    cudaStream_t cs = (cudaStream_t)stream;
    constexpr int kThreadsPerBlock = 256;
    const int64_t lanes = sp.vec ? P / 4 : P;
    const int64_t bx = (lanes + kThreadsPerBlock - 1) / kThreadsPerBlock;
    if (bx >= (1ll << 31)) return fail(MG_ERR_UNSUPPORTED, "too many outputs (%lld)", (long long)P);
    // enough blocks to keep every SM reading (4 per SM), each split >= 16 reduced rows
    int64_t splits = std::max<int64_t>(1, (4ll * dev->sm_count + bx - 1) / bx);
    splits = std::min<int64_t>(splits, std::max<int64_t>(1, R / 16));
    splits = std::min<int64_t>(splits, 65535);
    sp.rchunk = (R + splits - 1) / std::max<int64_t>(1, splits);
    sp.splits = (int)(sp.rchunk > 0 ? (R + sp.rchunk - 1) / sp.rchunk : 1);
    if (sp.splits < 1) sp.splits = 1;
    Workspace ws;
    ws.stream = stream;
    ws.pool = dev->pool;
    if (sp.splits > 1) {
        sp.part = static_cast<float*>(ws.get((size_t)sp.splits * (size_t)P * sizeof(float)));
        if (!sp.part) return fail(MG_ERR_ALLOC, "workspace allocation of %lld bytes failed",
                                  (long long)sp.splits * P * 4);
    }
    sum_into_kernel<<<dim3((unsigned)bx, (unsigned)sp.splits), kThreadsPerBlock, 0, cs>>>(sp);
    MG_CUDA_TRY(cudaGetLastError());
    g_launches++;
    if (sp.splits > 1) {
        sum_parts_kernel<<<(unsigned)((P + kThreadsPerBlock - 1) / kThreadsPerBlock), kThreadsPerBlock, 0, cs>>>(
            sp.part, dst, P, sp.splits, beta);
        MG_CUDA_TRY(cudaGetLastError());
        g_launches++;
    }
    return MG_OK;
}

mg_status mg_matmul_softmax(float* out, const float* A, const float* B, const float* bias,
                            const int32_t* out_shape, const int32_t* A_shape, const int32_t* B_shape,
                            const int32_t* bias_shape, int32_t rank, int32_t trans_a, int32_t trans_b,
                            float alpha, int32_t causal, void* stream)
{
    NvtxRange nvtx_range("mg_matmul_softmax");
    g_last_error.clear();
    mg_gemm_desc d;
    mg_status s = seam_desc(&d, out_shape, A_shape, B_shape, bias ? bias_shape : nullptr, rank,
                            trans_a, trans_b);
    if (s != MG_OK) return s;
    if (bias && !bias_shape) return fail(MG_ERR_INVALID, "bias_shape is NULL");
    d.alpha = alpha;
    d.epilogue = MG_EPI_SOFTMAX | (bias ? MG_EPI_BIAS : 0) | (causal ? MG_EPI_CAUSAL : 0);
    return mg_gemm(&d, out, A, B, bias, stream);
}

mg_status mg_matmul_softmax_backward(float* dS, const float* A, const float* B, const float* P,
                                     const int32_t* out_shape, const int32_t* A_shape, const int32_t* B_shape,
                                     int32_t rank, int32_t trans_a, int32_t trans_b, float alpha, void* stream)
{
    NvtxRange nvtx_range("mg_matmul_softmax_backward");
    g_last_error.clear();
    if (!P) return fail(MG_ERR_INVALID, "P is NULL");
    mg_gemm_desc d;
    mg_status s = seam_desc(&d, out_shape, A_shape, B_shape, nullptr, rank, trans_a, trans_b);
    if (s != MG_OK) return s;
    d.alpha = alpha;
    d.epilogue = mg::kEpiSoftmaxBwd;
    return gemm_impl(&d, dS, A, B, nullptr, stream, nullptr, 0, nullptr, P);
}

// mg_matmul without any allocation: its scratch (the padded copy of an
// operand whose rows break TMA's 16-byte rule, then the K-split partial slots
// and counters) comes from g_noalloc_scratch; a re-layout that does not fit is
// refused, split slots that do not fit leave the launch unsplit, and the lo
// planes of MG_GEMM_PRESPLIT are never made. The array's device address is
// looked up on this entry point's first call on each device
// (cudaGetSymbolAddress, with that device current) and cached; that first
// call should therefore come before any stream capture.
mg_status mg_matmul_noalloc(float* out, const float* A, const float* B, const int32_t* out_shape,
                            const int32_t* A_shape, const int32_t* B_shape, int32_t rank,
                            int32_t trans_a, int32_t trans_b, void* stream)
{
    NvtxRange nvtx_range("mg_matmul_noalloc");
    g_last_error.clear();
    mg_gemm_desc d;
    mg_status s = seam_desc(&d, out_shape, A_shape, B_shape, nullptr, rank, trans_a, trans_b);
    if (s != MG_OK) return s;
    int dev = 0;
    MG_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(MG_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    uint8_t* scratch = g_noalloc_ptr[dev].load(std::memory_order_acquire);
    if (scratch == nullptr) {
        std::lock_guard<std::mutex> lk(g_mu);
        scratch = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
        if (scratch == nullptr) {
            void* p = nullptr;
            MG_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
            scratch = static_cast<uint8_t*>(p);
            g_noalloc_ptr[dev].store(scratch, std::memory_order_release);
        }
    }
    return gemm_impl(&d, out, A, B, nullptr, stream, scratch, MG_NOALLOC_SCRATCH_BYTES);
}

// Copy-engine form of the row-sharded GEMM (MG_GEMM_EXPORT=2). The rank's
// rows are computed band by band (mg::plan_bands: whole 256-wide tile
// columns, one launch each) into this GPU's own full C; when a band is done,
// every other rank's C receives it by cudaMemcpy2DAsync on a stream per
// destination, so the copies run on the copy engines beside the next band's
// GEMM and no SM issues a remote store. The caller's stream waits for the
// copies before this returns, as it waits for the fused forms' kernel.
static mg_status scatter_by_bands(const mg_gemm_desc* d, const float* A, const float* B, const float* bias,
                                  const ScatterSpec& sc, int local, cudaStream_t st)
{
    DeviceState* dev = nullptr;
    mg_status s = device_state(&dev);
    if (s != MG_OK) return s;
    s = copy_engine_state(dev);
    if (s != MG_OK) return s;
    // the same choice gemm_impl makes for each band (one matrix, the rank's rows)
    const int32_t mode = d->mode == MG_MODE_DEFAULT ? resolve_default_mode() : d->mode;
    const bool pair = use_pair(d, 1, dev->sm_count, mode);
    const int tile_rows = pair ? 2 * mg::kBM : mg::kBM;
    const int m_tiles = (int)((d->M + tile_rows - 1) / tile_rows);
    const int n_tiles = (int)((d->N + 255) / 256);
    mg::BandPlan bp;
    // the deepest K split a band's launch can make (as plan_split allows it)
    const int num_kb = (int)((d->K + mg::kBK - 1) / mg::kBK);
    const int min_kb = tuning_int("MG_GEMM_SPLIT", 1, 0, 1) ? tuning_int("MG_GEMM_SPLIT_MIN_KB", 16, 1, 1 << 20) : 0;
    const int max_split = min_kb > 0 ? std::max(1, num_kb / min_kb) : 1;
    mg::plan_bands(bp, m_tiles, n_tiles, pair ? dev->sm_count / 2 : dev->sm_count, max_split,
                   tuning_int("MG_GEMM_BAND_COLS", 0, 1, 1 << 20));
    const int64_t ld = d->ldc;
    const size_t pitch = (size_t)ld * sizeof(float);
    float* own = sc.peers[local] + sc.row0 * ld;
    mg_status result = MG_OK;
    for (int b = 0; b < bp.nbands; ++b) {
        const int64_t c0 = (int64_t)bp.col0[b] * 256;
        const int64_t c1 = std::min<int64_t>(d->N, (int64_t)bp.col0[b + 1] * 256);
        mg_gemm_desc db = *d;
        db.N = (int32_t)(c1 - c0);
        const float* Bb = B + (d->trans_b ? c0 * d->ldb : c0);
        const float* biasb = (d->epilogue & MG_EPI_BIAS) ? bias + c0 * d->bias_cs : bias;
        result = gemm_impl(&db, own + c0, A, Bb, biasb, st, nullptr, 0);
        if (result != MG_OK) break;
        cudaError_t e = cudaEventRecord(dev->band_done[b], st);
        for (int q = 0; q < sc.npeers && e == cudaSuccess; ++q) {
            if (q == local) continue;
            e = cudaStreamWaitEvent(dev->copy_stream[q], dev->band_done[b], 0);
            if (e == cudaSuccess)
                e = cudaMemcpy2DAsync(sc.peers[q] + sc.row0 * ld + c0, pitch, own + c0, pitch,
                                      (size_t)(c1 - c0) * sizeof(float), (size_t)d->M, cudaMemcpyDeviceToDevice,
                                      dev->copy_stream[q]);
        }
        if (e != cudaSuccess) {
            result = fail(MG_ERR_CUDA, "copy of band %d to the other ranks failed: %s", b, cudaGetErrorString(e));
            break;
        }
    }
    // the caller's stream continues once every copy enqueued above has landed
    // (also after a failure, so that nothing is left in flight behind it)
    for (int q = 0; q < sc.npeers; ++q) {
        if (q == local) continue;
        cudaError_t e = cudaEventRecord(dev->copies_done[q], dev->copy_stream[q]);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(st, dev->copies_done[q], 0);
        if (e != cudaSuccess && result == MG_OK)
            result = fail(MG_ERR_CUDA, "joining the copy streams failed: %s", cudaGetErrorString(e));
    }
    return result;
}

mg_status mg_gemm_scatter_rows(const mg_gemm_desc* d, const float* A, const float* B, const float* bias,
                               float* const* peer_C, int32_t npeers, int64_t row0, int64_t rows_full,
                               void* stream)
{
    NvtxRange nvtx_range("mg_gemm_scatter_rows");
    g_last_error.clear();
    if (!d) return fail(MG_ERR_INVALID, "descriptor is NULL");
    if (npeers < 1 || npeers > mg::kMaxPeers)
        return fail(MG_ERR_INVALID, "npeers %d outside [1, %d]", npeers, mg::kMaxPeers);
    if (!peer_C) return fail(MG_ERR_INVALID, "peer_C is NULL");
    if (row0 < 0 || row0 + d->M > rows_full)
        return fail(MG_ERR_INVALID, "rows [%lld, %lld) are not inside the %lld rows of the full C",
                    (long long)row0, (long long)(row0 + d->M), (long long)rows_full);
    if (d->beta != 0.f) return fail(MG_ERR_INVALID, "the scattering GEMM does not accumulate (beta must be 0)");
    ScatterSpec sc;
    sc.npeers = npeers;
    sc.row0 = row0;
    sc.rows_full = rows_full;
    for (int q = 0; q < npeers; ++q) {
        if (!peer_C[q]) return fail(MG_ERR_INVALID, "peer_C[%d] is NULL", q);
        sc.peers[q] = peer_C[q];
    }
    if (d->K == 0) return fail(MG_ERR_UNSUPPORTED, "K = 0 is not supported by the scattering GEMM");
    // copy engines instead of the kernel's export warps: a 2-D C without a
    // row epilogue (bands cut the rows), one destination in this process. By
    // default for jobs of 4 ranks, where it measured fastest (8192^3 over 4
    // B200s: 772 TFLOP/s against 730 for the export warps and 663 for NCCL;
    // with 2 and 8 ranks the export warps led: 427 / 1134 against 411 / 979)
    const int export_dflt = npeers == 4 ? 2 : 1;
    if (tuning_int("MG_GEMM_EXPORT", export_dflt, 0, 2) == 2 && d->batch_rank == 0 &&
        (d->epilogue & (MG_EPI_SOFTMAX | mg::kEpiSoftmaxBwd)) == 0) {
        int local = -1;
        for (int q = 0; q < npeers && local < 0; ++q)
            if (!ipc_imported(peer_C[q])) local = q;
        if (local >= 0) {
            mg_status s = validate(d, peer_C[local] + row0 * d->ldc, A, B, bias);
            if (s != MG_OK) return s;
            if (d->M == 0 || d->N == 0) return MG_OK;
            return scatter_by_bands(d, A, B, bias, sc, local, (cudaStream_t)stream);
        }
    }
    return gemm_impl(d, peer_C[0], A, B, bias, stream, nullptr, 0, &sc);
}

static_assert(sizeof(cudaIpcMemHandle_t) <= sizeof(mg_ipc_handle), "IPC handle does not fit");

// The allocation containing a device pointer (driver cuMemGetAddressRange).
static mg_status address_range(const void* p, CUdeviceptr* base, size_t* size)
{
    // looked up once (thread-safe static initialisation); null if unavailable
    static const PFN_cuMemGetAddressRange_v3020 get_range = []() -> PFN_cuMemGetAddressRange_v3020 {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
    }();
    if (!get_range) return fail(MG_ERR_CUDA, "cuMemGetAddressRange unavailable");
    if (get_range(base, size, (CUdeviceptr)p) != CUDA_SUCCESS)
        return fail(MG_ERR_INVALID, "pointer is not device memory");
    return MG_OK;
}

mg_status mg_ipc_export(const void* dev_ptr, mg_ipc_handle* handle, uint64_t* offset)
{
    g_last_error.clear();
    if (!dev_ptr || !handle || !offset) return fail(MG_ERR_INVALID, "NULL argument");
    CUdeviceptr base = 0;
    size_t size = 0;
    mg_status s = address_range(dev_ptr, &base, &size);
    if (s != MG_OK) return s;
    cudaIpcMemHandle_t h;
    MG_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    std::memset(handle, 0, sizeof(*handle));
    std::memcpy(handle->bytes, &h, sizeof(h));
    *offset = (uint64_t)((CUdeviceptr)dev_ptr - base);
    return MG_OK;
}

mg_status mg_ipc_import(const mg_ipc_handle* handle, uint64_t offset, void** dev_ptr)
{
    g_last_error.clear();
    if (!handle || !dev_ptr) return fail(MG_ERR_INVALID, "NULL argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle->bytes, sizeof(h));
    void* base = nullptr;
    MG_CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    *dev_ptr = static_cast<uint8_t*>(base) + offset;
    CUdeviceptr rb = 0;
    size_t rsize = 0;
    if (address_range(base, &rb, &rsize) != MG_OK || rb != (CUdeviceptr)base) rsize = 0;
    g_last_error.clear();
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto& m : g_ipc_maps) {
        if (!m.user) {
            m.user = *dev_ptr;
            m.base = base;
            m.size = rsize;
            return MG_OK;
        }
    }
    cudaIpcCloseMemHandle(base);
    *dev_ptr = nullptr;
    return fail(MG_ERR_UNSUPPORTED, "too many imported buffers");
}

mg_status mg_ipc_close(void* dev_ptr)
{
    g_last_error.clear();
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto& m : g_ipc_maps) {
        if (m.user == dev_ptr && dev_ptr) {
            void* base = m.base;
            m.user = m.base = nullptr;
            m.size = 0;
            MG_CUDA_TRY(cudaIpcCloseMemHandle(base));
            return MG_OK;
        }
    }
    return fail(MG_ERR_INVALID, "pointer was not returned by mg_ipc_import");
}

void mg_set_allocator(mg_alloc_fn alloc_fn, mg_free_fn free_fn, void* ctx)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (alloc_fn && free_fn) {
        g_alloc = alloc_fn;
        g_free = free_fn;
        g_alloc_ctx = ctx;
    } else {
        g_alloc = nullptr;
        g_free = nullptr;
        g_alloc_ctx = nullptr;
    }
}

mg_status mg_set_mode(int32_t mode)
{
    if (mode != MG_MODE_TF32X3 && mode != MG_MODE_TF32) return fail(MG_ERR_INVALID, "unknown mode %d", mode);
    g_mode.store(mode);
    return MG_OK;
}

int32_t mg_get_mode(void) { return resolve_default_mode(); }

const char* mg_last_error(void) { return g_last_error.c_str(); }

mg_status mg_device_status(int32_t* detail, int32_t reset)
{
    DeviceState* dev = nullptr;
    mg_status s = device_state(&dev);
    if (s != MG_OK) return s;
    MG_CUDA_TRY(cudaDeviceSynchronize());
    int h[2] = {0, 0};
    MG_CUDA_TRY(cudaMemcpyFromSymbol(h, g_device_status, sizeof(h)));
    if (detail) *detail = h[1];
    if (reset) {
        int z[2] = {0, 0};
        MG_CUDA_TRY(cudaMemcpyToSymbol(g_device_status, z, sizeof(z)));
    }
    return (mg_status)h[0];
}

uint64_t mg_launch_count(void) { return g_launches.load(); }

const char* mg_version(void) { return "mg_gemm 0.1.0 (sm_100a tcgen05 tf32 / 3xtf32)"; }

}  // extern "C"

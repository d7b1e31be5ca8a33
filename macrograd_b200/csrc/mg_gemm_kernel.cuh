// mg_gemm_kernel.cuh -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
// Computes, per output tile of 128 x BN, C = alpha * op(A) op(B) (+ bias)
// (+ beta * C) or a fused row softmax of it, on fp32 operands through the TF32
// tensor cores: one product per term (TF32 mode), or the 3xTF32 split
// hi*hi + hi*lo + lo*hi (fp32-accurate mode; hi = x with its 13 low mantissa
// bits cleared, lo = x - hi, which is exact in fp32).
//
// Roles (320 threads, one CTA per SM):
//   warps 0-3  epilogue: TMEM -> registers -> bias / scale / softmax -> HBM;
//              warp w reads TMEM lanes 32w..32w+31 = tile rows 32w..32w+31.
//   warps 4-7  split: on each landed stage, write lo tiles and clear the low
//              bits of the raw tiles in place (3xTF32 mode only).
//   warp 8     TMA producer (one lane): A and B tiles, 32 K-elements deep,
//              128-byte swizzled, into a ring of STAGES stages.
//   warp 9     TMEM allocator; one lane issues tcgen05.mma into one of two
//              TMEM accumulators (double-buffered so the epilogue of tile i
//              overlaps the main loop of tile i+1).
//
// Operand layouts in shared memory (per stage, 1024-byte aligned):
//   K-major tile (op(X) rows contiguous in K): R rows x 128 B, one TMA box
//     {32, R}; descriptor LBO 16 B, SBO 1024 B; +32 B per 8-deep K step.
//   MN-major tile (X stored with M or N contiguous, i.e. the transposed views
//     the backward pass produces): R/32 boxes {32 (MN), 32 (K)} of 4 KB at
//     4 KB spacing; descriptor LBO 4096 B (next 32 MN), SBO 1024 B (next 8 K);
//     +1024 B per 8-deep K step.
// Transposed views are therefore read in place; nothing is materialised.
//
// Every wait is bounded (global timer). On expiry the kernel records
// MG_ERR_TIMEOUT in the device status word, every role stops, in-flight TMA
// and MMA work is drained (with its own bound), TMEM is freed and the CTA exits.
#pragma once

#include <stdint.h>

#include "mg_ptx.cuh"

namespace mg {

constexpr int kBM = 128;            // tile rows (MMA M)
constexpr int kBK = 32;             // K elements per stage (128 bytes of fp32)
constexpr int kMaxStages = 8;
constexpr int kThreads = 320;
constexpr int kMaxBatchDims = 6;
constexpr uint64_t kWaitLimitNs = 4000000000ull;   // 4 s: far above any legitimate wait
constexpr uint64_t kDrainLimitNs = 200000000ull;   // 200 ms for draining after an abort

enum : int { kEpiBias = 1, kEpiCausal = 2, kEpiSoftmax = 4 };

// Wait sites, reported in the status detail word when a wait gives up.
enum : int {
    kWaitProducerEmpty = 1,
    kWaitSplitFull = 2,
    kWaitMmaAccEmpty = 3,
    kWaitMmaStage = 4,
    kWaitEpilogueFull = 5,
    kWaitDrain = 6
};

struct GemmParams {
    int M, N, K;
    int num_kb;                 // ceil(K / 32)
    int m_tiles, n_tiles;
    int tiles_per_batch;
    int total_tiles;
    int group_m;                // tile raster: group_m m-tiles sweep all n-tiles
    int stages;
    int split;                  // 1 = 3xTF32
    int a_mn, b_mn;             // 1 = operand tile is MN-major (transposed view)
    int a_rank, b_rank;         // tensor-map ranks (2 + mapped batch dims)
    uint32_t idesc;
    int nbd;                    // output batch dims
    int bsize[kMaxBatchDims];
    int8_t a_map[kMaxBatchDims], b_map[kMaxBatchDims];   // batch dim -> map dim (-1: broadcast)
    int32_t a_mult[kMaxBatchDims], b_mult[kMaxBatchDims];
    float* C;
    int64_t ldc;
    int64_t c_bs[kMaxBatchDims];
    const float* bias;
    int64_t bias_rs, bias_cs;
    int64_t bias_bs[kMaxBatchDims];
    float alpha, beta;
    int epi;
    int* status;                // device status word pair {code, detail}
};

struct TileCoord {
    int batch, mt, nt;
};

__device__ __forceinline__ TileCoord decode_tile(int t, const GemmParams& p)
{
    TileCoord tc;
    tc.batch = t / p.tiles_per_batch;
    const int r = t - tc.batch * p.tiles_per_batch;
    const int span = p.group_m * p.n_tiles;
    const int g = r / span;
    const int first_m = g * p.group_m;
    const int gm = min(p.group_m, p.m_tiles - first_m);
    const int rr = r - g * span;
    tc.mt = first_m + rr % gm;
    tc.nt = rr / gm;
    return tc;
}

// Output batch multi-index of a flat batch number (row-major over bsize).
__device__ __forceinline__ void batch_index(int b, const GemmParams& p, int* idx)
{
#pragma unroll
    for (int d = kMaxBatchDims - 1; d >= 0; --d) {
        if (d < p.nbd) {
            idx[d] = b % p.bsize[d];
            b /= p.bsize[d];
        } else {
            idx[d] = 0;
        }
    }
}

struct SharedState {
    uint64_t full[kMaxStages];
    uint64_t split_done[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    volatile int abort_flag;
};

__device__ __forceinline__ void record_failure(const GemmParams& p, SharedState* ss, int where)
{
    ss->abort_flag = 1;
    if (p.status != nullptr) {
        if (atomicCAS(p.status, 0, 5 /* MG_ERR_TIMEOUT */) == 0) atomicExch(p.status + 1, where);
    }
}

// Bounded wait for the phase of parity `parity` of `bar`. Returns false when
// the CTA is aborting (another role gave up) or this wait itself ran out.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, SharedState* ss,
                                           const GemmParams& p, int where)
{
    if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_test(bar, parity)) return true;
        if (ss->abort_flag) return false;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            record_failure(p, ss, where);
            return false;
        }
    }
}

// Wait used only while draining after an abort: ignores the abort flag.
__device__ __forceinline__ void drain_phase(uint32_t bar, uint32_t parity)
{
    const uint64_t t0 = global_timer_ns();
    while (!mbar_test(bar, parity)) {
        if (global_timer_ns() - t0 > kDrainLimitNs) return;
    }
}

template <int BN>
struct Layout {
    static constexpr uint32_t kABytes = kBM * 128;          // 16 KB
    static constexpr uint32_t kBBytes = BN * 128;
    static constexpr uint32_t kStageBytes = kABytes + kBBytes;
    static constexpr uint32_t kTmemCols = 2 * BN;           // double-buffered accumulator
};

template <int BN>
__device__ __forceinline__ void store_row_chunk(float* crow, int gn0, int nvalid, const float* v)
{
    if (nvalid == 32 && ((reinterpret_cast<uintptr_t>(crow + gn0) & 15u) == 0)) {
        float4* dst = reinterpret_cast<float4*>(crow + gn0);
#pragma unroll
        for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < nvalid) crow[gn0 + j] = v[j];
    }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    mg_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ GemmParams p)
{
    using L = Layout<BN>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the 128-byte swizzle atoms.
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const uint32_t smem_base = smem_u32(smem);
    const int stages = p.stages;
    const uint32_t raw_region = (uint32_t)stages * L::kStageBytes;
    SharedState* ss = reinterpret_cast<SharedState*>(smem + raw_region * (p.split ? 2u : 1u));

    auto a_raw = [&](int s) { return smem_base + (uint32_t)s * L::kStageBytes; };
    auto b_raw = [&](int s) { return smem_base + (uint32_t)s * L::kStageBytes + L::kABytes; };
    auto a_lo = [&](int s) { return a_raw(s) + raw_region; };
    auto b_lo = [&](int s) { return b_raw(s) + raw_region; };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(&ss->full[s]), 1);
            mbar_init(smem_u32(&ss->split_done[s]), 128);
            mbar_init(smem_u32(&ss->empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&ss->acc_full[a]), 1);
            mbar_init(smem_u32(&ss->acc_empty[a]), 128);
        }
        mbar_init(smem_u32(&ss->drain), 1);
        ss->abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 8 && lane == 0) {
        tma_prefetch_map(&tmA);
        tma_prefetch_map(&tmB);
    }
    if (warp == 9) {
        tmem_alloc(smem_u32(&ss->tmem_base), L::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = ss->tmem_base;

    if (warp == 8) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0, issued_par = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x) {
                const TileCoord tc = decode_tile(t, p);
                int idx[kMaxBatchDims];
                batch_index(tc.batch, p, idx);
                int32_t ca[5] = {0, 0, 0, 0, 0}, cb[5] = {0, 0, 0, 0, 0};
#pragma unroll
                for (int d = 0; d < kMaxBatchDims; ++d) {
                    if (d < p.nbd && p.a_map[d] >= 0) ca[2 + p.a_map[d]] += idx[d] * p.a_mult[d];
                    if (d < p.nbd && p.b_map[d] >= 0) cb[2 + p.b_map[d]] += idx[d] * p.b_mult[d];
                }
                const int m0 = tc.mt * kBM;
                const int n0 = tc.nt * BN;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!wait_phase(smem_u32(&ss->empty[stage]), phase ^ 1u, ss, p, kWaitProducerEmpty)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = smem_u32(&ss->full[stage]);
                    mbar_arrive_expect_tx(fb, L::kStageBytes);
                    const int k0 = kb * kBK;
                    if (!p.a_mn) {
                        ca[0] = k0; ca[1] = m0;
                        tma_load(&tmA, fb, a_raw(stage), p.a_rank, ca);
                    } else {
                        ca[1] = k0;
#pragma unroll
                        for (int j = 0; j < kBM / 32; ++j) {
                            ca[0] = m0 + 32 * j;
                            tma_load(&tmA, fb, a_raw(stage) + 4096u * j, p.a_rank, ca);
                        }
                    }
                    if (!p.b_mn) {
                        cb[0] = k0; cb[1] = n0;
                        tma_load(&tmB, fb, b_raw(stage), p.b_rank, cb);
                    } else {
                        cb[1] = k0;
#pragma unroll
                        for (int j = 0; j < BN / 32; ++j) {
                            cb[0] = n0 + 32 * j;
                            tma_load(&tmB, fb, b_raw(stage) + 4096u * j, p.b_rank, cb);
                        }
                    }
                    issued |= 1u << stage;
                    issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == stages) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {
                // let every issued copy land before the CTA's shared memory goes away
                for (int s = 0; s < stages; ++s)
                    if (issued & (1u << s)) drain_phase(smem_u32(&ss->full[s]), (issued_par >> s) & 1u);
            }
        }
        __syncwarp();
    } else if (warp == 9) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            const bool split = p.split != 0;
            const uint32_t a_lbo = p.a_mn ? 4096u : 16u;
            const uint32_t b_lbo = p.b_mn ? 4096u : 16u;
            const uint32_t a_kstep = p.a_mn ? 1024u : 32u;
            const uint32_t b_kstep = p.b_mn ? 1024u : 32u;
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x) {
                if (!wait_phase(smem_u32(&ss->acc_empty[acc]), acc_phase ^ 1u, ss, p, kWaitMmaAccEmpty)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    const uint32_t ready = split ? smem_u32(&ss->split_done[stage]) : smem_u32(&ss->full[stage]);
                    if (!wait_phase(ready, phase, ss, p, kWaitMmaStage)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < kBK / 8; ++ks) {
                        const uint32_t accum = (kb > 0 || ks > 0) ? 1u : 0u;
                        const uint64_t da = smem_desc_sw128(a_raw(stage) + ks * a_kstep, a_lbo, 1024u);
                        const uint64_t db = smem_desc_sw128(b_raw(stage) + ks * b_kstep, b_lbo, 1024u);
                        if (split) {
                            const uint64_t dal = smem_desc_sw128(a_lo(stage) + ks * a_kstep, a_lbo, 1024u);
                            const uint64_t dbl = smem_desc_sw128(b_lo(stage) + ks * b_kstep, b_lbo, 1024u);
                            tc_mma_tf32(d_tmem, dal, db, p.idesc, accum);   // lo * hi
                            tc_mma_tf32(d_tmem, da, dbl, p.idesc, 1u);      // hi * lo
                            tc_mma_tf32(d_tmem, da, db, p.idesc, 1u);       // hi * hi
                        } else {
                            tc_mma_tf32(d_tmem, da, db, p.idesc, accum);
                        }
                    }
                    tc_commit(smem_u32(&ss->empty[stage]));   // frees the stage when these MMAs finish
                    if (++stage == stages) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                tc_commit(smem_u32(&ss->acc_full[acc]));      // accumulator ready for the epilogue
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
            // every MMA this thread issued has finished before TMEM is freed
            tc_commit(smem_u32(&ss->drain));
            drain_phase(smem_u32(&ss->drain), 0);
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ------------------------------------------------ 3xTF32 split
        if (p.split) {
            const int tid = threadIdx.x - 128;
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x) {
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!wait_phase(smem_u32(&ss->full[stage]), phase, ss, p, kWaitSplitFull)) {
                        ok = false;
                        break;
                    }
                    // A and B raw tiles are contiguous in the stage; their lo
                    // tiles sit at the same offsets one raw region higher.
                    uint4* raw = reinterpret_cast<uint4*>(smem + (size_t)stage * L::kStageBytes);
                    uint4* lo = reinterpret_cast<uint4*>(smem + (size_t)stage * L::kStageBytes + raw_region);
                    constexpr int n4 = (int)(L::kStageBytes / 16);
#pragma unroll 4
                    for (int i = tid; i < n4; i += 128) {
                        const uint4 x = raw[i];
                        uint4 h, l;
                        h.x = x.x & 0xFFFFE000u; h.y = x.y & 0xFFFFE000u;
                        h.z = x.z & 0xFFFFE000u; h.w = x.w & 0xFFFFE000u;
                        // lo = x - hi exactly; 0 for +-inf / nan so they pass through hi alone
                        const float fx = __uint_as_float(x.x), fy = __uint_as_float(x.y);
                        const float fz = __uint_as_float(x.z), fw = __uint_as_float(x.w);
                        l.x = __float_as_uint(isfinite(fx) ? fx - __uint_as_float(h.x) : 0.f);
                        l.y = __float_as_uint(isfinite(fy) ? fy - __uint_as_float(h.y) : 0.f);
                        l.z = __float_as_uint(isfinite(fz) ? fz - __uint_as_float(h.z) : 0.f);
                        l.w = __float_as_uint(isfinite(fw) ? fw - __uint_as_float(h.w) : 0.f);
                        raw[i] = h;
                        lo[i] = l;
                    }
                    fence_proxy_async_smem();
                    mbar_arrive(smem_u32(&ss->split_done[stage]));
                    if (++stage == stages) { stage = 0; phase ^= 1u; }
                }
            }
        }
    } else {
        // ------------------------------------------------ epilogue (warps 0-3)
        const int row = warp * 32 + lane;
        int acc = 0;
        uint32_t acc_phase = 0;
        const bool has_bias = (p.epi & kEpiBias) != 0;
        for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
            const TileCoord tc = decode_tile(t, p);
            int idx[kMaxBatchDims];
            batch_index(tc.batch, p, idx);
            int64_t coff = 0, boff = 0;
#pragma unroll
            for (int d = 0; d < kMaxBatchDims; ++d) {
                if (d < p.nbd) {
                    coff += (int64_t)idx[d] * p.c_bs[d];
                    boff += (int64_t)idx[d] * p.bias_bs[d];
                }
            }
            const int m0 = tc.mt * kBM;
            const int n0 = tc.nt * BN;
            const int gm = m0 + row;
            const bool rok = gm < p.M;
            float* crow = p.C + coff + (int64_t)(rok ? gm : 0) * p.ldc;
            const float* brow = has_bias ? p.bias + boff + (int64_t)(rok ? gm : 0) * p.bias_rs : nullptr;

            // every lane waits; the warp leaves together if any lane gave up, so
            // the .sync.aligned TMEM loads below always run converged
            const bool got = wait_phase(smem_u32(&ss->acc_full[acc]), acc_phase, ss, p, kWaitEpilogueFull);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)(acc * BN);

            if (p.epi & kEpiSoftmax) {
                // One thread owns one full row (N <= BN, single n-tile): the
                // row softmax needs no cross-thread reduction.
                const bool causal = (p.epi & kEpiCausal) != 0;
                float mx = -INFINITY;
                for (int c = 0; c < BN && c < p.N; c += 32) {
                    uint32_t r[32];
                    tmem_ld32(taddr + c, r);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int gn = c + j;
                        if (gn < p.N) {
                            float v = p.alpha * __uint_as_float(r[j]);
                            if (has_bias && rok) v += brow[(int64_t)gn * p.bias_cs];
                            if (causal && gn > gm) v = -INFINITY;
                            mx = fmaxf(mx, v);
                        }
                    }
                }
                float sum = 0.f;
                for (int c = 0; c < BN && c < p.N; c += 32) {
                    uint32_t r[32];
                    tmem_ld32(taddr + c, r);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int gn = c + j;
                        if (gn < p.N) {
                            float v = p.alpha * __uint_as_float(r[j]);
                            if (has_bias && rok) v += brow[(int64_t)gn * p.bias_cs];
                            if (causal && gn > gm) v = -INFINITY;
                            sum += expf(v - mx);
                        }
                    }
                }
                for (int c = 0; c < BN && c < p.N; c += 32) {
                    uint32_t r[32];
                    tmem_ld32(taddr + c, r);
                    float v[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int gn = c + j;
                        float x = p.alpha * __uint_as_float(r[j]);
                        if (gn < p.N && has_bias && rok) x += brow[(int64_t)gn * p.bias_cs];
                        if (causal && gn > gm) x = -INFINITY;
                        v[j] = expf(x - mx) / sum;
                    }
                    if (rok) store_row_chunk<BN>(crow, c, min(32, p.N - c), v);
                }
            } else {
                for (int c = 0; c < BN; c += 32) {
                    const int gn0 = n0 + c;
                    if (gn0 >= p.N) break;   // uniform across the warp
                    uint32_t r[32];
                    tmem_ld32(taddr + c, r);
                    if (rok) {
                        const int nvalid = min(32, p.N - gn0);
                        float v[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = p.alpha * __uint_as_float(r[j]);
                        if (has_bias) {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (j < nvalid) v[j] += brow[(int64_t)(gn0 + j) * p.bias_cs];
                        }
                        if (p.beta != 0.f) {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (j < nvalid) v[j] += p.beta * crow[gn0 + j];
                        }
                        store_row_chunk<BN>(crow, gn0, nvalid, v);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&ss->acc_empty[acc]));
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem_base, L::kTmemCols);
    }
}

}  // namespace mg

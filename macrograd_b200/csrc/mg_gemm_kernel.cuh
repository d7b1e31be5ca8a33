// mg_gemm_kernel.cuh -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
// Computes C = alpha * op(A) op(B) (+ bias) (+ beta * C), a fused row softmax
// of it, or the fused softmax backward P * (G - rowsum(P * G)) of it, on fp32
// operands through the TF32 tensor cores: one product per term (TF32 mode), or
// the 3xTF32 split hi*hi + hi*lo + lo*hi (fp32-accurate mode).
//
// Two variants of one template:
//   kPair = false  one CTA per SM, output tile 128 x BN, MMA M=128
//                  (tcgen05.mma.cta_group::1);
//   kPair = true   a cluster of two CTAs on two SMs shares a 256 x BN tile
//                  (tcgen05.mma.cta_group::2, M=256): each CTA loads its 128
//                  rows of A and half of the BN columns of B, holds 128 rows of
//                  D in its TMEM, and the leader CTA (rank 0) issues the MMAs.
//                  Per SM this halves the B tile in shared memory, so stages
//                  are smaller (more of them fit) and the tensor core reads
//                  less shared memory per flop.
//
// Two hardware facts shape the fp32-accurate mode (both pinned by GPU tests):
//  * a TF32 MMA reads an fp32 operand truncated to its top 19 bits, so the raw
//    tile already is `hi` and only lo = x - hi (exact in fp32) is written;
//  * the MMA's accumulate into TMEM truncates, so the error of one accumulator
//    grows with the number of MMAs added into it. The main loop therefore
//    accumulates at most kChunkKb K-blocks (256 K-elements) into a TMEM
//    *partial*, which the epilogue warps add into a TMEM *master* with fp32
//    round-to-nearest adds; the error then no longer grows with K.
//
// Roles (512 threads = 16 warps per CTA, one CTA per SM):
//   warps 0-7   epilogue: warp w owns TMEM lanes 32(w%4).. (tile rows) and the
//               column half w/4. Per chunk: master (+)= partial. Per tile:
//               alpha / bias / beta / store from the master; for the row
//               softmax (and its backward) warps w and w^4 reduce their halves
//               of each row and meet through shared memory.
//   warps 8-11  split (3xTF32): lo tile of every landed stage; in both modes
//               they report the landed stage to the MMA issuer.
//   warp 12     TMA producer (one lane), into this CTA's shared memory.
//   warp 13     TMEM allocator; one lane (of the leader CTA) issues tcgen05.mma.
//   warps 14-15 export (fused all-gather): once the epilogue has written a tile
//               into this GPU's C, copy its rows into every peer's C over
//               NVLink, so the epilogue never waits on the fabric.
// TMEM: columns [0, BN) partial, [BN, 2BN) master; when every tile is a
// single chunk (p.dbuf) the two regions are alternate accumulators instead,
// so one tile's MMAs run during the previous tile's epilogue.
//
// Work units: whole tiles, dealt round-robin; the last partial wave may be
// split over K into ranges whose fp32 partials the tile's final range adds
// (unit_at, GemmParams::nlev), the grid then launched cooperatively.
//
// Operand layouts in shared memory (per stage, 1024-byte aligned):
//   K-major tile (op(X) rows contiguous in K): R rows x 128 B, one TMA box
//     {32, R}, 128-byte swizzle of 16-byte chunks; descriptor LBO 16 B,
//     SBO 1024 B; +32 B per 8-deep K step.
//   MN-major tile (X stored with M or N contiguous, i.e. the transposed views
//     the backward pass produces): R/32 boxes {32 (MN), 32 (K)} of 4 KB at
//     4 KB spacing, 128-byte rows swizzled in 32-byte chunks; descriptor
//     LBO 4096 B (next 32 MN), SBO 512 B (next 4 K rows); +1024 B per 8-deep
//     K step.
// Transposed views are therefore read in place; nothing is materialised. All
// TMA loads are plain loads from this GPU's memory into the loading CTA's own
// shared memory (no multicast).
//
// Every wait is bounded (global timer). On expiry the kernel records
// MG_ERR_TIMEOUT in the device status word, every role stops, in-flight TMA
// and MMA work is drained (with its own bound), TMEM is freed and the CTA exits.
#pragma once

#include <stdint.h>

#include "mg_plan.h"
#include "mg_ptx.cuh"

namespace mg {

constexpr int kBM = 128;            // tile rows per CTA (MMA M per SM)
constexpr int kBK = 32;             // K elements per stage (128 bytes of fp32)
constexpr int kChunkKb = 8;         // default K-blocks accumulated in TMEM before promotion
constexpr int kMaxStages = 8;
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kSplitWarp0 = 8;
constexpr int kSplitThreads = 128;
constexpr int kProducerWarp = 12;
constexpr int kMmaWarp = 13;
constexpr int kExportWarp0 = 14;
constexpr int kExportThreads = 64;
constexpr int kThreads = 16 * 32;
constexpr int kMaxBatchDims = 6;
// Softmax backward with P loaded by TMA (GemmParams::p_tma): a ring of two
// slots in shared memory after the epilogue staging blocks, each one step of
// both column halves -- two boxes of 128 rows x 32 columns (128-byte rows,
// 128-byte swizzle: the staging blocks' layout).
constexpr int kPRingSlots = 2;
constexpr uint32_t kPBoxBytes = 128u * 128u;
constexpr uint32_t kPSlotBytes = 2u * kPBoxBytes;
constexpr int kMaxPeers = 8;
constexpr uint64_t kWaitLimitNs = 4000000000ull;   // 4 s, the default limit: far above any legitimate wait
constexpr uint64_t kDrainLimitNs = 200000000ull;   // 200 ms for draining after an abort
constexpr uint32_t kSleepHintNs = 20000u;          // try_wait suspend hint

enum : int { kEpiBias = 1, kEpiCausal = 2, kEpiSoftmax = 4, kEpiSoftmaxBwd = 8 };

// Wait sites, reported in the status detail word when a wait gives up.
enum : int {
    kWaitProducerEmpty = 1,
    kWaitSplitFull = 2,
    kWaitMmaPartialFree = 3,
    kWaitMmaStage = 4,
    kWaitEpiloguePartial = 5,
    // 6: no longer used
    kWaitEpilogueRows = 7,
    kWaitExportTile = 8,
    kWaitPartials = 9
};

struct GemmParams {
    int M, N, K;
    int num_kb;                 // ceil(K / 32)
    int m_tiles, n_tiles;       // tiles of (128 or 256 for pairs) x BN
    int tiles_per_batch;
    int total_tiles;
    int group_m;                // tile raster: group_m m-tiles sweep all n-tiles
    int stages;
    int chunk_kb;               // K-blocks per TMEM partial (promotion interval)
    int relay_spin;             // split warps poll without suspend hints
    int split;                  // 1 = 3xTF32
    int presplit;               // 3xTF32 with lo planes precomputed in HBM (tmAlo / tmBlo)
    int a_tmem;                 // 3xTF32, tiles up to 128 wide: the split warps write each stage's
                                // A hi and lo tiles into TMEM (columns a_col0 + 64 * stage) and
                                // the MMAs read A from there; shared memory serves only B
    int a_col0;                 // first TMEM column of those A tiles
    int b2;                     // with A in TMEM, width 64, plain epilogue: B's lo tile follows B's
                                // tile in the stage, and each K-step is two MMAs of width 2 BN
                                // (A hi, then A lo, times [B hi | B lo]); the accumulator is 2 BN
                                // wide and its two halves are added for the result
    uint32_t idesc2;            // instruction descriptor of those width-2 BN MMAs
    int tmem_cols;              // TMEM columns allocated (a power of two >= 32)
    int dbuf;                   // every unit is one chunk: two accumulators, no promotion
    int a_mn, b_mn;             // 1 = operand tile is MN-major (transposed view)
    int a_rank, b_rank;         // tensor-map ranks (2 + mapped batch dims)
    uint32_t idesc;
    int nbd;                    // batch dims of the product
    int bsize[kMaxBatchDims];   // their sizes over the output tiles (1 for a reduction dim)
    // Reduction dims: batch dims of the product that C does not have (stride 0
    // in C): C receives the sum over them, folded into the K loop -- K-block kb
    // is K-block kb % kb_per of reduction step kb / kb_per, whose indices run
    // row-major over rsize (1 for the other dims).
    int rsize[kMaxBatchDims];
    int red_steps;              // product of rsize (1: no reduction)
    int kb_per;                 // K-blocks of one reduction step: ceil(K / 32)
    int8_t a_map[kMaxBatchDims], b_map[kMaxBatchDims];   // batch dim -> map dim (-1: broadcast)
    int32_t a_mult[kMaxBatchDims], b_mult[kMaxBatchDims];
    float* C;
    int64_t ldc;
    int64_t c_bs[kMaxBatchDims];
    const float* bias;
    const float* aux;           // kEpiSoftmaxBwd: the softmax output P, laid out like C
    int c_tma;                  // output blocks leave by TMA tensor stores (map tmC): beta 0, C mappable
    int c_rank;                 // tmC's rank (2 + mapped batch dims)
    int8_t c_map[kMaxBatchDims];
    int32_t c_mult[kMaxBatchDims];
    int stage_blocks;           // epilogue staging blocks per warp: 2 lets two TMA stores of C
                                // be in flight per warp (row softmax backward: always 1)
    int p_tma;                  // kEpiSoftmaxBwd: P streamed by TMA (map tmP) into the P ring
    int p_rank;                 // tmP's rank (2 + mapped batch dims)
    int8_t p_map[kMaxBatchDims];
    int32_t p_mult[kMaxBatchDims];
    int64_t bias_rs, bias_cs;
    int64_t bias_bs[kMaxBatchDims];
    float alpha, beta;
    int epi;
    int* status;                // device status word pair {code, detail}
    uint64_t wait_limit_ns;     // limit of every bounded wait (kWaitLimitNs unless a test shortens it)
    int test_stall;             // failure-path test: each CTA's producer stops after its first K-block
    // Fused all-gather of a row-sharded GEMM: when npeers > 0, every output
    // row chunk is written to each peers[q] (the full C of every rank, this
    // rank's own included) at row peer_row0 + m instead of to C.
    // With export_peers the epilogue writes only C (this GPU's full C, at row
    // peer_row0 + m) and the export warps copy each finished tile from there
    // into peers[0..npeers) (the other ranks' full C).
    int npeers;
    int64_t peer_row0;
    int peer_tma;               // full 32-row blocks go out as TMA bulk stores (PeerMaps)
    int export_peers;
    int export_vec;             // N, ldc and every destination allow 16-byte copies
    float* peers[kMaxPeers];
    // Work units: whole tiles, then the K-split levels of the last partial
    // wave (mg_plan.h; units = CTAs, or CTA pairs).
    UnitPlan plan;
    float* part_ws;             // [slot][cta rank][BN/32 chunks][128 rows][32] floats
    unsigned int* part_flag;    // [slot][cta rank]: epilogue warps that stored their part
    // Fused all-gather with split levels: the last level's tiles finish last,
    // so every CTA's export warps (not only the owners') send a share of
    // their rows, each once its tile half is in C (tail_flag[tile][cta rank]
    // counts the owner's epilogue warps).
    int tail_share;
    unsigned int* tail_flag;
    int export_threads;         // export threads in use (32 or 64)
    int export_stream;          // remote 16-byte stores with the streaming (evict-first) hint
};

// 2-D tensor maps over every rank's full C (fused all-gather with TMA stores).
struct PeerMaps {
    CUtensorMap m[kMaxPeers];
};

struct TileCoord {
    int batch, mt, nt;
};

// The i-th unit of CTA (pair) u0 of ustep; false past the last one. Every role
// of the CTA walks the same list.
__device__ __forceinline__ bool unit_at(const GemmParams& p, int u0, int ustep, int i, Unit& u)
{
    return plan_unit_at(p.plan, u0, ustep, i, u);
}

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

// Tensor-map coordinates (map dims 2, 3, 4) that batch multi-index idx adds
// to operand X's loads.
__device__ __forceinline__ void batch_coords(const GemmParams& p, const int* idx, const int8_t* map,
                                             const int32_t* mult, int32_t* c)
{
#pragma unroll
    for (int d = 0; d < kMaxBatchDims; ++d) {
        if (d < p.nbd) {
            const int32_t v = idx[d] * mult[d];
            c[0] += map[d] == 0 ? v : 0;
            c[1] += map[d] == 1 ? v : 0;
            c[2] += map[d] == 2 ? v : 0;
        }
    }
}

// Multi-index of reduction step r (row-major over rsize; 0 on the other dims).
__device__ __forceinline__ void reduction_index(int r, const GemmParams& p, int* idx)
{
#pragma unroll
    for (int d = kMaxBatchDims - 1; d >= 0; --d) {
        if (d < p.nbd && p.rsize[d] > 1) {
            idx[d] = r % p.rsize[d];
            r /= p.rsize[d];
        } else {
            idx[d] = 0;
        }
    }
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

constexpr int kSharedStateBytes = 1024;  // SharedState, padded; the epilogue staging blocks follow
                                         // (1024-byte aligned: TMA stores read them 128B-swizzled)

// What the epilogue warps need of one work unit, worked out ahead of time by
// the producer thread (tile decoding and batch offsets take divisions and
// parameter loads: hundreds of cycles of one warp's latency per tile, which
// the epilogue would otherwise spend between tiles). kind -1: no more units.
struct UnitRec {
    int kind, slot, nsib;   // Unit::kind, slot, nsib
    int n_chunks;           // promotion chunks of the unit's K-range
    int tile, mt, nt;
    int cc[3];              // C tensor map batch coordinates (p.c_tma)
    int64_t coff, boff;     // C and bias batch offsets (elements)
};
constexpr int kRecSlots = 4;

struct SharedState {
    uint64_t full[kMaxStages];        // local: TMA landed
    uint64_t split_done[kMaxStages];  // MMA issuer's CTA: stage ready in every CTA
    uint64_t empty[kMaxStages];       // local: the MMAs reading the stage are done
    uint64_t part_full;               // local: partial accumulator complete
    uint64_t part_free;               // MMA issuer's CTA: every epilogue took the partial
    uint64_t part_full1;              // the same for the second accumulator (p.dbuf)
    uint64_t part_free1;
    uint64_t drain;
    uint32_t tmem_base;
    volatile int abort_flag;
    unsigned int tiles_stored;        // epilogue warps x tiles written to C (export mode)
    uint64_t pair_bar[kEpiWarps / 2]; // row epilogues: epilogue warps w and w ^ 4 met (64 arrivals)
    uint64_t p_full[kPRingSlots];     // softmax backward: a step of P landed in the ring slot
    uint64_t p_empty[kPRingSlots];    // ... every epilogue warp is done with the slot
    uint64_t rec_full[kRecSlots];     // the producer wrote unit record `rec` of the slot
    uint64_t rec_empty[kRecSlots];    // ... every epilogue warp has read it
    UnitRec rec[kRecSlots];
};

static_assert(sizeof(SharedState) <= kSharedStateBytes, "SharedState outgrew its slot");

__device__ __forceinline__ void record_failure(const GemmParams& p, SharedState* ss, int where)
{
    ss->abort_flag = 1;
    if (p.status != nullptr) {
        if (atomicCAS(p.status, 0, 5 /* MG_ERR_TIMEOUT */) == 0) atomicExch(p.status + 1, where);
    }
}

// Bounded wait for the phase of parity `parity` of `bar`. Returns false when
// the CTA is aborting (another role gave up) or this wait itself ran out.
// kHow: 0 = poll (latency-critical single threads), 1 = poll with a suspend
// hint (groups of waiting warps), 2 = poll with cluster-scope acquire (the
// arrivals come from both CTAs of a pair).
template <int kHow>
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, SharedState* ss,
                                           const GemmParams& p, int where)
{
    auto test = [&]() {
        if (kHow == 2) return mbar_test_cluster(bar, parity);
        return mbar_test(bar, parity);
    };
    if (test()) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (kHow == 1) {
            if (mbar_test_sleep(bar, parity, kSleepHintNs)) return true;
        } else {
#pragma unroll 1
            for (int i = 0; i < 16; ++i)
                if (test()) return true;
        }
        if (ss->abort_flag) return false;
        if (global_timer_ns() - t0 > p.wait_limit_ns) {
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

// Producer side of the unit records: waits until the epilogue warps have read
// the slot's previous record, writes unit ui's (u null: the end marker) and
// marks it written (the arrive releases the writes). Single thread.
__device__ __forceinline__ bool post_unit_rec(SharedState* ss, const GemmParams& p, int ui, const Unit* u,
                                              const TileCoord& tc, const int* idx)
{
    const int rs = ui % kRecSlots;
    if (!wait_phase<0>(smem_u32(&ss->rec_empty[rs]), ((uint32_t)(ui / kRecSlots) & 1u) ^ 1u, ss, p,
                       kWaitProducerEmpty))
        return false;
    UnitRec& r = ss->rec[rs];
    if (u == nullptr) {
        r.kind = -1;
    } else {
        r.kind = u->kind;
        r.slot = u->slot;
        r.nsib = u->nsib;
        r.n_chunks = (u->kb1 - u->kb0 + p.chunk_kb - 1) / p.chunk_kb;
        r.tile = u->tile;
        r.mt = tc.mt;
        r.nt = tc.nt;
        int64_t coff = 0, boff = 0;
#pragma unroll
        for (int d = 0; d < kMaxBatchDims; ++d) {
            if (d < p.nbd) {
                coff += (int64_t)idx[d] * p.c_bs[d];
                boff += (int64_t)idx[d] * p.bias_bs[d];
            }
        }
        r.coff = coff;
        r.boff = boff;
        int32_t cc[3] = {0, 0, 0};
        if (p.c_tma) batch_coords(p, idx, p.c_map, p.c_mult, cc);
        r.cc[0] = cc[0];
        r.cc[1] = cc[1];
        r.cc[2] = cc[2];
    }
    mbar_arrive(smem_u32(&ss->rec_full[rs]));
    return true;
}

// Epilogue side: unit ui's record (bounded wait), then the slot goes back.
// Warp-collective; false when the wait gave up.
__device__ __forceinline__ bool take_unit_rec(SharedState* ss, const GemmParams& p, int ui, UnitRec& r)
{
    const int rs = ui % kRecSlots;
    const bool got = wait_phase<1>(smem_u32(&ss->rec_full[rs]), (uint32_t)(ui / kRecSlots) & 1u, ss, p,
                                   kWaitEpiloguePartial);
    if (!__all_sync(0xffffffffu, got)) return false;
    r = ss->rec[rs];
    __syncwarp();   // every lane holds the record before the slot is handed back
    if ((threadIdx.x & 31) == 0) mbar_arrive(smem_u32(&ss->rec_empty[rs]));
    return true;
}

__host__ __device__ constexpr uint32_t pow2_at_least(uint32_t x, uint32_t p = 32)
{
    return p >= x ? p : pow2_at_least(x, 2 * p);
}

template <int BN, bool kPair>
struct Layout {
    static_assert(BN % 32 == 0 && (!kPair || BN % 32 == 0), "tile width must be a multiple of 32");
    static constexpr int kBRows = kPair ? BN / 2 : BN;       // B rows (N) this CTA's MMA operand has
    static constexpr int kBBoxes = (kBRows + 31) / 32;       // MN-major: 32-wide TMA boxes
    static constexpr uint32_t kABytes = kBM * 128;          // 16 KB
    static constexpr uint32_t kBBytes = kBBoxes * 32 * 128;  // room for whole MN-major boxes
    static constexpr uint32_t kStageBytes = kABytes + kBBytes;
    static constexpr uint32_t kTmemCols = pow2_at_least(2 * BN);   // partial + master (A in TMEM: p.tmem_cols)
    static constexpr int kTileRows = kPair ? 2 * kBM : kBM;  // output rows per tile
    static constexpr int kChunks = BN / 32;                  // 32-column epilogue chunks
    static constexpr int kHalfChunks = (kChunks + 1) / 2;    // chunks of column half 0
    // bytes one stage's TMA loads deliver (K-major B: kBRows rows; MN-major:
    // whole 32-wide boxes, the last one partly past this CTA's columns)
    static constexpr uint32_t kLoadA = kABytes;
    __host__ __device__ static constexpr uint32_t load_b(bool mn) { return mn ? kBBytes : (uint32_t)kBRows * 128u; }
};

// lo = x - hi of the 3xTF32 split, hi = x with its 13 low mantissa bits
// cleared; exact in fp32. Non-finite x gives lo = 0, so it passes through hi.
__device__ __forceinline__ uint32_t split_lo(uint32_t x)
{
    const float d = __uint_as_float(x) - __uint_as_float(x & 0xFFFFE000u);
    return d == d ? __float_as_uint(d) : 0u;
}

constexpr int kStageFloatsPerWarp = 32 * 32;   // epilogue staging block per warp

// largest divisor of n that is at most 16 (16-byte loads a split thread keeps in flight)
__host__ __device__ constexpr int batch_of(int n, int b = 16)
{
    return (b <= 1 || n % b == 0) ? (b < 1 ? 1 : b) : batch_of(n, b - 1);
}

// A warp's 32-row block of the output tile: its first row in C (`blk`; in
// export mode this GPU's full C, at this rank's row offset), how many of its
// rows are inside the matrix, its first row within the batch's matrix, the
// batch's element offset in C, and -- for TMA stores -- C's map and the
// batch's map coordinates.
struct OutRows {
    float* blk;
    int rows;
    int row0;
    int64_t coff;
    const CUtensorMap* map;
    int32_t cc[3];
};

// Before a warp writes its staging block: with TMA stores, the previous
// store's read of the block must be over (the write of C itself may still be
// in flight -- that is the point). Warp-collective.
// `pending`: how many of the warp's most recent stores may still be reading
// their blocks (0 .. 3) -- those that did not read the block about to be
// written.
__device__ __forceinline__ void staging_free(const GemmParams& p, int pending = 0)
{
    if (p.c_tma) {
        if ((threadIdx.x & 31) == 0) {
            switch (pending) {
            case 3: bulk_wait_read_n<3>(); break;
            case 2: bulk_wait_read_n<2>(); break;
            case 1: bulk_wait_read_n<1>(); break;
            default: bulk_wait_read_all(); break;
            }
        }
        __syncwarp();
    }
}

// The staging block of this warp's next output store (plain epilogue). With
// two blocks a warp (p.stage_blocks) they alternate, so a TMA store reads one
// while the warp fills the other: only the store before last must be done
// reading (`pending` 1).
__device__ __forceinline__ float* next_staging(const GemmParams& p, float* stage_w, unsigned int& seq, int& pending)
{
    pending = 0;
    if (p.stage_blocks < 2) return stage_w;
    float* blk = stage_w + (seq & 1u) * kStageFloatsPerWarp;
    ++seq;
    pending = 1;
    return blk;
}

// Row epilogues: the warp's k-th store of a tile goes to staging block
// k % S (S = p.stage_blocks); every tile makes the same number nb of stores.
// The stores since block k % S was last written -- the previous tile's from
// the next one of the same block on, this tile's first k -- may still be
// reading theirs.
__device__ __forceinline__ int row_store_pending(int k, int nb, int S)
{
    return k >= S ? S - 1 : (nb - 1 - k) % S + k;
}

// Warp-collective store of a 32 x 32 output block (v[j] = column gn0 + j of
// row row0 + lane). The TMEM layout gives each lane one row; written as is,
// one warp store would touch 32 rows at 16 bytes each. The block is staged in
// shared memory instead -- 16-byte chunks XOR-swizzled by row, conflict-free
// both ways, which is also the 128-byte-swizzled layout of a TMA {32, 32} box
// -- and then (a) handed to the TMA engine as one tensor store into C
// (p.c_tma: the warp moves on while the write drains), (b) handed to it once
// per rank for a fused all-gather (p.peer_tma), or (c) written back
// row-contiguous by the warp, each store 4 rows x 128 bytes, into C or every
// rank's C. All 32 lanes must call it.
__device__ __forceinline__ void store_block_out(const GemmParams& p, const PeerMaps& pm, float* stage,
                                                const float* v, const OutRows& o, int gn0, int nvalid,
                                                int pending = 0)
{
    const int lane = threadIdx.x & 31;
    staging_free(p, pending);
#pragma unroll
    for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4*>(stage + lane * 32)[q ^ (lane & 7)] =
            make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    if (p.c_tma) {
        // rows past M and columns past N are clipped by the map
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && o.rows > 0) {   // (a block wholly past M stores nothing)
            tma_store(o.map, smem_u32(stage), p.c_rank, gn0, o.row0, o.cc[0], o.cc[1], o.cc[2]);
            bulk_commit_group();
        }
        __syncwarp();
        return;
    }
    __syncwarp();
    const bool to_peers = p.npeers > 0 && !p.export_peers;   // the epilogue itself writes every rank's C
    if (to_peers && p.peer_tma && o.row0 + 32 <= p.M) {
        // The staging block is laid out as a TMA 128B-swizzled {32, 32} box:
        // hand it to the TMA engine once per destination (columns past N are
        // clipped by the map), and wait only until it has been read.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            const uint32_t src = smem_u32(stage);
            for (int q = 0; q < p.npeers; ++q)
                tma_store_2d(&pm.m[q], src, gn0, (int32_t)(p.peer_row0 + o.row0));
            bulk_commit_group();
            bulk_wait_read_all();
        }
        __syncwarp();
        return;
    }
    const int ndst = to_peers ? p.npeers : 1;
    const int q = lane & 7;
    const int r_lane = lane >> 3;   // row of this lane within each 4-row store
    // the block's row pieces out of shared memory first, then the global stores
    float4 vals[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = i * 4 + r_lane;
        vals[i] = reinterpret_cast<const float4*>(stage + r * 32)[q ^ (r & 7)];
    }
#pragma unroll 1
    for (int dsti = 0; dsti < ndst; ++dsti) {
        float* base = to_peers ? p.peers[dsti] + o.coff + (p.peer_row0 + o.row0) * p.ldc : o.blk;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = i * 4 + r_lane;
            const float4 val = vals[i];
            if (r >= o.rows || 4 * q >= nvalid) continue;
            float* dst = base + (int64_t)r * p.ldc + gn0 + 4 * q;
            if (4 * q + 4 <= nvalid && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
                *reinterpret_cast<float4*>(dst) = val;
            } else {
                const float e[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (4 * q + j < nvalid) dst[j] = e[j];
            }
        }
    }
    __syncwarp();
}

// Bounded wait until the shared counter reaches `target`.
__device__ __forceinline__ bool wait_count(const unsigned int* ctr, unsigned int target, SharedState* ss,
                                           const GemmParams& p, int where)
{
    const volatile unsigned int* c = ctr;
    if (*c >= target) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        __nanosleep(1000);
        if (*c >= target) return true;
        if (ss->abort_flag) return false;
        if (global_timer_ns() - t0 > p.wait_limit_ns) {
            record_failure(p, ss, where);
            return false;
        }
    }
}

// Export of one finished tile (rows x cols of this CTA, already in this GPU's
// C at src) to every peer's C at the same element offset: the export threads
// read 16-byte pieces from L2 (ld.cg: the epilogue wrote them moments ago)
// and store them over NVLink, kUnroll pieces in flight per thread.
template <bool kVec>
__device__ __forceinline__ void export_tile(const GemmParams& p, int64_t off, int rows, int cols, int et)
{
    constexpr int kUnroll = 8;
    const int nt = p.export_threads;
    if (et >= nt) return;
    const float* src = p.C + off;
    if (kVec) {
        const int c4 = cols >> 2;
        const int items = rows * c4;
#pragma unroll 1
        for (int base = et; base < items; base += nt * kUnroll) {
            float4 v[kUnroll];
            int64_t eo[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int i = base + u * nt;
                const int r = i / c4;
                eo[u] = (int64_t)r * p.ldc + 4 * (i - r * c4);
                if (i < items) v[u] = __ldcg(reinterpret_cast<const float4*>(src + eo[u]));
            }
#pragma unroll 1
            for (int q = 0; q < p.npeers; ++q) {
                float* dst = p.peers[q] + off;
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    if (base + u * nt >= items) continue;
                    float4* d4 = reinterpret_cast<float4*>(dst + eo[u]);
                    if (p.export_stream) __stcs(d4, v[u]);   // evict-first at the destination
                    else *d4 = v[u];
                }
            }
        }
    } else {
        const int items = rows * cols;
#pragma unroll 1
        for (int base = et; base < items; base += nt * kUnroll) {
            float v[kUnroll];
            int64_t eo[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int i = base + u * nt;
                const int r = i / cols;
                eo[u] = (int64_t)r * p.ldc + (i - r * cols);
                if (i < items) v[u] = __ldcg(src + eo[u]);
            }
#pragma unroll 1
            for (int q = 0; q < p.npeers; ++q) {
                float* dst = p.peers[q] + off;
#pragma unroll
                for (int u = 0; u < kUnroll; ++u)
                    if (base + u * nt < items) dst[eo[u]] = v[u];
            }
        }
    }
}

// K-split partial sums. A slot holds one CTA's 128 x BN fp32 partial in the
// epilogue threads' own layout: [32-column chunk][8 float4 columns][128 rows]
// of float4, so one warp instruction moves 32 consecutive rows x 16 bytes --
// 512 contiguous bytes -- and the final range's same thread reads back what
// the partial range's same thread wrote. Kept out of line: they run once per
// split unit and would otherwise crowd the epilogue main loop's registers.
__device__ __noinline__ void store_partial(float* slot, uint32_t t_master, int c_lo, int c_hi, int row)
{
    float4* base = reinterpret_cast<float4*>(slot) + row;
    for (int c = c_lo; c < c_hi; ++c) {
        uint32_t r[32];
        tmem_ld32(t_master + (uint32_t)(32 * c), r);
#pragma unroll
        for (int q = 0; q < 8; ++q)
            base[(size_t)(c * 8 + q) * kBM] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                                          __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
    }
}

// master += slots 0 .. nsib-1 (slot_stride floats apart), in slot order; two
// slots' loads in flight at a time.
__device__ __noinline__ void add_partials(const float* slot0, int nsib, size_t slot_stride, uint32_t t_master,
                                          int c_lo, int c_hi, int row)
{
    const float4* base = reinterpret_cast<const float4*>(slot0) + row;
    const size_t stride4 = slot_stride / 4;
    for (int c = c_lo; c < c_hi; ++c) {
        uint32_t r[32];
        const uint32_t tcol = t_master + (uint32_t)(32 * c);
        tmem_ld32(tcol, r);
        auto add = [&](const float4& x, int e) {
            r[4 * e] = __float_as_uint(__uint_as_float(r[4 * e]) + x.x);
            r[4 * e + 1] = __float_as_uint(__uint_as_float(r[4 * e + 1]) + x.y);
            r[4 * e + 2] = __float_as_uint(__uint_as_float(r[4 * e + 2]) + x.z);
            r[4 * e + 3] = __float_as_uint(__uint_as_float(r[4 * e + 3]) + x.w);
        };
        int q = 0;
        for (; q + 1 < nsib; q += 2) {
            const float4* s0 = base + q * stride4 + (size_t)c * 8 * kBM;
            const float4* s1 = s0 + stride4;
            float4 x0[8], x1[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                x0[e] = __ldcg(s0 + (size_t)e * kBM);
                x1[e] = __ldcg(s1 + (size_t)e * kBM);
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) add(x0[e], e);   // slot q before slot q + 1
#pragma unroll
            for (int e = 0; e < 8; ++e) add(x1[e], e);
        }
        if (q < nsib) {
            const float4* s0 = base + q * stride4 + (size_t)c * 8 * kBM;
            float4 x0[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) x0[e] = __ldcg(s0 + (size_t)e * kBM);
#pragma unroll
            for (int e = 0; e < 8; ++e) add(x0[e], e);
        }
        tmem_st32(tcol, r);
    }
}

// Meeting of the two epilogue warps that hold the two column halves of the
// same 32 rows (warps w and w ^ 4; both read the same TMEM lanes): each has
// posted what the other needs in its own staging block before calling. Only
// the pair waits -- the other row groups run on -- and it waits suspended on
// its mbarrier: the two warps share an SM sub-partition, so a polling loop
// would take issue slots from the very warp it waits for. `meets` counts this
// warp's meetings (both warps of a pair make the same number, so its parity
// is the barrier's phase). Warp-collective.
__device__ __forceinline__ bool pair_meet(SharedState* ss, int warp, unsigned int& meets, const GemmParams& p)
{
    const uint32_t bar = smem_u32(&ss->pair_bar[warp & 3]);
    mbar_arrive(bar);   // release: this thread's posts
    const bool met = wait_phase<1>(bar, meets & 1u, ss, p, kWaitEpilogueRows);
    ++meets;
    return __all_sync(0xffffffffu, met);
}

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32: relative error
// about 2^-22; results below 2^-126 flush to 0). With e^t = 2^(t log2 e) it is
// the row softmax's exponential: one FMA for the argument, one ex2.
__device__ __forceinline__ float exp2_approx(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
constexpr float kLog2e = 1.4426950408889634f;

// Row softmax passes over one thread's TMEM row. The two warps that share a
// row's TMEM lanes take every other 32-column block of it: this warp the
// blocks c = c0, c0 + 64, ... below c1 (c0 = 0 or 32; c1 warp-uniform, as
// the TMEM loads are warp-collective), so under a causal mask both warps
// keep about the same number of live blocks. Column n's logit is
// alpha * acc[n] + brow[n * bcs] (brow null: no bias); columns n >= lim
// (past N, or past the causal diagonal; per lane) are -inf and their bias is
// never read. Blocks that end at or before `full` (warp-uniform: no lane of
// the warp masks them) skip the per-column test. Max, sum: four interleaved
// partial results per block, so no pass is one long dependency chain.
__device__ __forceinline__ float logit_of(uint32_t acc, int n, int lim, float alpha, const float* brow, int64_t bcs)
{
    if (n >= lim) return -INFINITY;
    float x = alpha * __uint_as_float(acc);
    if (brow) x += brow[(int64_t)n * bcs];
    return x;
}

__device__ __forceinline__ void block_max(const uint32_t (&r)[32], int c, int lim, int full, float (&m)[4])
{
    if (c + 32 <= full) {
#pragma unroll
        for (int j = 0; j < 32; ++j) m[j & 3] = fmaxf(m[j & 3], __uint_as_float(r[j]));
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) m[j & 3] = fmaxf(m[j & 3], c + j < lim ? __uint_as_float(r[j]) : -INFINITY);
    }
}

// Max of the live logits. `plain` (no bias, alpha >= 0; warp-uniform) takes
// it on the raw accumulators: rounding is monotone, so
// max_n fl(alpha acc[n]) = fl(alpha max_n acc[n]) exactly. Otherwise each
// column's logit is formed first (some lanes of a biased warp may have no
// bias row).
__device__ __forceinline__ float softmax_row_max(uint32_t t_row, int c0, int c1, int lim, int full, float alpha,
                                                 const float* brow, int64_t bcs, bool plain)
{
    float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    if (plain) {
        int c = c0;
        for (; c + 64 < c1; c += 128) {
            uint32_t r[32], q[32];
            tmem_ld32x2(t_row + c, r, t_row + c + 64, q);
            block_max(r, c, lim, full, m);
            block_max(q, c + 64, lim, full, m);
        }
        if (c < c1) {
            uint32_t r[32];
            tmem_ld32(t_row + c, r);
            block_max(r, c, lim, full, m);
        }
        const float mx = fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
        return mx == -INFINITY ? mx : alpha * mx;
    }
    for (int c = c0; c < c1; c += 64) {
        uint32_t r[32];
        tmem_ld32(t_row + c, r);
#pragma unroll
        for (int j = 0; j < 32; ++j) m[j & 3] = fmaxf(m[j & 3], logit_of(r[j], c + j, lim, alpha, brow, bcs));
    }
    return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}

// exp(logit - mx) of one 32-column block, in place (0 for the -inf
// columns), added into the four partial sums.
__device__ __forceinline__ void exp_block(uint32_t (&r)[32], int c, int lim, int full, float alpha, const float* brow,
                                          int64_t bcs, bool plain, float mx2, float (&s)[4])
{
    if (plain) {
        const float a2 = alpha * kLog2e;
        if (c + 32 <= full) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float e = exp2_approx(fmaf(__uint_as_float(r[j]), a2, -mx2));
                s[j & 3] += e;
                r[j] = __float_as_uint(e);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float e = c + j < lim ? exp2_approx(fmaf(__uint_as_float(r[j]), a2, -mx2)) : 0.f;
                s[j & 3] += e;
                r[j] = __float_as_uint(e);
            }
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float x = logit_of(r[j], c + j, lim, alpha, brow, bcs);
        const float e = x != -INFINITY ? exp2_approx(fmaf(x, kLog2e, -mx2)) : 0.f;
        s[j & 3] += e;
        r[j] = __float_as_uint(e);
    }
}

// exp(logit - mx) back into this warp's blocks of the row; returns their sum.
__device__ __forceinline__ float softmax_row_exp(uint32_t t_row, int c0, int c1, int lim, int full, float alpha,
                                                 const float* brow, int64_t bcs, bool plain, float mx)
{
    const float mx2 = mx * kLog2e;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = c0; c < c1; c += 64) {
        uint32_t r[32];
        tmem_ld32(t_row + c, r);
        exp_block(r, c, lim, full, alpha, brow, bcs, plain, mx2, s);
        tmem_st32_async(t_row + c, r);
    }
    tmem_wait_st();   // the exps are in TMEM before the scaling pass reads them
    return (s[0] + s[1]) + (s[2] + s[3]);
}

// This lane's row of a 32 x 32 block of P (rows blk_row0 .., columns c ..):
// the warp reads the block row-contiguously (each load instruction 4 rows x
// 128 bytes) into its staging block, then each lane takes its own row -- the
// transposition of the output stores, reversed. Rows at or past `rows` and
// columns at or past `ncols` read as 0. Warp-collective; `stage` is free.
__device__ __forceinline__ void load_row_block(const float* blk, int64_t ld, int rows, int ncols, bool vec,
                                               float* stage, float (&pr)[32])
{
    const int lane = threadIdx.x & 31;
    const int q = lane & 7;
    // all eight loads first, then the stores: a shared store between two
    // global loads would hold the second back (the compiler cannot move a
    // load above a store through a pointer that may alias it), turning one
    // memory round trip per block into eight
    float4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = i * 4 + (lane >> 3);
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < rows) {
            const float* src = blk + (int64_t)r * ld + 4 * q;
            if (vec && 4 * q + 4 <= ncols) {
                v[i] = __ldg(reinterpret_cast<const float4*>(src));
            } else {
                if (4 * q + 0 < ncols) v[i].x = __ldg(src + 0);
                if (4 * q + 1 < ncols) v[i].y = __ldg(src + 1);
                if (4 * q + 2 < ncols) v[i].z = __ldg(src + 2);
                if (4 * q + 3 < ncols) v[i].w = __ldg(src + 3);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = i * 4 + (lane >> 3);
        reinterpret_cast<float4*>(stage + r * 32)[q ^ (r & 7)] = v[i];
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float4 v = reinterpret_cast<const float4*>(stage + lane * 32)[k ^ (lane & 7)];
        pr[4 * k] = v.x, pr[4 * k + 1] = v.y, pr[4 * k + 2] = v.z, pr[4 * k + 3] = v.w;
    }
    __syncwarp();   // every lane has its row before the block is reused
}

// Softmax backward, first pass: sum over this thread's row half of
// P[n] * G[n], G = alpha * acc, in column order (columns [c0, c1), c1 <= N).
__device__ __forceinline__ float softmax_bwd_rowsum(uint32_t t_row, int c0, int c1, const float* pblk, int64_t ld,
                                                 int rows, int ncols, bool vec, float* stage, float alpha)
{
    float sum = 0.f;
    for (int c = c0; c < c1; c += 32) {
        float pr[32];
        load_row_block(pblk + c, ld, rows, ncols - c, vec, stage, pr);
        uint32_t r[32];
        tmem_ld32(t_row + c, r);
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (c + j < ncols) sum += pr[j] * (alpha * __uint_as_float(r[j]));
    }
    return sum;
}

// Softmax backward, second pass: dS = P * (G - sum) for this thread's row
// half, columns [c0, c1), stored like any output block.
__device__ __forceinline__ void softmax_bwd_out(const GemmParams& p, const PeerMaps& pm, uint32_t t_row, int c0, int c1,
                                             const float* pblk, int rows, bool vec, float* stage, float sum,
                                             const OutRows& o)
{
    for (int c = c0; c < c1; c += 32) {
        float pr[32];
        staging_free(p);
        load_row_block(pblk + c, p.ldc, rows, p.N - c, vec, stage, pr);
        uint32_t r[32];
        tmem_ld32(t_row + c, r);
#pragma unroll
        for (int j = 0; j < 32; ++j) pr[j] = pr[j] * (p.alpha * __uint_as_float(r[j]) - sum);
        store_block_out(p, pm, stage, pr, o, c, min(32, p.N - c));
    }
}

// The row softmax epilogue of one tile, for the thread's row gm (TMEM row
// t_row; the warp's rows start at o.row0). A row lives in one TMEM lane; warp
// w and its partner w ^ 4 hold its 32-column blocks alternately (warp w the
// blocks from col0 = 32 * (w >> 2) on, every 64 columns). Each thread takes
// the max over its blocks, the pair meets (pair_meet: posts in the warps'
// staging blocks), exp(x - max) goes back into the blocks' TMEM columns while
// summing, the pair meets for the sum (and once more before the staging block
// is reused), then the scaled values leave. Semantics of Tensor::softmax
// (tensor_ops.cpp:2093-2112): max, expf, sum, divide (here: multiply by the
// rounded reciprocal); the sum is formed as eight partial sums (four per
// warp), so its rounding differs from the reference's single running sum by
// a few ulp. Returns false when a meeting gave up (abort).
__device__ __forceinline__ bool softmax_tile(const GemmParams& p, const PeerMaps& pm, SharedState* ss, int warp,
                                          unsigned int& meet_seq, uint32_t t_row, int col0, int gm,
                                          const float* bias_row, const OutRows& o, float* stage_w)
{
    const int wrow0 = o.row0;
    const int lane = threadIdx.x & 31;
    const int half = warp >> 2;
    // the warp's stores a tile: its blocks below N; the posts below go into
    // staging block 0, free once the previous tile's store from it has read it
    const int S = p.stage_blocks;
    const int nb = (p.N - col0 + 63) / 64;
    staging_free(p, nb > 0 ? (nb - 1) % S : 0);
    const bool causal = (p.epi & kEpiCausal) != 0;
    float* xch = stage_w;                                                    // my posts
    const float* pxch = stage_w + (half ? -4 : 4) * p.stage_blocks * kStageFloatsPerWarp;   // partner's
    // live columns: [0, N), and up to the diagonal when causal. wlim bounds
    // every lane of the warp (rows wrow0 .. + 31), so the block loops -- and
    // their warp-collective TMEM loads -- stay warp-uniform; below `full` no
    // lane masks a column
    const int lim = causal ? min(p.N, gm + 1) : p.N;
    const int wlim = causal ? min(p.N, wrow0 + 32) : p.N;
    const int full = causal ? min(p.N, wrow0 + 1) : p.N;
    // the bias path for the whole warp when any of its rows has a bias row
    // (rows past M have none): a warp-uniform choice of code with collective loads
    const bool plain = !__any_sync(0xffffffffu, bias_row != nullptr) && p.alpha >= 0.f;
    float mx = softmax_row_max(t_row, col0, wlim, lim, full, p.alpha, bias_row, p.bias_cs, plain);
    xch[lane] = mx;
    if (!pair_meet(ss, warp, meet_seq, p)) return false;
    mx = fmaxf(mx, pxch[lane]);
    float sum = softmax_row_exp(t_row, col0, wlim, lim, full, p.alpha, bias_row, p.bias_cs, plain, mx);
    xch[32 + lane] = sum;
    if (!pair_meet(ss, warp, meet_seq, p)) return false;
    // the row's sum, added in the same order by both warps
    sum = half ? pxch[32 + lane] + sum : sum + pxch[32 + lane];
    // the partner has read this block before the stores reuse it
    if (!pair_meet(ss, warp, meet_seq, p)) return false;
    const float inv = 1.f / sum;
    const float dead = 0.f * inv;   // columns no lane of the warp reaches (NaN if the whole row is)
    for (int k = 0, c = col0; c < p.N; ++k, c += 64) {
        float v[32];
        if (c < wlim) {
            uint32_t r[32];
            tmem_ld32(t_row + c, r);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * inv;
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = dead;
        }
        store_block_out(p, pm, stage_w + (k % S) * kStageFloatsPerWarp, v, o, c, min(32, p.N - c),
                        row_store_pending(k, nb, S));
    }
    return true;
}

// The fused softmax backward of one tile (dP = dO V^T, N <= BN, one n-tile):
// dS = P * (dP - rowsum(P * dP)), the derivative SoftOp::_backward applies
// (tensor_ops.cpp:2056-2059), P read from p.aux (laid out like C) as
// row-contiguous 32 x 32 blocks through the warp's staging block
// (load_row_block). The two column halves of a row meet like the forward
// softmax's. Arguments as softmax_tile.
__device__ __forceinline__ bool softmax_bwd_tile(const GemmParams& p, const PeerMaps& pm, SharedState* ss, int warp,
                                              unsigned int& meet_seq, uint32_t t_row, int col0, int col1,
                                              const OutRows& o, float* stage_w)
{
    const int wrow0 = o.row0;
    const int64_t coff = o.coff;
    staging_free(p);
    const int lane = threadIdx.x & 31;
    const int half = warp >> 2;
    float* xch = stage_w;
    const float* pxch = stage_w + (half ? -4 : 4) * p.stage_blocks * kStageFloatsPerWarp;
    const int wrows = max(0, min(32, p.M - wrow0));     // the warp's rows inside the matrix
    const float* pblk = p.aux + coff + (int64_t)min(wrow0, max(p.M - 1, 0)) * p.ldc;
    const bool pvec = (p.ldc & 3) == 0 && (coff & 3) == 0 && (reinterpret_cast<uintptr_t>(p.aux) & 15u) == 0;
    const int c1 = min(col1, p.N);
    float sum = softmax_bwd_rowsum(t_row, col0, c1, pblk, p.ldc, wrows, p.N, pvec, stage_w, p.alpha);
    xch[lane] = sum;
    if (!pair_meet(ss, warp, meet_seq, p)) return false;
    sum = half ? pxch[lane] + sum : sum + pxch[lane];   // first half's columns first
    if (!pair_meet(ss, warp, meet_seq, p)) return false;
    softmax_bwd_out(p, pm, t_row, col0, c1, pblk, wrows, pvec, stage_w, sum, o);
    return true;
}

// The softmax backward of one tile with P streamed into the ring by the P
// producer (p.p_tma): the same arithmetic and order as softmax_bwd_tile, P
// read from the ring slot's box of this warp's column half (row sub * 32 +
// lane, the staging layout) instead of from global memory. Each pass consumes
// `nsteps` slots -- every step, also one past N -- and releases each slot once
// the warp has its rows; `slot` / `phase` follow the ring across tiles.
__device__ __forceinline__ bool softmax_bwd_tile_ring(const GemmParams& p, const PeerMaps& pm, SharedState* ss,
                                                   int warp, unsigned int& meet_seq, int& slot, uint32_t& phase,
                                                   int nsteps, uint32_t t_row, int col0, const OutRows& o,
                                                   float* stage_w)
{
    staging_free(p);
    const int lane = threadIdx.x & 31;
    const int half = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    float* xch = stage_w;
    const float* pxch = stage_w + (half ? -4 : 4) * p.stage_blocks * kStageFloatsPerWarp;
    const float* ring = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(ss) + kSharedStateBytes +
                                                       (size_t)kEpiWarps * p.stage_blocks * kStageFloatsPerWarp * 4);
    // this lane's 32 P values of the slot's box for this half; then the slot goes back
    auto take = [&](float (&pr)[32]) -> bool {
        const bool landed = wait_phase<1>(smem_u32(&ss->p_full[slot]), phase, ss, p, kWaitEpiloguePartial);
        if (!__all_sync(0xffffffffu, landed)) return false;
        const float* box = ring + (size_t)slot * (kPSlotBytes / 4) + (size_t)half * (kPBoxBytes / 4);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float4 v = reinterpret_cast<const float4*>(box + row * 32)[k ^ (row & 7)];
            pr[4 * k] = v.x, pr[4 * k + 1] = v.y, pr[4 * k + 2] = v.z, pr[4 * k + 3] = v.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ss->p_empty[slot]));
        if (++slot == kPRingSlots) { slot = 0; phase ^= 1u; }
        return true;
    };
    float sum = 0.f;
    for (int s = 0; s < nsteps; ++s) {
        const int c = col0 + 32 * s;
        float pr[32];
        if (!take(pr)) return false;
        if (c < p.N) {
            uint32_t r[32];
            tmem_ld32(t_row + c, r);
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (c + j < p.N) sum += pr[j] * (p.alpha * __uint_as_float(r[j]));
        }
    }
    xch[lane] = sum;
    if (!pair_meet(ss, warp, meet_seq, p)) return false;
    sum = half ? pxch[lane] + sum : sum + pxch[lane];   // first half's columns first
    if (!pair_meet(ss, warp, meet_seq, p)) return false;
    for (int s = 0; s < nsteps; ++s) {
        const int c = col0 + 32 * s;
        float pr[32];
        if (!take(pr)) return false;
        if (c < p.N) {
            uint32_t r[32];
            tmem_ld32(t_row + c, r);
#pragma unroll
            for (int j = 0; j < 32; ++j) pr[j] = pr[j] * (p.alpha * __uint_as_float(r[j]) - sum);
            store_block_out(p, pm, stage_w, pr, o, c, min(32, p.N - c));
        }
    }
    return true;
}

// tmA / tmB map the operands; in pre-split 3xTF32 mode (p.presplit) tmAlo /
// tmBlo map their lo planes (same layout), which the producer loads next to
// the raw tiles instead of the split warps computing them.

// kRow: the row epilogue this instantiation carries -- kRowNone (alpha, bias,
// beta), kRowSoftmax (softmax_tile) or kRowSoftmaxBwd (softmax_bwd_tile) --
// so that each variant holds only its own epilogue code.
enum : int { kRowNone = 0, kRowSoftmax = 1, kRowSoftmaxBwd = 2 };

template <int BN, bool kPair, int kRow>
__global__ void __launch_bounds__(kThreads, 1)
    mg_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmAlo,
                      const __grid_constant__ CUtensorMap tmBlo,
                      const __grid_constant__ CUtensorMap tmP,
                      const __grid_constant__ CUtensorMap tmC,
                      const __grid_constant__ GemmParams p,
                      const __grid_constant__ PeerMaps pm)
{
    using L = Layout<BN, kPair>;
    // A in TMEM (p.a_tmem) exists for tiles up to 128 wide only: the wider
    // instantiations compile without any of its branches
    constexpr bool kATmem = BN <= 128;
    const bool a_tmem = kATmem && p.a_tmem != 0;
    const uint32_t tmem_cols = kATmem ? (uint32_t)p.tmem_cols : L::kTmemCols;
    // p.b2 exists for the single-SM plain-epilogue kernel of width 64 only
    constexpr bool kB2 = BN == 64 && !kPair && kRow == kRowNone;
    const bool b2 = kB2 && a_tmem && p.b2 != 0;
    const uint32_t acc_w = b2 ? 2u * BN : (uint32_t)BN;   // TMEM columns of one accumulator
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the 128-byte swizzle atoms.
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const uint32_t smem_base = smem_u32(smem);
    const int stages = p.stages;
    // shared memory: raw stages, then (3xTF32) one lo tile per stage, then the
    // barriers; with A in TMEM the lo region holds only B's lo tiles (kBBytes a
    // stage), and with b2 each stage is A, B, B's lo tile and there is no lo region
    const uint32_t stage_stride = b2 ? L::kStageBytes + L::kBBytes : L::kStageBytes;
    const uint32_t raw_region = (uint32_t)stages * stage_stride;
    const uint32_t lo_stride = a_tmem ? L::kBBytes : L::kStageBytes;
    SharedState* ss =
        reinterpret_cast<SharedState*>(smem + raw_region + (p.split && !b2 ? (uint32_t)stages * lo_stride : 0u));

    auto a_raw = [&](int s) { return smem_base + (uint32_t)s * stage_stride; };
    auto b_raw = [&](int s) { return smem_base + (uint32_t)s * stage_stride + L::kABytes; };
    auto a_lo = [&](int s) { return a_raw(s) + raw_region; };
    auto b_lo = [&](int s) {
        return b2 ? b_raw(s) + L::kBBytes
                  : (a_tmem ? smem_base + raw_region + (uint32_t)s * L::kBBytes : b_raw(s) + raw_region);
    };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = kPair ? cluster_ctarank() : 0u;
    const bool issuer = rank == 0;
    // work unit: a tile per CTA, or a tile per pair (both CTAs walk the same list)
    const int unit0 = kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int unit_step = kPair ? (int)(gridDim.x >> 1) : (int)gridDim.x;

    // split warps that report each landed stage to the MMA issuer: all of them
    // when they compute lo tiles, else a single thread relays it
    const int relay_threads = (p.split && !p.presplit) ? kSplitThreads : 1;
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(&ss->full[s]), 1);
            mbar_init(smem_u32(&ss->split_done[s]), relay_threads * (kPair ? 2 : 1));
            mbar_init(smem_u32(&ss->empty[s]), 1);
        }
        mbar_init(smem_u32(&ss->part_full), 1);
        mbar_init(smem_u32(&ss->part_free), kEpiThreads * (kPair ? 2 : 1));
        mbar_init(smem_u32(&ss->part_full1), 1);
        mbar_init(smem_u32(&ss->part_free1), kEpiThreads * (kPair ? 2 : 1));
        mbar_init(smem_u32(&ss->drain), 1);
        ss->abort_flag = 0;
        ss->tiles_stored = 0u;
        for (int q = 0; q < kEpiWarps / 2; ++q) mbar_init(smem_u32(&ss->pair_bar[q]), 64);
        for (int q = 0; q < kPRingSlots; ++q) {
            mbar_init(smem_u32(&ss->p_full[q]), 1);
            mbar_init(smem_u32(&ss->p_empty[q]), kEpiWarps);
        }
        for (int q = 0; q < kRecSlots; ++q) {
            mbar_init(smem_u32(&ss->rec_full[q]), 1);
            mbar_init(smem_u32(&ss->rec_empty[q]), kEpiWarps);
        }
        mbar_fence_init();
    }
    if (warp == kProducerWarp && lane == 0) {
        tma_prefetch_map(&tmA);
        tma_prefetch_map(&tmB);
        if (p.presplit) {
            tma_prefetch_map(&tmAlo);
            tma_prefetch_map(&tmBlo);
        }
    }
    if (kRow == kRowSoftmaxBwd && p.p_tma && warp == kExportWarp0 && lane == 0) tma_prefetch_map(&tmP);
    if (p.c_tma && threadIdx.x == 0) tma_prefetch_map(&tmC);
    if (warp == kMmaWarp) {
        if (kPair) {
            tmem_alloc_pair(smem_u32(&ss->tmem_base), tmem_cols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(&ss->tmem_base), tmem_cols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (kPair) cluster_sync_all();   // the peer's barriers exist before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = ss->tmem_base;
    // barriers of the MMA issuer's CTA, as shared::cluster addresses
    const uint32_t split_done0 = kPair ? cluster_map(smem_u32(&ss->split_done[0]), 0) : smem_u32(&ss->split_done[0]);
    const uint32_t part_free0 = kPair ? cluster_map(smem_u32(&ss->part_free), 0) : smem_u32(&ss->part_free);
    const uint32_t part_free1_0 = kPair ? cluster_map(smem_u32(&ss->part_free1), 0) : smem_u32(&ss->part_free1);

    if (warp == kProducerWarp) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0, issued_par = 0;
            bool ok = true;
            Unit u;
            int ui = 0;
            for (; ok && unit_at(p, unit0, unit_step, ui, u); ++ui) {
                const TileCoord tc = decode_tile(u.tile, p);
                int idx[kMaxBatchDims];
                batch_index(tc.batch, p, idx);
                if (!post_unit_rec(ss, p, ui, &u, tc, idx)) {
                    ok = false;
                    break;
                }
                int32_t ta[3] = {0, 0, 0}, tb[3] = {0, 0, 0};   // the tile's batch coordinates
                batch_coords(p, idx, p.a_map, p.a_mult, ta);
                batch_coords(p, idx, p.b_map, p.b_mult, tb);
                int32_t a2 = ta[0], a3 = ta[1], a4 = ta[2], b2 = tb[0], b3 = tb[1], b4 = tb[2];
                const int m0 = tc.mt * L::kTileRows + (int)rank * kBM;
                const int n0 = tc.nt * BN + (int)rank * L::kBRows;
                int red_step = -1;
                for (int kb = u.kb0; kb < u.kb1; ++kb) {
                    if (p.test_stall && ui == 0 && kb > u.kb0) {
                        // failure-path test: this stage is never loaded, so the
                        // roles waiting for it run out their (shortened) limit
                        ok = false;
                        break;
                    }
                    if (!wait_phase<0>(smem_u32(&ss->empty[stage]), phase ^ 1u, ss, p, kWaitProducerEmpty)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = smem_u32(&ss->full[stage]);
                    mbar_arrive_expect_tx(fb, (L::kLoadA + L::load_b(p.b_mn != 0)) * (p.presplit ? 2u : 1u));
                    int kk = kb;
                    if (p.red_steps > 1) {
                        // K-block kk of reduction step r: the operands' batch
                        // coordinates move to that step's matrices
                        const int r = kb / p.kb_per;
                        kk = kb - r * p.kb_per;
                        if (r != red_step) {
                            red_step = r;
                            int ridx[kMaxBatchDims];
                            reduction_index(r, p, ridx);
                            int32_t ra[3] = {ta[0], ta[1], ta[2]}, rb[3] = {tb[0], tb[1], tb[2]};
                            batch_coords(p, ridx, p.a_map, p.a_mult, ra);
                            batch_coords(p, ridx, p.b_map, p.b_mult, rb);
                            a2 = ra[0], a3 = ra[1], a4 = ra[2], b2 = rb[0], b3 = rb[1], b4 = rb[2];
                        }
                    }
                    const int k0 = kk * kBK;
                    // raw tiles, and in pre-split mode the lo tiles one region higher
                    for (int plane = 0; plane < (p.presplit ? 2 : 1); ++plane) {
                        const CUtensorMap* ma = plane ? &tmAlo : &tmA;
                        const CUtensorMap* mb = plane ? &tmBlo : &tmB;
                        const uint32_t da = plane ? a_lo(stage) : a_raw(stage);
                        const uint32_t db = plane ? b_lo(stage) : b_raw(stage);
                        if (!p.a_mn) {
                            tma_load(ma, fb, da, p.a_rank, k0, m0, a2, a3, a4);
                        } else {
#pragma unroll
                            for (int j = 0; j < kBM / 32; ++j)
                                tma_load(ma, fb, da + 4096u * j, p.a_rank, m0 + 32 * j, k0, a2, a3, a4);
                        }
                        if (!p.b_mn) {
                            tma_load(mb, fb, db, p.b_rank, k0, n0, b2, b3, b4);
                        } else {
#pragma unroll
                            for (int j = 0; j < L::kBBoxes; ++j)
                                tma_load(mb, fb, db + 4096u * j, p.b_rank, n0 + 32 * j, k0, b2, b3, b4);
                        }
                    }
                    issued |= 1u << stage;
                    issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == stages) { stage = 0; phase ^= 1u; }
                }
            }
            if (ok) ok = post_unit_rec(ss, p, ui, nullptr, TileCoord{}, nullptr);   // no more units
            if (!ok) {
                // let every issued copy land before the CTA's shared memory goes away
                for (int s = 0; s < stages; ++s)
                    if (issued & (1u << s)) drain_phase(smem_u32(&ss->full[s]), (issued_par >> s) & 1u);
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------ MMA issuer (leader CTA)
        if (lane == 0 && issuer) {
            const bool split = p.split != 0;
            const uint32_t a_lbo = p.a_mn ? 4096u : 16u;
            const uint32_t b_lbo = p.b_mn ? 4096u : 16u;
            const uint32_t a_sbo = p.a_mn ? 512u : 1024u;
            const uint32_t b_sbo = p.b_mn ? 512u : 1024u;
            const uint32_t a_lay = p.a_mn ? kLayoutSw128Base32 : kLayoutSw128;
            const uint32_t b_lay = p.b_mn ? kLayoutSw128Base32 : kLayoutSw128;
            const uint32_t a_kstep = p.a_mn ? 1024u : 32u;
            const uint32_t b_kstep = p.b_mn ? 1024u : 32u;
            uint32_t d_tmem = tmem_base;   // accumulator: the partial, columns [0, BN)
            auto mma = [&](uint64_t da, uint64_t db, uint32_t acc) {
                if (kPair) tc_mma_tf32_pair(d_tmem, da, db, p.idesc, acc);
                else tc_mma_tf32(d_tmem, da, db, p.idesc, acc);
            };
            auto commit_all = [&](uint32_t bar) {   // arrive in every CTA of the pair
                if (kPair) tc_commit_pair_all(bar, (uint16_t)0x3);
                else tc_commit(bar);
            };
            int stage = 0;
            uint32_t phase = 0;
            uint32_t chunk_phase = 0;
            bool ok = true;
            Unit u;
            for (int ui = 0; ok && unit_at(p, unit0, unit_step, ui, u); ++ui) {
                // p.dbuf: whole tiles of one chunk alternate between the two
                // accumulators, so a tile's MMAs run during the previous
                // tile's epilogue
                const int rg = p.dbuf ? (ui & 1) : 0;
                d_tmem = tmem_base + (uint32_t)rg * acc_w;
                const uint32_t acc_free = smem_u32(rg ? &ss->part_free1 : &ss->part_free);
                const uint32_t acc_full = smem_u32(rg ? &ss->part_full1 : &ss->part_full);
                for (int kb = u.kb0; kb < u.kb1; ++kb) {
                    const int rel = kb - u.kb0;   // chunks restart with every unit
                    const bool chunk_start = (rel % p.chunk_kb) == 0;
                    const bool chunk_end = (rel % p.chunk_kb) == p.chunk_kb - 1 || kb == u.kb1 - 1;
                    if (chunk_start) {
                        // every epilogue has taken the previous partial (p.dbuf: has
                        // finished with this accumulator two tiles ago)
                        const uint32_t fpar = p.dbuf ? ((((uint32_t)ui >> 1) & 1u) ^ 1u) : (chunk_phase ^ 1u);
                        if (!wait_phase<kPair ? 2 : 0>(acc_free, fpar, ss, p, kWaitMmaPartialFree)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                    }
                    if (!wait_phase<kPair ? 2 : 0>(smem_u32(&ss->split_done[stage]), phase, ss, p, kWaitMmaStage)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < kBK / 8; ++ks) {
                        const uint32_t accum = (!chunk_start || ks > 0) ? 1u : 0u;
                        const uint64_t da = smem_desc(a_raw(stage) + ks * a_kstep, a_lbo, a_sbo, a_lay);
                        const uint64_t db = smem_desc(b_raw(stage) + ks * b_kstep, b_lbo, b_sbo, b_lay);
                        if (split && a_tmem) {
                            // A's hi and lo tiles from TMEM (the split warps wrote them;
                            // in a pair each CTA's rows in its own TMEM)
                            const uint32_t t_hi = tmem_base + (uint32_t)(p.a_col0 + 64 * stage + 8 * ks);
                            auto mma_ta = [&](uint32_t ta, uint64_t db_, uint32_t acc, uint32_t idesc) {
                                if (kPair) tc_mma_tf32_pair_ta(d_tmem, ta, db_, idesc, acc);
                                else tc_mma_tf32_ta(d_tmem, ta, db_, idesc, acc);
                            };
                            if (b2) {
                                // [B hi | B lo] is one operand 2 BN wide (db): two MMAs
                                // give hi*hi | hi*lo and add lo*hi | lo*lo
                                mma_ta(t_hi, db, accum, p.idesc2);
                                mma_ta(t_hi + 32u, db, 1u, p.idesc2);
                            } else {
                                const uint64_t dbl = smem_desc(b_lo(stage) + ks * b_kstep, b_lbo, b_sbo, b_lay);
                                mma_ta(t_hi + 32u, db, accum, p.idesc);   // lo * hi
                                mma_ta(t_hi, dbl, 1u, p.idesc);           // hi * lo
                                mma_ta(t_hi, db, 1u, p.idesc);            // hi * hi
                            }
                        } else if (split) {
                            const uint64_t dal = smem_desc(a_lo(stage) + ks * a_kstep, a_lbo, a_sbo, a_lay);
                            const uint64_t dbl = smem_desc(b_lo(stage) + ks * b_kstep, b_lbo, b_sbo, b_lay);
                            mma(dal, db, accum);   // lo * hi
                            mma(da, dbl, 1u);      // hi * lo
                            mma(da, db, 1u);       // hi * hi
                        } else {
                            mma(da, db, accum);
                        }
                    }
                    commit_all(smem_u32(&ss->empty[stage]));   // frees the stage in every CTA
                    if (++stage == stages) { stage = 0; phase ^= 1u; }
                    if (chunk_end) {
                        commit_all(acc_full);  // partial ready for promotion (p.dbuf: for the output)
                        chunk_phase ^= 1u;
                    }
                }
            }
            // every MMA this thread issued has finished before TMEM is freed
            if (kPair) tc_commit_pair(smem_u32(&ss->drain));
            else tc_commit(smem_u32(&ss->drain));
            drain_phase(smem_u32(&ss->drain), 0);
        }
        __syncwarp();
    } else if (warp >= kExportWarp0) {
        if (kRow == kRowSoftmaxBwd && p.p_tma) {
            // -------------------------------------------- P producer (softmax backward)
            // One lane streams, for every tile of this CTA, its 128 rows of P
            // into the ring twice (the epilogue's two passes), a step -- the
            // next 32 columns of both halves -- per slot, in the order the
            // epilogue warps consume them; plain TMA loads from this GPU's P.
            if (warp == kExportWarp0 && lane == 0) {
                uint8_t* ring = reinterpret_cast<uint8_t*>(ss) + kSharedStateBytes +
                                (size_t)kEpiWarps * p.stage_blocks * kStageFloatsPerWarp * 4;
                int slot = 0;
                uint32_t phase = 0, issued = 0, issued_par = 0;
                bool ok = true;
                Unit u;
                for (int ui = 0; ok && unit_at(p, unit0, unit_step, ui, u); ++ui) {
                    const TileCoord tc = decode_tile(u.tile, p);
                    int idx[kMaxBatchDims];
                    batch_index(tc.batch, p, idx);
                    int32_t pc[3] = {0, 0, 0};
                    batch_coords(p, idx, p.p_map, p.p_mult, pc);
                    const int m0 = tc.mt * L::kTileRows + (int)rank * kBM;
                    for (int step = 0; ok && step < 2 * L::kHalfChunks; ++step) {
                        const int s = step % L::kHalfChunks;   // both passes walk the same columns
                        if (!wait_phase<1>(smem_u32(&ss->p_empty[slot]), phase ^ 1u, ss, p, kWaitProducerEmpty)) {
                            ok = false;
                            break;
                        }
                        const uint32_t fb = smem_u32(&ss->p_full[slot]);
                        mbar_arrive_expect_tx(fb, kPSlotBytes);
                        const uint32_t dst = smem_u32(ring + (size_t)slot * kPSlotBytes);
                        tma_load(&tmP, fb, dst, p.p_rank, 32 * s, m0, pc[0], pc[1], pc[2]);
                        tma_load(&tmP, fb, dst + kPBoxBytes, p.p_rank, 32 * (L::kHalfChunks + s), m0, pc[0], pc[1],
                                 pc[2]);
                        issued |= 1u << slot;
                        issued_par = (issued_par & ~(1u << slot)) | (phase << slot);
                        if (++slot == kPRingSlots) { slot = 0; phase ^= 1u; }
                    }
                }
                if (!ok) {
                    // let every issued copy land before the CTA's shared memory goes away
                    for (int q = 0; q < kPRingSlots; ++q)
                        if (issued & (1u << q)) drain_phase(smem_u32(&ss->p_full[q]), (issued_par >> q) & 1u);
                }
            }
            __syncwarp();
        } else if (p.export_peers && p.npeers > 0) {
        // ------------------------------------------------ export (fused all-gather)
        // Follows the epilogue tile by tile: tile j of this CTA may be copied
        // once all eight epilogue warps have counted it into tiles_stored.
            const int et = threadIdx.x - kExportWarp0 * 32;
            unsigned int j = 0;
            Unit u;
            for (int ui = 0; unit_at(p, unit0, unit_step, ui, u); ++ui, ++j) {
                if (!wait_count(&ss->tiles_stored, (unsigned int)kEpiWarps * (j + 1u), ss, p, kWaitExportTile))
                    break;
                if (u.kind == 1) continue;   // a partial K-range: its tile leaves with the final range
                if (p.tail_share && u.tile >= p.plan.lev_tile0[p.plan.nlev - 1]) continue;   // shared below
                __threadfence();
                const TileCoord tc = decode_tile(u.tile, p);
                int idx[kMaxBatchDims];
                batch_index(tc.batch, p, idx);
                int64_t coff = 0;
#pragma unroll
                for (int d = 0; d < kMaxBatchDims; ++d)
                    if (d < p.nbd) coff += (int64_t)idx[d] * p.c_bs[d];
                const int m0 = tc.mt * L::kTileRows + (int)rank * kBM;
                const int n0 = tc.nt * BN;
                const int rows = min(kBM, p.M - m0);
                const int cols = min(BN, p.N - n0);
                if (rows <= 0 || cols <= 0) continue;
                const int64_t off = coff + (p.peer_row0 + m0) * p.ldc + n0;
                if (p.export_vec) export_tile<true>(p, off, rows, cols, et);
                else export_tile<false>(p, off, rows, cols, et);
            }
            if (p.tail_share) {
                // this CTA's share of the last level's rows (every CTA of the grid)
                constexpr int kHalves = kPair ? 2 : 1;
                const int t0 = p.plan.lev_tile0[p.plan.nlev - 1];
                const int R = p.plan.lev_tiles[p.plan.nlev - 1] * kHalves * kBM;
                const int G = (int)gridDim.x, b = (int)blockIdx.x;
                const int r_end = (int)((int64_t)R * (b + 1) / G);
                for (int r = (int)((int64_t)R * b / G); r < r_end;) {
                    const int piece = r / kBM;   // (tile, half) of the level
                    const int cnt = min(r_end, (piece + 1) * kBM) - r;
                    if (!wait_count(&p.tail_flag[piece], (unsigned int)kEpiWarps, ss, p, kWaitExportTile)) break;
                    __threadfence();
                    const TileCoord tc = decode_tile(t0 + piece / kHalves, p);
                    int idx[kMaxBatchDims];
                    batch_index(tc.batch, p, idx);
                    int64_t coff = 0;
#pragma unroll
                    for (int d = 0; d < kMaxBatchDims; ++d)
                        if (d < p.nbd) coff += (int64_t)idx[d] * p.c_bs[d];
                    const int m0 = tc.mt * L::kTileRows + (piece % kHalves) * kBM + (r - piece * kBM);
                    const int n0 = tc.nt * BN;
                    const int rows = min(cnt, p.M - m0);
                    const int cols = min(BN, p.N - n0);
                    if (rows > 0 && cols > 0) {
                        const int64_t off = coff + (p.peer_row0 + m0) * p.ldc + n0;
                        if (p.export_vec) export_tile<true>(p, off, rows, cols, et);
                        else export_tile<false>(p, off, rows, cols, et);
                    }
                    r += cnt;
                }
            }
            // the peers' rows have landed before the kernel is seen as complete
            __threadfence_system();
        }
    } else if (warp >= kSplitWarp0) {
        // ------------------------------------------------ split / stage relay
        // When the warps split (3xTF32), every thread waits for the stage
        // itself and reports its share itself: a warp-wide wait / arrive is one
        // warp instruction, and no thread is held back by another's wake-up
        // (one elected arrival per warp or per CTA measured slower there).
        // With nothing to split, one thread relays each stage (relay_threads).
        const int tid = threadIdx.x - kSplitWarp0 * 32;
        const bool compute_lo = p.split && !p.presplit;
        int stage = 0;
        uint32_t phase = 0;
        bool ok = tid < relay_threads;   // without lo tiles to compute, one thread relays
        Unit u;
        for (int ui = 0; ok && unit_at(p, unit0, unit_step, ui, u); ++ui) {
            for (int kb = u.kb0; kb < u.kb1; ++kb) {
                bool landed = p.relay_spin
                    ? wait_phase<0>(smem_u32(&ss->full[stage]), phase, ss, p, kWaitSplitFull)
                    : wait_phase<1>(smem_u32(&ss->full[stage]), phase, ss, p, kWaitSplitFull);
                if (!landed) {
                    ok = false;
                    break;
                }
                if (compute_lo && a_tmem) {
                    // A into TMEM: this thread's row (TMEM lane tid: warp 8 + g
                    // writes lanes 32g ..) as hi (truncated to TF32) and
                    // lo = x - hi, 32 columns each; from the 128-byte-swizzled
                    // K-major tile, or the unswizzled MN-major one (32-row boxes
                    // of 4 KB, K steps of 128 bytes)
                    uint32_t hi[32], lw[32];
                    if (!p.a_mn) {
                        const uint4* arow = reinterpret_cast<const uint4*>(smem + (size_t)stage * stage_stride) + tid * 8;
#pragma unroll
                        for (int c = 0; c < 8; ++c) {
                            const uint4 x = arow[c ^ (tid & 7)];
                            const uint32_t e[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                            for (int j = 0; j < 4; ++j) hi[4 * c + j] = e[j];
                        }
                    } else {
                        const uint32_t* acol = reinterpret_cast<const uint32_t*>(smem + (size_t)stage * stage_stride) +
                                               (tid >> 5) * 1024 + (tid & 31);
#pragma unroll
                        for (int k = 0; k < 32; ++k) hi[k] = acol[k * 32];
                    }
#pragma unroll
                    for (int k = 0; k < 32; ++k) {
                        lw[k] = split_lo(hi[k]);
                        hi[k] &= 0xFFFFE000u;
                    }
                    const uint32_t t_a = tmem_base + ((uint32_t)((tid >> 5) * 32) << 16) +
                                         (uint32_t)(p.a_col0 + 64 * stage);
                    tmem_st32_async(t_a, hi);
                    tmem_st32_async(t_a + 32u, lw);
                    // and the B tile's lo beside it in shared memory, as below
                    const uint4* raw = reinterpret_cast<const uint4*>(smem + (size_t)stage * stage_stride) +
                                       L::kABytes / 16;
                    uint4* lo = b2 ? const_cast<uint4*>(raw) + L::kBBytes / 16   // right after B (b2)
                                   : reinterpret_cast<uint4*>(smem + raw_region + (size_t)stage * L::kBBytes);
                    constexpr int n4 = (int)(L::kBBytes / 16);
                    static_assert(n4 % kSplitThreads == 0, "B tile not a whole number of split rounds");
                    constexpr int kPer = n4 / kSplitThreads;
#pragma unroll
                    for (int u = 0; u < kPer; ++u) {
                        const uint4 x = raw[tid + u * kSplitThreads];
                        lo[tid + u * kSplitThreads] =
                            make_uint4(split_lo(x.x), split_lo(x.y), split_lo(x.z), split_lo(x.w));
                    }
                    fence_proxy_async_smem();
                    tmem_wait_st();
                    tc_fence_before();   // the TMEM writes before the MMA issuer's reads
                } else if (compute_lo) {
                    // The MMA reads the raw tile as hi (the TF32 datapath drops the
                    // 13 low mantissa bits); lo = x - hi is exact.
                    const uint4* raw = reinterpret_cast<const uint4*>(smem + (size_t)stage * L::kStageBytes);
                    uint4* lo = reinterpret_cast<uint4*>(smem + raw_region + (size_t)stage * L::kStageBytes);
                    constexpr int n4 = (int)(L::kStageBytes / 16);
                    static_assert(n4 % kSplitThreads == 0, "stage not a whole number of split rounds");
                    // all of this thread's loads first (they queue behind the
                    // tensor core's reads of shared memory), then the stores
                    constexpr int kPer = n4 / kSplitThreads;
                    constexpr int kBatch = batch_of(kPer);
                    static_assert(kPer % kBatch == 0, "split batches must tile the stage");
#pragma unroll 1
                    for (int i0 = 0; i0 < kPer; i0 += kBatch) {
                        uint4 x[kBatch];
#pragma unroll
                        for (int u = 0; u < kBatch; ++u) x[u] = raw[tid + (i0 + u) * kSplitThreads];
#pragma unroll
                        for (int u = 0; u < kBatch; ++u)
                            lo[tid + (i0 + u) * kSplitThreads] =
                                make_uint4(split_lo(x[u].x), split_lo(x[u].y), split_lo(x[u].z), split_lo(x[u].w));
                    }
                    fence_proxy_async_smem();
                }
                // stage ready (in this CTA) for the MMA issuer
                if (kPair) mbar_arrive_cluster(split_done0 + (uint32_t)stage * 8u);
                else mbar_arrive(smem_u32(&ss->split_done[stage]));
                if (++stage == stages) { stage = 0; phase ^= 1u; }
            }
        }
    } else {
        // ------------------------------------------------ epilogue (warps 0-7)
        const int sub = warp & 3;                    // TMEM sub-partition = row group
        const int half = warp >> 2;                  // column half
        // column half h owns 32-column chunks [c_lo, c_hi) (BN / 32 may be odd)
        const int c_lo = half * L::kHalfChunks;
        const int c_hi = half ? L::kChunks : L::kHalfChunks;
        const int row = sub * 32 + lane;
        const uint32_t lane_base = tmem_base + ((uint32_t)(sub * 32) << 16);
        const uint32_t t_part = lane_base;
        const uint32_t t_master = lane_base + acc_w;   // (b2: the partial is 2 BN wide)
        float* stage_w = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ss) + kSharedStateBytes) +
                         warp * p.stage_blocks * kStageFloatsPerWarp;   // this warp's store staging block(s)
        const bool has_bias = (p.epi & kEpiBias) != 0;
        constexpr bool softmax = kRow == kRowSoftmax;
        constexpr bool softmax_bwd = kRow == kRowSoftmaxBwd;
        uint32_t chunk_phase = 0;
        unsigned int meet_seq = 0;   // row epilogues: meetings with the partner warp so far
        unsigned int out_seq = 0;    // output stores so far (alternating staging blocks)
        int p_slot = 0;              // softmax backward with the P ring: the next slot and its phase
        uint32_t p_phase = 0;
        bool ok = true;
        for (int ui = 0; ok; ++ui) {
            UnitRec u;   // the unit, decoded by the producer
            if (!take_unit_rec(ss, p, ui, u)) {
                ok = false;
                break;
            }
            if (u.kind < 0) break;
            const int n_chunks = u.n_chunks;
            const int rg = p.dbuf ? (ui & 1) : 0;
            if (p.dbuf) {
                // one chunk: the accumulator itself is the result
                const bool got = wait_phase<1>(smem_u32(rg ? &ss->part_full1 : &ss->part_full),
                                               ((uint32_t)ui >> 1) & 1u, ss, p, kWaitEpiloguePartial);
                if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
                tc_fence_after();
            }
            // ---- promotions: master = sum of the tile's partials (fp32 round-to-nearest)
            for (int c = 0; c < (p.dbuf ? 0 : n_chunks); ++c) {
                const bool got = wait_phase<1>(smem_u32(&ss->part_full), chunk_phase, ss, p, kWaitEpiloguePartial);
                if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
                tc_fence_after();
#pragma unroll 1
                // the MMAs wait for this hand-off at every chunk, so it is kept
                // short: both loads behind one wait, master stores not waited
                // for until the partial has been released
                for (int j = 32 * c_lo; j < 32 * c_hi; j += 32) {
                    uint32_t r[32];
                    if (b2) {
                        // the partial's two halves first (hi * B | lo * B terms)
                        uint32_t q[32];
                        tmem_ld32x2(t_part + j, r, t_part + (uint32_t)BN + j, q);
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            r[i] = __float_as_uint(__uint_as_float(r[i]) + __uint_as_float(q[i]));
                        if (c > 0) {
                            tmem_ld32(t_master + j, q);
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                r[i] = __float_as_uint(__uint_as_float(q[i]) + __uint_as_float(r[i]));
                        }
                    } else if (c > 0) {
                        uint32_t m[32];
                        tmem_ld32x2(t_part + j, r, t_master + j, m);
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            r[i] = __float_as_uint(__uint_as_float(m[i]) + __uint_as_float(r[i]));
                    } else {
                        tmem_ld32(t_part + j, r);
                    }
                    tmem_st32_async(t_master + j, r);
                }
                tc_fence_before();
                // the MMA may overwrite the partial once every epilogue thread has it
                if (kPair) mbar_arrive_cluster(part_free0);
                else mbar_arrive(smem_u32(&ss->part_free));
                tmem_wait_st();   // the master is complete before this thread reads it again
                chunk_phase ^= 1u;
            }
            if (!ok) break;

            if (u.kind == 1) {
                // A partial K-range: the master goes to its workspace slot for
                // the tile's final range to add; nothing is written to C.
                store_partial(p.part_ws + (size_t)(u.slot * 2 + (int)rank) * (kBM * BN), t_master,
                              c_lo, c_hi, row);
                __threadfence();
                __syncwarp();
                if (lane == 0) atomicAdd(&p.part_flag[u.slot * 2 + (int)rank], 1u);
                tc_fence_before();
                if (p.export_peers) {
                    __syncwarp();
                    if (lane == 0) atomicAdd(&ss->tiles_stored, 1u);
                }
                continue;
            }
            if (u.kind == 2) {
                // the final range: every other range of the tile has stored its part
                bool ready = true;
                if (lane == 0)
                    for (int q = 0; q < u.nsib && ready; ++q)
                        ready = wait_count(&p.part_flag[(u.slot + q) * 2 + (int)rank], (unsigned int)kEpiWarps, ss, p,
                                           kWaitPartials);
                if (!__shfl_sync(0xffffffffu, ready ? 1 : 0, 0)) {
                    ok = false;
                    break;
                }
                __threadfence();
                // master += the other ranges' partials, in range order
                add_partials(p.part_ws + (size_t)(u.slot * 2 + (int)rank) * (kBM * BN), u.nsib,
                             (size_t)2 * kBM * BN, t_master, c_lo, c_hi, row);
            }

            // ---- output epilogue from the master
            const int64_t coff = u.coff, boff = u.boff;
            const int m0 = u.mt * L::kTileRows + (int)rank * kBM;
            const int n0 = u.nt * BN;
            const int gm = m0 + row;
            const bool rok = gm < p.M;
            // this warp's 32-row output block: its first row in C (export
            // mode: this GPU's full C, at this rank's row offset) and how many
            // of its rows are inside the matrix
            const int wrow0 = m0 + sub * 32;
            const int brows = max(0, min(32, p.M - wrow0));
            OutRows orow;
            orow.blk = p.C + coff + (int64_t)(brows > 0 ? wrow0 + (p.export_peers ? p.peer_row0 : 0) : 0) * p.ldc;
            orow.rows = brows;
            orow.row0 = wrow0;
            orow.coff = coff;
            orow.map = &tmC;
            orow.cc[0] = u.cc[0];
            orow.cc[1] = u.cc[1];
            orow.cc[2] = u.cc[2];
            // export mode: this GPU's full C, at this rank's row offset
            const int64_t crow_idx = rok ? gm + (p.export_peers ? p.peer_row0 : 0) : 0;
            float* crow = p.C + coff + crow_idx * p.ldc;
            const float* brow = has_bias ? p.bias + boff + (int64_t)(rok ? gm : 0) * p.bias_rs : nullptr;
            // the result, column 0: the master, or (p.dbuf) this tile's accumulator
            const uint32_t t_row = p.dbuf ? lane_base + (uint32_t)rg * acc_w : t_master;
            // b2 with one chunk: the accumulator's two halves are added here
            const bool sum_halves = b2 && p.dbuf;

            if constexpr (softmax) {
                // row softmax (N <= BN, one n-tile): softmax_tile
                if (!softmax_tile(p, pm, ss, warp, meet_seq, t_row, 32 * half, gm, has_bias && rok ? brow : nullptr,
                                  orow, stage_w)) {
                    ok = false;
                    break;
                }
            } else if constexpr (softmax_bwd) {
                // fused softmax backward (N <= BN, one n-tile): softmax_bwd_tile
                const bool done = p.p_tma
                    ? softmax_bwd_tile_ring(p, pm, ss, warp, meet_seq, p_slot, p_phase, L::kHalfChunks, t_row,
                                            c_lo * 32, orow, stage_w)
                    : softmax_bwd_tile(p, pm, ss, warp, meet_seq, t_row, c_lo * 32, c_hi * 32, orow, stage_w);
                if (!done) {
                    ok = false;
                    break;
                }
            } else {
                for (int c = 32 * c_lo; c < 32 * c_hi; c += 32) {
                    const int gn0 = n0 + c;
                    if (gn0 >= p.N) break;   // uniform across the warp
                    uint32_t r[32];
                    float v[32];
                    if (sum_halves) {
                        uint32_t q[32];
                        tmem_ld32x2(t_row + c, r, t_row + (uint32_t)BN + c, q);
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            v[j] = p.alpha * (__uint_as_float(r[j]) + __uint_as_float(q[j]));
                    } else {
                        tmem_ld32(t_row + c, r);
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = p.alpha * __uint_as_float(r[j]);
                    }
                    const int nvalid = min(32, p.N - gn0);
                    if (rok && has_bias) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < nvalid) v[j] += brow[(int64_t)(gn0 + j) * p.bias_cs];
                    }
                    if (rok && p.beta != 0.f) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < nvalid) v[j] += p.beta * crow[gn0 + j];
                    }
                    int pending;
                    float* blk = next_staging(p, stage_w, out_seq, pending);
                    store_block_out(p, pm, blk, v, orow, gn0, nvalid, pending);
                }
            }
            tc_fence_before();
            if (p.tail_share && u.kind == 2 && u.tile >= p.plan.lev_tile0[p.plan.nlev - 1]) {
                // a last-level tile half is in C: any CTA's export warps may send it
                __threadfence();
                __syncwarp();
                if (lane == 0) atomicAdd(&p.tail_flag[(u.tile - p.plan.lev_tile0[p.plan.nlev - 1]) * (kPair ? 2 : 1) + (int)rank], 1u);
            }
            if (p.dbuf) {
                // done with this accumulator: the MMAs of the tile after next may use it
                if (kPair) mbar_arrive_cluster(rg ? part_free1_0 : part_free0);
                else mbar_arrive(smem_u32(rg ? &ss->part_free1 : &ss->part_free));
            }
            if (p.export_peers) {
                // this warp's part of the tile is in C (visible GPU-wide) for the export warps
                __threadfence();
                __syncwarp();
                if (lane == 0) atomicAdd(&ss->tiles_stored, 1u);
            }
        }
        // this CTA's TMA stores of C have completed before it exits
        if (p.c_tma) {
            if (lane == 0) bulk_wait_all();
            __syncwarp();
        }
        // remote rows (fused all-gather) have landed and are visible
        // system-wide before the kernel is seen as complete
        if (p.npeers > 0 && !p.export_peers) {
            if (lane == 0) bulk_wait_all();
            __syncwarp();
            __threadfence_system();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (kPair) cluster_sync_all();   // the leader's MMAs no longer touch the peer
    if (warp == kMmaWarp) {
        tc_fence_after();
        if (kPair) tmem_dealloc_pair(tmem_base, tmem_cols);
        else tmem_dealloc(tmem_base, tmem_cols);
    }
}

}  // namespace mg

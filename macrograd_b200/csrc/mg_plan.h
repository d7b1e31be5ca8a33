// mg_plan.h -- the GEMM kernel's work units, the K split of its last wave, and
// the column bands of the copy-engine all-gather.
//
// Plain C++ shared by the kernel (device), the launcher (host) and the CPU
// tests (tests/plan_check.cpp), so the tests check the code the GPU runs.
//
// T output tiles go to U resident units (CTAs, or CTA pairs). Whole tiles fill
// floor(T / U) waves, dealt round-robin. The R < U leftover tiles would keep
// U - R units idle for a whole tile time; instead they may be cut along K into
// ranges, in up to kMaxLevels levels: level l takes lev_tiles[l] tiles (from
// tile lev_tile0[l]) and cuts each into lev_split[l] ranges, one range to each
// of the units 0 .. lev_tiles[l] * lev_split[l] - 1. A range accumulates its
// own fp32 sum; the non-final ranges of a tile store theirs in workspace slots
// (lev_slot0[l] + tile-in-level * (split - 1) + range), and the tile's final
// range adds them, in range order, before writing the output.
#pragma once

#ifdef __CUDACC__
#define MG_HD __host__ __device__ __forceinline__
#else
#define MG_HD inline
#endif

namespace mg {

constexpr int kMaxLevels = 4;

struct UnitPlan {
    int full_tiles;     // whole tiles [0, full_tiles), round-robin
    int mirror;         // odd waves dealt in reverse unit order (unit u takes position U - 1 - u)
    int nlev;           // split levels after them
    int num_kb;         // K-blocks of a whole tile
    int lev_split[kMaxLevels], lev_tiles[kMaxLevels], lev_tile0[kMaxLevels], lev_slot0[kMaxLevels];
};

// One work unit: K-blocks [kb0, kb1) of a tile; kind 0 = the whole tile,
// 1 = a partial range (stores its fp32 sum in workspace slot `slot`),
// 2 = the final range (adds slots slot .. slot + nsib - 1 and writes C).
struct Unit {
    int tile, kb0, kb1, kind, slot, nsib;
};

// The i-th unit of unit u0 out of ustep; false past its last one.
MG_HD bool plan_unit_at(const UnitPlan& w, int u0, int ustep, int i, Unit& u)
{
    // whole tiles: wave v holds tiles [v * ustep, (v + 1) * ustep); the unit's
    // position in wave v is u0, or ustep - 1 - u0 on odd waves when mirrored
    // (a unit then alternates between even and odd tile positions)
    const int waves = w.full_tiles / ustep, rem = w.full_tiles - waves * ustep;
    const int last_pos = (w.mirror && (waves & 1)) ? ustep - 1 - u0 : u0;
    const int nw = waves + (last_pos < rem ? 1 : 0);
    if (i < nw) {
        u.tile = i * ustep + ((w.mirror && (i & 1)) ? ustep - 1 - u0 : u0);
        u.kb0 = 0;
        u.kb1 = w.num_kb;
        u.kind = 0;
        u.slot = 0;
        u.nsib = 0;
        return true;
    }
    int j = i - nw;
    for (int l = 0; l < w.nlev; ++l) {
        const int S = w.lev_split[l];
        if (u0 >= w.lev_tiles[l] * S) continue;
        if (j-- > 0) continue;
        const int tl = u0 / S, part = u0 - tl * S;
        u.tile = w.lev_tile0[l] + tl;
        u.kb0 = (int)((long long)w.num_kb * part / S);
        u.kb1 = (int)((long long)w.num_kb * (part + 1) / S);
        const int base = w.lev_slot0[l] + tl * (S - 1);
        u.kind = part == S - 1 ? 2 : 1;
        u.slot = part == S - 1 ? base : base + part;
        u.nsib = part == S - 1 ? S - 1 : 0;
        return true;
    }
    return false;
}

// Plans the split for `units` resident units: all R leftover tiles at once in
// floor(units / R) ranges when that is >= 2 (at most 8), else level by level in
// 2, 4, 8, ... ranges per tile, as many tiles per level as the units allow;
// ranges of at least min_kb K-blocks. Kept only when every leftover tile is
// placed and the plan saves at least 5 % of the time of whole-tile waves.
// Returns the workspace slots needed (0: no split; w then holds whole tiles).
inline int plan_k_split(UnitPlan& w, int total_tiles, int units, int num_kb, int min_kb)
{
    w.full_tiles = total_tiles;
    w.nlev = 0;
    w.num_kb = num_kb;
    if (units < 2 || min_kb < 1) return 0;
    const int waves = total_tiles / units, R = total_tiles - waves * units;
    if (R == 0) return 0;
    int S[kMaxLevels], Rl[kMaxLevels], n = 0, rem = R;
    double t = 0.0;
    if (units / R >= 2) {
        int s = units / R < 8 ? units / R : 8;
        if (num_kb / min_kb < s) s = num_kb / min_kb;
        if (s >= 2) {
            S[0] = s;
            Rl[0] = R;
            n = 1;
            rem = 0;
            t = 1.0 / s;
        }
    } else {
        for (int s = 2; rem > 0 && n < kMaxLevels && num_kb / s >= min_kb; s *= 2) {
            const int r = rem < units / s ? rem : units / s;
            if (r == 0) break;
            S[n] = s;
            Rl[n] = r;
            ++n;
            rem -= r;
            t += 1.0 / s;
        }
    }
    if (rem > 0 || n == 0) return 0;
    if (waves + t > 0.95 * (waves + 1)) return 0;   // not worth the partial sums
    w.full_tiles = waves * units;
    int tile0 = w.full_tiles, slot0 = 0;
    for (int l = 0; l < n; ++l) {
        w.lev_split[l] = S[l];
        w.lev_tiles[l] = Rl[l];
        w.lev_tile0[l] = tile0;
        w.lev_slot0[l] = slot0;
        tile0 += Rl[l];
        slot0 += Rl[l] * (S[l] - 1);
    }
    w.nlev = n;
    return slot0;
}

// Column bands of a row-sharded GEMM whose rows reach the other ranks through
// the copy engines: the GEMM runs as one launch per band of whole n-tile
// columns (m_tiles x columns tiles), and a finished band is copied to the
// peers while the next band computes, so only the last band's copy is not
// overlapped. Full bands hold w waves of `units` tiles: the smallest w <= 4
// whose whole columns fill at least 95 % of them, else the fullest. When the
// launches can split tiles along K (max_split >= 2: a tile's K-blocks make at
// least two ranges of the shortest length), the columns after the full bands
// -- or the last full band, when there are none left over -- are cut into
// bands of about units / 2^k tiles, k = 1, 2, ... (2^k <= max_split), each
// of which its launch can spread over every unit by a 2^k-way split; the
// bands shrink towards the end and the last one is a single column at best.
// Without the split the leftover columns form one last band.
// Returns the number of bands; 1 when a single band holds the whole GEMM.
// force_cols > 0 sets the band width in columns instead (a tuning knob).
constexpr int kMaxBands = 16;

struct BandPlan {
    int nbands;
    int col0[kMaxBands + 1];   // band b: n-tile columns [col0[b], col0[b + 1])
};

inline int plan_bands(BandPlan& bp, int m_tiles, int n_tiles, int units, int max_split = 1, int force_cols = 0)
{
    bp.nbands = 1;
    bp.col0[0] = 0;
    bp.col0[1] = n_tiles;
    if (m_tiles < 1 || n_tiles < 2 || units < 1) return 1;
    int cols = 0;
    double best = -1.0;
    for (int w = 1; w <= 4; ++w) {
        const int c = (int)((long long)w * units / m_tiles);
        if (c < 1) continue;
        const double fill = (double)c * m_tiles / ((double)w * units);
        if (fill >= 0.95) {
            cols = c;
            break;
        }
        if (fill > best) {
            best = fill;
            cols = c;
        }
    }
    if (cols < 1) cols = 1;   // a single column already holds more than 4 waves
    const bool taper = force_cols <= 0 && max_split >= 2;
    if (force_cols > 0) cols = force_cols;
    if (cols >= n_tiles && !taper) return 1;
    int full = n_tiles / cols, rem = n_tiles - full * cols;
    if (taper && rem == 0) {   // the last full band tapers instead
        --full;
        rem = cols;
    }
    if (full > kMaxBands - 1) full = kMaxBands - 1;
    rem = n_tiles - full * cols;
    int n = 0, c = 0;
    for (; n < full; ++n, c += cols) bp.col0[n] = c;
    for (int k = taper ? 1 : 0; rem > 0;) {
        long long t = rem;
        if (taper && k < 30 && (1 << k) <= max_split) {
            t = units / ((long long)m_tiles << k);
            if (t >= rem) {   // a smaller band first
                ++k;
                continue;
            }
            if (t < 1) t = rem;
        }
        if (n == kMaxBands - 1) t = rem;   // past the band limit the last one takes the rest
        bp.col0[n++] = c;
        c += (int)t;
        rem -= (int)t;
    }
    bp.col0[n] = n_tiles;
    bp.nbands = n;
    return n;
}

}  // namespace mg

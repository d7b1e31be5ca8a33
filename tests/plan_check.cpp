// plan_check.cpp -- CPU check of the GEMM kernel's work-unit plan
// (macrograd_b200/csrc/mg_plan.h, the same code the kernel and the launcher
// use). Built and run by tests/test_plan.py; prints "ok" or the first failure.
#include <cstdio>
#include <map>
#include <vector>

#include "mg_plan.h"

using mg::Unit;
using mg::UnitPlan;

static int fail(const char* what, int T, int U, int KB, int mk)
{
    std::printf("FAIL %s (tiles %d, units %d, num_kb %d, min_kb %d)\n", what, T, U, KB, mk);
    return 1;
}

// Every (tile, K-block) is covered exactly once; partial slots are written by
// exactly one range of their tile and read by that tile's final range; a
// split never makes any unit's work longer than whole-tile waves would. With
// `mirror` the whole-tile waves alternate direction: a unit's tiles then
// alternate between even and odd positions (when the unit count is even).
static int check(int T, int U, int KB, int mk, int* nsplit, int mirror = 0)
{
    UnitPlan w{};
    w.mirror = mirror;
    const int nslots = mg::plan_k_split(w, T, U, KB, mk);
    if (w.nlev > 0) ++*nsplit;
    if ((nslots > 0) != (w.nlev > 0)) return fail("slot count vs levels", T, U, KB, mk);
    const int grid = w.nlev > 0 ? U : (T < U ? T : U);
    std::vector<int> cover((size_t)T * KB, 0);
    std::map<int, int> slot_writer;            // slot -> tile
    std::map<int, std::pair<int, int>> finals; // tile -> (first slot, count)
    int worst = 0;
    for (int u0 = 0; u0 < grid; ++u0) {
        Unit u;
        int work = 0, prev_whole = -1;
        for (int i = 0; mg::plan_unit_at(w, u0, grid, i, u); ++i) {
            if (mirror && u.kind == 0 && grid % 2 == 0 && prev_whole >= 0 && (u.tile - prev_whole) % 2 == 0)
                return fail("mirrored waves: consecutive whole tiles of a unit share a parity", T, U, KB, mk);
            if (u.kind == 0) prev_whole = u.tile;
            if (u.tile < 0 || u.tile >= T || u.kb0 < 0 || u.kb1 > KB || u.kb0 >= u.kb1)
                return fail("unit out of range", T, U, KB, mk);
            for (int kb = u.kb0; kb < u.kb1; ++kb) cover[(size_t)u.tile * KB + kb]++;
            work += u.kb1 - u.kb0;
            if (u.kind == 1) {
                if (slot_writer.count(u.slot)) return fail("slot written twice", T, U, KB, mk);
                slot_writer[u.slot] = u.tile;
            } else if (u.kind == 2) {
                if (u.kb1 != KB) return fail("final range does not end the tile", T, U, KB, mk);
                finals[u.tile] = {u.slot, u.nsib};
            } else if (u.kb0 != 0 || u.kb1 != KB) {
                return fail("whole tile with a partial range", T, U, KB, mk);
            }
        }
        worst = work > worst ? work : worst;
    }
    for (size_t i = 0; i < cover.size(); ++i)
        if (cover[i] != 1) return fail("K-block not covered exactly once", T, U, KB, mk);
    int read = 0;
    for (auto& f : finals) {
        for (int q = 0; q < f.second.second; ++q) {
            auto it = slot_writer.find(f.second.first + q);
            if (it == slot_writer.end() || it->second != f.first) return fail("final reads a foreign slot", T, U, KB, mk);
        }
        read += f.second.second;
    }
    if (read != (int)slot_writer.size() || (int)slot_writer.size() != nslots)
        return fail("slots written / read / planned disagree", T, U, KB, mk);
    const int whole = ((T + grid - 1) / grid) * KB;   // K-blocks of the busiest unit without a split
    if (w.nlev > 0 && worst > whole) return fail("split made the busiest unit slower", T, U, KB, mk);
    return 0;
}

static int expect(int T, int U, int KB, int mk, int nlev, const int* split, const int* tiles)
{
    UnitPlan w{};
    mg::plan_k_split(w, T, U, KB, mk);
    if (w.nlev != nlev) return fail("unexpected level count", T, U, KB, mk);
    for (int l = 0; l < nlev; ++l)
        if (w.lev_split[l] != split[l] || w.lev_tiles[l] != tiles[l]) return fail("unexpected level", T, U, KB, mk);
    return 0;
}

static int fail_bands(const char* what, int m, int n, int U)
{
    std::printf("FAIL %s (m-tiles %d, n-tiles %d, units %d)\n", what, m, n, U);
    return 1;
}

// Column bands: contiguous, non-empty, cover every column once; widths never
// grow towards the end (unless the band cap merged the rest into the last);
// the first band holds at most 4 waves (or one column).
static int check_bands(int m, int n, int U, int ms)
{
    mg::BandPlan bp;
    const int nb = mg::plan_bands(bp, m, n, U, ms);
    if (nb != bp.nbands || nb < 1 || nb > mg::kMaxBands) return fail_bands("band count", m, n, U);
    if (bp.col0[0] != 0 || bp.col0[nb] != n) return fail_bands("bands do not cover the columns", m, n, U);
    for (int b = 0; b < nb; ++b)
        if (bp.col0[b + 1] <= bp.col0[b]) return fail_bands("empty band", m, n, U);
    const int last = nb < mg::kMaxBands ? nb : nb - 1;   // bands that must not grow
    for (int b = 1; b < last; ++b)
        if (bp.col0[b + 1] - bp.col0[b] > bp.col0[b] - bp.col0[b - 1]) return fail_bands("band wider than the one before", m, n, U);
    const int w0 = bp.col0[1] - bp.col0[0];
    if (nb > 1 && (long long)w0 * m > 4ll * U && w0 > 1) return fail_bands("band above 4 waves", m, n, U);
    if (ms < 2 && nb > 1) {   // no split: equal bands, then the leftover
        for (int b = 0; b + 1 < nb; ++b)
            if (bp.col0[b + 1] - bp.col0[b] != w0) return fail_bands("unequal full bands", m, n, U);
    }
    return 0;
}

static int expect_bands(int m, int n, int U, int ms, int nb, const int* col0)
{
    mg::BandPlan bp;
    if (mg::plan_bands(bp, m, n, U, ms) != nb) return fail_bands("unexpected band count", m, n, U);
    for (int b = 0; b <= nb; ++b)
        if (bp.col0[b] != col0[b]) return fail_bands("unexpected band edge", m, n, U);
    return 0;
}

int main()
{
    int nsplit = 0;
    const int units[] = {1, 2, 3, 37, 74, 148};
    const int kbs[] = {1, 8, 12, 32, 256};
    const int mks[] = {1, 4, 16};
    for (int T = 1; T < 320; ++T)
        for (int U : units)
            for (int KB : kbs)
                for (int mk : mks)
                    if (check(T, U, KB, mk, &nsplit) || check(T, U, KB, mk, &nsplit, 1)) return 1;
    for (int T : {512, 1024, 1184, 2048})
        for (int U : units)
            if (check(T, U, 256, 16, &nsplit) || check(T, U, 256, 16, &nsplit, 1)) return 1;
    // the row-sharded 8192^3 shapes on 74 SM pairs
    const int s8[] = {2, 4}, t8[] = {37, 17};
    const int s4[] = {2}, t4[] = {34};
    if (expect(128, 74, 256, 16, 2, s8, t8)) return 1;    // 8 GPUs: 1 wave + halves + quarters
    if (expect(256, 74, 256, 16, 1, s4, t4)) return 1;    // 4 GPUs: 3 waves + halves
    if (expect(1024, 74, 256, 16, 0, nullptr, nullptr)) return 1;   // 1 GPU: saves < 5 %
    if (nsplit == 0) return fail("no case split at all", 0, 0, 0, 0);
    int nbanded = 0;
    for (int m = 1; m < 160; ++m)
        for (int n = 1; n < 160; ++n)
            for (int U : units)
                for (int ms : {1, 2, 8, 16}) {
                    if (check_bands(m, n, U, ms)) return 1;
                    mg::BandPlan bp;
                    nbanded += mg::plan_bands(bp, m, n, U, ms) > 1;
                }
    // 8192^3 row-sharded over 8 / 4 / 2 GPUs: 256 x 256 pair tiles on 74 SM pairs,
    // 256 K-blocks (up to a 16-way split at the default 16-block minimum)
    const int b8[] = {0, 18, 27, 31, 32}, b8s[] = {0, 18, 32};
    const int b4[] = {0, 9, 18, 27, 31, 32}, b2[] = {0, 9, 18, 27, 29, 31, 32};
    if (expect_bands(4, 32, 74, 16, 4, b8)) return 1;     // 72 tiles (1 wave), 36, 16, 4
    if (expect_bands(4, 32, 74, 1, 2, b8s)) return 1;     // no K split: 72, then the 56 left
    if (expect_bands(8, 32, 74, 16, 5, b4)) return 1;     // 3 x 72 tiles, 32, 8
    if (expect_bands(16, 32, 74, 16, 6, b2)) return 1;    // 3 x 144 tiles (2 waves), 32, 32, 16
    const int one[] = {0, 16}, taper1[] = {0, 9, 13, 15, 16};
    if (expect_bands(4, 16, 74, 1, 1, one)) return 1;     // one wave, no split: a single band
    if (expect_bands(4, 16, 74, 16, 4, taper1)) return 1; // one wave, split: 36, 16, 8, 4 tiles
    if (nbanded == 0) return fail_bands("no case banded at all", 0, 0, 0);
    std::printf("ok %d split plans, %d band plans checked\n", nsplit, nbanded);
    return 0;
}

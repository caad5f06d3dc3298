// Coverage check of the decode kernel's static work plans, on the CPU.
//
// The plan functions of csrc/dev.cuh are the ones the producer warp, the
// consumer warps and the loader all evaluate; here they run as plain C++ for
// one model shape (the shape of one rank under tensor parallelism) and every
// CTA of the grid, and the program checks that each weight phase's tiles are
// split over the grid exactly once, that every CTA's K-slices cover the
// blocks of a row exactly once and that every chunk fits one ring slot.
//
//   plan_check H qd kvd FF V nh hd grid qtype
//
// prints "ok" and exits 0, or prints the first violated property and exits 1.
// `plan_check selftest` feeds the partition check two overlapping ranges and
// a gap and exits 0 only if both are reported.
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include <vector_types.h>  // uint2 of the device structs (CUDA include directory)

#include "../ai-agent-framework_b200/csrc/dev.cuh"

using namespace b2;

namespace {

int g_fail = 0;

void fail(const std::string& what) {
    if (!g_fail) std::printf("FAIL %s\n", what.c_str());
    g_fail = 1;
}

// One CTA's plan: its K-slices cover nb blocks (every slice non-empty) and a
// chunk of nt tiles x bpk blocks fits a slot.
void check_plan(const TPlan& p, int nb, int tbb, int slot, const std::string& where) {
    if (p.n == 0) {
        if (p.nchunks != 0) fail(where + ": empty plan with chunks");
        return;
    }
    if (p.bpk < 1 || p.nks < 1 || p.nt < 1) fail(where + ": non-positive plan field");
    if ((long long)p.nks * p.bpk < nb) fail(where + ": K-slices leave blocks uncovered");
    if ((long long)(p.nks - 1) * p.bpk >= nb) fail(where + ": empty K-slice");
    if ((long long)p.nt * p.bpk * tbb > slot) fail(where + ": chunk larger than a ring slot");
    if (p.nks > 1 && p.nt != 1) fail(where + ": several tiles per chunk with a split K");
    if (p.nchunks != (p.n + p.nt - 1) / p.nt * p.nks) fail(where + ": chunk count");
}

// The CTAs' tile ranges of one phase, in CTA order, partition [first, first + tiles).
void check_partition(const std::vector<std::pair<int, int>>& r, int first, int tiles, const std::string& where) {
    std::vector<int> seen(tiles, 0);
    for (const auto& x : r) {
        if (x.second < 0) fail(where + ": negative tile count");
        for (int u = x.first; u < x.first + x.second; u++) {
            if (u < first || u >= first + tiles) {
                fail(where + ": tile out of range");
                return;
            }
            seen[u - first]++;
        }
    }
    for (int u = 0; u < tiles; u++)
        if (seen[u] != 1) {
            fail(where + ": tile " + std::to_string(first + u) + " covered " + std::to_string(seen[u]) + " times");
            return;
        }
}

}  // namespace

int main(int argc, char** argv) {
    if (argc == 2 && std::string(argv[1]) == "selftest") {
        check_partition({{0, 3}, {2, 2}}, 0, 4, "overlap");
        const int overlap = g_fail;
        g_fail = 0;
        check_partition({{0, 1}, {2, 2}}, 0, 4, "gap");
        const int gap = g_fail;
        std::printf("%s\n", overlap && gap ? "selftest ok" : "selftest missed a planted error");
        return overlap && gap ? 0 : 1;
    }
    if (argc != 10) {
        std::printf("usage: plan_check H qd kvd FF V nh hd grid qtype\n");
        return 2;
    }
    const int H = std::atoi(argv[1]), qd = std::atoi(argv[2]), kvd = std::atoi(argv[3]), FF = std::atoi(argv[4]);
    const int V = std::atoi(argv[5]), nh = std::atoi(argv[6]), hd = std::atoi(argv[7]), grid = std::atoi(argv[8]);
    const int qt = std::atoi(argv[9]);
    const int slot = 8192, warps = kConsumerWarps;
    const int tbb = kTileRows * tile_qb(qt) + 2 * kTileRows;  // one (tile, block) unit with its scales

    // plan slots are distinct and inside the table
    {
        std::vector<int> used(kPlanSlots, 0);
        for (int k = PH_WO; k <= PH_DOWN; k++) used[plan_slot(k, 1)]++;
        for (int s = 0; s < kMaxLmSub; s++) used[plan_slot(PH_LMHEAD, s)]++;
        for (int S = 1; S <= kMaxSplits; S++) used[plan_slot(PH_QA, S)]++;
        for (int i = 0; i < kPlanSlots; i++)
            if (used[i] != 1) fail("plan slot " + std::to_string(i) + " used " + std::to_string(used[i]) + " times");
    }

    struct Phase {
        const char* name;
        int tiles, nb;
        bool own;
    };
    const Phase phases[] = {
        {"wo", H / kTileRows, qd / 32, true},
        {"gateup", 2 * FF / kTileRows, H / 32, false},
        {"down", H / kTileRows, FF / 32, true},
        {"lm_head", (int)(tiled_rows(V) / kTileRows), H / 32, false},
    };
    for (const Phase& ph : phases) {
        std::vector<std::pair<int, int>> r;
        for (int cta = 0; cta < grid; cta++) {
            const TPlan p = ph.own ? own_plan(ph.tiles, ph.nb, tbb, cta, grid, slot, warps)
                                   : tile_plan(ph.tiles, ph.nb, tbb, cta, grid, slot, warps);
            check_plan(p, ph.nb, tbb, slot, std::string(ph.name) + " cta " + std::to_string(cta));
            r.push_back({p.u0, p.n});
        }
        check_partition(r, 0, ph.tiles, ph.name);
        if (ph.own && ph.tiles <= grid)
            for (int cta = 0; cta < grid; cta++)
                if ((r[cta].second == 1) != (cta >= grid - ph.tiles))
                    fail(std::string(ph.name) + ": residual rows not owned by the last CTAs");
    }

    // gate/up with the owners' share cut to own_pct percent (gu_plan)
    for (int own_pct : {0, 10, 25, 50, 100}) {
        const int tiles = 2 * FF / kTileRows;
        std::vector<std::pair<int, int>> r;
        for (int cta = 0; cta < grid; cta++) {
            const TPlan p = gu_plan(tiles, H / 32, tbb, cta, grid, slot, warps, H / kTileRows, own_pct);
            check_plan(p, H / 32, tbb, slot, "gateup own " + std::to_string(own_pct) + " cta " + std::to_string(cta));
            r.push_back({p.u0, p.n});
        }
        check_partition(r, 0, tiles, "gateup own " + std::to_string(own_pct));
    }

    // down split over K (dn_split_plan): each residual tile's blocks are
    // covered exactly once by its kDownSplit CTAs, whose slice index matches
    if (kDownSplit * (H / kTileRows) <= grid) {
        const int ht = H / kTileRows, nb = FF / 32;
        std::vector<std::vector<int>> cover(ht, std::vector<int>(nb, 0));
        for (int cta = 0; cta < grid; cta++) {
            const TPlan p = dn_split_plan(ht, nb, tbb, cta, grid, slot, warps);
            const std::string where = "down split cta " + std::to_string(cta);
            if (p.n == 0) {
                if (dn_slice_of(cta, grid, ht) >= 0) fail(where + ": slice index without work");
                continue;
            }
            check_plan(p, p.kbn, tbb, slot, where);
            if (p.n != 1 || p.u0 < 0 || p.u0 >= ht) fail(where + ": not one residual tile");
            if (p.kb0 != dn_slice_of(cta, grid, ht) * nb / kDownSplit) fail(where + ": slice index mismatch");
            for (int b = p.kb0; b < p.kb0 + p.kbn; b++) {
                if (b < 0 || b >= nb) fail(where + ": block out of range");
                else cover[p.u0][b]++;
            }
        }
        for (int t = 0; t < ht; t++)
            for (int b = 0; b < nb; b++)
                if (cover[t][b] != 1) fail("down split: tile " + std::to_string(t) + " block " + std::to_string(b) +
                                           " covered " + std::to_string(cover[t][b]) + " times");
    }

    // QA phase: every split count the kernel can pick, fused and distributed forms
    const int tph = hd / kTileRows, qtiles = qd / kTileRows, kvtiles = 2 * kvd / kTileRows;
    for (int dist = 0; dist <= 1; dist++)
        for (int S = 1; S <= kMaxSplits && nh * S < grid; S++) {
            const std::string where = std::string(dist ? "qa dist" : "qa fused") + " S=" + std::to_string(S);
            std::vector<std::pair<int, int>> kv;
            for (int cta = 0; cta < grid; cta++) {
                int u0 = 0, n = 0;
                qa_tiles(nh, hd, qd, kvd, S, cta, grid, &u0, &n, dist);
                check_plan(tile_plan_range(u0, n, H / 32, tbb, slot, warps), H / 32, tbb, slot,
                           where + " cta " + std::to_string(cta));
                if (dist || cta >= nh * S) {
                    kv.push_back({u0, n});
                } else if (u0 != (cta / S) * tph || n != tph) {
                    fail(where + ": q CTA " + std::to_string(cta) + " does not hold its head's q tiles");
                }
            }
            if (dist) check_partition(kv, 0, qtiles + kvtiles, where);
            else check_partition(kv, qtiles, kvtiles, where);
        }

    if (!g_fail) std::printf("ok\n");
    return g_fail;
}

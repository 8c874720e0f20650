// Exhaustive host-side check of the cross-CTA schedule of a persistent trunk
// launch (alphazero_b200/csrc/trunk_schedule.cuh), over the geometries the
// two trunk kernels derive (conv_pix.cu: balanced 16-row ranges cut into
// tiles of at most 256 rows; conv_tc.cu: ranges of whole 128-row tiles).
//
// For every tile of every layer l >= 1 it checks, with the header's own
// functions:
//   - coverage: every row of layer l-1 the tile reads lies in a tile that
//     the waited-for counts include (so the TMA load sees finished rows);
//   - the reverse hazard: every tile of layer l-1 whose input rows include a
//     row this tile overwrites is included too;
//   - bounds: a target never asks for a tile of layer l or later;
// and, by simulating the CTAs publishing tiles in their own order, that the
// waits can always be met (no CTA set waits on itself in a cycle).
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../../alphazero_b200/csrc/trunk_schedule.cuh"

namespace {

struct Geom {
    int m_total, span, npx;
};

int fails = 0;

void check(bool ok, const char* what, const Geom& g, int halo, int l, int c, int q) {
    if (ok) return;
    if (++fails <= 20)
        std::printf("FAIL %s: m_total %d span %d npx %d halo %d layer %d cta %d q %d\n", what,
                    g.m_total, g.span, g.npx, halo, l, c, q);
}

// conv_pix.cu's launcher: balanced ranges of 16-row units, tiles of at most
// max_npx rows.
Geom pix_geom(int m_total, int grid_limit, int max_npx) {
    const int unit = 16;
    const int units = (m_total + unit - 1) / unit;
    int grid = units < grid_limit ? units : grid_limit;
    if (grid < 1) grid = 1;
    const int span = (units + grid - 1) / grid * unit;
    const int tiles = (span + max_npx - 1) / max_npx;
    const int npx = ((span + tiles - 1) / tiles + 15) / 16 * 16;
    return {m_total, span, npx};
}

// conv_tc.cu's launcher for several layers: whole 128-row tiles per CTA.
Geom tc_geom(int m_total, int grid_limit) {
    const int units = (m_total + 127) / 128;
    int grid = units < grid_limit ? units : grid_limit;
    if (grid < 1) grid = 1;
    const int upc = (units + grid - 1) / grid;
    return {m_total, upc * 128, 128};
}

void check_geometry(const Geom& g, int halo, int layers) {
    using mgb::cta_tiles;
    using mgb::input_rows;
    using mgb::order_of;
    using mgb::tile_at;
    using mgb::tile_rows;
    using mgb::wait_target;
    const int grid = (g.m_total + g.span - 1) / g.span;
    // The tiles partition the rows.
    std::vector<int> owner_tile(g.m_total, -1);
    for (int c = 0; c < grid; ++c)
        for (int j = 0; j < cta_tiles(g, c); ++j) {
            int m0, len;
            tile_rows(g, c, j, m0, len);
            check(len > 0 && m0 >= 0 && m0 + len <= g.m_total, "tile inside the tensor", g, halo, 0, c, j);
            for (int r = m0; r < m0 + len && r < g.m_total; ++r) {
                check(owner_tile[r] < 0, "rows owned once", g, halo, 0, c, j);
                owner_tile[r] = j;
            }
        }
    for (int r = 0; r < g.m_total; ++r) check(owner_tile[r] >= 0, "every row owned", g, halo, 0, r, 0);

    // Finished-tile count of layer l-1 that covers tile j of CTA c.
    auto done_count = [&](int c, int j, int l) {
        return (unsigned)((l - 1) * cta_tiles(g, c) + order_of(c, j, cta_tiles(g, c)) + 1);
    };
    for (int l = 1; l < layers; ++l)
        for (int c = 0; c < grid; ++c) {
            const int nt = cta_tiles(g, c);
            for (int q = 0; q < nt; ++q) {
                int m0, len, lo, hi;
                tile_rows(g, c, tile_at(c, q, nt), m0, len);
                input_rows(g, m0, len, halo, lo, hi);
                const int c0 = lo / g.span, c1 = hi / g.span;
                std::vector<unsigned> target(grid, 0);
                for (int cc = c0; cc <= c1; ++cc) {
                    target[cc] = wait_target(g, cc, lo, hi, l);
                    check(target[cc] <= (unsigned)(l * cta_tiles(g, cc)), "target within layer l-1", g,
                          halo, l, c, q);
                }
                // Coverage: every input row's producing tile is waited for.
                for (int r = lo; r <= hi; ++r) {
                    const int oc = r / g.span;
                    check(done_count(oc, owner_tile[r], l) <= target[oc], "input rows covered", g, halo,
                          l, c, q);
                }
                // Reverse hazard: tiles of layer l-1 that read any row this
                // tile writes are finished.  A reader's rows lie within halo
                // of ours, so its CTA is among those owning [lo, hi]; the
                // scan takes one more CTA on each side to show that.
                const int s0 = c0 > 0 ? c0 - 1 : 0, s1 = c1 + 1 < grid ? c1 + 1 : grid - 1;
                for (int oc = s0; oc <= s1; ++oc)
                    for (int j = 0; j < cta_tiles(g, oc); ++j) {
                        int a0, alen, alo, ahi;
                        tile_rows(g, oc, j, a0, alen);
                        input_rows(g, a0, alen, halo, alo, ahi);
                        const bool reads_ours = alo < m0 + len && ahi >= m0;
                        if (reads_ours)
                            check(oc >= c0 && oc <= c1 && done_count(oc, j, l) <= target[oc],
                                  "readers of overwritten rows finished", g, halo, l, c, q);
                    }
            }
        }

    // Progress: CTAs publish their tiles in order; a tile of layer l >= 1
    // starts once its targets are met.  Some CTA can always move.
    std::vector<unsigned> published(grid, 0);
    std::vector<int> next(grid, 0);  // next (layer * nt + q) of each CTA
    long remaining = 0;
    for (int c = 0; c < grid; ++c) remaining += (long)layers * cta_tiles(g, c);
    while (remaining > 0) {
        bool moved = false;
        for (int c = 0; c < grid; ++c) {
            const int nt = cta_tiles(g, c);
            if (nt == 0 || next[c] == layers * nt) continue;
            const int l = next[c] / nt, q = next[c] % nt;
            bool ready = true;
            if (l > 0) {
                int m0, len, lo, hi;
                tile_rows(g, c, tile_at(c, q, nt), m0, len);
                input_rows(g, m0, len, halo, lo, hi);
                for (int cc = lo / g.span; cc <= hi / g.span && ready; ++cc)
                    ready = published[cc] >= wait_target(g, cc, lo, hi, l);
            }
            if (ready) {
                ++published[c];
                ++next[c];
                --remaining;
                moved = true;
            }
        }
        if (!moved) {
            check(false, "progress (no CTA can move)", g, halo, -1, -1, -1);
            return;
        }
    }
}

}  // namespace

int main() {
    int cases = 0;
    // Boards 5, 9, 13, 19 (row stride RS = board + 1, frame IS = RS^2,
    // halo RS + 1), batches from 1 to 1024, launch limits from a few CTAs to
    // the B200's 148.
    const int boards[] = {5, 9, 13, 19};
    const int batches[] = {1, 2, 5, 16, 17, 64, 100, 256, 300, 512, 1024};
    const int grid_limits[] = {3, 7, 13, 64, 148};
    for (int board : boards)
        for (int n : batches)
            for (int gl : grid_limits) {
                const int rs = board + 1, is = rs * rs, halo = rs + 1, m_total = n * is;
                for (int max_npx : {256, 96, 64}) {
                    check_geometry(pix_geom(m_total, gl, max_npx), halo, 4);
                    ++cases;
                }
                check_geometry(tc_geom(m_total, gl), halo, 4);
                ++cases;
            }
    std::printf("%d geometries checked, %d failures\n", cases, fails);
    return fails == 0 ? 0 : 1;
}

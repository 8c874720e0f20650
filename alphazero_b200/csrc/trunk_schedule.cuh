// Work split and cross-CTA ordering of a persistent trunk launch (several
// 3x3 convolution layers in one cooperative launch), shared by the
// 128-channel kernel (conv_pix.cu) and the 64/256-channel kernel (conv_tc.cu).
//
// CTA c owns the rows [c * span, min((c + 1) * span, m_total)) in every
// layer, cut into tiles of npx rows (the last may be shorter).  Even CTAs
// take their tiles left to right, odd CTAs right to left.  A tile of layer l
// reads layer l-1's rows [m0 - halo, m0 + len + halo): the CTA's own
// neighbouring tiles and, at the ends of its range, the nearest tiles of
// the neighbouring CTAs.  After its epilogue has stored a tile, a CTA
// publishes its count of finished tiles (release, GPU scope); before loading
// a tile's input of layer l, the slab producer waits (acquire, bounded) until
// every CTA owning some of those rows has published the tiles of layer l-1
// that hold them.  The same wait covers the reverse hazard: a tile's outputs
// overwrite rows that only those tiles of the layer before read.  Because
// neighbouring CTAs run in opposite directions, the first tile of layer l
// needs only tiles that were among the first finished in layer l-1.
//
// The geometry type G has int fields m_total, span and npx.
#pragma once

#include "ptx_sm100.cuh"

namespace mgb {

// The index arithmetic below is host-callable too, so that the protocol can
// be checked exhaustively on the CPU (tests/cpp/test_trunk_schedule.cu).

// Number of tiles of CTA c (those of the last CTA may be fewer).
template <typename G>
__host__ __device__ __forceinline__ int cta_tiles(const G& g, int c) {
    const int start = c * g.span;
    const int end = start + g.span < g.m_total ? start + g.span : g.m_total;
    return end > start ? (end - start + g.npx - 1) / g.npx : 0;
}

// Rows [m0, m0 + len) of CTA c's tile j.
template <typename G>
__host__ __device__ __forceinline__ void tile_rows(const G& g, int c, int j, int& m0, int& len) {
    const int start = c * g.span;
    const int end = start + g.span < g.m_total ? start + g.span : g.m_total;
    m0 = start + j * g.npx;
    len = end - m0 < g.npx ? end - m0 : g.npx;
}

// The tile CTA c takes q-th in each layer, and the position of tile j in
// that order: even CTAs left to right, odd CTAs right to left.
__host__ __device__ __forceinline__ int tile_at(int c, int q, int nt) {
    return (c & 1) ? nt - 1 - q : q;
}
__host__ __device__ __forceinline__ int order_of(int c, int j, int nt) {
    return (c & 1) ? nt - 1 - j : j;
}

// Rows [lo, hi] (inclusive) of layer l-1's output that the tile [m0, m0 +
// len) of layer l reads: its own rows and `halo` rows on either side,
// clipped to the tensor.
template <typename G>
__host__ __device__ __forceinline__ void input_rows(const G& g, int m0, int len, int halo, int& lo,
                                                    int& hi) {
    lo = m0 - halo > 0 ? m0 - halo : 0;
    hi = (m0 + len + halo < g.m_total ? m0 + len + halo : g.m_total) - 1;
}

// The count of finished tiles CTA c (which owns some of rows [lo, hi]) must
// have published before a tile of layer l (>= 1) reads those rows: all its
// tiles of layers before l-1, and its tiles of layer l-1 up to the last one,
// in its order, that holds any of the rows.
template <typename G>
__host__ __device__ __forceinline__ unsigned wait_target(const G& g, int c, int lo, int hi, int l) {
    const int start = c * g.span;
    const int nt = cta_tiles(g, c);
    const int j0 = ((lo > start ? lo : start) - start) / g.npx;
    const int j1 = ((hi < start + g.span - 1 ? hi : start + g.span - 1) - start) / g.npx;
    const int last = (c & 1) ? order_of(c, j0, nt) : order_of(c, j1, nt);
    return (unsigned)((l - 1) * nt + last + 1);
}

// Before a tile of layer l (>= 1) reads rows [m0 - halo, m0 + len + halo)
// of layer l-1's output: waits until every CTA owning some of those rows has
// published the tiles that hold them.  False (with kErrWaitDep recorded in
// *err) if a wait gave up.
template <typename G>
__device__ __forceinline__ bool wait_inputs(const G& g, const unsigned* progress, int* err, int l,
                                            int m0, int len, int halo) {
    int lo, hi;
    input_rows(g, m0, len, halo, lo, hi);
    const int c0 = lo / g.span, n = hi / g.span - c0 + 1;
    auto target = [&](int c) { return wait_target(g, c, lo, hi, l); };
    constexpr int kPoll = 4;
    if (n > kPoll) {  // many small ranges: one acquire wait per CTA
        for (int c = c0; c < c0 + n; ++c)
            if (!wait_counter(&progress[c], target(c), err, kErrWaitDep)) return false;
        return true;
    }
    // Up to kPoll counters (the CTA's own and its neighbours'), polled
    // together with relaxed loads, all in flight at once; once every one has
    // reached its target, one fence makes the reads an acquire of each
    // (a strong read followed by fence.acq_rel).  Acquire loads one counter
    // after another took a round trip to L2 each.
    unsigned tgt[kPoll];
#pragma unroll
    for (int i = 0; i < kPoll; ++i) tgt[i] = i < n ? target(c0 + i) : 0u;
    const uint64_t t0 = global_timer_ns();
    for (int round = 0;; ++round) {
        unsigned v[kPoll];
#pragma unroll
        for (int i = 0; i < kPoll; ++i) v[i] = i < n ? ld_relaxed_gpu(&progress[c0 + i]) : 0u;
        bool all = true;
#pragma unroll
        for (int i = 0; i < kPoll; ++i) all = all && v[i] >= tgt[i];
        if (all) {
            fence_acq_rel_gpu();
            return true;
        }
        if ((round & 7) == 7 && global_timer_ns() - t0 > kWaitLimitNs) {
            atomicCAS(err, 0, kErrWaitDep);
            return false;
        }
    }
}

}  // namespace mgb

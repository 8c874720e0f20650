// 3x3 convolutions with 128 output channels as implicit GEMMs on the sm_100a
// tensor cores, pixels on the MMA's N side; one launch runs one layer or a
// whole run of trunk layers.
//
//   D[co][px] = sum_{cb, tap, k} W[co][tap][cb*64 + k] * X[px + off(tap)][cb*64 + k]
//
// A = weights (M = 128 output channels), B = pixels (N = up to 256 framed
// pixels per tile), K = 9 taps x input channels.  Per 64-channel block the
// producer loads ONE activation slab of N + 2*(RS+1) rows (the tile's rows
// plus a halo of one frame row and one pixel on each side) and every one of
// the 9 taps reads it through a descriptor whose start row is shifted by
// dy*RS + dx, so activations cross L2 -> SMEM once per block instead of
// nine times.  (The MMA derives the 128-byte swizzle phase from the absolute
// shared-memory address, as TMA does when it writes the slab, so a start
// address moved by whole 128-byte rows needs no descriptor base offset.)
// Weight K blocks (128 x 64) stream through a 4-deep ring.
//
// The accumulator is [co lanes][px columns] in TMEM, double-buffered across
// tiles (2 x 256 columns).  Each epilogue warp works on its own: it owns 32
// channels (its TMEM lanes) of every third 16-pixel chunk (lane = channel,
// so each 16-bit load of a warp covers 64 contiguous bytes of a pixel row).
// The residual stream is a pair of 16-bit planes, x = hi + lo with hi = x
// rounded to the operand type (the next layer's input) and lo = x - hi
// rounded to fp16.  A chunk's residual hi / lo values are loaded one chunk
// ahead into registers; each thread adds bias and residual, applies ReLU and
// the frame mask, and re-splits the sum into hi and lo.  The hi values go
// through one of the warp's two 1 KB shared-memory staging buffers and one
// TMA store per chunk; the lo values (16-pixel blocks, contiguous per warp)
// are stored from registers.  In the last trunk layer the fp32 sums go
// through shared memory to the policy / value 1x1 head projection instead.
//
// Warp roles (480 threads): warp 0 weight TMA producer, warp 1 TMEM
// allocator + MMA issuer, warps 2-13 epilogue (warp w reads TMEM lanes
// [32*(w%4), +32) of chunks (w-2)/4, (w-2)/4 + 3, ...; three warps per lane
// quarter hide more of each other's latency than two did), warp 14
// activation slab TMA producer (two slab buffers).  All waits are bounded.
//
// Work split: CTA b owns the contiguous pixel range [b*span, (b+1)*span) in
// every layer, cut into equal tiles of at most 256 pixels, so every SM gets
// the same number of pixels.  Even CTAs take their tiles left to right, odd
// CTAs right to left.
//
// Several layers in one launch (a cooperative launch, so every CTA is
// resident): a tile of layer l reads layer l-1's rows [m0 - RS - 1, m0 + len
// + RS + 1), i.e. the CTA's own neighbouring tiles and, at the ends of its
// range, the nearest tiles of the neighbouring CTAs.  After all 12 epilogue
// warps have stored a tile, the CTA publishes its count of finished tiles
// (release, GPU scope); the slab producer waits until the tiles it needs
// are counted (relaxed polls of every counter it needs, then one acquire
// fence) before loading a slab.  The same wait covers the
// reverse hazard: a tile's outputs overwrite rows that only those tiles of
// the layer before read.  Because neighbouring CTAs run in opposite
// directions, the first tile of layer l needs only tiles that were among the
// first finished in layer l-1, so the MMA moves on to layer l while the
// epilogue finishes layer l-1.  Single-layer launches are ordinary
// programmatic dependent launches: a CTA's prologue overlaps the previous
// kernel's tail.
#include "kernels.cuh"
#include "ptx_sm100.cuh"
#include "trunk_schedule.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

namespace mgb {
namespace {

constexpr int kCo = 128;        // output channels (MMA M)
constexpr int kBK = 64;         // K per stage / slab channel block
constexpr int kMaxPx = 256;     // MMA N limit
// Weight ring depth, measured: 4 beats 3 and every deeper ring.  With the
// ring index advanced incrementally (no division) and the head layer's
// slots aliased onto the store staging, 5, 6 and 8 stages ran the 19x19
// batch-512 trunk in 1040, 1045 and 1094 us against 1015 us, and the 9x9
// batch-256 trunk in 254, 256 and 260 us against 252 us, though a stage's
// round trip (about 1 us from its TMA load to the commit that frees it)
// bounds a ring of 4 near the MMA's rate.  Weight loads further ahead take
// L2 bandwidth from the slab and residual loads that the layer waits on.
constexpr int kStages = 4;
constexpr int kSlabs = 2;       // activation slab ring depth
constexpr int kEpiWarps = 12;   // epilogue warps: kPar per TMEM lane quarter
constexpr int kPar = kEpiWarps / 4;
constexpr int kThreads = 32 * (3 + kEpiWarps);
constexpr int kChunk = 16;      // pixels per epilogue chunk
constexpr uint32_t kWBytes = kCo * kBK * 2;            // 16 KB weight stage
constexpr int kSlot = kChunk * 32;  // one warp's chunk: 16 pixels x 32 channels
constexpr int kMagicShift = 40;     // n / d == (n * ceil(2^40 / d)) >> 40 here
constexpr int kMaxLayers = 44;      // layers per launch (kernel parameter space)
constexpr int kMaxBufs = 4;         // TMEM accumulator buffers (512 columns / tile width)

// One layer of a launch.
struct PixLayer {
    const float* bias;       // [128]
    const uint16_t* res_hi;  // residual stream [m_total][128] hi plane, or nullptr
    const uint16_t* res_lo;  // and its fp16 remainder plane (16-pixel blocks, see lo_block)
    uint16_t* out16;         // output [m_total][128] (hi plane), or nullptr
    uint16_t* out_lo;        // its fp16 remainder plane (16-pixel blocks), or nullptr
    int cin;                 // 64 or 128
    int xmap;                // activation tensor map of the input slabs (0..2)
    int wmap;                // weight tensor map (0 or 1)
    int wrow;                // first row of this layer's weights in that map
    int head;                // fused head projection (last trunk layer)
    int omap;                // tensor map of out16 (0 or 1) for the epilogue's TMA stores
};
static_assert(sizeof(PixLayer) == 64, "PixLayer layout");

struct PixArgs {
    int m_total;
    int span;           // pixels per CTA (multiple of 16): CTA b owns [b*span, (b+1)*span)
    int tiles_per_cta;  // tiles a full range is cut into
    int npx;            // pixels per tile (multiple of 16, <= 256; the last tile may be shorter)
    int rs, is, board;
    int slab_rows;                // rows per slab (multiple of 16)
    int nbuf;                     // TMEM accumulator buffers, npx columns each
    uint64_t is_magic, rs_magic;  // ceil(2^40 / is), ceil(2^40 / rs)
    int n_layers;
    int own_frames;      // 1: CTA ranges are whole frames; a tile waits only on its own CTA
    int* err;
    unsigned* progress;  // [grid] tiles finished per CTA (several layers), else nullptr
    int withhold_cta;    // test hook: this CTA never publishes its progress (-1: none)
    const float* head_w;  // [3][128] or nullptr (fused head projection)
    const float* head_b;
    float* feat;
    PixLayer layer[kMaxLayers];
};

// The launch geometry, copied out of the parameters once: kept in registers,
// it is not re-read after every store the way fields reached through a
// reference to the parameter block can be.
struct Geo {
    int m_total, span, npx, rs, is, board, nbuf;
    uint64_t is_magic, rs_magic;
};

// The rows of the previous layer a tile reads, as wait_inputs takes them.
// With CTA ranges of whole frames (own_frames), only the CTA's own rows: the
// halo rows past either end of its range are either zero padding rows of a
// neighbouring frame (the frame stride is padded to whole 16-row chunks, and
// every layer writes frame rows as zero) or inputs of frame pixels, whose
// outputs are masked to zero whatever they read.
__device__ __forceinline__ bool wait_tile_inputs(const Geo& G, const PixArgs& a, int l, int m0,
                                                 int len, int halo) {
    if (!a.own_frames) return wait_inputs(G, a.progress, a.err, l, m0, len, halo);
    // Tiles of whole frames read no other tile's rows at all.
    if (G.npx % G.is == 0) halo = 0;
    const int start = blockIdx.x * G.span;
    const int end = min(start + G.span, G.m_total);
    const int lo = max(m0 - halo, start), hi = min(m0 + len + halo, end);
    return wait_inputs(G, a.progress, a.err, l, lo, hi - lo, 0);
}

__device__ __forceinline__ Geo geo_of(const PixArgs& a) {
    Geo g;
    g.m_total = a.m_total;
    g.span = a.span;
    g.npx = a.npx;
    g.rs = a.rs;
    g.is = a.is;
    g.board = a.board;
    g.nbuf = a.nbuf;
    g.is_magic = a.is_magic;
    g.rs_magic = a.rs_magic;
    return g;
}

template <bool FP16>
__device__ __forceinline__ float from16(uint16_t h);
template <>
__device__ __forceinline__ float from16<false>(uint16_t h) {
    return __uint_as_float((uint32_t)h << 16);
}
template <>
__device__ __forceinline__ float from16<true>(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}
// Two values rounded in one conversion; the first in the low half.
template <bool FP16>
__device__ __forceinline__ uint32_t to16x2(float a, float b);
template <>
__device__ __forceinline__ uint32_t to16x2<false>(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t to16x2<true>(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t lo_bits2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float lo_value(uint16_t l) { return __half2float(__ushort_as_half(l)); }

// The lo plane is read and written only by the epilogue, one channel per
// lane and 16 pixels at a time, so it is stored in 16-pixel blocks:
// element (pixel px, channel c) at (px / 16) * 16 * 128 + c * 16 + px % 16.
// A lane's 16 values of a chunk are then 32 contiguous bytes (two 16-byte
// accesses instead of sixteen 2-byte ones).  Chunks start at multiples of
// 16 pixels; the plane holds whole blocks (rows rounded up to 16).
__device__ __forceinline__ size_t lo_block(int px0, int co) {
    return (size_t)(px0 >> 4) * (16 * kCo) + (size_t)co * 16;
}

// n / d for 0 <= n < 2^23 and d <= 1200 (the launcher checks both).
__device__ __forceinline__ int div_magic(int n, uint64_t magic) {
    return (int)(((uint64_t)(uint32_t)n * magic) >> kMagicShift);
}

// One layer of the epilogue for one warp (see the kernel's epilogue): t
// counts the CTA's tiles so far.  Returns false when a wait gave up.
template <bool FP16, bool HEAD>
__device__ __forceinline__ bool epilogue_layer(const PixArgs& a, const Geo G, int l, int nt, int& t,
                                               uint64_t* tfull, uint64_t* tempty, uint32_t* tcount,
                                               uint32_t tmem_base, float* hslot, const float* shead,
                                               uint16_t* ostage, int& sc, const CUtensorMap* omap,
                                               int warp, int lane) {
    const int quarter = warp & 3;  // channels [32*quarter, +32)
    const int ew = warp - 2;       // 0..kEpiWarps-1
    const int par = ew >> 2;       // chunks par, par+kPar, ...
    const int co = quarter * 32 + lane;
    const int hw = G.board * G.board;
    int* const err = a.err;
    unsigned* const progress = a.progress;
    float* const feat = a.feat;
    const float* const head_b = a.head_b;
    float* slot = hslot + ew * kSlot;  // head layer: this warp's fp32 sums [16][32]
    // This warp's two staging buffers for the hi plane, [16 pixels][32
    // channels] each: lane = channel writes them, and one TMA store per chunk
    // moves the 16 x 64-byte block to global memory, so the output bypasses
    // the load/store unit.  Buffer sc & 1 is written only once the store
    // issued from it two chunks earlier has read it.
    uint16_t* const ost = ostage + ew * (2 * kSlot);
    const int bar_a = 2 + 2 * par, bar_b = 3 + 2 * par;  // head layer only
    bool ok = true;
    // The layer's parameters in registers (read once, not after every
    // store or wait).
    const uint16_t* const res_hi = a.layer[l].res_hi;
    const uint16_t* const res_lo = a.layer[l].res_lo;
    uint16_t* const out_lo = a.layer[l].out_lo;
    const float bias = a.layer[l].bias[co];
    const bool has_res = res_hi != nullptr;
    const bool has_lo = out_lo != nullptr;
    // Residual of the next chunk (tile order position lq, chunk lc),
    // loaded one chunk ahead into registers.
    uint16_t nh[kChunk];
    uint4 nl0, nl1;  // lo values of pixels 0-7 and 8-15, two per word
    auto load_res = [&](int px) {
        const uint16_t* ph = res_hi + (size_t)px * kCo + co;
        const uint16_t* pl = res_lo + lo_block(px, co);
        nl0 = ld_cg_v4_early(pl);
        nl1 = ld_cg_v4_early(pl + 8);
        if (px + kChunk <= G.m_total) {
#pragma unroll
            for (int j = 0; j < kChunk; ++j) nh[j] = ld_cg_u16_early(ph + j * kCo);
        } else {
#pragma unroll
            for (int j = 0; j < kChunk; ++j)
                nh[j] = px + j < G.m_total ? ld_cg_u16_early(ph + j * kCo) : (uint16_t)0;
        }
    };
    // Advances (lq, lc) to this warp's next chunk of the layer.
    auto next_chunk = [&](int& lq, int& lc) {
        lc += kPar;
        while (lq < nt) {
            int m, n;
            tile_rows(G, blockIdx.x, tile_at(blockIdx.x, lq, nt), m, n);
            if (lc * kChunk < n) return true;
            ++lq;
            lc = par;
        }
        return false;
    };
    int lq = 0, lc = par - kPar;
    bool lvalid = next_chunk(lq, lc);
    if (has_res && lvalid) {
        int m, n;
        tile_rows(G, blockIdx.x, tile_at(blockIdx.x, lq, nt), m, n);
        load_res(m + lc * kChunk);
        lvalid = next_chunk(lq, lc);
    }
    for (int q = 0; q < nt && ok; ++q, ++t) {
        int m0, len;
        tile_rows(G, blockIdx.x, tile_at(blockIdx.x, q, nt), m0, len);
        const int nchunks = (len + kChunk - 1) / kChunk;
        const int acc = t % G.nbuf;
        const int use = t / G.nbuf;  // earlier tiles of this accumulator buffer
        ok = mbar_wait(smem_u32(&tfull[acc]), use & 1, err, kErrWaitEpilogue);
        if (HEAD ? bar_any(bar_a, 128, !ok) : __any_sync(0xffffffffu, !ok)) {
            ok = false;
            break;
        }
        tc_fence_after();
        const uint32_t tcol =
            tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * G.npx);
#pragma unroll 1
        for (int c = par; c < nchunks; c += kPar) {
            const int px0 = m0 + c * kChunk;
            uint32_t v[16];
            tmem_ld_16cols(tcol + (uint32_t)(c * kChunk), v);
            float f[16];
            if (has_res) {
                const uint32_t lw[8] = {nl0.x, nl0.y, nl0.z, nl0.w, nl1.x, nl1.y, nl1.z, nl1.w};
#pragma unroll
                for (int j = 0; j < kChunk; ++j)
                    f[j] = from16<FP16>(nh[j]) +
                           lo_value((uint16_t)(lw[j >> 1] >> (16 * (j & 1))));
                if (lvalid) {  // next chunk's residual, in flight during this one
                    int m1, len1;
                    tile_rows(G, blockIdx.x, tile_at(blockIdx.x, lq, nt), m1, len1);
                    load_res(m1 + lc * kChunk);
                    lvalid = next_chunk(lq, lc);
                }
            } else {
#pragma unroll
                for (int j = 0; j < kChunk; ++j) f[j] = 0.f;
            }
            // lanes 0..15 classify pixels px0 + lane
            bool onb = false;
            if (c * kChunk + (lane & 15) < len) {
                const int mj = px0 + (lane & 15);
                const int qq = mj - div_magic(mj, G.is_magic) * G.is;
                const int y = div_magic(qq, G.rs_magic);
                onb = (y < G.board) && (qq - y * G.rs < G.board);
            }
            const uint32_t board_mask = __ballot_sync(0xffffffffu, onb) & 0xffffu;
            tmem_ld_wait(v);
#pragma unroll
            for (int j = 0; j < kChunk; ++j) {
                const float x = __uint_as_float(v[j]) + bias + f[j];
                f[j] = ((board_mask >> j) & 1) ? fmaxf(x, 0.f) : 0.f;
            }
            if (!HEAD) {
                uint16_t* const sb = ost + (sc & 1) * kSlot;
                if (lane == 0) bulk_wait_read_n<1>();  // the store from sb two chunks ago has read it
                __syncwarp();
                uint32_t lw[8];
#pragma unroll
                for (int j = 0; j < kChunk; j += 2) {
                    // two pixels per conversion: hi pair, then lo pair
                    const uint32_t hp = to16x2<FP16>(f[j], f[j + 1]);
                    const uint16_t h0 = (uint16_t)(hp & 0xffffu), h1 = (uint16_t)(hp >> 16);
                    sb[j * 32 + lane] = h0;
                    sb[(j + 1) * 32 + lane] = h1;
                    // rows past the end (f = 0) fill the last block
                    lw[j >> 1] = lo_bits2(f[j] - from16<FP16>(h0), f[j + 1] - from16<FP16>(h1));
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    // rows past the tensor's end are not written
                    tma_store_2d(omap, smem_u32(sb), quarter * 32, px0);
                    bulk_commit();
                }
                ++sc;
                if (has_lo) {
                    uint4* ol = reinterpret_cast<uint4*>(out_lo + lo_block(px0, co));
                    ol[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                    ol[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
                }
            } else {
                // Policy / value 1x1 convs of the chunk's 16 pixels:
                // thread (pixel g/8, channel segment g%8) of the group
                // sums 16 channels, which sit in the slot of the warp
                // owning that channel quarter; the 8 segments of a
                // pixel combine by shuffles.  The first barrier keeps
                // the slots from being rewritten while the previous
                // chunk's sums still read them.
                named_barrier_sync(bar_b, 128);
#pragma unroll
                for (int j = 0; j < kChunk; ++j) slot[j * 32 + lane] = f[j];
                named_barrier_sync(bar_a, 128);
                const int g = ((warp - 2) & 3) * 32 + lane;
                const int p = g >> 3, seg = g & 7, sq = seg >> 1;
                const float* row =
                    hslot + (par * 4 + ((sq + 2) & 3)) * kSlot + p * 32 + (seg & 1) * 16;
                const float* hw0 = shead + seg * 16;
                float d0 = 0.f, d1 = 0.f, d2 = 0.f;
#pragma unroll 4
                for (int k = 0; k < 16; ++k) {
                    const int kq = (k + 4 * sq + (p & 3)) & 15;  // spread banks
                    const float xv = row[kq];
                    d0 = fmaf(xv, hw0[kq], d0);
                    d1 = fmaf(xv, hw0[kCo + kq], d1);
                    d2 = fmaf(xv, hw0[2 * kCo + kq], d2);
                }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) {
                    d0 += __shfl_xor_sync(0xffffffffu, d0, o);
                    d1 += __shfl_xor_sync(0xffffffffu, d1, o);
                    d2 += __shfl_xor_sync(0xffffffffu, d2, o);
                }
                if (seg == 0 && ((board_mask >> p) & 1)) {
                    const int mp = px0 + p;
                    const int pos = div_magic(mp, G.is_magic);
                    const int qq = mp - pos * G.is;
                    const int y = div_magic(qq, G.rs_magic), x = qq - y * G.rs;
                    float* fr = feat + (size_t)pos * 3 * hw + y * G.board + x;
                    fr[0] = fmaxf(d0 + head_b[0], 0.f);
                    fr[hw] = fmaxf(d1 + head_b[1], 0.f);
                    fr[2 * hw] = fmaxf(d2 + head_b[2], 0.f);
                }
            }
        }
        // The accumulator has been read: hand it back to the MMA warp first.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
        if (!HEAD && lane == 0) {
            // this warp's TMA stores of the tile have landed in global memory
            bulk_wait_all();
            fence_proxy_async_global();
        }
        if (progress != nullptr) {
            // This warp's stores of the tile are done (the warp barrier
            // orders every lane's stores before lane 0's release).  The
            // epilogue warps count themselves in at CTA scope; the last one,
            // whose acquire sees the others' stores, publishes the CTA's
            // count of finished tiles with a GPU-scope release.  Causality
            // order is transitive, so that release covers every warp's
            // stores: no full fence is needed (one before it cost 0.5 us per
            // tile, measured; a full fence in every warp stalled the
            // epilogue).
            __syncwarp();
            if (lane == 0) {
                const unsigned before = atom_add_acq_rel_cta(smem_u32(&tcount[acc]), 1u);
                if (before == (unsigned)(kEpiWarps * use + kEpiWarps - 1) &&
                    (int)blockIdx.x != a.withhold_cta) {
                    fence_proxy_async_global();
                    red_max_release_gpu(&progress[blockIdx.x], (unsigned)(l * nt + q + 1));
                }
            }
        }
        __syncwarp();
    }
    return ok;
}

// The head-projection layer's epilogue kept out of line: inlined next to
// the other layers' epilogue it made the compiler schedule that hot loop
// worse (measured: the residual layers' epilogue 20% slower).
template <bool FP16>
__device__ __noinline__ bool epilogue_head_layer(const PixArgs& a, const Geo G, int l, int nt,
                                                 int& t, uint64_t* tfull, uint64_t* tempty,
                                                 uint32_t* tcount, uint32_t tmem_base, float* hslot,
                                                 const float* shead, uint16_t* ostage, int& sc,
                                                 const CUtensorMap* omap, int warp, int lane) {
    return epilogue_layer<FP16, true>(a, G, l, nt, t, tfull, tempty, tcount, tmem_base, hslot,
                                      shead, ostage, sc, omap, warp, lane);
}

template <bool FP16>
__global__ void __launch_bounds__(kThreads, 1)
    conv3x3_pix_kernel(const __grid_constant__ CUtensorMap tmW0,
                       const __grid_constant__ CUtensorMap tmW1,
                       const __grid_constant__ CUtensorMap tmX0,
                       const __grid_constant__ CUtensorMap tmX1,
                       const __grid_constant__ CUtensorMap tmX2,
                       const __grid_constant__ CUtensorMap tmO0,
                       const __grid_constant__ CUtensorMap tmO1, const __grid_constant__ PixArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t slab_bytes = (uint32_t)a.slab_rows * 128u;
    uint8_t* wring = smem;                                   // kStages x 16 KB
    uint8_t* slab0 = wring + kStages * kWBytes;              // kSlabs slabs
    float* hslot = reinterpret_cast<float*>(slab0 + kSlabs * slab_bytes);  // [kEpiWarps][16][32]
    uint16_t* ostage = reinterpret_cast<uint16_t*>(hslot + kEpiWarps * kSlot);  // [kEpiWarps][2][16][32]
    uint64_t* bars = reinterpret_cast<uint64_t*>(ostage + kEpiWarps * 2 * kSlot);
    uint64_t* wfull = bars;
    uint64_t* wempty = bars + kStages;
    uint64_t* sfull = bars + 2 * kStages;
    uint64_t* sempty = sfull + kSlabs;
    uint64_t* tfull = sempty + kSlabs;
    uint64_t* tempty = tfull + kMaxBufs;
    uint64_t* done = tempty + kMaxBufs;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    uint32_t* tcount = tmem_slot + 1;  // [kMaxBufs] epilogue warps done, per buffer
    float* shead = reinterpret_cast<float*>(tmem_slot + 8);  // [3][128]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const Geo G = geo_of(a);
    int* const err = a.err;
    const int nt = cta_tiles(G, blockIdx.x);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&wfull[s]), 1);
            mbar_init(smem_u32(&wempty[s]), 1);
        }
        for (int i = 0; i < kSlabs; ++i) {
            mbar_init(smem_u32(&sfull[i]), 1);
            mbar_init(smem_u32(&sempty[i]), 1);
        }
        for (int i = 0; i < kMaxBufs; ++i) {
            mbar_init(smem_u32(&tfull[i]), 1);
            mbar_init(smem_u32(&tempty[i]), kEpiWarps);
            tcount[i] = 0;
        }
        mbar_init(smem_u32(done), 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), 512);
        tmem_relinquish();
    }
    if (a.head_w != nullptr)
        for (int i = threadIdx.x; i < 3 * kCo; i += kThreads) shead[i] = a.head_w[i];
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Everything above touches only this CTA's resources and the launch's
    // constant parameters.  Activations written by the previous kernel are
    // read, and activations it may still read are overwritten, only after
    // it has completed.
    griddep_launch_dependents();
    griddep_wait();

    const int halo = G.rs + 1;
    const int half_rows = a.slab_rows / 2;

    if (warp == 0) {
        // ---------------- weight producer ----------------
        if (lane == 0) {
            prefetch_tensormap(&tmW0);
            prefetch_tensormap(&tmW1);
            int iw = 0;
            bool ok = true;
            for (int l = 0; l < a.n_layers && ok; ++l) {
                const int cin = a.layer[l].cin, wrow = a.layer[l].wrow;
                const CUtensorMap* map = a.layer[l].wmap ? &tmW1 : &tmW0;
                for (int q = 0; q < nt && ok; ++q) {
                    for (int cb = 0; cb < cin / kBK && ok; ++cb) {
                        for (int tap = 0; tap < 9; ++tap, ++iw) {
                            const int s = iw % kStages;
                            if (!mbar_wait(smem_u32(&wempty[s]), ((iw / kStages) & 1) ^ 1, err,
                                           kErrWaitProducer)) {
                                ok = false;
                                break;
                            }
                            const uint32_t wfb = smem_u32(&wfull[s]);
                            mbar_arrive_expect_tx(wfb, kWBytes);
                            tma_load_2d(smem_u32(wring + s * kWBytes), map, wfb, tap * cin + cb * kBK,
                                        wrow);
                        }
                    }
                }
            }
            // Drain every copy still in flight before the CTA exits.
            for (int j = (iw > kStages ? iw - kStages : 0); j < iw; ++j)
                mbar_wait(smem_u32(&wfull[j % kStages]), (j / kStages) & 1, err, kErrWaitDrain);
        }
        __syncwarp();
    } else if (warp == 2 + kEpiWarps) {
        // ---------------- activation slab producer ----------------
        // Separate from the weight producer so a slab load is issued as soon
        // as a slab buffer frees up, not behind the weight ring's waits.
        if (lane == 0) {
            prefetch_tensormap(&tmX0);
            prefetch_tensormap(&tmX1);
            prefetch_tensormap(&tmX2);
            int is = 0;
            bool ok = true;
            for (int l = 0; l < a.n_layers && ok; ++l) {
                const int cin = a.layer[l].cin, xmap = a.layer[l].xmap;
                const CUtensorMap* map = xmap == 0 ? &tmX0 : (xmap == 1 ? &tmX1 : &tmX2);
                for (int q = 0; q < nt && ok; ++q) {
                    int m0, len;
                    tile_rows(G, blockIdx.x, tile_at(blockIdx.x, q, nt), m0, len);
                    if (l > 0 && a.progress != nullptr) {
                        if (!wait_tile_inputs(G, a, l, m0, len, halo)) {
                            ok = false;
                            break;
                        }
                        // the rows were written through the generic proxy
                        fence_proxy_async_global();
                    }
                    for (int cb = 0; cb < cin / kBK; ++cb, ++is) {
                        const int sb = is % kSlabs;
                        if (!mbar_wait(smem_u32(&sempty[sb]), ((is / kSlabs) & 1) ^ 1, err,
                                       kErrWaitProducer)) {
                            ok = false;
                            break;
                        }
                        const uint32_t sfb = smem_u32(&sfull[sb]);
                        uint8_t* slab = slab0 + sb * slab_bytes;
                        mbar_arrive_expect_tx(sfb, slab_bytes);
                        tma_load_2d(smem_u32(slab), map, sfb, cb * kBK, m0 - halo);
                        tma_load_2d(smem_u32(slab + half_rows * 128), map, sfb, cb * kBK,
                                    m0 - halo + half_rows);
                    }
                }
            }
            for (int j = (is > kSlabs ? is - kSlabs : 0); j < is; ++j)
                mbar_wait(smem_u32(&sfull[j % kSlabs]), (j / kSlabs) & 1, err, kErrWaitDrain);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int iw = 0, is = 0, t = 0;
            bool ok = true;
            for (int l = 0; l < a.n_layers && ok; ++l) {
                const int cblocks = a.layer[l].cin / kBK;
                for (int q = 0; q < nt && ok; ++q, ++t) {
                    int m0, len;
                    tile_rows(G, blockIdx.x, tile_at(blockIdx.x, q, nt), m0, len);
                    // MMA N = the tile's pixels rounded up to 16
                    const uint32_t idesc = idesc_f16(kCo, (len + 15) & ~15, !FP16);
                    const int acc = t % G.nbuf;
                    if (!mbar_wait(smem_u32(&tempty[acc]), ((t / G.nbuf) & 1) ^ 1, err, kErrWaitMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(acc * G.npx);
                    for (int cb = 0; cb < cblocks && ok; ++cb, ++is) {
                        const int sb = is % kSlabs;
                        if (!mbar_wait(smem_u32(&sfull[sb]), (is / kSlabs) & 1, err, kErrWaitMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        // Descriptor of the slab's first row; a row-shifted
                        // start (base offset 0, see file comment) adds its
                        // byte offset / 16 to the address field, which cannot
                        // carry out since every start lies inside shared memory.
                        const uint64_t bd0 = smem_desc_sw128(smem_u32(slab0 + sb * slab_bytes));
                        // A compile-time trip count keeps the issue loop free
                        // of per-tap index arithmetic (measured: 4-5 % on the
                        // whole layer, the MMA queue otherwise runs dry).
#pragma unroll
                        for (int tap = 0; tap < 9; ++tap, ++iw) {
                            const int s = iw % kStages;
                            if (!mbar_wait(smem_u32(&wfull[s]), (iw / kStages) & 1, err,
                                           kErrWaitMma)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const int r0 = halo + (tap / 3 - 1) * G.rs + (tap % 3 - 1);
                            const uint64_t ad = smem_desc_sw128(smem_u32(wring + s * kWBytes));
                            const uint64_t bd = bd0 + (uint64_t)(r0 * 8);  // r0 * 128 B / 16
#pragma unroll
                            for (int kk = 0; kk < kBK / 16; ++kk)
                                mma_f16(d, ad + (uint64_t)(2 * kk), bd + (uint64_t)(2 * kk), idesc,
                                        (cb | tap | kk) != 0);
                            mma_commit(smem_u32(&wempty[s]));
                        }
                        if (ok) mma_commit(smem_u32(&sempty[sb]));
                    }
                    if (ok) mma_commit(smem_u32(&tfull[acc]));
                }
            }
            mma_commit(smem_u32(done));
            mbar_wait(smem_u32(done), 0, err, kErrWaitDrain);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        // Each warp finishes its 32 channels (its TMEM lanes) of every third
        // chunk on its own, straight between registers and global memory.
        // Only the head-projection layer, which sums over all 128 channels,
        // couples the warps (through shared memory).
        int t = 0, sc = 0;
        bool ok = true;
        if (lane == 0) {
            prefetch_tensormap(&tmO0);
            prefetch_tensormap(&tmO1);
        }
        for (int l = 0; l < a.n_layers && ok; ++l) {
            const CUtensorMap* omap = a.layer[l].omap ? &tmO1 : &tmO0;
            ok = a.layer[l].head != 0
                     ? epilogue_head_layer<FP16>(a, G, l, nt, t, tfull, tempty, tcount, tmem_base,
                                                  hslot, shead, ostage, sc, omap, warp, lane)
                     : epilogue_layer<FP16, false>(a, G, l, nt, t, tfull, tempty, tcount, tmem_base,
                                                   hslot, shead, ostage, sc, omap, warp, lane);
        }
        // every TMA store has landed before the CTA exits
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
    }
}

int slab_rows_for(int npx, int rs) {
    const int need = npx + 2 * (rs + 1);
    return (need + 15) / 16 * 16;
}

size_t pix_smem_bytes(int npx, int rs) {
    const size_t slab = (size_t)slab_rows_for(npx, rs) * 128;
    return (size_t)kStages * kWBytes + kSlabs * slab + (size_t)kEpiWarps * kSlot * (4 + 2 * 2) +
           (2 * kStages + 2 * kSlabs + 2 * kMaxBufs + 1) * 8 + 32 + 3 * kCo * 4 + 1024;
}

// 2-D tensor map [rows][inner] of `esize`-byte elements.
bool encode(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
            uint64_t rows, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    return encode_tiled_2d(map, dt, esize, base, inner, rows, box_inner, box_rows, sw);
}

bool layer_ok(const ConvLayer& L, const ConvLayer& first) {
    // The residual stream is the hi / lo pair; fp32 residuals are not read.
    return L.cout == kCo && (L.cin == 64 || L.cin == 128) && L.m_total == first.m_total &&
           L.g.rs == first.g.rs && L.res32 == nullptr && L.out32 == nullptr &&
           (L.res_hi == nullptr) == (L.res_lo == nullptr) &&
           (L.out_lo == nullptr || L.out16 != nullptr) &&
           (L.head_w != nullptr || L.out16 != nullptr) && L.g.is <= 1200 &&
           L.m_total < (1 << 23) - 2 * kMaxPx;
}

// Launches layers[0..n) (n <= kMaxLayers) as one kernel.  Layer 0 may have
// any supported cin; layers 1.. must have cin 128 and weights laid out back
// to back from layers[1].weight.  With several layers, progress must point
// at grid_limit counters.
// Whether CTA ranges can be whole frames: frames of whole 16-row chunks that
// fit one tile.
bool frames_fit(const FrameGeom& g, int m_total) {
    return g.is % kChunk == 0 && g.is <= kMaxPx && m_total % g.is == 0;
}

cudaError_t launch_layers(const ConvLayer* layers, int n, int max_npx, bool fp16, int grid_limit,
                          unsigned* progress, cudaStream_t stream, int withhold_cta = -1,
                          bool own_frames = false) {
    if (n < 1 || n > kMaxLayers || (n > 1 && progress == nullptr)) return cudaErrorInvalidValue;
    const ConvLayer& F = layers[0];
    if (own_frames && !frames_fit(F.g, F.m_total)) return cudaErrorInvalidValue;
    // Balanced ranges: each CTA takes span pixels (a multiple of 16, or of
    // whole frames) cut into equal tiles of at most max_npx.
    const int unit = own_frames ? F.g.is : 16;
    const int units = (F.m_total + unit - 1) / unit;
    int grid = units < grid_limit ? units : grid_limit;
    if (grid < 1) grid = 1;
    const int span = (units + grid - 1) / grid * unit;
    grid = (F.m_total + span - 1) / span;
    const int tiles = (span + max_npx - 1) / max_npx;
    const int npx = ((span + tiles - 1) / tiles + 15) / 16 * 16;
    if (npx % kChunk != 0 || npx < 16 || npx > kMaxPx ||
        pix_smem_bytes(npx, F.g.rs) > 227 * 1024)
        return cudaErrorInvalidValue;
    PixArgs a;
    a.m_total = F.m_total;
    a.span = span;
    a.tiles_per_cta = tiles;
    a.npx = npx;
    a.rs = F.g.rs;
    a.is = F.g.is;
    a.board = F.g.board;
    a.slab_rows = slab_rows_for(npx, F.g.rs);
    a.nbuf = 512 / npx < kMaxBufs ? 512 / npx : kMaxBufs;
    a.is_magic = ((1ull << kMagicShift) + (uint64_t)F.g.is - 1) / (uint64_t)F.g.is;
    a.rs_magic = ((1ull << kMagicShift) + (uint64_t)F.g.rs - 1) / (uint64_t)F.g.rs;
    a.n_layers = n;
    a.own_frames = own_frames ? 1 : 0;
    a.err = F.err;
    a.progress = n > 1 ? progress : nullptr;
    a.withhold_cta = n > 1 ? withhold_cta : -1;
    a.head_w = nullptr;
    a.head_b = nullptr;
    a.feat = nullptr;
    // Up to three distinct input buffers, each with its own tensor map, and
    // up to two distinct 16-bit output buffers (the epilogue's TMA stores).
    const void* xin[3] = {nullptr, nullptr, nullptr};
    int xcin[3] = {0, 0, 0};
    int nx = 0;
    const void* oout[2] = {nullptr, nullptr};
    int no = 0;
    const size_t wstride = (size_t)kCo * 9 * 128;  // elements per cin-128 layer
    for (int l = 0; l < n; ++l) {
        const ConvLayer& L = layers[l];
        if (!layer_ok(L, F)) return cudaErrorInvalidValue;
        if (L.head_w != nullptr && l != n - 1) return cudaErrorInvalidValue;
        PixLayer& P = a.layer[l];
        P = PixLayer{};
        P.bias = L.bias;
        P.res_hi = static_cast<const uint16_t*>(L.res_hi);
        P.res_lo = L.res_lo;
        P.out16 = static_cast<uint16_t*>(L.out16);
        P.out_lo = L.out_lo;
        P.cin = L.cin;
        int xm = 0;
        while (xm < nx && xin[xm] != L.in) ++xm;
        if (xm == nx) {
            if (nx == 3) return cudaErrorInvalidValue;
            xin[nx] = L.in;
            xcin[nx] = L.cin;
            ++nx;
        } else if (xcin[xm] != L.cin) {
            return cudaErrorInvalidValue;
        }
        P.xmap = xm;
        P.omap = 0;
        if (L.out16 != nullptr) {
            int om = 0;
            while (om < no && oout[om] != L.out16) ++om;
            if (om == no) {
                if (no == 2) return cudaErrorInvalidValue;
                oout[no++] = L.out16;
            }
            P.omap = om;
        }
        if (l == 0) {
            P.wmap = 0;
            P.wrow = 0;
        } else {
            if (L.cin != 128 ||
                L.weight != static_cast<const uint16_t*>(layers[1].weight) + (l - 1) * wstride)
                return cudaErrorInvalidValue;
            P.wmap = 1;
            P.wrow = (l - 1) * kCo;
        }
        if (L.head_w != nullptr) {
            P.head = 1;
            a.head_w = L.head_w;
            a.head_b = L.head_b;
            a.feat = L.feat;
        }
    }
    const CUtensorMapDataType t16 =
        fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap tmW[2], tmX[3];
    const uint64_t rows = (uint64_t)F.m_total;
    if (!encode(&tmW[0], t16, 2, F.weight, (uint64_t)9 * F.cin, (uint64_t)kCo, kBK, kCo,
                CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    // Maps that a launch does not use describe a valid dummy and are never read.
    if (!encode(&tmW[1], t16, 2, n > 1 ? layers[1].weight : F.weight,
                n > 1 ? (uint64_t)9 * 128 : (uint64_t)9 * F.cin,
                n > 1 ? (uint64_t)(n - 1) * kCo : (uint64_t)kCo, kBK, kCo,
                CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    for (int i = 0; i < 3; ++i) {
        const int k = i < nx ? i : 0;
        if (!encode(&tmX[i], t16, 2, xin[k], (uint64_t)xcin[k], rows, kBK,
                    (uint32_t)(a.slab_rows / 2), CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
    }
    // Output maps: [rows][128] 16-bit, box of 32 channels x 16 rows (one
    // epilogue warp's chunk), no swizzle; a map a launch does not use
    // describes a valid dummy and is never written.
    CUtensorMap tmO[2];
    for (int i = 0; i < 2; ++i) {
        const void* base = i < no ? oout[i] : (no > 0 ? oout[0] : xin[0]);
        if (!encode(&tmO[i], t16, 2, base, (uint64_t)kCo, rows, 32, kChunk, CU_TENSOR_MAP_SWIZZLE_NONE))
            return cudaErrorInvalidValue;
    }
    if (n > 1) {
        cudaError_t e = cudaMemsetAsync(progress, 0, (size_t)grid * sizeof(unsigned), stream);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pix_smem_bytes(npx, F.g.rs);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (n > 1) {
        // CTAs wait on one another's progress: all of them must be resident.
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
    } else {
        // Programmatic dependent launch: this kernel's CTAs may start (and
        // run their prologue) while the previous kernel in the stream
        // drains; they wait for its completion before touching activations.
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    auto fn = fp16 ? conv3x3_pix_kernel<true> : conv3x3_pix_kernel<false>;
    return cudaLaunchKernelEx(&cfg, fn, tmW[0], tmW[1], tmX[0], tmX[1], tmX[2], tmO[0], tmO[1], a);
}

// Whether launch_trunk_pix runs its layers as one persistent launch (at
// least min_tiles tiles per CTA) or as one launch per layer.
bool trunk_in_one_launch(int m_total, int max_npx, int grid_limit, int min_tiles) {
    const int units = (m_total + 15) / 16;
    const int grid = units < grid_limit ? (units < 1 ? 1 : units) : grid_limit;
    const int span = (((m_total + grid - 1) / grid) + 15) / 16 * 16;
    return (span + max_npx - 1) / max_npx >= min_tiles;
}

}  // namespace

int trunk_pix_launches(int m_total, int n, int max_npx, int grid_limit, int min_tiles,
                       bool own_frames) {
    if (n <= 0) return 0;
    if (own_frames) return (n + kMaxLayers - 1) / kMaxLayers;
    if (!trunk_in_one_launch(m_total, max_npx, grid_limit, min_tiles)) return n;
    return (n + kMaxLayers - 1) / kMaxLayers;
}

cudaError_t configure_conv_pix() {
    const int smem = 227 * 1024;
    const void* fns[2] = {(const void*)conv3x3_pix_kernel<false>,
                          (const void*)conv3x3_pix_kernel<true>};
    for (const void* f : fns) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

bool conv_pix_supported(const ConvLayer& L, int npx) {
    return layer_ok(L, L) && npx % kChunk == 0 && npx >= 16 && npx <= kMaxPx &&
           pix_smem_bytes(npx, L.g.rs) <= 227 * 1024;
}

cudaError_t launch_conv_pix(const ConvLayer& L, int max_npx, bool fp16, int grid_limit,
                            cudaStream_t stream) {
    return launch_layers(&L, 1, max_npx, fp16, grid_limit, nullptr, stream);
}

cudaError_t launch_trunk_pix(const ConvLayer* layers, int n, int max_npx, bool fp16,
                             int grid_limit, unsigned* progress, cudaStream_t stream,
                             int withhold_cta, int min_tiles, bool own_frames) {
    // CTA ranges of whole frames: no tile waits on another CTA, so the
    // layers run as one launch whatever the batch (each CTA goes through
    // them at its own pace).
    if (own_frames && n > 0 && frames_fit(layers[0].g, layers[0].m_total)) {
        for (int l0 = 0; l0 < n; l0 += kMaxLayers) {
            const int cnt = n - l0 < kMaxLayers ? n - l0 : kMaxLayers;
            cudaError_t e = launch_layers(layers + l0, cnt, max_npx, fp16, grid_limit,
                                          cnt > 1 ? progress : nullptr, stream, withhold_cta, true);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    // Below min_tiles tiles per CTA, one launch per layer (programmatic
    // dependent launches).  The engine's default of 1 never takes this path:
    // the persistent launch measured faster at every batch (19x19 batch 32
    // to 384 and 9x9 batch 64 to 768, 1 to 4 tiles per CTA: 1-3% at one
    // tile, 5-6% at two, 16-18% at three).
    if (n > 0 && !trunk_in_one_launch(layers[0].m_total, max_npx, grid_limit, min_tiles)) {
        for (int l = 0; l < n; ++l) {
            cudaError_t e = launch_layers(layers + l, 1, max_npx, fp16, grid_limit, nullptr, stream);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    // Runs of at most kMaxLayers layers per launch; a run's first layer
    // takes its weights through its own tensor map, so a run may start at
    // any layer.
    for (int l0 = 0; l0 < n; l0 += kMaxLayers) {
        const int cnt = n - l0 < kMaxLayers ? n - l0 : kMaxLayers;
        cudaError_t e = launch_layers(layers + l0, cnt, max_npx, fp16, grid_limit,
                                      cnt > 1 ? progress : nullptr, stream, withhold_cta);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace mgb

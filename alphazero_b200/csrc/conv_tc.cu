// 3x3 convolution as an implicit GEMM on the sm_100a tensor cores.
//
// GEMM view (the dominant cost of the reference forward pass,
// src/eigen_engine.cpp:174-178, there one position at a time):
//   M = positions * IS framed pixels, N = output channels,
//   K = 9 taps * input channels.
// Because of the framed layout, the A tile of tap (dy, dx) for output rows
// [m0, m0 + 128) is simply rows [m0 + dy*RS + dx, ... + 128) of the input
// activation matrix.  Per 64-channel block the producer loads ONE slab of
// the tile's rows plus a halo of RS + 1 rows on each side (one TMA box,
// 128-byte swizzle), and the 9 taps read it through A descriptors whose
// start row is shifted by dy*RS + dx (the MMA derives the swizzle phase from
// the absolute shared-memory address, as TMA does when it writes the slab):
// activations cross L2 -> SMEM once per block instead of nine times.
// Weights are [cout][9][cin], so a K block of B is a (64 x bn) box at column
// tap*cin + channel block; B stages stream through a ring.
//
// One persistent CTA per SM, warp-specialised:
//   warp 0     weight producer (one thread): a STAGES-deep ring of B
//              stages by TMA, and each layer's bias by a bulk copy;
//   warp 1     TMEM allocator and MMA issuer (one thread): 4 x
//              tcgen05.mma.kind::f16 (128 x bn x 16) per K block, fp32
//              accumulators in TMEM, double-buffered across tiles;
//   warps 2-9  epilogue: tcgen05.ld of the accumulator, folded-BN bias,
//              residual add (the stream is a 16-bit hi plane, the operand,
//              plus an fp16 remainder plane lo, both pixel-major), ReLU,
//              frame masking, the sum re-split into hi and lo, each plane
//              staged per warp in shared memory ([32 rows][32 channels],
//              64-byte swizzle) and written by one TMA store, and
//              optionally the fused policy/value 1x1 head
//              projection (one thread owns one pixel row, so when a tile
//              spans all output channels it sees the whole channel vector);
//   warp 10    activation producer (one thread): the two halo-slab buffers
//              by TMA, after waiting for the previous layer's tiles when
//              one launch runs several layers.
// The epilogue of tile t overlaps the main loop of tile t+1.
// Every mbarrier wait is bounded (ptx_sm100.cuh); on expiry the kernel
// records an error code, drains its in-flight copies and frees TMEM.
#include "kernels.cuh"
#include "ptx_sm100.cuh"
#include "trunk_schedule.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <type_traits>

namespace mgb {
namespace {

constexpr int kBM = 128;  // rows per tile (TMEM lanes)
constexpr int kBK = 64;   // K elements per stage (128 bytes of 16-bit data)
// weight producer, MMA, 8 epilogue warps, slab producer
constexpr int kEpiWarps = 8;
constexpr int kSlabWarp = 2 + kEpiWarps;
constexpr int kThreads = 32 * (kSlabWarp + 1);
constexpr int kMaxLayers = 44;  // layers per launch (kernel parameter space)

template <int BN>
struct TcConfig {
    // 4 stages at BN 256 keep the kernel under 196 KB of shared memory, so
    // the carve-out leaves more L1 to the epilogue (measured 8% faster
    // than 5 stages on 19x19 b20c256 batch 1024).
    static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 8 : 12);
    static constexpr uint32_t kBBytes = BN * kBK * 2;
    static constexpr uint32_t kTmemCols = 2 * BN;
    // B ring + output staging (kStageBytes per epilogue warp) + barriers,
    // tmem slot and tile counters (512) + head weights (3 x 256 floats) +
    // head exchange (2 x 128 x 3 floats) + two layers' biases (2 x 256
    // floats, 16-byte aligned) + 1 KB alignment slack; the two slabs come
    // on top (slab_bytes).
    static constexpr int kSmemFixed =
        kStages * kBBytes + kEpiWarps * 4096 + 512 + 3072 + 3072 + 2048 + 16 + 1024;
};

// Rows of an activation slab: the tile's 128 rows plus RS + 1 on each side,
// rounded up to 16.
__host__ __device__ constexpr int tc_slab_rows(int rs) { return (kBM + 2 * (rs + 1) + 15) / 16 * 16; }

// One layer of a launch.
struct TcLayer {
    const float* bias;       // [cout]
    const uint16_t* res_hi;  // residual stream x = hi + lo, pixel-major [m_total][cout], or nullptr
    const uint16_t* res_lo;
    uint16_t* out16;         // output hi plane (operand type) or nullptr
    uint16_t* out_lo;        // output lo plane (fp16 remainder) or nullptr
    int cin;
    int xmap;                // activation tensor map of the input slabs (0..2)
    int wmap;                // weight tensor map (0 or 1)
    int wrow;                // first row of this layer's weights in that map
    int head;                // fused head projection (last trunk layer)
    int omap;                // output tensor maps: hi plane (bits 0-1), lo plane (bits 2-3)
};
static_assert(sizeof(TcLayer) == 64, "TcLayer layout");

// Work units: unit u is row tile u / nsplit (rows [128 * (u / nsplit), +128))
// and column tile u % nsplit (output channels [BN * (u % nsplit), +BN)).
// CTA c owns units [c * upc, (c + 1) * upc).  With several layers per
// launch nsplit is 1, and the units are the row tiles of the schedule of
// trunk_schedule.cuh (span = 128 * upc, npx = 128).
struct RowSpan {
    int m_total, span, npx;
};

struct TcArgs {
    int m_total;
    int units, upc;  // work units in all, per CTA
    int nsplit;      // cout / BN column tiles per row tile (one layer per launch only)
    int cout;
    int rs, is, board;
    int n_layers;
    int* err;
    unsigned* progress;  // [grid] tiles finished per CTA (several layers), else nullptr
    int withhold_cta;    // test hook: this CTA never publishes its progress (-1: none)
    const float* head_w;  // [3][cout] or nullptr (fused head projection, last layer)
    const float* head_b;
    float* feat;
    TcLayer layer[kMaxLayers];
};

template <bool FP16>
struct Act16;
template <>
struct Act16<false> {
    using T = __nv_bfloat16;
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ float2 unpack(uint32_t u) {
        __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
        return __bfloat1622float2(h);
    }
};
template <>
struct Act16<true> {
    using T = __half;
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ float2 unpack(uint32_t u) {
        __half2 h = *reinterpret_cast<__half2*>(&u);
        return __half22float2(h);
    }
};

template <int BN, bool FP16>
__global__ void __launch_bounds__(kThreads, 1)
    conv3x3_tc_kernel(const __grid_constant__ CUtensorMap tmA0,
                      const __grid_constant__ CUtensorMap tmA1,
                      const __grid_constant__ CUtensorMap tmA2,
                      const __grid_constant__ CUtensorMap tmB0,
                      const __grid_constant__ CUtensorMap tmB1,
                      const __grid_constant__ CUtensorMap tmO0,
                      const __grid_constant__ CUtensorMap tmO1,
                      const __grid_constant__ CUtensorMap tmO2, const __grid_constant__ TcArgs a) {
    using Cfg = TcConfig<BN>;
    using P = Act16<FP16>;
    constexpr int S = Cfg::kStages;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int halo = a.rs + 1;
    const uint32_t slab_bytes = (uint32_t)tc_slab_rows(a.rs) * 128u;
    uint8_t* sSlab = smem;                   // 2 slabs (multiples of 2 KB: atoms stay aligned)
    uint8_t* sB = smem + 2 * slab_bytes;     // S B stages
    // Output staging, 4 KB per epilogue warp: two [32 rows][64 B] blocks in
    // the 64-byte swizzle of the output tensor maps (1 KB aligned).
    uint8_t* sOut = sB + S * Cfg::kBBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + kEpiWarps * 4096);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* tfull = bars + 2 * S;
    uint64_t* tempty = bars + 2 * S + 2;
    uint64_t* done = bars + 2 * S + 4;
    uint64_t* sfull = bars + 2 * S + 5;
    uint64_t* sempty = sfull + 2;
    uint64_t* bfull = sempty + 2;   // [2] a layer's bias has landed in sbias[l & 1]
    uint64_t* bempty = bfull + 2;   // [2] the epilogue is done with sbias[l & 1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bempty + 2);
    uint32_t* tcount = tmem_slot + 1;  // [2] epilogue warps done, per accumulator buffer
    float* shead = reinterpret_cast<float*>(tmem_slot + 4);  // [3][cout] fused head projection weights
    float* sxchg = shead + 768;  // [2][128][3] head partial-sum exchange
    // [2][256] folded-BN biases of layers l and l + 1 (bulk copies)
    float* sbias = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(sxchg + 768) + 15) & ~uintptr_t(15));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int u0 = blockIdx.x * a.upc;
    const int nt = max(0, min(a.upc, a.units - u0));  // this CTA's units per layer

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_u32(&tfull[i]), 1);
            mbar_init(smem_u32(&tempty[i]), kEpiWarps);
            mbar_init(smem_u32(&sfull[i]), 1);
            mbar_init(smem_u32(&sempty[i]), 1);
            mbar_init(smem_u32(&bfull[i]), 1);
            mbar_init(smem_u32(&bempty[i]), kEpiWarps);
            tcount[i] = 0;
        }
        mbar_init(smem_u32(done), 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
        tmem_relinquish();
    }
    if (a.head_w != nullptr)
        for (int i = threadIdx.x; i < 3 * a.cout; i += kThreads) shead[i] = a.head_w[i];
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Activations of the previous kernel are read (and ones it may still
    // read are overwritten) only after it has completed.
    griddep_launch_dependents();
    griddep_wait();

    if (warp == 0) {
        // ---------------- weight (B) producer ----------------
        if (lane == 0) {
            prefetch_tensormap(&tmB0);
            prefetch_tensormap(&tmB1);
            int it = 0, nb = 0;
            bool ok = true;
            for (int l = 0; l < a.n_layers && ok; ++l) {
                const int cin = a.layer[l].cin, wrow = a.layer[l].wrow;
                const CUtensorMap* map = a.layer[l].wmap ? &tmB1 : &tmB0;
                // the layer's bias into sbias[l & 1], once the epilogue is
                // done with layer l - 2's
                const int bb = l & 1;
                if (l >= 2 && !mbar_wait(smem_u32(&bempty[bb]), ((l >> 1) - 1) & 1, a.err,
                                         kErrWaitProducer)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(smem_u32(&bfull[bb]), (uint32_t)a.cout * 4u);
                bulk_load(smem_u32(sbias + bb * 256), a.layer[l].bias, (uint32_t)a.cout * 4u,
                          smem_u32(&bfull[bb]));
                ++nb;
                for (int q = 0; q < nt && ok; ++q) {
                    const int n0 = ((u0 + tile_at(blockIdx.x, q, nt)) % a.nsplit) * BN;
                    for (int cb = 0; cb < cin / kBK && ok; ++cb) {
                        for (int tap = 0; tap < 9; ++tap, ++it) {
                            const int s = it % S;
                            if (!mbar_wait(smem_u32(&empty[s]), ((it / S) & 1) ^ 1, a.err,
                                           kErrWaitProducer)) {
                                ok = false;
                                break;
                            }
                            const uint32_t fb = smem_u32(&full[s]);
                            mbar_arrive_expect_tx(fb, Cfg::kBBytes);
                            tma_load_2d(smem_u32(sB + s * Cfg::kBBytes), map, fb,
                                        tap * cin + cb * kBK, wrow + n0);
                        }
                    }
                }
            }
            // Drain: every copy issued has landed before exit.
            for (int j = (it > S ? it - S : 0); j < it; ++j)
                mbar_wait(smem_u32(&full[j % S]), (j / S) & 1, a.err, kErrWaitDrain);
            for (int j = (nb > 2 ? nb - 2 : 0); j < nb; ++j)
                mbar_wait(smem_u32(&bfull[j & 1]), (j >> 1) & 1, a.err, kErrWaitDrain);
        }
        __syncwarp();
    } else if (warp == kSlabWarp) {
        // ---------------- activation slab producer ----------------
        // Separate from the weight producer, so the wait for the previous
        // layer's tiles never holds back the weight ring.
        if (lane == 0) {
            prefetch_tensormap(&tmA0);
            prefetch_tensormap(&tmA1);
            prefetch_tensormap(&tmA2);
            int is = 0;
            bool ok = true;
            for (int l = 0; l < a.n_layers && ok; ++l) {
                const int cin = a.layer[l].cin, xmap = a.layer[l].xmap;
                const CUtensorMap* map = xmap == 0 ? &tmA0 : (xmap == 1 ? &tmA1 : &tmA2);
                for (int q = 0; q < nt && ok; ++q) {
                    const int m0 = ((u0 + tile_at(blockIdx.x, q, nt)) / a.nsplit) * kBM;
                    if (l > 0 && a.progress != nullptr) {
                        const RowSpan g{a.m_total, a.upc * kBM, kBM};
                        if (!wait_inputs(g, a.progress, a.err, l, m0, min(kBM, a.m_total - m0),
                                         halo)) {
                            ok = false;
                            break;
                        }
                        // the rows were written through the generic proxy
                        fence_proxy_async_global();
                    }
                    for (int cb = 0; cb < cin / kBK; ++cb, ++is) {
                        // the tile's halo slab of this channel block (rows
                        // before the first or past the last read as zeros)
                        const int sb = is & 1;
                        if (!mbar_wait(smem_u32(&sempty[sb]), ((is >> 1) & 1) ^ 1, a.err,
                                       kErrWaitProducer)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(smem_u32(&sfull[sb]), slab_bytes);
                        tma_load_2d(smem_u32(sSlab + sb * slab_bytes), map, smem_u32(&sfull[sb]),
                                    cb * kBK, m0 - halo);
                    }
                }
            }
            for (int j = (is > 2 ? is - 2 : 0); j < is; ++j)
                mbar_wait(smem_u32(&sfull[j & 1]), (j >> 1) & 1, a.err, kErrWaitDrain);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(kBM, BN, !FP16);
            int it = 0, is = 0, t = 0;
            bool ok = true;
            for (int l = 0; l < a.n_layers && ok; ++l) {
                const int cblocks = a.layer[l].cin / kBK;
                for (int q = 0; q < nt && ok; ++q, ++t) {
                    const int acc = t & 1;
                    if (!mbar_wait(smem_u32(&tempty[acc]), ((t >> 1) & 1) ^ 1, a.err, kErrWaitMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                    for (int cb = 0; cb < cblocks && ok; ++cb, ++is) {
                        const int sb = is & 1;
                        if (!mbar_wait(smem_u32(&sfull[sb]), (is >> 1) & 1, a.err, kErrWaitMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        // Descriptor of the slab's first row; a tap's shifted
                        // start adds its byte offset / 16 to the address field
                        // (no carry: every start lies inside shared memory).
                        const uint64_t ad0 = smem_desc_sw128(smem_u32(sSlab + sb * slab_bytes));
                        // compile-time trip count: no per-tap index arithmetic
                        // between the MMA groups
#pragma unroll
                        for (int tap = 0; tap < 9; ++tap, ++it) {
                            const int s = it % S;
                            if (!mbar_wait(smem_u32(&full[s]), (it / S) & 1, a.err, kErrWaitMma)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            // A: the slab from the tap's shifted start row (whole
                            // 128-byte rows, so no descriptor base offset)
                            const int r0 = halo + (tap / 3 - 1) * a.rs + (tap % 3 - 1);
                            const uint64_t bd = smem_desc_sw128(smem_u32(sB + s * Cfg::kBBytes));
                            const uint64_t ad = ad0 + (uint64_t)(r0 * 8);  // r0 * 128 B / 16
                            // advance 16 elements (32 bytes) along K inside the swizzle atom
#pragma unroll
                            for (int k = 0; k < kBK / 16; ++k)
                                mma_f16(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc,
                                        (cb | tap | k) != 0);
                            mma_commit(smem_u32(&empty[s]));
                        }
                        if (ok) mma_commit(smem_u32(&sempty[sb]));
                    }
                    if (ok) mma_commit(smem_u32(&tfull[acc]));
                }
            }
            // All MMAs complete before TMEM is released.
            mma_commit(smem_u32(done));
            mbar_wait(smem_u32(done), 0, a.err, kErrWaitDrain);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        // Two warps per TMEM lane quarter: warp w reads lanes
        // [32*(w%4), +32) (the lane-access rule of tcgen05.ld) and column half
        // (w-2)/4 of the tile, so one thread owns one pixel row's half.
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        constexpr int kCols = BN / 2;
        constexpr int kChunks = kCols / 32;
        const int row = quarter * 32 + lane;
        uint8_t* const stg = sOut + (warp - 2) * 4096;
        const CUtensorMap* const omaps[3] = {&tmO0, &tmO1, &tmO2};
        if (lane == 0)
            for (int i = 0; i < 3; ++i) prefetch_tensormap(omaps[i]);
        int t = 0, sc = 0;
        bool ok = true;
        for (int l = 0; l < a.n_layers && ok; ++l) {
            // the layer's bias (bulk-copied by the weight producer)
            const int bb = l & 1;
            ok = mbar_wait(smem_u32(&bfull[bb]), (l >> 1) & 1, a.err, kErrWaitEpilogue);
            if (bar_any(1, 32 * kEpiWarps, !ok)) {
                ok = false;
                break;
            }
            const float* const bias = sbias + bb * 256;
            // the layer's parameters, read once
            const uint16_t* const res_hi = a.layer[l].res_hi;
            const uint16_t* const res_lo = a.layer[l].res_lo;
            uint16_t* const out16 = a.layer[l].out16;
            uint16_t* const out_lo = a.layer[l].out_lo;
            const bool head = a.layer[l].head != 0;
            const CUtensorMap* const map_hi = omaps[a.layer[l].omap & 3];
            const CUtensorMap* const map_lo = omaps[(a.layer[l].omap >> 2) & 3];
            // The staging buffers change roles between layers (two hi
            // buffers without a lo plane, one each with it): every store
            // of the layer before has read its buffer first.
            if (lane == 0) bulk_wait_read();
            __syncwarp();
            for (int q = 0; q < nt; ++q, ++t) {
                const int u = u0 + tile_at(blockIdx.x, q, nt);
                const int m0 = (u / a.nsplit) * kBM;
                const int len = min(kBM, a.m_total - m0);
                const int n0 = (u % a.nsplit) * BN;
                const int cbase = n0 + half * kCols;
                const int acc = t & 1;
                const int use = t >> 1;  // earlier tiles of this accumulator buffer
                const int m = m0 + row;
                const bool in_range = row < len;
                bool board_px = false;
                int pos = 0, pix = 0;
                if (in_range) {
                    pos = m / a.is;
                    const int qq = m - pos * a.is;
                    const int y = qq / a.rs;
                    const int x = qq - y * a.rs;
                    board_px = (y < a.board) && (x < a.board);
                    pix = y * a.board + x;
                }
                const size_t off = (size_t)m * a.cout + cbase;
                const bool has_res = res_hi != nullptr && in_range;
                // The first chunk's residual (32 hi and 32 lo values: each
                // plane's 64 contiguous bytes of the row as two 32-byte,
                // whole-sector loads) is requested before the accumulator is
                // ready; each later chunk's one chunk ahead.  L2-only: a
                // launch of several layers reads the rows again two layers
                // on, after its own TMA stores (which bypass L1) rewrote
                // them.  Every address is 32-byte aligned: buffers are
                // 256-byte aligned, rows are cout * 2 bytes and chunks start
                // at multiples of 32 channels.
                uint32_t rh[16], rl[16];
                if (has_res) {
                    ld_cg_v8(res_hi + off, rh);
                    ld_cg_v8(res_hi + off + 16, rh + 8);
                    ld_cg_v8(res_lo + off, rl);
                    ld_cg_v8(res_lo + off + 16, rl + 8);
                }
                ok = mbar_wait(smem_u32(&tfull[acc]), use & 1, a.err, kErrWaitEpilogue);
                // Leave together: no epilogue warp may be left at a named barrier.
                if (bar_any(1, 32 * kEpiWarps, !ok)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                float h0 = 0.f, h1 = 0.f, h2 = 0.f;  // fused head projection partial sums
                const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) +
                                       (uint32_t)(acc * BN + half * kCols);
#pragma unroll 1
                for (int c = 0; c < kChunks; ++c) {
                    const int c0 = c * 32;
                    uint32_t v[32];
                    tmem_ld_32cols(tbase + (uint32_t)c0, v);
                    tmem_ld_wait();
                    // Rows past the end go through with zeros (the warp
                    // stages and stores together; the store clips them).
                    float f[32];
                    // the layer's folded-BN bias (the same 32 values in every lane)
#pragma unroll
                    for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]) + bias[cbase + c0 + j];
                    if (has_res) {
#pragma unroll
                        for (int w = 0; w < 16; ++w) {
                            const float2 hv = P::unpack(rh[w]);
                            const float2 lv = __half22float2(*reinterpret_cast<const __half2*>(&rl[w]));
                            f[2 * w] += hv.x + lv.x;
                            f[2 * w + 1] += hv.y + lv.y;
                        }
                        if (c + 1 < kChunks) {
                            ld_cg_v8(res_hi + off + c0 + 32, rh);
                            ld_cg_v8(res_hi + off + c0 + 48, rh + 8);
                            ld_cg_v8(res_lo + off + c0 + 32, rl);
                            ld_cg_v8(res_lo + off + c0 + 48, rl + 8);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 32; ++j) f[j] = board_px ? fmaxf(f[j], 0.0f) : 0.0f;
                    if (out16 != nullptr) {
                        // This warp's [32 rows][32 channels] block of each
                        // plane goes through a shared-memory block and one
                        // TMA store: 32 rows per instruction in 16-byte
                        // pieces made 32 separate writes each (measured: the
                        // hi/lo stores took 27% of the 256-filter trunk).
                        // Lane = row; its 16-byte piece q4 sits at chunk
                        // q4 ^ ((row >> 1) & 3) of the row (64-byte swizzle,
                        // conflict-free for the 8 lanes of a store phase).
                        // With a lo plane, hi uses block 0 and lo block 1;
                        // without, the hi blocks alternate.  A block is
                        // rewritten only after the store issued from it
                        // has read it (at most one newer group pending).
                        const int y0 = m0 + quarter * 32;
                        const bool store = y0 < a.m_total;  // warp-uniform
                        uint8_t* const sh = stg + (out_lo != nullptr ? 0 : (sc & 1)) * 2048 + lane * 64;
                        uint8_t* const sl = stg + 2048 + lane * 64;
                        const int swz = (lane >> 1) & 3;
                        if (lane == 0) bulk_wait_read_n<1>();
                        __syncwarp();
                        uint32_t lw[16];
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) {
                            uint32_t hw4[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float x0 = f[q4 * 8 + 2 * e], x1 = f[q4 * 8 + 2 * e + 1];
                                hw4[e] = P::pack(x0, x1);
                                const float2 hv = P::unpack(hw4[e]);
                                const __half2 lv = __floats2half2_rn(x0 - hv.x, x1 - hv.y);
                                lw[q4 * 4 + e] = *reinterpret_cast<const uint32_t*>(&lv);
                            }
                            *reinterpret_cast<uint4*>(sh + ((q4 ^ swz) << 4)) =
                                make_uint4(hw4[0], hw4[1], hw4[2], hw4[3]);
                        }
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0 && store) {
                            tma_store_2d(map_hi, smem_u32(stg + (out_lo != nullptr ? 0 : (sc & 1)) * 2048),
                                         cbase + c0, y0);
                            bulk_commit();
                        }
                        if (out_lo != nullptr) {
                            if (lane == 0) bulk_wait_read_n<1>();
                            __syncwarp();
#pragma unroll
                            for (int q4 = 0; q4 < 4; ++q4)
                                *reinterpret_cast<uint4*>(sl + ((q4 ^ swz) << 4)) =
                                    make_uint4(lw[q4 * 4], lw[q4 * 4 + 1], lw[q4 * 4 + 2], lw[q4 * 4 + 3]);
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0 && store) {
                                tma_store_2d(map_lo, smem_u32(stg + 2048), cbase + c0, y0);
                                bulk_commit();
                            }
                        }
                        ++sc;
                    }
                    if (head) {
                        const float* w0 = shead + cbase + c0;
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            h0 = fmaf(f[j], w0[j], h0);
                            h1 = fmaf(f[j], w0[a.cout + j], h1);
                            h2 = fmaf(f[j], w0[2 * a.cout + j], h2);
                        }
                    }
                }
                if (head) {
                    // Half 1 hands its partial sums to half 0 through a
                    // double-buffered exchange (indexed by accumulator).
                    float* xs = sxchg + acc * (kBM * 3) + row * 3;
                    if (half == 1) {
                        xs[0] = h0;
                        xs[1] = h1;
                        xs[2] = h2;
                    }
                    named_barrier_sync(1, 32 * kEpiWarps);
                    if (half == 0 && board_px) {
                        const int hw = a.board * a.board;
                        float* fr = a.feat + (size_t)pos * 3 * hw;
                        fr[pix] = fmaxf(h0 + xs[0] + a.head_b[0], 0.f);
                        fr[hw + pix] = fmaxf(h1 + xs[1] + a.head_b[1], 0.f);
                        fr[2 * hw + pix] = fmaxf(h2 + xs[2] + a.head_b[2], 0.f);
                    }
                }
                // The accumulator has been read: hand it back to the MMA warp.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
                if (a.progress != nullptr) {
                    if (lane == 0) {
                        // this warp's TMA stores of the tile have landed
                        bulk_wait_all();
                        fence_proxy_async_global();
                    }
                    // This warp's stores of the tile are done (the warp
                    // barrier orders every lane's stores before lane 0's
                    // release).  The epilogue warps count themselves in at CTA
                    // scope; the last one, whose acquire sees the others'
                    // stores, publishes the CTA's count of finished tiles with
                    // a GPU-scope release, which (causality order being
                    // transitive) covers every warp's stores.
                    __syncwarp();
                    if (lane == 0) {
                        const unsigned before = atom_add_acq_rel_cta(smem_u32(&tcount[acc]), 1u);
                        if (before == (unsigned)(kEpiWarps * use + kEpiWarps - 1) &&
                            (int)blockIdx.x != a.withhold_cta) {
                            fence_proxy_async_global();
                            red_max_release_gpu(&a.progress[blockIdx.x], (unsigned)(l * nt + q + 1));
                        }
                    }
                    __syncwarp();
                }
            }
            // this warp is done with the layer's bias
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(smem_u32(&bempty[bb]));
        }
        // every TMA store has landed before the CTA exits
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

bool encode_2d(CUtensorMap* map, bool fp16, const void* base, uint64_t inner, uint64_t rows,
               uint32_t box_inner, uint32_t box_rows, const char** why,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    if (!encode_tiled_2d(map, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                         2, base, inner, rows, box_inner, box_rows, swizzle)) {
        *why = "cuTensorMapEncodeTiled rejected the tensor map (or is unavailable)";
        return false;
    }
    return true;
}

// Output maps of a launch: up to three distinct 16-bit [m_total][cout]
// buffers (hi planes and lo planes alike; a store copies bytes), box of 32
// channels x 32 rows (one epilogue warp's chunk), 64-byte swizzle.  Sets
// each layer's omap; unused maps describe a valid dummy that is never
// written.
bool output_maps(const ConvLayer* layers, int n, TcArgs& a, bool fp16, CUtensorMap* tmO,
                 const char** why) {
    const void* outs[3] = {nullptr, nullptr, nullptr};
    int no = 0;
    auto slot = [&](const void* p) {
        if (p == nullptr) return 0;
        for (int i = 0; i < no; ++i)
            if (outs[i] == p) return i;
        if (no == 3) return -1;
        outs[no] = p;
        return no++;
    };
    for (int l = 0; l < n; ++l) {
        const int h = slot(layers[l].out16), lo = slot(layers[l].out_lo);
        if (h < 0 || lo < 0) {
            *why = "more than three output buffers in one launch";
            return false;
        }
        a.layer[l].omap = h | (lo << 2);
    }
    const ConvLayer& F = layers[0];
    for (int i = 0; i < 3; ++i) {
        const void* base = i < no ? outs[i] : (no > 0 ? outs[0] : F.in);
        const uint64_t inner = no > 0 ? (uint64_t)F.cout : (uint64_t)F.cin;
        if (!encode_2d(&tmO[i], fp16, base, inner, (uint64_t)F.m_total, 32, 32, why,
                       CU_TENSOR_MAP_SWIZZLE_64B))
            return false;
    }
    return true;
}

template <int BN, bool FP16>
cudaError_t configure_one() {
    return cudaFuncSetAttribute(conv3x3_tc_kernel<BN, FP16>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

// The residual stream is the hi / lo pair (16-bit operands only).
bool tc_layer_ok(const ConvLayer& L) {
    return L.res32 == nullptr && L.out32 == nullptr && (L.res_hi == nullptr) == (L.res_lo == nullptr) &&
           (L.out_lo == nullptr || L.out16 != nullptr) && L.cin % kBK == 0 && L.g.is <= 1200;
}

TcLayer tc_layer(const ConvLayer& L) {
    TcLayer t{};
    t.bias = L.bias;
    t.res_hi = static_cast<const uint16_t*>(L.res_hi);
    t.res_lo = L.res_lo;
    t.out16 = static_cast<uint16_t*>(L.out16);
    t.out_lo = L.out_lo;
    t.cin = L.cin;
    t.head = L.head_w != nullptr ? 1 : 0;
    return t;
}

// The launch's common fields; returns the grid (units spread evenly over at
// most grid_limit CTAs).
int tc_args(const ConvLayer& F, int nsplit, int grid_limit, TcArgs& a) {
    a.m_total = F.m_total;
    a.nsplit = nsplit;
    a.units = ((F.m_total + kBM - 1) / kBM) * nsplit;
    int grid = a.units < grid_limit ? a.units : grid_limit;
    if (grid < 1) grid = 1;
    a.upc = (a.units + grid - 1) / grid;
    grid = (a.units + a.upc - 1) / a.upc;
    a.cout = F.cout;
    a.rs = F.g.rs;
    a.is = F.g.is;
    a.board = F.g.board;
    a.err = F.err;
    a.progress = nullptr;
    a.withhold_cta = -1;
    a.head_w = nullptr;
    a.head_b = nullptr;
    a.feat = nullptr;
    return grid;
}

template <int BN, bool FP16>
cudaError_t launch_tc(const CUtensorMap* tmA, const CUtensorMap* tmB, const CUtensorMap* tmO,
                      const TcArgs& a, int grid, bool cooperative, cudaStream_t stream) {
    using Cfg = TcConfig<BN>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)Cfg::kSmemFixed + 2 * tc_slab_rows(a.rs) * 128;
    if (cfg.dynamicSmemBytes > 227 * 1024 || tc_slab_rows(a.rs) > 256) return cudaErrorInvalidValue;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (cooperative) {
        // CTAs wait on one another's progress: all of them must be resident.
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
    } else {
        // Programmatic dependent launch (see griddep_wait in the kernel).
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, conv3x3_tc_kernel<BN, FP16>, tmA[0], tmA[1], tmA[2], tmB[0],
                              tmB[1], tmO[0], tmO[1], tmO[2], a);
}

cudaError_t launch_tc_any(int bn, bool fp16, const CUtensorMap* tmA, const CUtensorMap* tmB,
                          const CUtensorMap* tmO, const TcArgs& a, int grid, bool cooperative,
                          cudaStream_t stream) {
    if (fp16) {
        switch (bn) {
            case 64: return launch_tc<64, true>(tmA, tmB, tmO, a, grid, cooperative, stream);
            case 128: return launch_tc<128, true>(tmA, tmB, tmO, a, grid, cooperative, stream);
            case 256: return launch_tc<256, true>(tmA, tmB, tmO, a, grid, cooperative, stream);
        }
    } else {
        switch (bn) {
            case 64: return launch_tc<64, false>(tmA, tmB, tmO, a, grid, cooperative, stream);
            case 128: return launch_tc<128, false>(tmA, tmB, tmO, a, grid, cooperative, stream);
            case 256: return launch_tc<256, false>(tmA, tmB, tmO, a, grid, cooperative, stream);
        }
    }
    return cudaErrorInvalidValue;
}

}  // namespace

bool encode_tiled_2d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base,
                     uint64_t inner, uint64_t rows, uint32_t box_inner, uint32_t box_rows,
                     CUtensorMapSwizzle swizzle) {
    static PFN_cuTensorMapEncodeTiled_v12000 enc = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        return cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                           cudaSuccess &&
                       q == cudaDriverEntryPointSuccess
                   ? reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p)
                   : nullptr;
    }();
    struct Entry {
        const void* base;
        uint64_t inner, rows;
        uint32_t box_inner, box_rows;
        int dt, esize, swizzle;
        CUtensorMap map;
    };
    constexpr int kEntries = 64;  // a network's launches use a few dozen maps
    thread_local Entry cache[kEntries];
    thread_local int used = 0, next = 0;
    for (int i = 0; i < used; ++i) {
        const Entry& e = cache[i];
        if (e.base == base && e.inner == inner && e.rows == rows && e.box_inner == box_inner &&
            e.box_rows == box_rows && e.dt == (int)dt && e.esize == esize && e.swizzle == (int)swizzle) {
            *map = e.map;
            return true;
        }
    }
    if (enc == nullptr) return false;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {inner * (uint64_t)esize};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    if (enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    Entry& e = cache[next];
    e = Entry{base, inner, rows, box_inner, box_rows, (int)dt, esize, (int)swizzle, *map};
    next = (next + 1) % kEntries;
    if (used < kEntries) ++used;
    return true;
}

cudaError_t configure_conv_tc() {
    cudaError_t e;
    if ((e = configure_one<64, false>()) != cudaSuccess) return e;
    if ((e = configure_one<128, false>()) != cudaSuccess) return e;
    if ((e = configure_one<256, false>()) != cudaSuccess) return e;
    if ((e = configure_one<64, true>()) != cudaSuccess) return e;
    if ((e = configure_one<128, true>()) != cudaSuccess) return e;
    return configure_one<256, true>();
}

int conv_tc_smem_bytes(int bn, int rs) {
    const int slabs = 2 * tc_slab_rows(rs) * 128;
    switch (bn) {
        case 64: return TcConfig<64>::kSmemFixed + slabs;
        case 128: return TcConfig<128>::kSmemFixed + slabs;
        case 256: return TcConfig<256>::kSmemFixed + slabs;
        default: return -1;
    }
}

bool make_conv_tensor_maps(const ConvLayer& L, int bn, bool fp16, CUtensorMap* tmA,
                           CUtensorMap* tmB, const char** why) {
    if (L.cin % kBK != 0 || L.cout % bn != 0 || bn % 64 != 0 || bn > 256) {
        *why = "unsupported channel counts for the tensor-core convolution";
        return false;
    }
    if (tc_slab_rows(L.g.rs) > 256) {
        *why = "board too large for the tensor-core convolution's halo slab";
        return false;
    }
    if (!encode_2d(tmA, fp16, L.in, (uint64_t)L.cin, (uint64_t)L.m_total, kBK,
                   (uint32_t)tc_slab_rows(L.g.rs), why))
        return false;
    return encode_2d(tmB, fp16, L.weight, (uint64_t)9 * L.cin, (uint64_t)L.cout, kBK,
                     (uint32_t)bn, why);
}

cudaError_t launch_conv_tc(const ConvLayer& L, const CUtensorMap& tmA, const CUtensorMap& tmB,
                           int bn, bool fp16, int grid_limit, cudaStream_t stream) {
    // The fused head projection needs every output channel of a row in one tile.
    if (!tc_layer_ok(L) || bn <= 0 || L.cout % bn != 0 || (L.head_w != nullptr && L.cout != bn))
        return cudaErrorInvalidValue;
    TcArgs a;
    const int grid = tc_args(L, L.cout / bn, grid_limit, a);
    a.n_layers = 1;
    a.layer[0] = tc_layer(L);
    a.head_w = L.head_w;
    a.head_b = L.head_b;
    a.feat = L.feat;
    const CUtensorMap A[3] = {tmA, tmA, tmA};
    const CUtensorMap B[2] = {tmB, tmB};
    CUtensorMap O[3];
    const char* why = "";
    if (!output_maps(&L, 1, a, fp16, O, &why)) return cudaErrorInvalidValue;
    return launch_tc_any(bn, fp16, A, B, O, a, grid, false, stream);
}

bool trunk_tc_supported(const ConvLayer* layers, int n) {
    if (n < 1 || n > kMaxLayers) return false;
    const ConvLayer& F = layers[0];
    const int bn = F.cout;
    if (bn != 64 && bn != 128 && bn != 256) return false;
    if (conv_tc_smem_bytes(bn, F.g.rs) > 227 * 1024 || tc_slab_rows(F.g.rs) > 256) return false;
    const size_t wstride = (size_t)bn * 9 * bn;  // elements per cin == cout layer
    for (int l = 0; l < n; ++l) {
        const ConvLayer& L = layers[l];
        if (!tc_layer_ok(L) || L.cout != bn || L.m_total != F.m_total || L.g.rs != F.g.rs ||
            (L.head_w != nullptr && l != n - 1))
            return false;
        if (l > 0 && (L.cin != bn ||
                      L.weight != static_cast<const uint16_t*>(layers[1].weight) + (l - 1) * wstride))
            return false;
    }
    return true;
}

cudaError_t launch_trunk_tc(const ConvLayer* layers, int n, bool fp16, int grid_limit,
                            unsigned* progress, cudaStream_t stream, int withhold_cta) {
    if (!trunk_tc_supported(layers, n) || (n > 1 && progress == nullptr)) return cudaErrorInvalidValue;
    const ConvLayer& F = layers[0];
    const int bn = F.cout;
    TcArgs a;
    const int grid = tc_args(F, 1, grid_limit, a);
    a.n_layers = n;
    a.progress = n > 1 ? progress : nullptr;
    a.withhold_cta = n > 1 ? withhold_cta : -1;
    // Up to three distinct input buffers, each with its own tensor map.
    const void* xin[3] = {nullptr, nullptr, nullptr};
    int xcin[3] = {0, 0, 0};
    int nx = 0;
    for (int l = 0; l < n; ++l) {
        const ConvLayer& L = layers[l];
        TcLayer& P = a.layer[l];
        P = tc_layer(L);
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
        P.wmap = l == 0 ? 0 : 1;
        P.wrow = l == 0 ? 0 : (l - 1) * bn;
        if (L.head_w != nullptr) {
            a.head_w = L.head_w;
            a.head_b = L.head_b;
            a.feat = L.feat;
        }
    }
    const char* why = "";
    CUtensorMap A[3], B[2];
    for (int i = 0; i < 3; ++i) {
        const int k = i < nx ? i : 0;  // maps a launch does not use describe a valid dummy
        if (!encode_2d(&A[i], fp16, xin[k], (uint64_t)xcin[k], (uint64_t)F.m_total, kBK,
                       (uint32_t)tc_slab_rows(F.g.rs), &why))
            return cudaErrorInvalidValue;
    }
    if (!encode_2d(&B[0], fp16, F.weight, (uint64_t)9 * F.cin, (uint64_t)bn, kBK, (uint32_t)bn, &why) ||
        !encode_2d(&B[1], fp16, n > 1 ? layers[1].weight : F.weight,
                   n > 1 ? (uint64_t)9 * bn : (uint64_t)9 * F.cin,
                   n > 1 ? (uint64_t)(n - 1) * bn : (uint64_t)bn, kBK, (uint32_t)bn, &why))
        return cudaErrorInvalidValue;
    CUtensorMap O[3];
    if (!output_maps(layers, n, a, fp16, O, &why)) return cudaErrorInvalidValue;
    if (n > 1) {
        cudaError_t e = cudaMemsetAsync(progress, 0, (size_t)grid * sizeof(unsigned), stream);
        if (e != cudaSuccess) return e;
    }
    return launch_tc_any(bn, fp16, A, B, O, a, grid, n > 1, stream);
}

int trunk_tc_max_layers() { return kMaxLayers; }

}  // namespace mgb

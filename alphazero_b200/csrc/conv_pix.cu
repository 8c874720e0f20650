// 3x3 convolution with 128 output channels as an implicit GEMM on the
// sm_100a tensor cores, pixels on the MMA's N side.
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
// Weight K blocks (128 x 64) stream through a 5-deep ring.
//
// The accumulator is [co lanes][px columns] in TMEM, double-buffered across
// tiles (2 x 256 columns).  Each epilogue warp works on its own: it owns 32
// channels (its TMEM lanes) of every other 16-pixel chunk and moves them
// straight between registers and global memory (lane = channel, so each
// 16-bit access of a warp covers 64 contiguous bytes of a pixel row).  The
// residual stream is a pair of 16-bit planes, x = hi + lo with hi = x
// rounded to the operand type (the next layer's input) and lo = x - hi
// rounded to fp16.  A chunk's residual hi / lo values are loaded one chunk
// ahead into registers; each thread adds bias and residual, applies
// ReLU and the frame mask, and stores the sum re-split into hi and lo.  In
// the last trunk layer the fp32 sums go through shared memory to the
// policy / value 1x1 head projection instead.
//
// Warp roles (352 threads): warp 0 weight TMA producer, warp 1 TMEM
// allocator + MMA issuer, warps 2-9 epilogue (warp w reads TMEM lanes
// [32*(w%4), +32) of chunks (w-2)/4, (w-2)/4 + 2, ...), warp 10 activation
// slab TMA producer (two slab buffers).  All waits are bounded.
//
// Work split: CTA b owns the contiguous pixel range [b*span, (b+1)*span),
// cut into equal tiles of at most 256 pixels, so every SM gets the same
// number of pixels (a fixed 256-pixel tiling left up to 10% of the last wave
// idle).  Launches are programmatic dependent launches: a CTA's prologue
// overlaps the previous kernel's tail.
#include "kernels.cuh"
#include "ptx_sm100.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

namespace mgb {
namespace {

constexpr int kCo = 128;        // output channels (MMA M)
constexpr int kBK = 64;         // K per stage / slab channel block
constexpr int kMaxPx = 256;     // MMA N limit
constexpr int kStages = 5;      // weight ring depth
constexpr int kSlabs = 2;       // activation slab ring depth
constexpr int kThreads = 352;
constexpr int kChunk = 16;      // pixels per epilogue chunk
constexpr uint32_t kWBytes = kCo * kBK * 2;            // 16 KB weight stage
constexpr int kSlot = kChunk * 32;  // one warp's chunk: 16 pixels x 32 channels
constexpr int kEpiWarps = 8;
constexpr int kMagicShift = 40;     // n / d == (n * ceil(2^40 / d)) >> 40 here

struct PixArgs {
    int m_total;
    int span;           // pixels per CTA (multiple of 16): CTA b owns [b*span, (b+1)*span)
    int tiles_per_cta;  // tiles its range is cut into
    int npx;            // pixels per tile (multiple of 16, <= 256; the last tile may be shorter)
    int cin;
    int rs, is, board;
    int slab_rows;  // rows per slab (multiple of 16)
    uint64_t is_magic, rs_magic;  // ceil(2^40 / is), ceil(2^40 / rs)
    const uint16_t* res_hi;  // residual stream [m_total][128] hi plane or nullptr
    const uint16_t* res_lo;  // and its fp16 remainder plane
    uint16_t* out16;         // output [m_total][128] (hi plane) or nullptr
    uint16_t* out_lo;        // its fp16 remainder plane or nullptr
    const float* bias;
    const float* head_w;  // [3][128] or nullptr (fused head projection)
    const float* head_b;
    float* feat;
    int* err;
};

template <bool FP16>
__device__ __forceinline__ uint16_t to16(float v);
template <>
__device__ __forceinline__ uint16_t to16<false>(float v) {
    __nv_bfloat16 h = __float2bfloat16_rn(v);
    return *reinterpret_cast<uint16_t*>(&h);
}
template <>
__device__ __forceinline__ uint16_t to16<true>(float v) {
    __half h = __float2half_rn(v);
    return *reinterpret_cast<uint16_t*>(&h);
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
__device__ __forceinline__ float lo_value(uint16_t l) { return __half2float(__ushort_as_half(l)); }
__device__ __forceinline__ uint16_t lo_bits(float r) { return __half_as_ushort(__float2half_rn(r)); }

// n / d for 0 <= n < 2^23 and d <= 1200 (the launcher checks both).
__device__ __forceinline__ int div_magic(int n, uint64_t magic) {
    return (int)(((uint64_t)(uint32_t)n * magic) >> kMagicShift);
}

// Tile k of this CTA's contiguous pixel range: rows [m0, m0 + len);
// len <= 0 when the range has no such tile.  Every CTA gets the same number
// of pixels (to within one tile), so the last wave is not mostly idle.
__device__ __forceinline__ void cta_tile(const PixArgs& a, int k, int& m0, int& len) {
    const int start = blockIdx.x * a.span;
    const int end = min(start + a.span, a.m_total);
    m0 = start + k * a.npx;
    len = min(a.npx, end - m0);
}

// Advances (k, c) to epilogue group grp's next chunk (chunks grp, grp+2, ...
// of each tile in turn); false when the CTA has none left.
__device__ __forceinline__ bool group_next(const PixArgs& a, int grp, int& k, int& c) {
    c += 2;
    while (k < a.tiles_per_cta) {
        int m0, len;
        cta_tile(a, k, m0, len);
        if (len <= 0) return false;
        if (c * kChunk < len) return true;
        ++k;
        c = grp;
    }
    return false;
}

template <bool FP16, bool HEAD>
__global__ void __launch_bounds__(kThreads, 1)
    conv3x3_pix_kernel(const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmX, const PixArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t slab_bytes = (uint32_t)a.slab_rows * 128u;
    uint8_t* wring = smem;                                   // kStages x 16 KB
    uint8_t* slab0 = wring + kStages * kWBytes;              // kSlabs slabs
    float* hslot = reinterpret_cast<float*>(slab0 + kSlabs * slab_bytes);  // [kEpiWarps][16][32]
    uint64_t* bars = reinterpret_cast<uint64_t*>(hslot + kEpiWarps * kSlot);
    uint64_t* wfull = bars;
    uint64_t* wempty = bars + kStages;
    uint64_t* sfull = bars + 2 * kStages;
    uint64_t* sempty = sfull + kSlabs;
    uint64_t* tfull = sempty + kSlabs;
    uint64_t* tempty = tfull + 2;
    uint64_t* done = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    float* sbias = reinterpret_cast<float*>(tmem_slot + 4);  // [128]
    float* shead = sbias + kCo;                              // [3][128]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&wfull[s]), 1);
            mbar_init(smem_u32(&wempty[s]), 1);
        }
        for (int i = 0; i < kSlabs; ++i) {
            mbar_init(smem_u32(&sfull[i]), 1);
            mbar_init(smem_u32(&sempty[i]), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_u32(&tfull[i]), 1);
            mbar_init(smem_u32(&tempty[i]), 8);
        }
        mbar_init(smem_u32(done), 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), 512);
        tmem_relinquish();
    }
    for (int i = threadIdx.x; i < kCo; i += kThreads) sbias[i] = a.bias[i];
    if (a.head_w != nullptr)
        for (int i = threadIdx.x; i < 3 * kCo; i += kThreads) shead[i] = a.head_w[i];
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Everything above touches only this CTA's resources and the layer's
    // constant parameters.  Activations written by the previous kernel are
    // read, and activations it may still read are overwritten, only after
    // it has completed.
    griddep_launch_dependents();
    griddep_wait();

    const int cblocks = a.cin / kBK;
    const int halo = a.rs + 1;
    const int half_rows = a.slab_rows / 2;

    if (warp == 0) {
        // ---------------- weight producer ----------------
        if (lane == 0) {
            prefetch_tensormap(&tmW);
            int iw = 0;
            bool ok = true;
            for (int k = 0; k < a.tiles_per_cta && ok; ++k) {
                int m0, len;
                cta_tile(a, k, m0, len);
                if (len <= 0) break;
                for (int cb = 0; cb < cblocks && ok; ++cb) {
                    for (int tap = 0; tap < 9; ++tap, ++iw) {
                        const int s = iw % kStages;
                        if (!mbar_wait(smem_u32(&wempty[s]), ((iw / kStages) & 1) ^ 1, a.err,
                                       kErrWaitProducer)) {
                            ok = false;
                            break;
                        }
                        const uint32_t wfb = smem_u32(&wfull[s]);
                        mbar_arrive_expect_tx(wfb, kWBytes);
                        tma_load_2d(smem_u32(wring + s * kWBytes), &tmW, wfb, tap * a.cin + cb * kBK,
                                    0);
                    }
                }
            }
            // Drain every copy still in flight before the CTA exits.
            for (int j = (iw > kStages ? iw - kStages : 0); j < iw; ++j)
                mbar_wait(smem_u32(&wfull[j % kStages]), (j / kStages) & 1, a.err, kErrWaitDrain);
        }
        __syncwarp();
    } else if (warp == 2 + kEpiWarps) {
        // ---------------- activation slab producer ----------------
        // Separate from the weight producer so a slab load is issued as soon
        // as a slab buffer frees up, not behind the weight ring's waits.
        if (lane == 0) {
            prefetch_tensormap(&tmX);
            int is = 0;
            bool ok = true;
            for (int k = 0; k < a.tiles_per_cta && ok; ++k) {
                int m0, len;
                cta_tile(a, k, m0, len);
                if (len <= 0) break;
                for (int cb = 0; cb < cblocks; ++cb, ++is) {
                    const int sb = is % kSlabs;
                    if (!mbar_wait(smem_u32(&sempty[sb]), ((is / kSlabs) & 1) ^ 1, a.err,
                                   kErrWaitProducer)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sfb = smem_u32(&sfull[sb]);
                    uint8_t* slab = slab0 + sb * slab_bytes;
                    mbar_arrive_expect_tx(sfb, slab_bytes);
                    tma_load_2d(smem_u32(slab), &tmX, sfb, cb * kBK, m0 - halo);
                    tma_load_2d(smem_u32(slab + half_rows * 128), &tmX, sfb, cb * kBK,
                                m0 - halo + half_rows);
                }
            }
            for (int j = (is > kSlabs ? is - kSlabs : 0); j < is; ++j)
                mbar_wait(smem_u32(&sfull[j % kSlabs]), (j / kSlabs) & 1, a.err, kErrWaitDrain);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int iw = 0, is = 0, t = 0;
            bool ok = true;
            for (int k = 0; k < a.tiles_per_cta && ok; ++k, ++t) {
                int m0, len;
                cta_tile(a, k, m0, len);
                if (len <= 0) break;
                // MMA N = the tile's pixels rounded up to 16
                const uint32_t idesc = idesc_f16(kCo, (len + 15) & ~15, !FP16);
                const int acc = t & 1;
                if (!mbar_wait(smem_u32(&tempty[acc]), ((t >> 1) & 1) ^ 1, a.err, kErrWaitMma)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * kMaxPx);
                for (int cb = 0; cb < cblocks && ok; ++cb, ++is) {
                    const int sb = is % kSlabs;
                    if (!mbar_wait(smem_u32(&sfull[sb]), (is / kSlabs) & 1, a.err, kErrWaitMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t slab = smem_u32(slab0 + sb * slab_bytes);
                    for (int tap = 0; tap < 9; ++tap, ++iw) {
                        const int s = iw % kStages;
                        if (!mbar_wait(smem_u32(&wfull[s]), (iw / kStages) & 1, a.err, kErrWaitMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const int r0 = halo + (tap / 3 - 1) * a.rs + (tap % 3 - 1);
                        const uint64_t ad = smem_desc_sw128(smem_u32(wring + s * kWBytes));
#pragma unroll
                        for (int kk = 0; kk < kBK / 16; ++kk) {
                            // row-shifted start, base offset 0 (see file comment)
                            const uint64_t bd = smem_desc_sw128(slab + (uint32_t)r0 * 128u + 32u * kk);
                            mma_f16(d, ad + (uint64_t)(2 * kk), bd, idesc, (cb | tap | kk) != 0);
                        }
                        mma_commit(smem_u32(&wempty[s]));
                    }
                    if (ok) mma_commit(smem_u32(&sempty[sb]));
                }
                if (ok) mma_commit(smem_u32(&tfull[acc]));
            }
            mma_commit(smem_u32(done));
            mbar_wait(smem_u32(done), 0, a.err, kErrWaitDrain);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        // Each warp finishes its 32 channels (its TMEM lanes) of every other
        // chunk on its own, straight between registers and global memory:
        // lane = channel, so each 16-bit access of the warp covers 64
        // contiguous bytes of a pixel row.  Only the head-projection layer,
        // which sums over all 128 channels, couples the warps (through
        // shared memory).
        const int quarter = warp & 3;  // channels [32*quarter, +32)
        const int ew = warp - 2;       // 0..7
        const int par = ew >> 2;       // chunks par, par+2, ...
        const int co = quarter * 32 + lane;
        const float bias = sbias[co];
        const int hw = a.board * a.board;
        const bool has_res = a.res_hi != nullptr;
        const bool has_lo = a.out_lo != nullptr;
        float* slot = hslot + ew * kSlot;  // head layer: this warp's fp32 sums [16][32]
        const int bar_a = 2 + 2 * par, bar_b = 3 + 2 * par;  // head layer only
        // Residual of the next chunk, loaded one chunk ahead into registers.
        uint16_t nh[kChunk], nl[kChunk];
        auto load_res = [&](int px) {
            const uint16_t* ph = a.res_hi + (size_t)px * kCo + co;
            const uint16_t* pl = a.res_lo + (size_t)px * kCo + co;
            if (px + kChunk <= a.m_total) {
#pragma unroll
                for (int j = 0; j < kChunk; ++j) {
                    nh[j] = __ldcg(ph + j * kCo);
                    nl[j] = __ldcg(pl + j * kCo);
                }
            } else {
#pragma unroll
                for (int j = 0; j < kChunk; ++j) {
                    const bool in = px + j < a.m_total;
                    nh[j] = in ? __ldcg(ph + j * kCo) : (uint16_t)0;
                    nl[j] = in ? __ldcg(pl + j * kCo) : (uint16_t)0;
                }
            }
        };
        int lk = 0, lc = par - 2;  // position of the next residual load
        bool lvalid = group_next(a, par, lk, lc);
        if (has_res && lvalid) {
            int m0, len;
            cta_tile(a, lk, m0, len);
            load_res(m0 + lc * kChunk);
            lvalid = group_next(a, par, lk, lc);
        }
        int t = 0;
        bool ok = true;
        for (int k = 0; k < a.tiles_per_cta && ok; ++k, ++t) {
            int m0, len;
            cta_tile(a, k, m0, len);
            if (len <= 0) break;
            const int nchunks = (len + kChunk - 1) / kChunk;
            const int acc = t & 1;
            ok = mbar_wait(smem_u32(&tfull[acc]), (t >> 1) & 1, a.err, kErrWaitEpilogue);
            if (HEAD ? bar_any(bar_a, 128, !ok) : __any_sync(0xffffffffu, !ok)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t tcol =
                tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * kMaxPx);
#pragma unroll 1
            for (int c = par; c < nchunks; c += 2) {
                const int px0 = m0 + c * kChunk;
                uint32_t v[16];
                tmem_ld_16cols(tcol + (uint32_t)(c * kChunk), v);
                float f[16];
                if (has_res) {
#pragma unroll
                    for (int j = 0; j < kChunk; ++j) f[j] = from16<FP16>(nh[j]) + lo_value(nl[j]);
                    if (lvalid) {  // next chunk's residual, in flight during this one
                        int m1, len1;
                        cta_tile(a, lk, m1, len1);
                        load_res(m1 + lc * kChunk);
                        lvalid = group_next(a, par, lk, lc);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < kChunk; ++j) f[j] = 0.f;
                }
                // lanes 0..15 classify pixels px0 + lane
                bool onb = false;
                if (c * kChunk + (lane & 15) < len) {
                    const int mj = px0 + (lane & 15);
                    const int q = mj - div_magic(mj, a.is_magic) * a.is;
                    const int y = div_magic(q, a.rs_magic);
                    onb = (y < a.board) && (q - y * a.rs < a.board);
                }
                const uint32_t board_mask = __ballot_sync(0xffffffffu, onb) & 0xffffu;
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < kChunk; ++j) {
                    const float x = __uint_as_float(v[j]) + bias + f[j];
                    f[j] = ((board_mask >> j) & 1) ? fmaxf(x, 0.f) : 0.f;
                }
                if (!HEAD) {
                    uint16_t* oh = a.out16 + (size_t)px0 * kCo + co;
                    uint16_t* ol = a.out_lo + (size_t)px0 * kCo + co;
                    const int nrow = min(kChunk, a.m_total - px0);
#pragma unroll
                    for (int j = 0; j < kChunk; ++j) {
                        if (j < nrow) {
                            const uint16_t h = to16<FP16>(f[j]);
                            oh[j * kCo] = h;
                            if (has_lo) ol[j * kCo] = lo_bits(f[j] - from16<FP16>(h));
                        }
                    }
                } else {
                    // Policy / value 1x1 convs of the chunk's 16 pixels:
                    // thread (pixel g/8, channel segment g%8) of the group
                    // sums 16 channels, which sit in the slot of the warp
                    // owning that channel quarter; the 8 segments of a pixel
                    // combine by shuffles.  The first barrier keeps the slots
                    // from being rewritten while the previous chunk's sums
                    // still read them.
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
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        const int kq = (q + 4 * sq + (p & 3)) & 15;  // spread banks
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
                        const int pos = div_magic(mp, a.is_magic);
                        const int qq = mp - pos * a.is;
                        const int y = div_magic(qq, a.rs_magic), x = qq - y * a.rs;
                        float* fr = a.feat + (size_t)pos * 3 * hw + y * a.board + x;
                        fr[0] = fmaxf(d0 + a.head_b[0], 0.f);
                        fr[hw] = fmaxf(d1 + a.head_b[1], 0.f);
                        fr[2 * hw] = fmaxf(d2 + a.head_b[2], 0.f);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
        }
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
    return (size_t)kStages * kWBytes + kSlabs * slab + (size_t)kEpiWarps * kSlot * 4 +
           (2 * kStages + 2 * kSlabs + 4 + 1) * 8 + 16 + (kCo + 3 * kCo) * 4 + 1024;
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D tensor map [rows][inner] of `esize`-byte elements.
bool encode(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
            uint64_t rows, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    auto enc = encoder();
    if (enc == nullptr) return false;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {inner * (uint64_t)esize};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t configure_conv_pix() {
    const int smem = 227 * 1024;
    const void* fns[4] = {(const void*)conv3x3_pix_kernel<false, false>,
                          (const void*)conv3x3_pix_kernel<false, true>,
                          (const void*)conv3x3_pix_kernel<true, false>,
                          (const void*)conv3x3_pix_kernel<true, true>};
    for (const void* f : fns) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

bool conv_pix_supported(const ConvLayer& L, int npx) {
    // The residual stream is the hi / lo pair; fp32 residuals are not read.
    return L.cout == kCo && L.cin % kBK == 0 && npx % kChunk == 0 && npx >= 16 &&
           npx <= kMaxPx && pix_smem_bytes(npx, L.g.rs) <= 227 * 1024 && L.res32 == nullptr &&
           L.out32 == nullptr && (L.res_hi == nullptr) == (L.res_lo == nullptr) &&
           (L.out_lo == nullptr || L.out16 != nullptr) && L.g.is <= 1200 &&
           L.m_total < (1 << 23) - 2 * kMaxPx;
}

cudaError_t launch_conv_pix(const ConvLayer& L, int max_npx, bool fp16, int grid_limit,
                            cudaStream_t stream) {
    // Balanced ranges: each CTA takes span pixels (a multiple of 16) cut into
    // equal tiles of at most max_npx.
    const int units = (L.m_total + 15) / 16;
    int grid = units < grid_limit ? units : grid_limit;
    if (grid < 1) grid = 1;
    const int span = (((L.m_total + grid - 1) / grid) + 15) / 16 * 16;
    grid = (L.m_total + span - 1) / span;
    const int tiles = (span + max_npx - 1) / max_npx;
    const int npx = ((span + tiles - 1) / tiles + 15) / 16 * 16;
    if (!conv_pix_supported(L, npx)) return cudaErrorInvalidValue;
    PixArgs a;
    a.m_total = L.m_total;
    a.span = span;
    a.tiles_per_cta = tiles;
    a.npx = npx;
    a.cin = L.cin;
    a.rs = L.g.rs;
    a.is = L.g.is;
    a.board = L.g.board;
    a.slab_rows = slab_rows_for(npx, L.g.rs);
    a.is_magic = ((1ull << kMagicShift) + (uint64_t)L.g.is - 1) / (uint64_t)L.g.is;
    a.rs_magic = ((1ull << kMagicShift) + (uint64_t)L.g.rs - 1) / (uint64_t)L.g.rs;
    a.res_hi = static_cast<const uint16_t*>(L.res_hi);
    a.res_lo = L.res_lo;
    a.out16 = static_cast<uint16_t*>(L.out16);
    a.out_lo = L.out_lo;
    a.bias = L.bias;
    a.head_w = L.head_w;
    a.head_b = L.head_b;
    a.feat = L.feat;
    a.err = L.err;
    const CUtensorMapDataType t16 =
        fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap tmW, tmX;
    const uint64_t rows = (uint64_t)L.m_total;
    if (!encode(&tmW, t16, 2, L.weight, (uint64_t)9 * L.cin, (uint64_t)kCo, kBK, kCo,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode(&tmX, t16, 2, L.in, (uint64_t)L.cin, rows, kBK, (uint32_t)(a.slab_rows / 2),
                CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    // Programmatic dependent launch: this kernel's CTAs may start (and run
    // their prologue) while the previous kernel in the stream drains; they
    // wait for its completion before touching activations (griddep_wait).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pix_smem_bytes(npx, L.g.rs);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const bool head = L.head_w != nullptr;
    auto fn = fp16 ? (head ? conv3x3_pix_kernel<true, true> : conv3x3_pix_kernel<true, false>)
                   : (head ? conv3x3_pix_kernel<false, true> : conv3x3_pix_kernel<false, false>);
    return cudaLaunchKernelEx(&cfg, fn, tmW, tmX, a);
}

}  // namespace mgb

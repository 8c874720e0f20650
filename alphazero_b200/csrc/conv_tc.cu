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
//   warp 0     TMA producer (one thread): two slab buffers and a
//              STAGES-deep ring of B stages;
//   warp 1     TMEM allocator and MMA issuer (one thread): 4 x
//              tcgen05.mma.kind::f16 (128 x bn x 16) per K block, fp32
//              accumulators in TMEM, double-buffered across tiles;
//   warps 2-9  epilogue: tcgen05.ld of the accumulator, folded-BN bias,
//              residual add (the stream is a 16-bit hi plane, the operand,
//              plus an fp16 remainder plane lo, both pixel-major), ReLU,
//              frame masking, the sum re-split into hi and lo and stored
//              with 16-byte accesses, and optionally the fused policy/value 1x1 head
//              projection (one thread owns one pixel row, so when a tile
//              spans all output channels it sees the whole channel vector).
// The epilogue of tile t overlaps the main loop of tile t+1.
// Every mbarrier wait is bounded (ptx_sm100.cuh); on expiry the kernel
// records an error code, drains its in-flight copies and frees TMEM.
#include "kernels.cuh"
#include "ptx_sm100.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <type_traits>

namespace mgb {
namespace {

constexpr int kBM = 128;  // rows per tile (TMEM lanes)
constexpr int kBK = 64;   // K elements per stage (128 bytes of 16-bit data)
constexpr int kThreads = 320;  // producer, MMA, 8 epilogue warps

template <int BN>
struct TcConfig {
    // 4 stages at BN 256 keep the kernel under 196 KB of shared memory, so
    // the carve-out leaves more L1 to the epilogue (measured 8% faster
    // than 5 stages on 19x19 b20c256 batch 1024).
    static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 8 : 12);
    static constexpr uint32_t kBBytes = BN * kBK * 2;
    static constexpr uint32_t kTmemCols = 2 * BN;
    // B ring + barriers and tmem slot (512) + bias (256 floats) + head weights
    // (3 x 256 floats) + head exchange (2 x 128 x 3 floats) + 1 KB alignment
    // slack; the two slabs come on top (slab_bytes).
    static constexpr int kSmemFixed = kStages * kBBytes + 512 + 1024 + 3072 + 3072 + 1024;
};

// Rows of an activation slab: the tile's 128 rows plus RS + 1 on each side,
// rounded up to 16.
__host__ __device__ constexpr int tc_slab_rows(int rs) { return (kBM + 2 * (rs + 1) + 15) / 16 * 16; }

struct TcArgs {
    int m_total;
    int num_tiles;
    int nsplit;  // cout / BN
    int cin;
    int cout;
    int rs, is, board;
    const float* bias;
    const uint16_t* res_hi;  // residual stream x = hi + lo, pixel-major [m_total][cout]
    const uint16_t* res_lo;
    uint16_t* out16;         // output hi plane (operand type) or nullptr
    uint16_t* out_lo;        // output lo plane (fp16 remainder) or nullptr
    const float* head_w;
    const float* head_b;
    float* feat;
    int* err;
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
    conv3x3_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB, const TcArgs a) {
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
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* tfull = bars + 2 * S;
    uint64_t* tempty = bars + 2 * S + 2;
    uint64_t* done = bars + 2 * S + 4;
    uint64_t* sfull = bars + 2 * S + 5;
    uint64_t* sempty = sfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sempty + 2);
    float* sbias = reinterpret_cast<float*>(tmem_slot + 4);
    float* shead = sbias + 256;  // [3][cout] fused head projection weights
    float* sxchg = shead + 768;  // [2][128][3] head partial-sum exchange

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_u32(&tfull[i]), 1);
            mbar_init(smem_u32(&tempty[i]), 8);
            mbar_init(smem_u32(&sfull[i]), 1);
            mbar_init(smem_u32(&sempty[i]), 1);
        }
        mbar_init(smem_u32(done), 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
        tmem_relinquish();
    }
    for (int i = threadIdx.x; i < a.cout; i += kThreads) sbias[i] = a.bias[i];
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

    const int cblocks = a.cin / kBK;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            prefetch_tensormap(&tmA);
            prefetch_tensormap(&tmB);
            int it = 0, is = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < a.num_tiles && ok; tile += gridDim.x) {
                const int mt = tile / a.nsplit;
                const int n0 = (tile - mt * a.nsplit) * BN;
                const int m0 = mt * kBM;
                for (int cb = 0; cb < cblocks && ok; ++cb, ++is) {
                    // the tile's halo slab of this channel block (rows before
                    // the first or past the last come back as zeros)
                    const int sb = is & 1;
                    if (!mbar_wait(smem_u32(&sempty[sb]), ((is >> 1) & 1) ^ 1, a.err,
                                   kErrWaitProducer)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(smem_u32(&sfull[sb]), slab_bytes);
                    tma_load_2d(smem_u32(sSlab + sb * slab_bytes), &tmA, smem_u32(&sfull[sb]),
                                cb * kBK, m0 - halo);
                    for (int tap = 0; tap < 9; ++tap, ++it) {
                        const int s = it % S;
                        const uint32_t ph = ((it / S) & 1) ^ 1;
                        if (!mbar_wait(smem_u32(&empty[s]), ph, a.err, kErrWaitProducer)) {
                            ok = false;
                            break;
                        }
                        const uint32_t fb = smem_u32(&full[s]);
                        mbar_arrive_expect_tx(fb, Cfg::kBBytes);
                        tma_load_2d(smem_u32(sB + s * Cfg::kBBytes), &tmB, fb,
                                    tap * a.cin + cb * kBK, n0);
                    }
                }
            }
            // Drain: every copy issued has landed before exit.
            for (int j = (it > S ? it - S : 0); j < it; ++j)
                mbar_wait(smem_u32(&full[j % S]), (j / S) & 1, a.err, kErrWaitDrain);
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
            for (int tile = blockIdx.x; tile < a.num_tiles && ok; tile += gridDim.x, ++t) {
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
        using T = typename P::T;
        int t = 0;
        for (int tile = blockIdx.x; tile < a.num_tiles; tile += gridDim.x, ++t) {
            const int mt = tile / a.nsplit;
            const int n0 = (tile - mt * a.nsplit) * BN;
            const int cbase = n0 + half * kCols;
            const int acc = t & 1;
            const int m = mt * kBM + row;
            const bool in_range = m < a.m_total;
            bool board_px = false;
            int pos = 0, pix = 0;
            if (in_range) {
                pos = m / a.is;
                const int q = m - pos * a.is;
                const int y = q / a.rs;
                const int x = q - y * a.rs;
                board_px = (y < a.board) && (x < a.board);
                pix = y * a.board + x;
            }
            const size_t off = (size_t)m * a.cout + cbase;
            const bool has_res = a.res_hi != nullptr && in_range;
            // The first chunk's residual (32 hi and 32 lo values, 4 + 4
            // 16-byte loads) is requested before the accumulator is ready;
            // each later chunk's one chunk ahead.  Ordinary L1-cached loads:
            // a lane's 16 bytes are half a sector whose other half the
            // next load reads (each row is read before it is overwritten in
            // place, and never read again by this kernel).
            uint4 rh[4], rl[4];
            if (has_res) {
                const uint4* ph = reinterpret_cast<const uint4*>(a.res_hi + off);
                const uint4* pl = reinterpret_cast<const uint4*>(a.res_lo + off);
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    rh[q4] = ph[q4];
                    rl[q4] = pl[q4];
                }
            }
            const bool ok = mbar_wait(smem_u32(&tfull[acc]), (t >> 1) & 1, a.err, kErrWaitEpilogue);
            // Leave together: no epilogue warp may be left at a named barrier.
            if (bar_any(1, 256, !ok)) break;
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
                if (!in_range) continue;
                float f[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]) + sbias[cbase + c0 + j];
                if (has_res) {
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const uint32_t hw4[4] = {rh[q4].x, rh[q4].y, rh[q4].z, rh[q4].w};
                        const uint32_t lw4[4] = {rl[q4].x, rl[q4].y, rl[q4].z, rl[q4].w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 hv = P::unpack(hw4[e]);
                            const float2 lv = __half22float2(*reinterpret_cast<const __half2*>(&lw4[e]));
                            f[q4 * 8 + 2 * e] += hv.x + lv.x;
                            f[q4 * 8 + 2 * e + 1] += hv.y + lv.y;
                        }
                    }
                    if (c + 1 < kChunks) {
                        const uint4* ph = reinterpret_cast<const uint4*>(a.res_hi + off + c0 + 32);
                        const uint4* pl = reinterpret_cast<const uint4*>(a.res_lo + off + c0 + 32);
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) {
                            rh[q4] = ph[q4];
                            rl[q4] = pl[q4];
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) f[j] = board_px ? fmaxf(f[j], 0.0f) : 0.0f;
                if (a.out16 != nullptr) {
                    uint4* oh = reinterpret_cast<uint4*>(a.out16 + off + c0);
                    uint4* ol = reinterpret_cast<uint4*>(a.out_lo + off + c0);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        uint32_t hw4[4], lw4[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float x0 = f[q4 * 8 + 2 * e], x1 = f[q4 * 8 + 2 * e + 1];
                            hw4[e] = P::pack(x0, x1);
                            const float2 hv = P::unpack(hw4[e]);
                            const __half2 lv = __floats2half2_rn(x0 - hv.x, x1 - hv.y);
                            lw4[e] = *reinterpret_cast<const uint32_t*>(&lv);
                        }
                        oh[q4] = make_uint4(hw4[0], hw4[1], hw4[2], hw4[3]);
                        if (a.out_lo != nullptr) ol[q4] = make_uint4(lw4[0], lw4[1], lw4[2], lw4[3]);
                    }
                }
                if (a.head_w != nullptr) {
                    const float* w0 = shead + cbase + c0;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        h0 = fmaf(f[j], w0[j], h0);
                        h1 = fmaf(f[j], w0[a.cout + j], h1);
                        h2 = fmaf(f[j], w0[2 * a.cout + j], h2);
                    }
                }
            }
            if (a.head_w != nullptr) {
                // Half 1 hands its partial sums to half 0 through a
                // double-buffered exchange (indexed by accumulator).
                float* xs = sxchg + acc * (kBM * 3) + row * 3;
                if (half == 1) {
                    xs[0] = h0;
                    xs[1] = h1;
                    xs[2] = h2;
                }
                named_barrier_sync(1, 256);
                if (half == 0 && board_px) {
                    const int hw = a.board * a.board;
                    float* fr = a.feat + (size_t)pos * 3 * hw;
                    fr[pix] = fmaxf(h0 + xs[0] + a.head_b[0], 0.f);
                    fr[hw + pix] = fmaxf(h1 + xs[1] + a.head_b[1], 0.f);
                    fr[2 * hw + pix] = fmaxf(h2 + xs[2] + a.head_b[2], 0.f);
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
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

template <int BN, bool FP16>
cudaError_t launch_bn(const ConvLayer& L, const CUtensorMap& tmA, const CUtensorMap& tmB,
                      int grid_limit, cudaStream_t stream) {
    using Cfg = TcConfig<BN>;
    // The fused head projection needs every output channel of a row in one tile.
    if (L.head_w != nullptr && L.cout != BN) return cudaErrorInvalidValue;
    TcArgs a;
    a.m_total = L.m_total;
    a.nsplit = L.cout / BN;
    a.num_tiles = ((L.m_total + kBM - 1) / kBM) * a.nsplit;
    a.cin = L.cin;
    a.cout = L.cout;
    a.rs = L.g.rs;
    a.is = L.g.is;
    a.board = L.g.board;
    a.bias = L.bias;
    // The residual stream is the hi / lo pair (16-bit operands only).
    if (L.res32 != nullptr || L.out32 != nullptr || (L.res_hi == nullptr) != (L.res_lo == nullptr) ||
        (L.out_lo != nullptr && L.out16 == nullptr))
        return cudaErrorInvalidValue;
    a.res_hi = static_cast<const uint16_t*>(L.res_hi);
    a.res_lo = L.res_lo;
    a.out16 = static_cast<uint16_t*>(L.out16);
    a.out_lo = L.out_lo;
    a.head_w = L.head_w;
    a.head_b = L.head_b;
    a.feat = L.feat;
    a.err = L.err;
    int grid = a.num_tiles < grid_limit ? a.num_tiles : grid_limit;
    if (grid < 1) grid = 1;
    // Programmatic dependent launch (see griddep_wait in the kernel).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)Cfg::kSmemFixed + 2 * tc_slab_rows(L.g.rs) * 128;
    if (cfg.dynamicSmemBytes > 227 * 1024 || tc_slab_rows(L.g.rs) > 256) return cudaErrorInvalidValue;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, conv3x3_tc_kernel<BN, FP16>, tmA, tmB, a);
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

bool encode_2d(CUtensorMap* map, bool fp16, const void* base, uint64_t inner, uint64_t rows,
               uint32_t box_inner, uint32_t box_rows, const char** why) {
    auto enc = tensor_map_encoder();
    if (enc == nullptr) {
        *why = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {inner * 2};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                     2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *why = "cuTensorMapEncodeTiled rejected the tensor map";
        return false;
    }
    return true;
}

template <int BN, bool FP16>
cudaError_t configure_one() {
    return cudaFuncSetAttribute(conv3x3_tc_kernel<BN, FP16>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

}  // namespace

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
    if (fp16) {
        switch (bn) {
            case 64: return launch_bn<64, true>(L, tmA, tmB, grid_limit, stream);
            case 128: return launch_bn<128, true>(L, tmA, tmB, grid_limit, stream);
            case 256: return launch_bn<256, true>(L, tmA, tmB, grid_limit, stream);
        }
    } else {
        switch (bn) {
            case 64: return launch_bn<64, false>(L, tmA, tmB, grid_limit, stream);
            case 128: return launch_bn<128, false>(L, tmA, tmB, grid_limit, stream);
            case 256: return launch_bn<256, false>(L, tmA, tmB, grid_limit, stream);
        }
    }
    return cudaErrorInvalidValue;
}

}  // namespace mgb

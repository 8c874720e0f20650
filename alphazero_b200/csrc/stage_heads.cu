// Input staging and the policy / value heads.
#include "kernels.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace mgb {
namespace {

__device__ __forceinline__ uint32_t pack2(float a, float b, ActType t) {
    if (t == ActType::BF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// One thread per (framed row, group of 8 channels): gathers up to 8 input
// planes of the row's pixel (strided across planes, coalesced across rows)
// and writes them as one 16-byte (16-bit types) or 32-byte (fp32) vector;
// channels >= planes, frame pixels and absent positions are zero.
// Frame geometry of a staging launch with the divisions by IS and RS done as
// multiply-shifts: n / d == (n * ceil(2^40 / d)) >> 40 for every row index
// below 2^23 and d <= 1200 (checked by the launchers).
struct StageGeom {
    FrameGeom g;
    uint64_t is_magic, rs_magic;
    int gshift;  // log2(cpad / 8)
};

StageGeom stage_geom(const FrameGeom& g, int cpad) {
    StageGeom s;
    s.g = g;
    s.is_magic = ((1ull << 40) + (uint64_t)g.is - 1) / (uint64_t)g.is;
    s.rs_magic = ((1ull << 40) + (uint64_t)g.rs - 1) / (uint64_t)g.rs;
    s.gshift = 0;
    while ((8 << s.gshift) < cpad) ++s.gshift;
    return s;
}

bool stage_geom_ok(const FrameGeom& g, int cpad, int rows) {
    return cpad >= 8 && (cpad & (cpad - 1)) == 0 && g.is <= 1200 && rows < (1 << 23);
}

__device__ __forceinline__ int stage_div(int n, uint64_t magic) {
    return (int)(((uint64_t)(uint32_t)n * magic) >> 40);
}

// Row m = idx >> gshift, channels [c8, c8 + 8) of a staging thread; returns
// false for a thread past the end.  Groups at or past `planes` only hold
// zeros and are written here without the frame arithmetic.
template <ActType T>
__device__ __forceinline__ bool stage_thread(const StageGeom& sg, int rows, int planes, int cpad,
                                             void* out, int& m, int& c8) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    m = idx >> sg.gshift;
    c8 = (idx - (m << sg.gshift)) * 8;
    if (m >= rows) return false;
    if (c8 >= planes) {
        if (T == ActType::FP32) {
            float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)m * cpad + c8);
            o[0] = make_float4(0.f, 0.f, 0.f, 0.f);
            o[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
            *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + (size_t)m * cpad + c8) =
                make_uint4(0u, 0u, 0u, 0u);
        }
        return false;
    }
    return true;
}

template <ActType T>
__global__ void stage_input_kernel(const float* __restrict__ states, int n_valid, int rows,
                                   int planes, StageGeom sg, int cpad, int eigen_order,
                                   void* __restrict__ out) {
    int m, c8;
    if (!stage_thread<T>(sg, rows, planes, cpad, out, m, c8)) return;
    const FrameGeom& g = sg.g;
    const int n = stage_div(m, sg.is_magic);
    const int q = m - n * g.is;
    const int y = stage_div(q, sg.rs_magic);
    const int x = q - y * g.rs;
    const bool live = (n < n_valid) && (y < g.board) && (x < g.board);
    const int hw = g.board * g.board;
    const int p = y * g.board + x;
    const float* s = states + (size_t)n * planes * hw;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int c = c8 + j;
        v[j] = (live && c < planes) ? (eigen_order ? s[c + (size_t)p * planes] : s[(size_t)c * hw + p])
                                    : 0.0f;
    }
    if (T == ActType::FP32) {
        float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)m * cpad + c8);
        o[0] = make_float4(v[0], v[1], v[2], v[3]);
        o[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint4 w;
        w.x = pack2(v[0], v[1], T);
        w.y = pack2(v[2], v[3], T);
        w.z = pack2(v[4], v[5], T);
        w.w = pack2(v[6], v[7], T);
        *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + (size_t)m * cpad + c8) = w;
    }
}

// As stage_input_kernel for bit-packed binary planes: position n's element
// j (plane-major, c*B*B + p) is bit (j & 31) of word j >> 5 of its
// words_per_pos words.
template <ActType T>
__global__ void stage_bits_kernel(const uint32_t* __restrict__ bits, int words_per_pos, int n_valid,
                                  int rows, int planes, StageGeom sg, int cpad, int eigen_order,
                                  void* __restrict__ out) {
    int m, c8;
    if (!stage_thread<T>(sg, rows, planes, cpad, out, m, c8)) return;
    const FrameGeom& g = sg.g;
    const int n = stage_div(m, sg.is_magic);
    const int q = m - n * g.is;
    const int y = stage_div(q, sg.rs_magic);
    const int x = q - y * g.rs;
    const bool live = (n < n_valid) && (y < g.board) && (x < g.board);
    const int hw = g.board * g.board;
    const int p = y * g.board + x;
    const uint32_t* w = bits + (size_t)n * words_per_pos;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int c = c8 + j;
        float val = 0.0f;
        if (live && c < planes) {
            const int e = eigen_order ? c + p * planes : c * hw + p;
            val = (float)((w[e >> 5] >> (e & 31)) & 1u);
        }
        v[j] = val;
    }
    if (T == ActType::FP32) {
        float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)m * cpad + c8);
        o[0] = make_float4(v[0], v[1], v[2], v[3]);
        o[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint4 wv;
        wv.x = pack2(v[0], v[1], T);
        wv.y = pack2(v[2], v[3], T);
        wv.z = pack2(v[4], v[5], T);
        wv.w = pack2(v[6], v[7], T);
        *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + (size_t)m * cpad + c8) = wv;
    }
}

// Value of input plane `plane` at board point `pt` of a position in the
// history wire format (kernels.cuh: launch_stage_history), computed as
// GoGame::encode writes it (src/game.cpp:229-256): planes 0-7 hold the
// stones of the player to move on the boards 0-7 moves back, planes 8-15
// the opponent's, plane 16 is all ones when black is to move.
__device__ __forceinline__ float history_plane_value(const uint32_t* w, int slot_words, uint32_t hdr,
                                                     int plane, int pt) {
    const uint32_t to_move = hdr & 3u;
    if (plane == 2 * kHistoryBoards) return to_move == 1u ? 1.0f : 0.0f;
    const int i = plane < kHistoryBoards ? plane : plane - kHistoryBoards;
    if (i >= (int)((hdr >> 4) & 15u)) return 0.0f;  // fewer boards played than i
    const int slot = ((int)((hdr >> 8) & 7u) - i) & (kHistoryBoards - 1);
    const uint32_t s = (w[1 + slot * slot_words + (pt >> 4)] >> (2 * (pt & 15))) & 3u;
    const uint32_t want = plane < kHistoryBoards ? to_move : 3u - to_move;
    return (s != 0u && s == want) ? 1.0f : 0.0f;
}

// As stage_input_kernel for the history wire format: position n's
// words_per_pos words are a header and the ring of its last 8 boards at 2
// bits per point; the planes are expanded here.
template <ActType T>
__global__ void stage_history_kernel(const uint32_t* __restrict__ hist, int words_per_pos,
                                     int slot_words, int n_valid, int rows, int planes, StageGeom sg,
                                     int cpad, int eigen_order, void* __restrict__ out) {
    int m, c8;
    if (!stage_thread<T>(sg, rows, planes, cpad, out, m, c8)) return;
    const FrameGeom& g = sg.g;
    const int n = stage_div(m, sg.is_magic);
    const int q = m - n * g.is;
    const int y = stage_div(q, sg.rs_magic);
    const int x = q - y * g.rs;
    const bool live = (n < n_valid) && (y < g.board) && (x < g.board);
    const int hw = g.board * g.board;
    const int p = y * g.board + x;
    const uint32_t* w = hist + (size_t)n * words_per_pos;
    const uint32_t hdr = live ? w[0] : 0u;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int c = c8 + j;
        float val = 0.0f;
        if (live && c < planes) {
            int plane = c, pt = p;
            if (eigen_order) {  // element (c, p) of the column-major reading
                const int e = c + p * planes;
                plane = e / hw;
                pt = e - plane * hw;
            }
            val = history_plane_value(w, slot_words, hdr, plane, pt);
        }
        v[j] = val;
    }
    if (T == ActType::FP32) {
        float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)m * cpad + c8);
        o[0] = make_float4(v[0], v[1], v[2], v[3]);
        o[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint4 wv;
        wv.x = pack2(v[0], v[1], T);
        wv.y = pack2(v[2], v[3], T);
        wv.z = pack2(v[4], v[5], T);
        wv.w = pack2(v[6], v[7], T);
        *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + (size_t)m * cpad + c8) = wv;
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// One warp per board pixel: the three 1x1 head convolutions over the fp32
// trunk row, lanes across channels.
__global__ void head_projection_kernel(const float* __restrict__ trunk, int positions, int c,
                                       FrameGeom g, const float* __restrict__ hw3,
                                       const float* __restrict__ hb, float* __restrict__ feat) {
    const int hw = g.board * g.board;
    const int job = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (job >= positions * hw) return;
    const int n = job / hw, p = job - n * hw;
    const int y = p / g.board, x = p - y * g.board;
    const float* t = trunk + ((size_t)n * g.is + (size_t)y * g.rs + x) * c;
    float d0 = 0.f, d1 = 0.f, d2 = 0.f;
    for (int ch = lane; ch < c; ch += 32) {
        const float v = t[ch];
        d0 = fmaf(v, hw3[ch], d0);
        d1 = fmaf(v, hw3[c + ch], d1);
        d2 = fmaf(v, hw3[2 * c + ch], d2);
    }
    d0 = warp_sum(d0);
    d1 = warp_sum(d1);
    d2 = warp_sum(d2);
    if (lane == 0) {
        float* fr = feat + (size_t)n * 3 * hw;
        fr[p] = fmaxf(d0 + hb[0], 0.f);
        fr[hw + p] = fmaxf(d1 + hb[1], 0.f);
        fr[2 * hw + p] = fmaxf(d2 + hb[2], 0.f);
    }
}

constexpr int kFcTN = 64;  // positions per tile
constexpr int kFcTO = 64;  // outputs per tile
constexpr int kFcTK = 32;  // K per shared-memory stage

// Partial sums of out[n][o] = sum_k feat[n][k] * W[o][k] over K slice
// blockIdx.z (of kHeadsFcSplits fixed slices) for a 64 x 64 tile; 256
// threads each own 4 positions x 4 outputs and read them from shared
// memory as float4s (2 shared loads per 16 FMAs).  K stages of 32 are
// double-buffered in shared memory while the next stage is fetched into
// registers (coalesced: a warp reads 32 consecutive k of one row).  Output
// tiles that lie wholly in the policy (o < actions) or value (o >= actions)
// rows only walk their own K block.  The slicing depends on nothing but
// the network, so a position's sums do not depend on the batch it is in.
__global__ void __launch_bounds__(256) heads_fc_kernel(const float* __restrict__ feat, HeadFc h,
                                                       int positions, float* __restrict__ out) {
    __shared__ __align__(16) float sF[2][kFcTK][kFcTN + 4];
    __shared__ __align__(16) float sW[2][kFcTK][kFcTO + 4];
    const int K = 3 * h.hw;
    const int O = h.actions + h.hidden;
    const int n0 = blockIdx.x * kFcTN;
    const int o0 = blockIdx.y * kFcTO;
    const int kb = (o0 >= h.actions) ? 2 * h.hw : 0;
    const int ke = (o0 + kFcTO <= h.actions) ? 2 * h.hw : K;
    const int slice = (ke - kb + kHeadsFcSplits - 1) / kHeadsFcSplits;
    const int kbeg = kb + blockIdx.z * slice;
    const int kend = min(ke, kbeg + slice);
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    // Each thread stages 8 feature and 8 weight values per stage: element
    // (row r = idx / 32, k = idx % 32) for idx = threadIdx.x + i * 256.
    float pF[8], pW[8];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = threadIdx.x + i * 256;
            const int r = idx >> 5, k = idx & 31;
            const int kk = k0 + k;
            const bool kin = kk < kend;
            const int n = n0 + r, o = o0 + r;
            pF[i] = (kin && n < positions) ? feat[(size_t)n * K + kk] : 0.f;
            pW[i] = (kin && o < O) ? h.w[(size_t)o * K + kk] : 0.f;
        }
    };
    auto stage = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = threadIdx.x + i * 256;
            const int r = idx >> 5, k = idx & 31;
            sF[buf][k][r] = pF[i];
            sW[buf][k][r] = pW[i];
        }
    };
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    int buf = 0;
    if (kbeg < kend) {
        fetch(kbeg);
        stage(0);
        __syncthreads();
    }
    for (int k0 = kbeg; k0 < kend; k0 += kFcTK, buf ^= 1) {
        const bool more = k0 + kFcTK < kend;
        if (more) fetch(k0 + kFcTK);
#pragma unroll 8
        for (int k = 0; k < kFcTK; ++k) {
            const float4 a = *reinterpret_cast<const float4*>(&sF[buf][k][ty * 4]);
            const float4 w = *reinterpret_cast<const float4*>(&sW[buf][k][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w}, wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
        }
        // The other buffer was last read in the previous stage, which every
        // thread has finished (the barrier at the end of that stage).
        if (more) stage(buf ^ 1);
        __syncthreads();
    }
    float* o_base = out + (size_t)blockIdx.z * positions * O;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int n = n0 + ty * 4 + i;
        if (n >= positions) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int o = o0 + tx * 4 + j;
            if (o < O) o_base[(size_t)n * O + o] = acc[i][j];
        }
    }
}

// One 128-thread block per position: the FC outputs (bias plus the K-slice
// partial sums, added in a fixed order), a max-subtracted softmax of the
// logits, and the value head's last two steps (ReLU of FC1, FC2, tanh).
constexpr int kFinishThreads = 128;

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
    v = is_max ? warp_max(v) : warp_sum(v);
    const int w = threadIdx.x >> 5;
    __syncthreads();  // red may still be read by the previous reduction
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    v = red[0];
#pragma unroll
    for (int i = 1; i < kFinishThreads / 32; ++i) v = is_max ? fmaxf(v, red[i]) : v + red[i];
    return v;
}

__global__ void __launch_bounds__(kFinishThreads)
    heads_finish_kernel(float* __restrict__ fc, HeadFc h, int positions, float* __restrict__ probs,
                        float* __restrict__ logits, float* __restrict__ value) {
    __shared__ float red[kFinishThreads / 32];
    const int n = blockIdx.x;
    const int A = h.actions, O = h.actions + h.hidden;
    // Finished outputs overwrite slice 0's row of this position.
    float* l = fc + (size_t)n * O;
    for (int o = threadIdx.x; o < O; o += kFinishThreads) {
        float x = h.b[o];
        for (int sl = 0; sl < kHeadsFcSplits; ++sl) x += fc[((size_t)sl * positions + n) * O + o];
        l[o] = x;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int a = threadIdx.x; a < A; a += kFinishThreads) mx = fmaxf(mx, l[a]);
    mx = block_reduce(mx, true, red);
    float sum = 0.f;
    for (int a = threadIdx.x; a < A; a += kFinishThreads) sum += expf(l[a] - mx);
    sum = block_reduce(sum, false, red);
    const float inv = 1.0f / sum;
    for (int a = threadIdx.x; a < A; a += kFinishThreads) {
        const float la = l[a];
        probs[(size_t)n * A + a] = expf(la - mx) * inv;
        logits[(size_t)n * A + a] = la;
    }
    float v = 0.f;
    for (int j = threadIdx.x; j < h.hidden; j += kFinishThreads)
        v = fmaf(fmaxf(l[A + j], 0.f), h.v2_w[j], v);
    v = block_reduce(v, false, red);
    if (threadIdx.x == 0) value[n] = tanhf(v + h.v2_b[0]);
}

}  // namespace

cudaError_t launch_stage_input(const float* states, int n_valid, int n_pos, int planes,
                               const FrameGeom& g, int cpad, bool eigen_order, ActType t,
                               void* out, cudaStream_t stream) {
    const long threads_total = (long)n_pos * g.is * (cpad / 8);
    const int threads = 256;
    const long blocks = (threads_total + threads - 1) / threads;
    if (blocks == 0) return cudaSuccess;
    const int rows = n_pos * g.is;
    if (!stage_geom_ok(g, cpad, rows)) return cudaErrorInvalidValue;
    const StageGeom sg = stage_geom(g, cpad);
    const int eo = eigen_order ? 1 : 0;
    switch (t) {
        case ActType::BF16:
            stage_input_kernel<ActType::BF16><<<(unsigned)blocks, threads, 0, stream>>>(
                states, n_valid, rows, planes, sg, cpad, eo, out);
            break;
        case ActType::FP16:
            stage_input_kernel<ActType::FP16><<<(unsigned)blocks, threads, 0, stream>>>(
                states, n_valid, rows, planes, sg, cpad, eo, out);
            break;
        case ActType::FP32:
            stage_input_kernel<ActType::FP32><<<(unsigned)blocks, threads, 0, stream>>>(
                states, n_valid, rows, planes, sg, cpad, eo, out);
            break;
    }
    return cudaGetLastError();
}

cudaError_t launch_stage_bits(const uint32_t* bits, int words_per_pos, int n_valid, int n_pos,
                              int planes, const FrameGeom& g, int cpad, bool eigen_order, ActType t,
                              void* out, cudaStream_t stream) {
    const long threads_total = (long)n_pos * g.is * (cpad / 8);
    const int threads = 256;
    const long blocks = (threads_total + threads - 1) / threads;
    if (blocks == 0) return cudaSuccess;
    const int rows = n_pos * g.is;
    if (!stage_geom_ok(g, cpad, rows)) return cudaErrorInvalidValue;
    const StageGeom sg = stage_geom(g, cpad);
    const int eo = eigen_order ? 1 : 0;
    switch (t) {
        case ActType::BF16:
            stage_bits_kernel<ActType::BF16><<<(unsigned)blocks, threads, 0, stream>>>(
                bits, words_per_pos, n_valid, rows, planes, sg, cpad, eo, out);
            break;
        case ActType::FP16:
            stage_bits_kernel<ActType::FP16><<<(unsigned)blocks, threads, 0, stream>>>(
                bits, words_per_pos, n_valid, rows, planes, sg, cpad, eo, out);
            break;
        case ActType::FP32:
            stage_bits_kernel<ActType::FP32><<<(unsigned)blocks, threads, 0, stream>>>(
                bits, words_per_pos, n_valid, rows, planes, sg, cpad, eo, out);
            break;
    }
    return cudaGetLastError();
}

cudaError_t launch_stage_history(const uint32_t* hist, int words_per_pos, int n_valid, int n_pos,
                                 const FrameGeom& g, int cpad, bool eigen_order, ActType t, void* out,
                                 cudaStream_t stream) {
    const int planes = 2 * kHistoryBoards + 1;
    const int slot_words = (g.board * g.board + 15) / 16;
    if (words_per_pos < 1 + kHistoryBoards * slot_words || cpad < planes) return cudaErrorInvalidValue;
    const long threads_total = (long)n_pos * g.is * (cpad / 8);
    const int threads = 256;
    const long blocks = (threads_total + threads - 1) / threads;
    if (blocks == 0) return cudaSuccess;
    const int rows = n_pos * g.is;
    if (!stage_geom_ok(g, cpad, rows)) return cudaErrorInvalidValue;
    const StageGeom sg = stage_geom(g, cpad);
    const int eo = eigen_order ? 1 : 0;
    switch (t) {
        case ActType::BF16:
            stage_history_kernel<ActType::BF16><<<(unsigned)blocks, threads, 0, stream>>>(
                hist, words_per_pos, slot_words, n_valid, rows, planes, sg, cpad, eo, out);
            break;
        case ActType::FP16:
            stage_history_kernel<ActType::FP16><<<(unsigned)blocks, threads, 0, stream>>>(
                hist, words_per_pos, slot_words, n_valid, rows, planes, sg, cpad, eo, out);
            break;
        case ActType::FP32:
            stage_history_kernel<ActType::FP32><<<(unsigned)blocks, threads, 0, stream>>>(
                hist, words_per_pos, slot_words, n_valid, rows, planes, sg, cpad, eo, out);
            break;
    }
    return cudaGetLastError();
}

cudaError_t launch_head_projection(const float* trunk, int positions, int c, const FrameGeom& g,
                                   const float* head_w, const float* head_b, float* feat,
                                   cudaStream_t stream) {
    const int jobs = positions * g.board * g.board;
    const int warps_per_block = 8;
    const int blocks = (jobs + warps_per_block - 1) / warps_per_block;
    if (blocks == 0) return cudaSuccess;
    head_projection_kernel<<<blocks, warps_per_block * 32, 0, stream>>>(trunk, positions, c, g,
                                                                        head_w, head_b, feat);
    return cudaGetLastError();
}

cudaError_t launch_heads_fc(const float* feat, const HeadFc& h, int positions, float* scratch,
                            float* probs, float* logits, float* value, cudaStream_t stream) {
    if (positions == 0) return cudaSuccess;
    dim3 grid((positions + kFcTN - 1) / kFcTN, (h.actions + h.hidden + kFcTO - 1) / kFcTO,
              kHeadsFcSplits);
    heads_fc_kernel<<<grid, 256, 0, stream>>>(feat, h, positions, scratch);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    heads_finish_kernel<<<positions, kFinishThreads, 0, stream>>>(scratch, h, positions, probs,
                                                                  logits, value);
    return cudaGetLastError();
}

}  // namespace mgb

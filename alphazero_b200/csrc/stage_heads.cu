// Input staging and the fused policy / value heads.
#include "kernels.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace mgb {
namespace {

template <typename T>
__device__ __forceinline__ T from_float(float v);
template <>
__device__ __forceinline__ float from_float<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_float<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_float(__half v) { return __half2float(v); }

// One thread per framed row: gathers the row's `planes` input values
// (strided across planes, coalesced across threads) and writes cpad
// channels, zero beyond `planes` and on frame pixels / absent positions.
template <typename T>
__global__ void stage_input_kernel(const float* __restrict__ states, int n_valid, int rows,
                                   int planes, FrameGeom g, int cpad, int eigen_order,
                                   T* __restrict__ out) {
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= rows) return;
    const int n = m / g.is;
    const int q = m - n * g.is;
    const int y = q / g.rs;
    const int x = q - y * g.rs;
    T* o = out + (size_t)m * cpad;
    const bool live = (n < n_valid) && (y < g.board) && (x < g.board);
    const int hw = g.board * g.board;
    const int p = y * g.board + x;
    const float* s = states + (size_t)n * planes * hw;
    for (int c = 0; c < cpad; ++c) {
        float v = 0.0f;
        if (live && c < planes) v = eigen_order ? s[c + (size_t)p * planes] : s[(size_t)c * hw + p];
        o[c] = from_float<T>(v);
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

constexpr int kHeadPos = 4;  // positions per CTA (shares the FC weight reads)
constexpr int kHeadWarps = 8;

// Fused heads for kHeadPos positions per CTA (src/eigen_engine.cpp:236-270):
//  1. policy 1x1 conv (c -> 2) and value 1x1 conv (c -> 1) with folded BN
//     and ReLU, one warp per pixel, lanes across channels;
//  2. policy FC (2*hw -> actions) and value FC1 (hw -> hidden) + ReLU, one
//     warp per output row, lanes across inputs, all positions of the CTA at
//     once so each weight row is read once per CTA;
//  3. per position: max-subtracted softmax over the logits, value FC2 and
//     tanh.  All arithmetic is fp32.
template <typename T>
__global__ void __launch_bounds__(kHeadWarps * 32)
    heads_kernel(const T* __restrict__ trunk, HeadParams h, int n_pos, float* __restrict__ probs,
                 float* __restrict__ logits, float* __restrict__ value) {
    extern __shared__ float sm[];
    const int c = h.c, hw = h.hw, A = h.actions, V = h.hidden;
    float* sw = sm;                         // 3*c
    float* pf = sw + 3 * c;                 // kHeadPos * 2*hw
    float* vf = pf + kHeadPos * 2 * hw;     // kHeadPos * hw
    float* lg = vf + kHeadPos * hw;         // kHeadPos * A
    float* hid = lg + kHeadPos * A;         // kHeadPos * V
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos0 = blockIdx.x * kHeadPos;

    for (int i = threadIdx.x; i < c; i += blockDim.x) {
        sw[i] = h.pconv_w[i];
        sw[c + i] = h.pconv_w[c + i];
        sw[2 * c + i] = h.vconv_w[i];
    }
    __syncthreads();

    const float pb0 = h.pconv_b[0], pb1 = h.pconv_b[1], vb = h.vconv_b[0];
    for (int job = warp; job < kHeadPos * hw; job += kHeadWarps) {
        const int pp = job / hw, p = job - pp * hw;
        const int n = pos0 + pp;
        float d0 = 0.f, d1 = 0.f, d2 = 0.f;
        if (n < n_pos) {
            const int y = p / h.board, x = p - y * h.board;
            const T* t = trunk + ((size_t)n * h.g.is + (size_t)y * h.g.rs + x) * c;
            for (int ch = lane; ch < c; ch += 32) {
                const float v = to_float(t[ch]);
                d0 = fmaf(v, sw[ch], d0);
                d1 = fmaf(v, sw[c + ch], d1);
                d2 = fmaf(v, sw[2 * c + ch], d2);
            }
        }
        d0 = warp_sum(d0);
        d1 = warp_sum(d1);
        d2 = warp_sum(d2);
        if (lane == 0) {
            pf[pp * 2 * hw + p] = fmaxf(d0 + pb0, 0.f);
            pf[pp * 2 * hw + hw + p] = fmaxf(d1 + pb1, 0.f);
            vf[pp * hw + p] = fmaxf(d2 + vb, 0.f);
        }
    }
    __syncthreads();

    for (int a = warp; a < A; a += kHeadWarps) {
        float acc[kHeadPos];
#pragma unroll
        for (int pp = 0; pp < kHeadPos; ++pp) acc[pp] = 0.f;
        const float* wr = h.pfc_w + (size_t)a * 2 * hw;
        for (int k = lane; k < 2 * hw; k += 32) {
            const float wv = wr[k];
#pragma unroll
            for (int pp = 0; pp < kHeadPos; ++pp) acc[pp] = fmaf(wv, pf[pp * 2 * hw + k], acc[pp]);
        }
#pragma unroll
        for (int pp = 0; pp < kHeadPos; ++pp) {
            const float s = warp_sum(acc[pp]);
            if (lane == 0) lg[pp * A + a] = s + h.pfc_b[a];
        }
    }
    for (int j = warp; j < V; j += kHeadWarps) {
        float acc[kHeadPos];
#pragma unroll
        for (int pp = 0; pp < kHeadPos; ++pp) acc[pp] = 0.f;
        const float* wr = h.v1_w + (size_t)j * hw;
        for (int k = lane; k < hw; k += 32) {
            const float wv = wr[k];
#pragma unroll
            for (int pp = 0; pp < kHeadPos; ++pp) acc[pp] = fmaf(wv, vf[pp * hw + k], acc[pp]);
        }
#pragma unroll
        for (int pp = 0; pp < kHeadPos; ++pp) {
            const float s = warp_sum(acc[pp]);
            if (lane == 0) hid[pp * V + j] = fmaxf(s + h.v1_b[j], 0.f);
        }
    }
    __syncthreads();

    for (int pp = warp; pp < kHeadPos; pp += kHeadWarps) {
        const int n = pos0 + pp;
        if (n >= n_pos) continue;
        const float* l = lg + pp * A;
        float mx = -INFINITY;
        for (int a = lane; a < A; a += 32) mx = fmaxf(mx, l[a]);
        mx = warp_max(mx);
        float sum = 0.f;
        for (int a = lane; a < A; a += 32) sum += expf(l[a] - mx);
        sum = warp_sum(sum);
        const float inv = 1.0f / sum;
        for (int a = lane; a < A; a += 32) {
            probs[(size_t)n * A + a] = expf(l[a] - mx) * inv;
            if (logits != nullptr) logits[(size_t)n * A + a] = l[a];
        }
        float v = 0.f;
        for (int j = lane; j < V; j += 32) v = fmaf(hid[pp * V + j], h.v2_w[j], v);
        v = warp_sum(v);
        if (lane == 0) value[n] = tanhf(v + h.v2_b[0]);
    }
}

}  // namespace

cudaError_t launch_stage_input(const float* states, int n_valid, int n_pos, int planes,
                               const FrameGeom& g, int cpad, bool eigen_order, ActType t,
                               void* out, cudaStream_t stream) {
    const int rows = n_pos * g.is;
    const int threads = 128;
    const int blocks = (rows + threads - 1) / threads;
    if (blocks == 0) return cudaSuccess;
    switch (t) {
        case ActType::BF16:
            stage_input_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(
                states, n_valid, rows, planes, g, cpad, eigen_order ? 1 : 0,
                reinterpret_cast<__nv_bfloat16*>(out));
            break;
        case ActType::FP16:
            stage_input_kernel<__half><<<blocks, threads, 0, stream>>>(
                states, n_valid, rows, planes, g, cpad, eigen_order ? 1 : 0,
                reinterpret_cast<__half*>(out));
            break;
        case ActType::FP32:
            stage_input_kernel<float><<<blocks, threads, 0, stream>>>(
                states, n_valid, rows, planes, g, cpad, eigen_order ? 1 : 0,
                reinterpret_cast<float*>(out));
            break;
    }
    return cudaGetLastError();
}

size_t heads_smem_bytes(const HeadParams& h) {
    return sizeof(float) *
           (size_t)(3 * h.c + kHeadPos * (2 * h.hw + h.hw + h.actions + h.hidden));
}

cudaError_t launch_heads(const void* trunk, ActType t, const HeadParams& h, int n_pos,
                         float* probs, float* logits, float* value, cudaStream_t stream) {
    const int blocks = (n_pos + kHeadPos - 1) / kHeadPos;
    if (blocks == 0) return cudaSuccess;
    const size_t smem = heads_smem_bytes(h);
    switch (t) {
        case ActType::BF16:
            heads_kernel<__nv_bfloat16><<<blocks, kHeadWarps * 32, smem, stream>>>(
                reinterpret_cast<const __nv_bfloat16*>(trunk), h, n_pos, probs, logits, value);
            break;
        case ActType::FP16:
            heads_kernel<__half><<<blocks, kHeadWarps * 32, smem, stream>>>(
                reinterpret_cast<const __half*>(trunk), h, n_pos, probs, logits, value);
            break;
        case ActType::FP32:
            heads_kernel<float><<<blocks, kHeadWarps * 32, smem, stream>>>(
                reinterpret_cast<const float*>(trunk), h, n_pos, probs, logits, value);
            break;
    }
    return cudaGetLastError();
}

}  // namespace mgb

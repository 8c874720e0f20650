// fp32 SIMT 3x3 convolution for the fp32 verification mode.
//
// Same framed-NHWC implicit GEMM as the tensor-core kernel (kernels.cuh),
// computed with fp32 FMAs: each 256-thread CTA owns 64 rows x 64 output
// channels and walks K = 9 taps x cin in slices of 16 channels staged in
// shared memory; each thread accumulates a 4 x 4 block.  It exists to meet an
// fp32-level tolerance against the CPU restatement of
// src/eigen_engine.cpp:174-194, not for speed.
#include "kernels.cuh"

namespace mgb {
namespace {

constexpr int kTileM = 64;
constexpr int kTileN = 64;
constexpr int kSliceK = 16;

__global__ void __launch_bounds__(256) conv3x3_simt_kernel(ConvLayer L) {
    __shared__ float sA[kSliceK][kTileM + 4];
    __shared__ float sB[kSliceK][kTileN + 4];
    const float* in = reinterpret_cast<const float*>(L.in);
    const float* w = reinterpret_cast<const float*>(L.weight);
    const int m0 = blockIdx.x * kTileM;
    const int n0 = blockIdx.y * kTileN;
    const int tx = threadIdx.x & 15;   // output-channel group
    const int ty = threadIdx.x >> 4;   // row group
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    for (int tap = 0; tap < 9; ++tap) {
        const int off = (tap / 3 - 1) * L.g.rs + (tap % 3 - 1);
        for (int c0 = 0; c0 < L.cin; c0 += kSliceK) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int idx = threadIdx.x + i * 256;
                const int r = idx >> 4, kk = idx & 15;
                const int src = m0 + r + off;
                sA[kk][r] = (src >= 0 && src < L.m_total) ? in[(size_t)src * L.cin + c0 + kk] : 0.0f;
                const int co = n0 + r;
                sB[kk][r] = (co < L.cout) ? w[((size_t)co * 9 + tap) * L.cin + c0 + kk] : 0.0f;
            }
            __syncthreads();
#pragma unroll
            for (int kk = 0; kk < kSliceK; ++kk) {
                float av[4], bv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) av[i] = sA[kk][ty * 4 + i];
#pragma unroll
                for (int j = 0; j < 4; ++j) bv[j] = sB[kk][tx * 4 + j];
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
            }
            __syncthreads();
        }
    }

    float* out = L.out32;
    const float* res = L.res32;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= L.m_total) continue;
        const int q = m % L.g.is;
        const int y = q / L.g.rs;
        const int x = q - y * L.g.rs;
        const bool board_px = (y < L.g.board) && (x < L.g.board);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int co = n0 + tx * 4 + j;
            if (co >= L.cout) continue;
            float v = acc[i][j] + L.bias[co];
            if (res != nullptr) v += res[(size_t)m * L.cout + co];
            out[(size_t)m * L.cout + co] = board_px ? fmaxf(v, 0.0f) : 0.0f;
        }
    }
}

}  // namespace

cudaError_t launch_conv_simt(const ConvLayer& L, cudaStream_t stream) {
    if (L.cin % kSliceK != 0) return cudaErrorInvalidValue;
    dim3 grid((L.m_total + kTileM - 1) / kTileM, (L.cout + kTileN - 1) / kTileN);
    conv3x3_simt_kernel<<<grid, 256, 0, stream>>>(L);
    return cudaGetLastError();
}

}  // namespace mgb

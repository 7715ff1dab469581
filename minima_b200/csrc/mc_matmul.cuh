// mc_matmul.cuh — the fp32 matrix product of forward.h's matmul
// (forward.c:24-40): out[i][j] = sum_k x[i][k] * w[j][k], k ascending, for
// any n, d_in, d_out.  A CTA computes a 64 x 64 output tile from 32-wide K
// tiles staged in shared memory; each thread holds a 4 x 4 block of
// outputs and accumulates with FMAs in K order (the reference multiplies
// and adds separately, so results agree to fp32 rounding, not bit for bit).
#pragma once

#include <cuda_runtime.h>

namespace mc {

constexpr int kMmTile = 64, kMmK = 32;

__global__ void __launch_bounds__(256) matmul_f32_kernel(const float* __restrict__ x,
                                                         const float* __restrict__ w,
                                                         float* __restrict__ out, int n, int d_in,
                                                         int d_out) {
    __shared__ float xs[kMmK][kMmTile + 1];
    __shared__ float ws[kMmK][kMmTile + 1];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int i0 = blockIdx.y * kMmTile, j0 = blockIdx.x * kMmTile;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < d_in; k0 += kMmK) {
        // 64 rows x 32 k of each operand: 8 elements per thread, k fastest
        for (int e = threadIdx.x; e < kMmTile * kMmK; e += 256) {
            const int r = e / kMmK, kk = e % kMmK, k = k0 + kk;
            xs[kk][r] = (i0 + r < n && k < d_in) ? x[(size_t)(i0 + r) * d_in + k] : 0.0f;
            ws[kk][r] = (j0 + r < d_out && k < d_in) ? w[(size_t)(j0 + r) * d_in + k] : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < kMmK; kk++) {
            float a[4], b[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                a[u] = xs[kk][ty * 4 + u];
                b[u] = ws[kk][tx * 4 + u];
            }
#pragma unroll
            for (int u = 0; u < 4; u++)
#pragma unroll
                for (int v = 0; v < 4; v++) acc[u][v] = fmaf(a[u], b[v], acc[u][v]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int i = i0 + ty * 4 + u;
        if (i >= n) continue;
#pragma unroll
        for (int v = 0; v < 4; v++) {
            const int j = j0 + tx * 4 + v;
            if (j < d_out) out[(size_t)i * d_out + j] = acc[u][v];
        }
    }
}

}  // namespace mc

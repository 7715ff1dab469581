// mc_checkpoint.cuh — device side of the checkpoint loader: each staged
// chunk of fp32 values is checked for non-finite entries (checkpoint_load
// rejects such files, checkpoint.c:403-405) and written to its model array,
// as fp32 or as bf16 (round to nearest even).  Moments are checked only.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace mc {

__global__ void __launch_bounds__(256) ckpt_ingest_kernel(const float* __restrict__ src, size_t n,
                                                          float* __restrict__ dst_f32,
                                                          __nv_bfloat16* __restrict__ dst_bf16,
                                                          unsigned* __restrict__ bad) {
    bool nonfinite = false;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float v = src[i];
        nonfinite |= !isfinite(v);
        if (dst_f32) dst_f32[i] = v;
        else if (dst_bf16) dst_bf16[i] = __float2bfloat16_rn(v);
    }
    if (__syncthreads_or(nonfinite) && threadIdx.x == 0) atomicAdd(bad, 1u);
}

}  // namespace mc

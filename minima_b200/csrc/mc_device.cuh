// mc_device.cuh — device helpers for the sm_100a decode token loop:
// grid-wide barrier with a %globaltimer deadline, warp/CTA reductions,
// 16-byte weight loads for fp32/bf16 rows, L2-only activation loads.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define MC_WARP 32
#define MC_MAX_TOPK_DEV 256

namespace mc {

// Device status word values (mirrors MC_* in minima_cuda.h).
enum : int { ST_OK = 0, ST_TIMEOUT = 4, ST_DEVICE = 5 };

// Paged KV cache (the reference's KVCache, generate.h:11-24, holds
// [layer][max_seq][kv_dim] per sequence).  Here the K and V pools are
// [n_pages][L][K][page_len][hd] fp32: a page holds page_len consecutive
// positions of one sequence for every layer and KV head, and a sequence's
// positions [i * page_len, (i + 1) * page_len) live in page table[b][i].
// page_len is a power of two and a multiple of 64, so every key run the
// attention kernels read (32 or 64 keys from a 64-aligned start) lies in
// one page; the cluster loop's bulk copies are split at page boundaries.
// A session without a page pool has the identity table (b * pps + i).
struct KvPages {
    const int* table;   // [Bcap][pps]
    int pps;            // table entries per sequence
    int shift;          // log2(page_len)
};
constexpr int kKvMinPageShift = 6;

// Row index (times head_dim: the element offset) of position t of
// (layer l, sequence b, KV head g).  t < pps << shift.
__device__ __forceinline__ size_t kv_row_at(int page, int shift, int L, int K, int l, int g, int t) {
    return ((((size_t)page * L + l) * K + g) << shift) + (size_t)(t & ((1 << shift) - 1));
}
__device__ __forceinline__ size_t kv_row(const KvPages& pg, int L, int K, int l, int b, int g, int t) {
    const int page = __ldg(pg.table + (size_t)b * pg.pps + (t >> pg.shift));
    return kv_row_at(page, pg.shift, L, K, l, g, t);
}

// Programmatic dependent launch (kernels launched with the programmatic
// stream serialization attribute): pdl_wait returns once the previous kernel
// in the stream has completed and its memory operations are visible (at
// once for an ordinary launch); pdl_trigger lets the next kernel's CTAs be
// scheduled.  Kernels call pdl_trigger only after pdl_wait, so the next
// kernel's work before its own pdl_wait overlaps this kernel alone and may
// read only what the kernels before this one wrote, or constant data.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add_u32(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_volatile_i32(const int* p) {
    return *reinterpret_cast<const volatile int*>(p);
}

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
    return *reinterpret_cast<const volatile unsigned long long*>(p);
}

// u16 written by another CTA in an earlier phase: read from L2.
__device__ __forceinline__ int ld_u16_cg(const uint16_t* p) {
    unsigned short v;
    asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return (int)v;
}

// Grid-wide barrier over a monotonically increasing arrival counter.
// Thread 0 of each CTA arrives (release) and spins (acquire) until every CTA
// of this epoch arrived.  The spin is bounded by a %globaltimer deadline: on
// expiry it records ST_TIMEOUT in *status and returns, so that a CTA that
// can never arrive makes the kernel exit instead of hang.  Returns false
// once *status is non-zero (every CTA then leaves the token loop).
struct GridSync {
    unsigned* counter;
    int* status;
    unsigned nblocks;
    unsigned epoch;
    unsigned long long timeout_ns;

    __device__ __forceinline__ bool sync() {
        __syncthreads();
        if (threadIdx.x == 0) {
            epoch++;
            const unsigned target = epoch * nblocks;
            __threadfence();
            red_release_add_u32(counter, 1u);
            const unsigned long long t0 = globaltimer_ns();
            unsigned spins = 0;
            while ((int)(ld_acquire_u32(counter) - target) < 0) {
                if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > timeout_ns) {
                    atomicMax(status, (int)ST_TIMEOUT);
                    break;
                }
            }
            __threadfence();
        }
        __syncthreads();
        return ld_volatile_i32(status) == ST_OK;
    }
};

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

// Ordering used by greedy selection (generate.c:447-460 with top_k == 1):
// larger value wins, equal values keep the lower id; NaN never wins.
__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
    if (va != va) return false;
    if (vb != vb) return true;
    return va > vb || (va == vb && ia < ib);
}

__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better(ov, oi, v, i)) { v = ov; i = oi; }
    }
}

// CTA-wide sum; `red` is >= 32 floats of shared scratch.  All threads get
// the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.0f;
    t = warp_sum(t);
    return t;
}

// Activations written by other CTAs in the previous phase are read from L2
// (ld.global.cg) so that no stale L1 line can be returned.
__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float4 ldcg4(const float* p) {
    return __ldcg(reinterpret_cast<const float4*>(p));
}

// ---- weight rows: VEC elements per 16-byte load ----
template <typename WT> struct WVec;
template <> struct WVec<float> {
    static constexpr int N = 4;
    __device__ __forceinline__ static void load(const float* p, float (&w)[4]) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(p));
        w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    }
};
template <> struct WVec<__nv_bfloat16> {
    static constexpr int N = 8;
    __device__ __forceinline__ static void load(const __nv_bfloat16* p, float (&w)[8]) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w[2 * i] = __uint_as_float(u[i] << 16);
            w[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
        }
    }
};

__device__ __forceinline__ float wload1(const float* p) { return __ldg(p); }
__device__ __forceinline__ float wload1(const __nv_bfloat16* p) {
    return __bfloat162float(__ldg(p));
}

}  // namespace mc

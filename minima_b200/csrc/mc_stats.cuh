// mc_stats.cuh — next-token distribution statistics on the device: the
// numbers generation_inspect_next_tokens prints (generate.c:291-388) from
// one row of logits, computed by a single 1024-thread CTA.
//
// The reference defines them over the "sampleable" ids (id >= 4, the
// reserved ids are masked to -inf): the maximum logit, the softmax
// denominator sum(exp(l - max)) and the entropy in bits, both in double
// precision, and the top_n (<= 20) ids by logit with ties going to the
// lower id (its insertion loop moves an entry up only past strictly smaller
// logits).  Any non-finite sampleable logit, or a denominator that is not
// positive and finite, rejects the row.
//
// Here every thread owns the ids tid, tid + 1024, ... (coalesced loads).
// The sums are reduced in a fixed tree (deterministic run to run; the
// reference sums id by id, so the last bits of the doubles can differ, far
// below the printed precision).  The top-n is found by n rounds of a block
// maximum over a 64-bit key that orders by logit and then by lower id
// (order-preserving bits of the float above, 2^32-1-id below); round r
// takes the largest key strictly below round r-1's, so no id is taken
// twice and no per-id state is kept.
#pragma once

#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>

#include "minima_cuda.h"

namespace mc {

constexpr int kStatsThreads = 1024;

__device__ __forceinline__ unsigned long long stats_key(float v, int id) {
    unsigned u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)id);
}

// Block-wide reductions over 1024 threads: a shuffle tree per warp, then
// warp 0 over the 32 warp results (fixed order, so deterministic).
template <typename T, typename Op>
__device__ T stats_reduce(T v, T* red, Op op) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = red[lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red[32] = v;
    }
    __syncthreads();
    const T r = red[32];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kStatsThreads)
next_token_stats_kernel(const float* __restrict__ logits, int V, int top_n,
                        mc_token_stats* __restrict__ out) {
    __shared__ double red_d[33];
    __shared__ float red_f[33];
    __shared__ unsigned long long red_k[33];
    __shared__ int red_i[33];
    const int tid = threadIdx.x;
    constexpr int kFirst = 4;    // tokenizer.h: ids 0..3 are reserved

    // max over the sampleable ids, and whether any of them is not finite
    float vmax = -INFINITY;
    int bad = 0;
    for (int id = kFirst + tid; id < V; id += kStatsThreads) {
        const float v = logits[id];
        if (!isfinite(v)) bad = 1;
        vmax = fmaxf(vmax, v);
    }
    bad = stats_reduce(bad, red_i, [](int a, int b) { return a | b; });
    vmax = stats_reduce(vmax, red_f, [](float a, float b) { return fmaxf(a, b); });
    if (bad) {
        if (tid == 0) out->status = 1;
        return;
    }
    const double m = (double)vmax;

    double s = 0.0;
    for (int id = kFirst + tid; id < V; id += kStatsThreads) s += exp((double)logits[id] - m);
    const double denom = stats_reduce(s, red_d, [](double a, double b) { return a + b; });
    if (!(denom > 0.0) || !isfinite(denom)) {
        if (tid == 0) out->status = 2;
        return;
    }

    const double ln2 = log(2.0);
    double h = 0.0;
    for (int id = kFirst + tid; id < V; id += kStatsThreads) {
        const double p = exp((double)logits[id] - m) / denom;
        if (p > 0.0) h -= p * (log(p) / ln2);
    }
    const double entropy = stats_reduce(h, red_d, [](double a, double b) { return a + b; });

    // top_n by (logit desc, id asc)
    __shared__ int top_ids[MC_STATS_MAX_TOP];
    __shared__ float top_logits[MC_STATS_MAX_TOP];
    unsigned long long below = ~0ull;
    int found = 0;
    for (int r = 0; r < top_n; r++) {
        unsigned long long best = 0;
        for (int id = kFirst + tid; id < V; id += kStatsThreads) {
            const unsigned long long k = stats_key(logits[id], id);
            if (k < below && k > best) best = k;
        }
        best = stats_reduce(best, red_k,
                            [](unsigned long long a, unsigned long long b) { return a > b ? a : b; });
        if (best == 0) break;                   // fewer sampleable ids than top_n
        if (tid == 0) {
            const int id = (int)(0xFFFFFFFFu - (unsigned)(best & 0xFFFFFFFFull));
            top_ids[r] = id;
            top_logits[r] = logits[id];
        }
        below = best;
        found++;
    }
    __syncthreads();
    if (tid == 0) {
        double cum = 0.0, top1 = 0.0, top5 = 0.0, top10 = 0.0;
        for (int i = 0; i < found; i++) {
            const double p = exp((double)top_logits[i] - m) / denom;
            out->ids[i] = top_ids[i];
            out->logits[i] = top_logits[i];
            out->probability[i] = p;
            cum += p;
            if (i == 0) top1 = cum;
            if (i == 4) top5 = cum;
            if (i == 9) top10 = cum;
        }
        out->found = found;
        out->max_logit = m;
        out->denominator = denom;
        out->entropy_bits = entropy;
        out->top1_mass = top1;
        out->top5_mass = top5;
        out->top10_mass = top10;
        out->status = 0;
    }
}

}  // namespace mc

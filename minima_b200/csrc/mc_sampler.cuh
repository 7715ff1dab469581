// mc_sampler.cuh — exact device restatement of the reference sampler
// sample_top_k_top_p (generate.c:414-516) for one sequence, run by one CTA.
//
// The value transform (penalties, no-repeat bans, temperature; generate.c:
// 438-446) and the tail (expf, min_p, top_p, the single rng_f32 draw;
// generate.c:480-515) use round-to-nearest intrinsics so that nvcc cannot
// contract them into FMAs: given the same logits, history and RNG state the
// result id and the RNG advance equal the reference's.
//
// Top-k (generate.c:447-468) is a streaming replace-min followed by a
// selection sort; with tied values its output order depends on the order in
// which candidates were inserted.  The fast path (radix select + bitonic
// sort) is taken only when the top-k values are pairwise distinct and
// strictly above the (k+1)-th value, where the reference's result is the
// unique descending order.  Otherwise the slow path replays the reference's
// streaming and sort exactly on one thread.
#pragma once

#include "mc_device.cuh"

namespace mc {

struct SamplingArgs {
    float temperature, top_p, rep, min_p, freq, pres;
    int top_k, min_new, ngram;
    const uint16_t* stop_ids;
    int stop_len;
    int pen_active;   // repetition_penalty > 1 || freq != 0 || pres != 0
};

// xorshift64* (util.c:11-27)
__device__ __forceinline__ unsigned long long rng_u64(unsigned long long& s) {
    unsigned long long x = s;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    s = x;
    return x * 0x2545F4914F6CDD1DULL;
}
__device__ __forceinline__ float rng_f32(unsigned long long& s) {
    return __fmul_rn((float)(rng_u64(s) >> 40), 1.0f / 16777216.0f);
}

// expf of the reference (glibc, ~correctly rounded): computed in double and
// rounded once to float.
__device__ __forceinline__ float exp_ref(float x) { return (float)exp((double)x); }

// Value transform of generate.c:439-446 for one id.
__device__ __forceinline__ float transform_value(float logit, unsigned count, bool banned,
                                                 const SamplingArgs& s) {
    float value = logit;
    if (s.pen_active && count > 0) {
        if (s.rep > 1.0f)
            value = value > 0.0f ? __fdiv_rn(value, s.rep) : __fmul_rn(value, s.rep);
        const float c = (float)(count < 65535u ? count : 65535u);
        value = __fsub_rn(value, __fadd_rn(__fmul_rn(s.freq, c), s.pres));
    }
    if (banned) value = -INFINITY;
    // x / 1 is x exactly (infinities and NaN included): skip the division
    return s.temperature == 1.0f ? value : __fdiv_rn(value, s.temperature);
}

__device__ __forceinline__ unsigned order_key(float v) {
    if (v == 0.0f) v = 0.0f;  // -0 and +0 compare equal in the reference
    const unsigned u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct SamplerSmem {
    float* vals;      // [V] transformed values
    float* kv;        // [256] top-k values
    int* ki;          // [256] top-k ids
    unsigned* hist;   // [256]
    int* misc;        // [8]
};

// Bytes of shared memory the sampler needs for a vocabulary of V.
__host__ __device__ inline size_t sampler_smem_bytes(int V) {
    return (size_t)V * 4 + 256 * 4 * 3 + 64;
}

__device__ __forceinline__ SamplerSmem sampler_carve(float* base, int V) {
    SamplerSmem s;
    s.vals = base;
    s.kv = base + V;
    s.ki = reinterpret_cast<int*>(s.kv + 256);
    s.hist = reinterpret_cast<unsigned*>(s.ki + 256);
    s.misc = reinterpret_cast<int*>(s.hist + 256);
    return s;
}

// Fill sm.vals with transformed values; returns (to all threads) whether any
// value is NaN.
__device__ bool sampler_fill(const float* logits, const unsigned* counts,
                             const unsigned* banned, bool use_bans, int V,
                             const SamplingArgs& s, SamplerSmem& sm) {
    if (threadIdx.x == 0) sm.misc[0] = 0;
    __syncthreads();
    int nan_seen = 0;
    if ((V & 3) == 0) {
        // four consecutive ids per load, eight loads per thread in flight
        constexpr int U = 8;
        const int V4 = V >> 2;
        for (int q0 = threadIdx.x; q0 < V4; q0 += U * blockDim.x) {
            float4 lg[U];
            uint4 c[U];
            unsigned w[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int q = q0 + u * blockDim.x;
                lg[u] = q < V4 ? ldcg4(logits + 4 * q) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                c[u] = s.pen_active && q < V4 ? __ldcg(reinterpret_cast<const uint4*>(counts) + q)
                                              : make_uint4(0u, 0u, 0u, 0u);
                w[u] = use_bans && q < V4 ? __ldcg(banned + ((4 * q) >> 5)) : 0u;
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int q = q0 + u * blockDim.x;
                if (q >= V4) break;
                const int i = 4 * q;
                float4 v;
                v.x = transform_value(lg[u].x, c[u].x, (w[u] >> (i & 31)) & 1u, s);
                v.y = transform_value(lg[u].y, c[u].y, (w[u] >> ((i + 1) & 31)) & 1u, s);
                v.z = transform_value(lg[u].z, c[u].z, (w[u] >> ((i + 2) & 31)) & 1u, s);
                v.w = transform_value(lg[u].w, c[u].w, (w[u] >> ((i + 3) & 31)) & 1u, s);
                *reinterpret_cast<float4*>(sm.vals + i) = v;
                nan_seen |= (v.x != v.x) | (v.y != v.y) | (v.z != v.z) | (v.w != v.w);
            }
        }
        return __syncthreads_or(nan_seen) != 0;
    }
    // eight elements per thread and round: their loads are all in flight
    // before the first is transformed
    constexpr int U = 8;
    for (int i0 = threadIdx.x; i0 < V; i0 += U * blockDim.x) {
        float lg[U];
        unsigned c[U], w[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int i = i0 + u * blockDim.x;
            lg[u] = i < V ? ldcg(logits + i) : 0.0f;
            c[u] = s.pen_active && i < V ? __ldcg(counts + i) : 0u;
            w[u] = use_bans && i < V ? __ldcg(banned + (i >> 5)) : 0u;
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int i = i0 + u * blockDim.x;
            if (i >= V) break;
            const float v = transform_value(lg[u], c[u], (w[u] >> (i & 31)) & 1u, s);
            sm.vals[i] = v;
            nan_seen |= (v != v);
        }
    }
    if (__syncthreads_or(nan_seen)) return true;
    return false;
}

// Exact replay of generate.c:447-468 on thread 0.  Leaves n entries in
// sm.kv/sm.ki in the reference's post-sort order.
__device__ void topk_replay(int V, int k, SamplerSmem& sm, int& n_out) {
    if (threadIdx.x == 0) {
        float* vals = sm.kv;
        int* idx = sm.ki;
        int n = 0, min_i = 0;
        for (int id = 0; id < V; ++id) {
            const float value = sm.vals[id];
            if (n < k) {
                idx[n] = id;
                vals[n] = value;
                ++n;
                if (n == k) {
                    min_i = 0;
                    for (int j = 1; j < n; ++j)
                        if (vals[j] < vals[min_i]) min_i = j;
                }
            } else if (value > vals[min_i]) {
                idx[min_i] = id;
                vals[min_i] = value;
                min_i = 0;
                for (int j = 1; j < n; ++j)
                    if (vals[j] < vals[min_i]) min_i = j;
            }
        }
        for (int i = 0; i < n; ++i)
            for (int j = i + 1; j < n; ++j)
                if (vals[j] > vals[i]) {
                    const float tv = vals[i]; vals[i] = vals[j]; vals[j] = tv;
                    const int ti = idx[i]; idx[i] = idx[j]; idx[j] = ti;
                }
        sm.misc[1] = n;
    }
    __syncthreads();
    n_out = sm.misc[1];
}

// Sort sm.kv/sm.ki[0, n) by value descending, then id ascending (bitonic,
// padded to the next power of two), and check the order is exact: the k
// first values distinct and, when n > k, strictly above the (k+1)-th.
__device__ bool topk_sort_check(int n, int k, SamplerSmem& sm) {
    int npad = 2;
    while (npad < n) npad <<= 1;
    for (int i = threadIdx.x + n; i < npad; i += blockDim.x) {
        sm.kv[i] = -INFINITY;
        sm.ki[i] = 0x7fffffff;
    }
    __syncthreads();
    for (int size = 2; size <= npad; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < npad; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned ki_ = order_key(sm.kv[i]), kj_ = order_key(sm.kv[j]);
                    const bool swap = desc ? (ki_ < kj_ || (ki_ == kj_ && sm.ki[i] > sm.ki[j]))
                                           : (ki_ > kj_ || (ki_ == kj_ && sm.ki[i] < sm.ki[j]));
                    if (swap) {
                        const float tv = sm.kv[i]; sm.kv[i] = sm.kv[j]; sm.kv[j] = tv;
                        const int ti = sm.ki[i]; sm.ki[i] = sm.ki[j]; sm.ki[j] = ti;
                    }
                }
            }
            __syncthreads();
        }
    }
    int dup = 0;
    for (int i = threadIdx.x; i < k && i + 1 < n; i += blockDim.x)
        dup |= (order_key(sm.kv[i]) == order_key(sm.kv[i + 1]));
    return !__syncthreads_or(dup);
}

// Exact top-k by radix select of the k-th largest key; succeeds only when
// the k largest values are distinct and strictly above the rest.  On
// success sm.kv/sm.ki hold them in descending order.
__device__ bool topk_radix(int V, int k, SamplerSmem& sm) {
    unsigned prefix = 0, mask = 0;
    int remaining = k;
    const int lane = threadIdx.x & 31;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) sm.hist[i] = 0;
        __syncthreads();
        // histogram of the next byte among keys under the prefix: the lanes
        // that share lane 0's byte add once (logits share their high bytes,
        // so plain per-key atomics would queue on a few bins)
        for (int i0 = 0; i0 < V; i0 += blockDim.x) {
            const int i = i0 + threadIdx.x;
            unsigned bin = 256u;                         // no bin
            if (i < V) {
                const unsigned key = order_key(sm.vals[i]);
                if ((key & mask) == prefix) bin = (key >> shift) & 255u;
            }
            const unsigned lead = __shfl_sync(0xffffffffu, bin, 0);
            const unsigned same = __ballot_sync(0xffffffffu, bin == lead);
            if (lane == 0 && lead < 256u) atomicAdd(&sm.hist[lead], (unsigned)__popc(same));
            if (bin != lead && bin < 256u) atomicAdd(&sm.hist[bin], 1u);
        }
        __syncthreads();
        // the first bin, from 255 down to 1, whose cumulative count reaches
        // `remaining` (else bin 0): warp 0, eight bins per lane, lane 0
        // holding the highest
        if (threadIdx.x < 32) {
            int c[8], tot = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                c[j] = (int)sm.hist[255 - 8 * lane - j];
                tot += c[j];
            }
            int incl = tot;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += y;
            }
            int cum = incl - tot, found = -1, rem = 0, before0 = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int bin = 255 - 8 * lane - j;
                if (bin == 0) before0 = cum;
                if (bin >= 1 && found < 0 && cum + c[j] >= remaining) {
                    found = bin;
                    rem = remaining - cum;
                }
                cum += c[j];
            }
            const unsigned hit = __ballot_sync(0xffffffffu, found >= 0);
            if (hit) {
                const int src = __ffs(hit) - 1;
                found = __shfl_sync(0xffffffffu, found, src);
                rem = __shfl_sync(0xffffffffu, rem, src);
            } else {
                found = 0;
                rem = remaining - __shfl_sync(0xffffffffu, before0, 31);
            }
            if (lane == 0) {
                sm.misc[2] = found;
                sm.misc[3] = rem;
            }
        }
        __syncthreads();
        prefix |= (unsigned)sm.misc[2] << shift;
        mask |= 255u << shift;
        remaining = sm.misc[3];
        __syncthreads();
    }
    // prefix = key of the k-th largest value; `remaining` of its copies are
    // needed.  Ties at the threshold beyond those make the order ambiguous.
    if (threadIdx.x == 0) { sm.misc[4] = 0; sm.misc[5] = 0; }
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const unsigned key = order_key(sm.vals[i]);
        if (key >= prefix) {
            const int slot = atomicAdd(&sm.misc[4], 1);
            if (slot < 256) { sm.ki[slot] = i; sm.kv[slot] = sm.vals[i]; }
        }
    }
    __syncthreads();
    const int cnt = sm.misc[4];
    if (cnt != k) return false;  // ties at the threshold
    return topk_sort_check(k, k, sm);
}

// Fast exact top-k.  The values are bucketed by their distance below the
// maximum (256 linear buckets spanning the finite range; bucket order is
// monotone in the value, so the first buckets holding k values contain the
// k largest); those candidates are collected and sorted.  More than 256
// candidates: the radix path.  Succeeds only when the k largest values are
// distinct and strictly above the rest; sm.kv/sm.ki then hold them in
// descending order.
__device__ bool topk_fast(int V, int k, SamplerSmem& sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    float mx = -INFINITY, mn = INFINITY;
    auto extent = [&](float v) {
        mx = fmaxf(mx, v);
        if (v != -INFINITY) mn = fminf(mn, v);
    };
    if ((V & 3) == 0) {
        for (int q = threadIdx.x; q < (V >> 2); q += blockDim.x) {
            const float4 v = *reinterpret_cast<const float4*>(sm.vals + 4 * q);
            extent(v.x); extent(v.y); extent(v.z); extent(v.w);
        }
    } else {
        for (int i = threadIdx.x; i < V; i += blockDim.x) extent(sm.vals[i]);
    }
    for (int off = 16; off > 0; off >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    }
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sm.hist[i] = 0;
    if (lane == 0) {
        sm.kv[warp] = mx;
        sm.kv[32 + warp] = mn;
    }
    if (threadIdx.x == 0) sm.misc[4] = 0;
    __syncthreads();
    mx = -INFINITY;
    mn = INFINITY;
    for (int w = 0; w < nw; w++) {
        mx = fmaxf(mx, sm.kv[w]);
        mn = fminf(mn, sm.kv[32 + w]);
    }
    __syncthreads();                                     // kv is reused below
    if (!(mx > mn) || !isfinite(mx) || !isfinite(mn)) return topk_radix(V, k, sm);
    const float sc = 256.0f / (mx - mn);
    auto bucket = [&](float v) -> int {
        const float d = mx - v;
        if (!(d > 0.0f)) return 0;
        const float f = d * sc;
        return f >= 255.0f ? 255 : (int)f;
    };
    if ((V & 3) == 0) {
        for (int q = threadIdx.x; q < (V >> 2); q += blockDim.x) {
            const float4 v = *reinterpret_cast<const float4*>(sm.vals + 4 * q);
            atomicAdd(&sm.hist[bucket(v.x)], 1u);
            atomicAdd(&sm.hist[bucket(v.y)], 1u);
            atomicAdd(&sm.hist[bucket(v.z)], 1u);
            atomicAdd(&sm.hist[bucket(v.w)], 1u);
        }
    } else {
        for (int i = threadIdx.x; i < V; i += blockDim.x) atomicAdd(&sm.hist[bucket(sm.vals[i])], 1u);
    }
    __syncthreads();
    // first bucket whose cumulative count reaches k: warp 0, eight per lane
    if (threadIdx.x < 32) {
        int c[8], tot = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            c[j] = (int)sm.hist[8 * lane + j];
            tot += c[j];
        }
        int incl = tot;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += y;
        }
        int cum = incl - tot, found = -1;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            cum += c[j];
            if (found < 0 && cum >= k) found = 8 * lane + j;
        }
        const unsigned hit = __ballot_sync(0xffffffffu, found >= 0);
        const int bmax = hit ? __shfl_sync(0xffffffffu, found, __ffs(hit) - 1) : 255;
        if (lane == 0) sm.misc[5] = bmax;
    }
    __syncthreads();
    const int bmax = sm.misc[5];
    // collect the candidates (a warp reserves its slots at once)
    for (int i0 = 0; i0 < V; i0 += blockDim.x) {
        const int i = i0 + threadIdx.x;
        const bool take = i < V && bucket(sm.vals[i]) <= bmax;
        const unsigned bal = __ballot_sync(0xffffffffu, take);
        int base = 0;
        if (lane == 0 && bal) base = atomicAdd(&sm.misc[4], __popc(bal));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (take) {
            const int slot = base + __popc(bal & ((1u << lane) - 1u));
            if (slot < 256) {
                sm.kv[slot] = sm.vals[i];
                sm.ki[slot] = i;
            }
        }
    }
    __syncthreads();
    const int cnt = sm.misc[4];
    if (cnt > 256) return topk_radix(V, k, sm);
    return topk_sort_check(cnt, k, sm);
}

// Tail of generate.c:469-515 on thread 0.  Returns the id; advances rng
// exactly when the reference draws.
__device__ int sampler_tail(int n, const SamplingArgs& s, SamplerSmem& sm,
                            unsigned long long& rng, bool& retry_without_bans,
                            bool bans_active) {
    retry_without_bans = false;
    const float* vals = sm.kv;
    const int* idx = sm.ki;
    if (n == 0) return 0;
    if (!isfinite(vals[0])) {
        if (bans_active) { retry_without_bans = true; return -1; }
        return idx[0];
    }
    float probs[MC_MAX_TOPK_DEV];
    const float maxv = vals[0];
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        probs[i] = exp_ref(__fsub_rn(vals[i], maxv));
        sum = __fadd_rn(sum, probs[i]);
    }
    if (!(sum > 0.0f) || !isfinite(sum)) return idx[0];
    if (s.min_p > 0.0f) {
        const float min_probability = __fmul_rn(__fdiv_rn(probs[0], sum), s.min_p);
        int keep = 1;
        for (int i = 1; i < n; ++i) {
            if (__fdiv_rn(probs[i], sum) < min_probability) break;
            ++keep;
        }
        n = keep;
        sum = 0.0f;
        for (int i = 0; i < n; ++i) sum = __fadd_rn(sum, probs[i]);
    }
    if (s.top_p < 1.0f) {
        float cumulative = 0.0f;
        int keep = 0;
        for (int i = 0; i < n; ++i) {
            cumulative = __fadd_rn(cumulative, __fdiv_rn(probs[i], sum));
            ++keep;
            if (cumulative >= s.top_p) break;
        }
        n = keep;
    }
    sum = 0.0f;
    for (int i = 0; i < n; ++i) sum = __fadd_rn(sum, probs[i]);
    float draw = __fmul_rn(rng_f32(rng), sum);
    for (int i = 0; i < n; ++i) {
        draw = __fsub_rn(draw, probs[i]);
        if (draw <= 0.0f) return idx[i];
    }
    return idx[n - 1];
}

}  // namespace mc

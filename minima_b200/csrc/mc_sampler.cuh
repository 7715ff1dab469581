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
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float lg = ldcg(logits + i);
        const unsigned c = s.pen_active ? __ldcg(counts + i) : 0u;
        const bool ban = use_bans && ((__ldcg(banned + (i >> 5)) >> (i & 31)) & 1u);
        const float v = transform_value(lg, c, ban, s);
        sm.vals[i] = v;
        nan_seen |= (v != v);
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

// Fast exact top-k: radix-select the k-th largest key; succeed only when the
// k largest values are distinct and strictly above the rest.  On success
// sm.kv/sm.ki hold them in descending order and the function returns true.
__device__ bool topk_fast(int V, int k, SamplerSmem& sm) {
    unsigned prefix = 0, mask = 0;
    int remaining = k;
    const int lane = threadIdx.x & 31;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) sm.hist[i] = 0;
        __syncthreads();
        // histogram of the next byte among keys under the prefix: lanes with
        // the same byte add once (logits share their high bytes, so plain
        // per-key atomics would queue on a few bins)
        for (int i0 = 0; i0 < V; i0 += blockDim.x) {
            const int i = i0 + threadIdx.x;
            unsigned bin = 256u;                         // no bin
            if (i < V) {
                const unsigned key = order_key(sm.vals[i]);
                if ((key & mask) == prefix) bin = (key >> shift) & 255u;
            }
            const unsigned peers = __match_any_sync(0xffffffffu, bin);
            if (bin < 256u && lane == __ffs(peers) - 1) atomicAdd(&sm.hist[bin], (unsigned)__popc(peers));
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
    // bitonic sort of the k entries padded to the next power of two
    int npad = 2;
    while (npad < k) npad <<= 1;
    for (int i = threadIdx.x + k; i < npad; i += blockDim.x) {
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
    for (int i = threadIdx.x; i + 1 < k; i += blockDim.x)
        dup |= (order_key(sm.kv[i]) == order_key(sm.kv[i + 1]));
    return !__syncthreads_or(dup);
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

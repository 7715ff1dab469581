// mc_batched.cuh — batched decode step on the tensor cores (B >= 32 is the
// intended use; MINIMA_CUDA_DECODE=tcgen05 selects it).
//
// The grid-barrier loop runs each layer's matvecs for at most 8 sequences
// per pass over the weights, so a large batch repeats its weight reads and
// its latency chain per chunk of 8.  Here one decode step is a sequence of
// kernels in which every matrix product covers the whole batch as one GEMM
// on tcgen05 (mc_tcgen05.cuh, rows = sequences, fused decode epilogues):
//
//   lists (who runs, ids fed at position t)
//   per layer: norm -> QKV GEMM (+RoPE, K/V append) -> attention (the grid
//              loop's phase_att) -> proj GEMM (+residual) -> norm ->
//              up/gate GEMM (+SwiGLU) -> down GEMM (+residual)
//   final norm -> lm_head GEMM -> reserved-id mask + greedy partials ->
//   sampler and bookkeeping (the grid loop's phase_sample)
//
// The step's position lives in device memory (lists[2]), so every step
// launches the same kernels with the same arguments.
#pragma once

#include "mc_token_loop.cuh"

namespace mc {

// lists layout (ints): [0] nf, [1] nh, [2] t, [3] spare, then fwd[Bcap],
// head[Bcap], act_fwd[Bcap], act_head[Bcap], tok[Bcap]
__host__ __device__ inline size_t bd_lists_ints(int Bcap) { return 4 + 5 * (size_t)Bcap; }
struct BdLists {
    int* base;
    int Bcap;
    __device__ int* fwd() const { return base + 4; }
    __device__ int* head() const { return base + 4 + Bcap; }
    __device__ int* act_fwd() const { return base + 4 + 2 * Bcap; }
    __device__ int* act_head() const { return base + 4 + 3 * Bcap; }
    __device__ int* tok() const { return base + 4 + 4 * Bcap; }
};

// Sequences that run a forward at the current position and those that
// sample after it (the token loop's step lists), the ids they feed, and the
// position itself (first call: t0; then one more per call).
template <typename WT>
__global__ void __launch_bounds__(1024) bd_lists_kernel(const LoopParams<WT> p, BdLists L, int first) {
    __shared__ int flag[1024];
    const int t = first ? p.t0 : L.base[2] + 1;
    __syncthreads();                     // every thread has read the previous position
    // a thread per sequence: does it run a forward, does it sample, which id
    for (int b = threadIdx.x; b < p.B; b += blockDim.x) {
        const SeqState* st = p.seq + b;
        int f = 0;
        if (!st->done) {
            const int P = st->P, nnew = st->nnew;
            if (t < P + nnew - 1) {
                f = 1 | (t >= P - 1 ? 2 : 0);
                int tok = t < P ? (int)p.prompts[(size_t)b * p.prompt_stride + t] : st->tok;
                if (tok < 0 || tok >= p.V) {
                    atomicMax(p.status, (int)ST_DEVICE);
                    tok = 0;
                }
                L.tok()[b] = tok;
            }
        }
        L.act_fwd()[b] = f & 1;
        L.act_head()[b] = (f >> 1) & 1;
        if (b < 1024) flag[b] = f;
    }
    __syncthreads();
    if (threadIdx.x == 0) {              // compact, in sequence order
        int nf = 0, nh = 0;
        for (int b = 0; b < p.B; b++) {
            const int f = b < 1024 ? flag[b] : (L.act_fwd()[b] | (L.act_head()[b] << 1));
            if (f & 1) L.fwd()[nf++] = b;
            if (f & 2) L.head()[nh++] = b;
        }
        L.base[0] = nf;
        L.base[1] = nh;
        L.base[2] = t;
        if (p.stamps && t < p.T) p.stamps[t] = globaltimer_ns();
    }
}

// xn[b] = rmsnorm(x[b]) * scale (generate.c:57-63) for the listed sequences,
// plus a bf16 copy when xn16 is set; with embed, x[b] is first set to the
// embedding row of the id fed (generate.c:86-88).  One CTA per sequence.
template <typename WT>
__global__ void __launch_bounds__(kThreads) bd_norm_kernel(const LoopParams<WT> p, BdLists L, int head,
                                                           const float* scale, int embed, float* xn,
                                                           __nv_bfloat16* xn16) {
    __shared__ float red[32];
    const int b = blockIdx.x;
    if (b >= p.B || !(head ? L.act_head() : L.act_fwd())[b]) return;
    float* x = p.x + (size_t)b * p.D;
    if (embed) {
        const int tok = L.tok()[b];
        for (int k = threadIdx.x; k < p.D; k += blockDim.x) x[k] = wload1(p.tok_emb + (size_t)tok * p.D + k);
        __syncthreads();
    }
    float ss = 0.0f;
    for (int k = threadIdx.x; k < p.D; k += blockDim.x) ss += x[k] * x[k];
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)p.D + 1e-5f);
    for (int k = threadIdx.x; k < p.D; k += blockDim.x) {
        const float v = x[k] * inv * scale[k];
        xn[(size_t)b * p.D + k] = v;
        if (xn16) xn16[(size_t)b * p.D + k] = __float2bfloat16_rn(v);
    }
}

__device__ inline LoopSmem bd_smem(float* smem_f, int Bcap) {
    LoopSmem sm;
    sm.red = smem_f;
    sm.fwd = reinterpret_cast<int*>(smem_f + 64);
    sm.head = sm.fwd + Bcap;
    sm.ints = sm.head + Bcap;
    sm.xs = smem_f + loop_fixed_bytes(Bcap) / 4;
    return sm;
}

// Attention of the listed sequences at position t (the token loop's phase).
template <typename WT>
__global__ void __launch_bounds__(kThreads, 1) bd_att_kernel(const LoopParams<WT> p, BdLists L, int l) {
    extern __shared__ __align__(16) float smem_f[];
    LoopSmem sm = bd_smem(smem_f, p.Bcap);
    const int nf = L.base[0], t = L.base[2];
    for (int i = threadIdx.x; i < nf; i += blockDim.x) sm.fwd[i] = L.fwd()[i];
    __syncthreads();
    if (nf == 0) return;
    phase_att<WT>(p, l, t, sm, nf);
}

// bf16 copy of the attention output of the listed sequences (the A operand
// of a kind::f16 proj GEMM).
template <typename WT>
__global__ void __launch_bounds__(kThreads) bd_cvt_kernel(const LoopParams<WT> p, BdLists L, __nv_bfloat16* dst) {
    const int b = blockIdx.x;
    if (b >= p.B || !L.act_fwd()[b]) return;
    for (int k = threadIdx.x; k < p.D; k += blockDim.x)
        dst[(size_t)b * p.D + k] = __float2bfloat16_rn(p.att[(size_t)b * p.D + k]);
}

// After the lm_head GEMM: ids 0..3 masked (generate.c:580-581) and, for
// greedy sampling, each CTA's best transformed value over its share of the
// vocabulary (generate.c:438-460), the partials phase_sample reduces.
template <typename WT>
__global__ void __launch_bounds__(kThreads) bd_head_kernel(const LoopParams<WT> p, BdLists L) {
    const int nh = L.base[1];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int per = (p.V + gridDim.x - 1) / gridDim.x;
    const int v0 = min(p.V, blockIdx.x * per), v1 = min(p.V, v0 + per);
    const int nwords = (p.V + 31) >> 5;
    const bool greedy = p.s.top_k == 1;
    // a warp per head sequence over this CTA's share of the vocabulary
    for (int i = warp; i < nh; i += kWarps) {
        const int b = L.head()[i];
        float* lg = p.logits + (size_t)b * p.V;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int v = v0 + lane; v < v1; v += 32) {
            float x = lg[v];
            if (v < 4) {
                x = -INFINITY;
                lg[v] = x;
            }
            if (greedy) {
                const unsigned cnt = p.s.pen_active ? p.counts[(size_t)b * p.V + v] : 0u;
                const bool ban = p.s.ngram > 0 && ((p.banned[(size_t)b * nwords + (v >> 5)] >> (v & 31)) & 1u);
                const float tv = transform_value(x, cnt, ban, p.s);
                if (better(tv, v, bv, bi)) { bv = tv; bi = v; }
            }
        }
        if (!greedy) continue;
        warp_argmax(bv, bi);
        if (lane == 0) {
            p.amax_v[(size_t)b * gridDim.x + blockIdx.x] = bv;
            p.amax_i[(size_t)b * gridDim.x + blockIdx.x] = bi;
        }
    }
}

// Sampling and bookkeeping of the head sequences (the token loop's phase).
template <typename WT>
__global__ void __launch_bounds__(kThreads, 1) bd_sample_kernel(const LoopParams<WT> p, BdLists L) {
    extern __shared__ __align__(16) float smem_f[];
    LoopSmem sm = bd_smem(smem_f, p.Bcap);
    const int nh = L.base[1], t = L.base[2];
    for (int i = threadIdx.x; i < nh; i += blockDim.x) sm.head[i] = L.head()[i];
    __syncthreads();
    if (nh > 0) phase_sample<WT>(p, t, sm, nh);
    if (p.stamps && t + 1 == p.T && blockIdx.x == 0 && threadIdx.x == 0) p.stamps[p.T] = globaltimer_ns();
}

template <typename WT>
__global__ void __launch_bounds__(kThreads) bd_prologue_kernel(const LoopParams<WT> p) {
    loop_prologue(p);
}

}  // namespace mc

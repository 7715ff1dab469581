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
//   final norm -> lm_head GEMM (+ reserved-id mask and greedy partials) ->
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
    pdl_wait();
    pdl_trigger();
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

constexpr int kBdMaxParts = 16;              // K-slice partials of a decode GEMM
constexpr int kBdNormCols = 4;               // float4 columns per norm thread (D <= 16 * kThreads)

// The bf16 operands of the kind::f16 decode GEMMs carry each fp32
// activation as two bf16 numbers, hi = bf16(v) and lo = bf16(v - hi), in
// rows b and Bcap + b of the same buffer; the GEMM multiplies both by the
// weight tile into one accumulator, so the activation keeps ~16 significant
// bits instead of 8 (the error of a single bf16 copy, compounded over 24
// layers, moved config 4's logits by ~3e-2).
__device__ __forceinline__ void bf16_split_store(__nv_bfloat16* hi, size_t lo_off, float v) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[0] = h;
    hi[lo_off] = __float2bfloat16_rn(v - __bfloat162float(h));
}

// An attention output element: fp32 for the next kernels, and its bf16
// hi/lo pair when the proj GEMM takes bf16 operands (att16 set).
template <typename WT>
__device__ __forceinline__ void att_store(const LoopParams<WT>& p, __nv_bfloat16* att16, size_t i, float v) {
    p.att[i] = v;
    if (att16) bf16_split_store(att16 + i, (size_t)p.Bcap * p.D, v);
}

// xn[b] = rmsnorm(x[b]) * scale (generate.c:57-63) for the listed sequences,
// plus its bf16 hi/lo pair when xn16 is set.  With embed, x[b] is first set to the
// embedding row of the id fed (generate.c:86-88); with nparts > 0, the
// K-slice partials of the residual GEMM before it are first added to x[b]
// in slice order (part + (s * B + b) * D).  One CTA per sequence; a thread
// keeps its float4 columns in registers and issues all partial loads of a
// column before adding them.
template <typename WT>
__global__ void __launch_bounds__(kThreads) bd_norm_kernel(const LoopParams<WT> p, BdLists L, int head,
                                                           const float* scale, int embed, float* xn,
                                                           __nv_bfloat16* xn16, const float* part,
                                                           int nparts) {
    __shared__ float red[32];
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.x;
    if (b >= p.B || !(head ? L.act_head() : L.act_fwd())[b]) return;
    float* x = p.x + (size_t)b * p.D;
    const int nv = p.D >> 2;
    float4 keep[kBdNormCols];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kBdNormCols; i++) {
        const int c = threadIdx.x + i * blockDim.x;
        keep[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (c >= nv) continue;
        float4 v;
        if (embed) {
            const WT* e = p.tok_emb + (size_t)L.tok()[b] * p.D + 4 * c;
            v = make_float4(wload1(e), wload1(e + 1), wload1(e + 2), wload1(e + 3));
        } else {
            v = ldcg4(x + 4 * c);
            float4 r[kBdMaxParts];
#pragma unroll
            for (int s = 0; s < kBdMaxParts; s++)
                r[s] = s < nparts ? ldcg4(part + ((size_t)s * p.B + b) * p.D + 4 * c)
                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int s = 0; s < kBdMaxParts; s++)
                if (s < nparts) {
                    a.x += r[s].x; a.y += r[s].y; a.z += r[s].z; a.w += r[s].w;
                }
            v.x += a.x; v.y += a.y; v.z += a.z; v.w += a.w;
        }
        if (embed || nparts > 0) *reinterpret_cast<float4*>(x + 4 * c) = v;
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        keep[i] = v;
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)p.D + 1e-5f);
#pragma unroll
    for (int i = 0; i < kBdNormCols; i++) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c >= nv) continue;
        const float4 sc4 = *reinterpret_cast<const float4*>(scale + 4 * c);
        const float4 v = make_float4(keep[i].x * inv * sc4.x, keep[i].y * inv * sc4.y, keep[i].z * inv * sc4.z,
                                     keep[i].w * inv * sc4.w);
        *reinterpret_cast<float4*>(xn + (size_t)b * p.D + 4 * c) = v;
        if (xn16) {
            __nv_bfloat16* o = xn16 + (size_t)b * p.D + 4 * c;
            const size_t lo = (size_t)p.Bcap * p.D;
            bf16_split_store(o, lo, v.x);
            bf16_split_store(o + 1, lo, v.y);
            bf16_split_store(o + 2, lo, v.z);
            bf16_split_store(o + 3, lo, v.w);
        }
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

// Attention of the running sequences at position t (generate.c:122-160).
// One CTA per (sequence, KV head, key split) — a split is klen keys, and a
// (sequence, KV head) has one split unless there are too few pairs to fill
// the GPU.  The split's keys stream through shared memory in tiles of
// kBdTile rows through a ring of kBdRing buffers filled by cp.async (the
// next tiles' K and V rows are in flight while one is scored), and each of
// the G query heads
// keeps an online softmax (running max, sum and P.V rows).  With several
// splits the last one to finish merges the partial states (flash-decoding).
// The unit comes from blockIdx directly; sequences that do not run at t
// return before writing anything.
// With nq > 0 the QKV GEMM left nq K-slice partials of each sequence's
// [q | k | v] row in qkvp (slice r at qkvp + r * B * Q): every unit sums the
// partials of its queries and rotates them (RoPE, rotary.h:26-40), and the
// unit holding key t also builds that key's K (rotated) and V rows, appends
// them to the cache (generate.c:108-120) and places them in its last tile.
constexpr int kBdAttThreads = 128;
constexpr int kBdTile = 64;                  // keys per shared-memory tile
constexpr int kBdRing = 2;                   // tiles in the ring
constexpr int kBdAttMaxO = 4;                // P.V outputs per thread (G * hd <= 512)

// [flag, pad x3] then K, V [kBdRing][kBdTile][hd], q [G][hd], probabilities
// [G][kBdTile], the new K and V rows [hd] each, running max / sum / rescale
// [G] each
__host__ __device__ inline size_t bd_att_smem(int G, int hd) {
    return 16 + ((size_t)2 * kBdRing * kBdTile * hd + (size_t)G * hd + (size_t)G * kBdTile + 2 * (size_t)hd +
                 3 * (size_t)G) * 4;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <typename WT>
__global__ void __launch_bounds__(kBdAttThreads) bd_att_kernel(const LoopParams<WT> p, BdLists L, int l, int t,
                                                               int klen, const float* qkvp, int nq,
                                                               __nv_bfloat16* att16) {
    extern __shared__ __align__(16) float smem_f[];
    const int nkeys = t + 1;
    const int nsplit = (nkeys + klen - 1) / klen;
    const int u = blockIdx.x;
    const int G = p.G, hd = p.hd, q4 = hd / 4;
    const int s = u % nsplit;
    const int g = (u / nsplit) % p.K;
    const int b = u / (nsplit * p.K);
    if (b >= p.B) return;
    const int j0 = s * klen, j1 = min(nkeys, j0 + klen);
    const int ntiles = (j1 - j0 + kBdTile - 1) / kBdTile;
    // tiles of kBdTile (64) keys from j0 (a multiple of 64): each in one page
    auto krow_of = [&](int j) { return kv_row(p.pg, p.L, p.K, l, b, g, j); };
    const float* kb = p.kc + krow_of(j0) * hd;
    const float* vb = p.vc + krow_of(j0) * hd;
    int* flag = reinterpret_cast<int*>(smem_f);
    float* kt = smem_f + 4;                  // [kBdRing][kBdTile][hd], 16-byte aligned
    float* vt = kt + kBdRing * kBdTile * hd;
    float* qs = vt + kBdRing * kBdTile * hd;
    float* sc = qs + G * hd;
    float* krow = sc + G * kBdTile;          // key t's K and V rows (nq > 0)
    float* vrow = krow + hd;
    float* rm = vrow + hd;                   // running max
    float* rl = rm + G;                      // running sum
    float* ra = rl + G;                      // rescale of this tile
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int nwarps = kBdAttThreads / 32;
    const bool vec = (hd & 3) == 0;          // rows are whole 16-byte units
    {
        // every access below stays inside the launch's shared memory, the
        // cache and the query rows; a failed check records its number in
        // lists[3] and the CTA returns before touching anything
        uint32_t dyn = 0;
        asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
        int bad = 0;
        if ((size_t)dyn < bd_att_smem(G, hd)) bad = 1;
        else if (b >= p.Bcap || l < 0 || l >= p.L) bad = 2;
        else if (nkeys > p.cap || j1 <= j0) bad = 3;
        else if (vec && ((reinterpret_cast<uintptr_t>(kb) | reinterpret_cast<uintptr_t>(vb)) & 15)) bad = 4;
        else if (G * hd > kBdAttMaxO * kBdAttThreads || G > kBdAttThreads || (size_t)p.K * G * hd > (size_t)p.D)
            bad = 6;
        else if (s >= p.max_split) bad = 7;
        else if (nq > kBdMaxParts || (nq > 0 && (t >= p.rope_len || (hd & 1)))) bad = 8;
        if (bad) {
            if (threadIdx.x == 0) {
                atomicMax(L.base + 3, bad);
                atomicMax(p.status, (int)ST_DEVICE);
            }
            return;
        }
    }
    // key t (the last key of the last split) is built here when nq > 0
    const bool has_t = nq > 0 && s == nsplit - 1;
    // tile i of this split -> buffer i % kBdRing; one commit group per tile
    // (empty past the last tile), so tile i is complete once at most
    // kBdRing - 1 newer groups are pending
    auto load_tile = [&](int i) {
        const int k0 = i * kBdTile;
        const int nt = i < ntiles ? min(kBdTile, j1 - j0 - k0) - (has_t && i == ntiles - 1 ? 1 : 0) : 0;
        float* kd = kt + (i % kBdRing) * kBdTile * hd;
        float* vd = vt + (i % kBdRing) * kBdTile * hd;
        const size_t r0 = nt > 0 ? krow_of(j0 + k0) : 0;
        const float* ks = p.kc + r0 * hd;
        const float* vs = p.vc + r0 * hd;
        if (vec) {
            for (int e = threadIdx.x; e < nt * q4; e += blockDim.x) {
                cp_async16(kd + 4 * e, ks + 4 * e);
                cp_async16(vd + 4 * e, vs + 4 * e);
            }
        } else {
            for (int e = threadIdx.x; e < nt * hd; e += blockDim.x) {
                kd[e] = ldcg(ks + e);
                vd[e] = ldcg(vs + e);
            }
        }
        cp_async_commit();
    };
    // the first tiles' rows precede t and were written at earlier steps, so
    // they are requested before waiting for the previous kernel
    for (int i = 0; i < kBdRing - 1; i++) load_tile(i);
    pdl_wait();
    pdl_trigger();
    const int active = L.act_fwd()[b];
    const int hp = hd / 2;
    const int nitems = G * hp + (has_t ? hd : 0);   // gather items; K/V ones stay with their thread
    if (nq > 0) {
        // q (and key t's rows): sums of the partials in slice order, then RoPE
        const float* pb = qkvp + (size_t)b * p.Q;
        const size_t pst = (size_t)p.B * p.Q;
        const float2* rot = p.rope + (size_t)t * hp;
        auto gather = [&](int col, float& x0, float& x1) {
            x0 = 0.0f;
            x1 = 0.0f;
#pragma unroll
            for (int r = 0; r < kBdMaxParts; r++)
                if (r < nq) {
                    const float2 v = __ldcg(reinterpret_cast<const float2*>(pb + r * pst + col));
                    x0 += v.x;
                    x1 += v.y;
                }
        };
        // one pass: q pairs, then (for the unit holding key t) K and V pairs
        for (int i = threadIdx.x; i < nitems; i += blockDim.x) {
            if (i < G * hp) {
                const int h = i / hp, pr = i - h * hp;
                float x0, x1;
                gather((g * G + h) * hd + 2 * pr, x0, x1);
                const float2 r = rot[pr];
                qs[h * hd + 2 * pr] = x0 * r.x - x1 * r.y;
                qs[h * hd + 2 * pr + 1] = x0 * r.y + x1 * r.x;
            } else {
                const int k = i - G * hp;
                const bool isk = k < hp;
                const int pr = isk ? k : k - hp;
                float x0, x1;
                gather((isk ? p.H + g : p.H + p.K + g) * hd + 2 * pr, x0, x1);
                float* row = isk ? krow : vrow;
                if (isk) {
                    const float2 r = rot[pr];
                    row[2 * pr] = x0 * r.x - x1 * r.y;
                    row[2 * pr + 1] = x0 * r.y + x1 * r.x;
                } else {
                    row[2 * pr] = x0;
                    row[2 * pr + 1] = x1;
                }
            }
        }
    } else {
        for (int i = threadIdx.x; i < G * hd; i += blockDim.x)
            qs[i] = ldcg(p.q + (size_t)b * p.D + (size_t)g * G * hd + i);
    }
    if (threadIdx.x < G) {
        rm[threadIdx.x] = -INFINITY;
        rl[threadIdx.x] = 0.0f;
    }
    if (!active) {                           // block-uniform
        cp_async_wait<0>();
        return;
    }
    // key t's rows into the cache (this thread's own entries)
    const int tl = (t - j0) - (ntiles - 1) * kBdTile;       // its row in the last tile
    if (has_t)
        for (int i = threadIdx.x; i < nitems; i += blockDim.x) {
            if (i < G * hp) continue;
            const int k = i - G * hp;
            const bool isk = k < hp;
            const int d = 2 * (isk ? k : k - hp);
            float* dst = (isk ? p.kc : p.vc) + krow_of(t) * hd + d;
            const float* row = isk ? krow : vrow;
            dst[0] = row[d];
            dst[1] = row[d + 1];
        }
    const float scale = 1.0f / sqrtf((float)hd);
    float o[kBdAttMaxO];
#pragma unroll
    for (int k = 0; k < kBdAttMaxO; k++) o[k] = 0.0f;
    for (int it = 0; it < ntiles; it++) {
        load_tile(it + kBdRing - 1);         // into the buffer tile it - 1 used
        cp_async_wait<kBdRing - 1>();        // this thread's copies of tile it have landed
        if (has_t && it == ntiles - 1)       // key t's rows (this thread's own entries)
            for (int i = threadIdx.x; i < nitems; i += blockDim.x) {
                if (i < G * hp) continue;
                const int k = i - G * hp;
                const bool isk = k < hp;
                const int d = 2 * (isk ? k : k - hp);
                float* dst = (isk ? kt : vt) + (it % kBdRing) * kBdTile * hd + tl * hd + d;
                const float* row = isk ? krow : vrow;
                dst[0] = row[d];
                dst[1] = row[d + 1];
            }
        __syncthreads();                     // tile it (and q, stats) visible to all
        const int nt = min(kBdTile, j1 - j0 - it * kBdTile);
        const float* ks = kt + (it % kBdRing) * kBdTile * hd;
        const float* vs = vt + (it % kBdRing) * kBdTile * hd;
        // scores: a thread per (head, key); its key row is read starting at
        // element (j mod hd) so that neighbouring keys fall in different banks
        for (int e = threadIdx.x; e < G * nt; e += blockDim.x) {
            const int h = e / nt, j = e - h * nt;
            const float* kr = ks + j * hd;
            const float* qh = qs + h * hd;
            float part = 0.0f;
            if (vec) {
                int cc = j % q4;
#pragma unroll 4
                for (int c = 0; c < q4; c++) {
                    const float4 k4 = *reinterpret_cast<const float4*>(kr + 4 * cc);
                    const float4 x4 = *reinterpret_cast<const float4*>(qh + 4 * cc);
                    part += x4.x * k4.x + x4.y * k4.y + x4.z * k4.z + x4.w * k4.w;
                    cc = cc + 1 == q4 ? 0 : cc + 1;
                }
            } else {
                int d = j % hd;
                for (int c = 0; c < hd; c++) {
                    part += qh[d] * kr[d];
                    d = d + 1 == hd ? 0 : d + 1;
                }
            }
            sc[h * kBdTile + j] = part * scale;
        }
        __syncthreads();
        // online softmax per head: new max, rescale of the old state, exps
        for (int h = warp; h < G; h += nwarps) {
            float mx = -INFINITY;
            for (int j = lane; j < nt; j += 32) mx = fmaxf(mx, sc[h * kBdTile + j]);
            mx = warp_max(mx);
            const float mold = rm[h], mnew = fmaxf(mold, mx);
            float lsum = 0.0f;
            for (int j = lane; j < nt; j += 32) {
                const float e = expf(sc[h * kBdTile + j] - mnew);
                sc[h * kBdTile + j] = e;
                lsum += e;
            }
            lsum = warp_sum(lsum);
            if (lane == 0) {
                const float a = expf(mold - mnew);
                ra[h] = a;
                rl[h] = rl[h] * a + lsum;
                rm[h] = mnew;
            }
        }
        __syncthreads();
        // P.V into the running rows
#pragma unroll
        for (int k = 0; k < kBdAttMaxO; k++) {
            const int i = threadIdx.x + k * kBdAttThreads;
            if (i < G * hd) {
                const int h = i / hd, d = i - h * hd;
                const float* ph = sc + h * kBdTile;
                float acc = 0.0f;
#pragma unroll 8
                for (int j = 0; j < nt; j++) acc += ph[j] * vs[j * hd + d];
                o[k] = o[k] * ra[h] + acc;
            }
        }
        __syncthreads();                     // buffer it % kBdRing is refilled next
    }
    const bool combine = nsplit > 1;
#pragma unroll
    for (int k = 0; k < kBdAttMaxO; k++) {
        const int i = threadIdx.x + k * kBdAttThreads;
        if (i < G * hd) {
            const int h = i / hd, d = i - h * hd;
            if (!combine) att_store(p, att16, (size_t)b * p.D + (g * G + h) * hd + d, o[k] / rl[h]);
            else p.part_o[(((size_t)b * p.H + g * G + h) * p.max_split + s) * hd + d] = o[k];
        }
    }
    if (!combine) return;
    if (threadIdx.x < G) {
        const size_t pi = ((size_t)b * p.H + g * G + threadIdx.x) * p.max_split + s;
        p.part_m[pi] = rm[threadIdx.x];
        p.part_l[pi] = rl[threadIdx.x];
    }
    // the last split to finish merges (flash-decoding reduction)
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(&p.att_cnt[b * p.K + g], 1u);
        *flag = prev == (unsigned)nsplit - 1;
    }
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
        const int h = i / hd, d = i - h * hd;
        const size_t pb = ((size_t)b * p.H + g * G + h) * p.max_split;
        float M = -INFINITY;
        for (int s2 = 0; s2 < nsplit; s2++) M = fmaxf(M, ldcg(p.part_m + pb + s2));
        float num = 0.0f, den = 0.0f;
        for (int s2 = 0; s2 < nsplit; s2++) {
            const float w = expf(ldcg(p.part_m + pb + s2) - M);
            den += w * ldcg(p.part_l + pb + s2);
            num += w * ldcg(p.part_o + (pb + s2) * hd + d);
        }
        att_store(p, att16, (size_t)b * p.D + (g * G + h) * hd + d, num / den);
    }
    if (threadIdx.x == 0) p.att_cnt[b * p.K + g] = 0u;
}

// The same attention with a lane per key, for head_dim 32 or 64 and at
// most kBdWMaxG query heads per KV head.  A CTA of kBdWWarps warps takes one
// (sequence, KV head, key split) unit; warp w takes the split's 32-key
// chunks w, w + kBdWWarps, ...  Per chunk, the chunk's K and V rows stream
// into the warp's shared-memory tiles by cp.async (coalesced; K rows padded
// by 4 floats so that a lane reading its own key's row hits distinct banks),
// each lane scores its key against the G queries (broadcast reads), the warp
// updates its online softmax per head with shuffles, then P.V reads the
// probabilities four keys at a time and V as one HD/32-float piece per lane
// and key.  The warps' states merge in shared
// memory in warp order, then as in bd_att_kernel (direct output, or split
// partials merged by the last split to finish).  Key t's K and V rows are
// built from the QKV partials and written to the cache before any warp
// reads them.
constexpr int kBdWWarps = 4;
constexpr int kBdWMaxG = 4;

// q [G][HD], then per warp: K tile [32][HD + 4], V tile [32][HD] and
// probabilities [kBdWMaxG][32]; the merge reuses the tiles; flag at the end
__host__ __device__ inline size_t bd_attw_warp_floats(int hd) { return 32 * (hd + 4) + 32 * (size_t)hd + kBdWMaxG * 32; }
__host__ __device__ inline size_t bd_attw_smem(int G, int hd) {
    return ((size_t)G * hd + (size_t)kBdWWarps * bd_attw_warp_floats(hd) + 4) * 4;
}

template <typename WT, int HD>
__global__ void __launch_bounds__(kBdWWarps * 32) bd_attw_kernel(const LoopParams<WT> p, BdLists L, int l, int t,
                                                                 int klen, const float* qkvp, int nq,
                                                                 __nv_bfloat16* att16) {
    static_assert(HD == 32 || HD == 64, "a lane holds HD/32 output dimensions");
    constexpr int E = HD / 32;
    constexpr int Q4 = HD / 4;
    extern __shared__ __align__(16) float smem_f[];
    const int nkeys = t + 1;
    const int nsplit = (nkeys + klen - 1) / klen;
    const int u = blockIdx.x;
    const int G = p.G;
    const int s = u % nsplit;
    const int g = (u / nsplit) % p.K;
    const int b = u / (nsplit * p.K);
    if (b >= p.B) return;
    const int j0 = s * klen, j1 = min(nkeys, j0 + klen);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int KLD = HD + 4;                           // K tile row stride
    float* qs = smem_f;                                   // [G][HD]
    float* wk = qs + G * HD + warp * bd_attw_warp_floats(HD);   // this warp's K tile
    float* wv = wk + 32 * KLD;                            // this warp's V tile
    float* wp = wv + 32 * HD;                             // this warp's probabilities
    int* flag = reinterpret_cast<int*>(smem_f + G * HD + kBdWWarps * bd_attw_warp_floats(HD));
    {
        uint32_t dyn = 0;
        asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
        int bad = 0;
        if ((size_t)dyn < bd_attw_smem(G, HD)) bad = 11;
        else if (b >= p.Bcap || l < 0 || l >= p.L || p.hd != HD || G > kBdWMaxG) bad = 12;
        else if (nkeys > p.cap || j1 <= j0 || s >= p.max_split) bad = 13;
        else if (nq > kBdMaxParts || (nq > 0 && t >= p.rope_len)) bad = 14;
        if (bad) {
            if (threadIdx.x == 0) {
                atomicMax(L.base + 3, bad);
                atomicMax(p.status, (int)ST_DEVICE);
            }
            return;
        }
    }
    const bool has_t = nq > 0 && s == nsplit - 1;
    const int nchunks = (j1 - j0 + 31) / 32;
    // K and V rows [r0, r1) of chunk c -> this warp's tiles (16-byte pieces, coalesced)
    // chunk c holds keys j0 + 32 c ... (32-aligned, so in one page)
    auto issue = [&](int c, int r0, int r1) {
        if (r1 <= r0) {
            cp_async_commit();
            return;
        }
        const size_t row = kv_row(p.pg, p.L, p.K, l, b, g, j0 + 32 * c);
        const float* ksrc = p.kc + row * HD;
        const float* vsrc = p.vc + row * HD;
        for (int e = r0 * Q4 + lane; e < r1 * Q4; e += 32) {
            const int r = e / Q4, c4 = e - r * Q4;
            cp_async16(wk + r * KLD + 4 * c4, ksrc + 4 * e);
            cp_async16(wv + 4 * e, vsrc + 4 * e);
        }
        cp_async_commit();
    };
    // Each warp's first chunk holds rows written at earlier steps (key t,
    // built below, is held back), so it is requested before waiting for
    // the previous kernel.
    const int nv0 = warp < nchunks ? min(32, j1 - (j0 + 32 * warp)) : 0;
    const bool t_first = has_t && warp < nchunks && j0 + 32 * warp + nv0 - 1 == t;
    if (warp < nchunks) issue(warp, 0, nv0 - (t_first ? 1 : 0));
    pdl_wait();
    pdl_trigger();
    if (!L.act_fwd()[b]) {                                // block-uniform
        cp_async_wait<0>();
        return;
    }
    constexpr int HP = HD / 2;
    if (nq > 0) {
        // q pairs, then (for the unit holding key t) K and V pairs: sums of
        // the partials in slice order, RoPE on q and K; key t's rows go to
        // the cache, where the warps read them below
        const float* pb = qkvp + (size_t)b * p.Q;
        const size_t pst = (size_t)p.B * p.Q;
        const float2* rot = p.rope + (size_t)t * HP;
        const int nitems = G * HP + (has_t ? HD : 0);
        for (int i = threadIdx.x; i < nitems; i += blockDim.x) {
            int col;
            bool rope = true;
            float* dst;
            if (i < G * HP) {
                const int h = i / HP, pr = i - h * HP;
                col = (g * G + h) * HD + 2 * pr;
                dst = qs + h * HD + 2 * pr;
            } else {
                const int k = i - G * HP;
                const bool isk = k < HP;
                const int pr = isk ? k : k - HP;
                col = (isk ? p.H + g : p.H + p.K + g) * HD + 2 * pr;
                dst = (isk ? p.kc : p.vc) + kv_row(p.pg, p.L, p.K, l, b, g, t) * HD + 2 * pr;
                rope = isk;
            }
            float x0 = 0.0f, x1 = 0.0f;
#pragma unroll
            for (int r = 0; r < kBdMaxParts; r++)
                if (r < nq) {
                    const float2 v = __ldcg(reinterpret_cast<const float2*>(pb + r * pst + col));
                    x0 += v.x;
                    x1 += v.y;
                }
            if (rope) {
                const float2 r = rot[(col % HD) / 2];
                const float y0 = x0 * r.x - x1 * r.y, y1 = x0 * r.y + x1 * r.x;
                x0 = y0;
                x1 = y1;
            }
            dst[0] = x0;
            dst[1] = x1;
        }
        if (has_t) __threadfence();                       // key t's rows before any warp reads them
    } else {
        for (int i = threadIdx.x; i < G * HD; i += blockDim.x)
            qs[i] = ldcg(p.q + (size_t)b * p.D + (size_t)g * G * HD + i);
    }
    __syncthreads();
    const float scale = 1.0f / sqrtf((float)HD);
    float m[kBdWMaxG], lsum[kBdWMaxG], o[kBdWMaxG][E];
#pragma unroll
    for (int h = 0; h < kBdWMaxG; h++) {
        m[h] = -INFINITY;
        lsum[h] = 0.0f;
#pragma unroll
        for (int e = 0; e < E; e++) o[h][e] = 0.0f;
    }
    for (int c = warp; c < nchunks; c += kBdWWarps) {
        const int key0 = j0 + 32 * c;
        const int nv = min(32, j1 - key0);               // warp-uniform
        if (c != warp) issue(c, 0, nv);
        else if (t_first) issue(c, nv - 1, nv);          // key t, now in the cache
        cp_async_wait<0>();
        __syncwarp();                                     // the tiles are visible to the warp
        // scores: lane = key
        const bool valid = lane < nv;
        const float* krow = wk + (valid ? lane : 0) * KLD;
        float4 k4[Q4];
#pragma unroll
        for (int i = 0; i < Q4; i++) k4[i] = *reinterpret_cast<const float4*>(krow + 4 * i);
        float sv[kBdWMaxG];
#pragma unroll
        for (int h = 0; h < kBdWMaxG; h++) {
            sv[h] = -INFINITY;
            if (h < G) {
                const float4* q4p = reinterpret_cast<const float4*>(qs + h * HD);
                float a = 0.0f;
#pragma unroll
                for (int i = 0; i < Q4; i++) {
                    const float4 q = q4p[i];
                    a += q.x * k4[i].x + q.y * k4[i].y + q.z * k4[i].z + q.w * k4[i].w;
                }
                if (valid) sv[h] = a * scale;
            }
        }
        // online softmax per head
#pragma unroll
        for (int h = 0; h < kBdWMaxG; h++) {
            if (h < G) {
                const float mnew = fmaxf(m[h], warp_max(sv[h]));
                const float alpha = expf(m[h] - mnew);
                const float pv = valid ? expf(sv[h] - mnew) : 0.0f;
                lsum[h] = lsum[h] * alpha + warp_sum(pv);
                m[h] = mnew;
#pragma unroll
                for (int e = 0; e < E; e++) o[h][e] *= alpha;
                wp[h * 32 + lane] = pv;
            }
        }
        __syncwarp();                                     // probabilities visible to the warp
        // P.V: lane owns dimensions [E * lane, E * lane + E)
        for (int j = 0; j < nv; j += 4) {
#pragma unroll
            for (int h = 0; h < kBdWMaxG; h++) {
                if (h < G) {
                    const float4 p4 = *reinterpret_cast<const float4*>(wp + h * 32 + j);
                    const float pj[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
                    for (int jj = 0; jj < 4; jj++) {
                        if (j + jj < nv) {
                            const float* vr = wv + (j + jj) * HD + E * lane;
#pragma unroll
                            for (int e = 0; e < E; e++) o[h][e] += pj[jj] * vr[e];
                        }
                    }
                }
            }
        }
        __syncwarp();                                     // the tile is refilled by the next chunk
    }
    // merge the warps' states in warp order
    __syncthreads();
    float* ms = qs + G * HD;                              // [kBdWWarps][G] max, then sums, then outputs
    float* ls = ms + kBdWWarps * kBdWMaxG;
    float* os = ls + kBdWWarps * kBdWMaxG;                // [kBdWWarps][G][HD]
#pragma unroll
    for (int h = 0; h < kBdWMaxG; h++) {
        if (h < G) {
            if (lane == 0) {
                ms[warp * kBdWMaxG + h] = m[h];
                ls[warp * kBdWMaxG + h] = lsum[h];
            }
#pragma unroll
            for (int e = 0; e < E; e++) os[(warp * G + h) * HD + E * lane + e] = o[h][e];
        }
    }
    __syncthreads();
    const bool combine = nsplit > 1;
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
        const int h = i / HD, d = i - h * HD;
        float M = -INFINITY;
        for (int w = 0; w < kBdWWarps; w++) M = fmaxf(M, ms[w * kBdWMaxG + h]);
        float num = 0.0f, den = 0.0f;
        for (int w = 0; w < kBdWWarps; w++) {
            const float mw = ms[w * kBdWMaxG + h];
            if (mw == -INFINITY) continue;                // a warp without keys
            const float wgt = expf(mw - M);
            den += wgt * ls[w * kBdWMaxG + h];
            num += wgt * os[(w * G + h) * HD + d];
        }
        if (!combine) {
            att_store(p, att16, (size_t)b * p.D + (g * G + h) * HD + d, num / den);
        } else {
            const size_t pi = ((size_t)b * p.H + g * G + h) * p.max_split + s;
            p.part_o[pi * HD + d] = num;
            if (d == 0) {
                p.part_m[pi] = M;
                p.part_l[pi] = den;
            }
        }
    }
    if (!combine) return;
    // the last split to finish merges (flash-decoding reduction)
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(&p.att_cnt[b * p.K + g], 1u);
        *flag = prev == (unsigned)nsplit - 1;
    }
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
        const int h = i / HD, d = i - h * HD;
        const size_t pb2 = ((size_t)b * p.H + g * G + h) * p.max_split;
        float M = -INFINITY;
        for (int s2 = 0; s2 < nsplit; s2++) M = fmaxf(M, ldcg(p.part_m + pb2 + s2));
        float num = 0.0f, den = 0.0f;
        for (int s2 = 0; s2 < nsplit; s2++) {
            const float w = expf(ldcg(p.part_m + pb2 + s2) - M);
            den += w * ldcg(p.part_l + pb2 + s2);
            num += w * ldcg(p.part_o + (pb2 + s2) * HD + d);
        }
        att_store(p, att16, (size_t)b * p.D + (g * G + h) * HD + d, num / den);
    }
    if (threadIdx.x == 0) p.att_cnt[b * p.K + g] = 0u;
}

// f[b] = SiLU(gate) * up (generate.c:165-179) of the running sequences, from
// the nparts K-slice partials the up/gate GEMM left in part (slice r, row b
// at part + (r * B + b) * 2F: up in [0, F), gate in [F, 2F)), summed in
// slice order; plus its bf16 hi/lo pair when f16 is set (the operand of a
// kind::f16 down GEMM).
template <typename WT>
__global__ void __launch_bounds__(kThreads) bd_swiglu_kernel(const LoopParams<WT> p, BdLists L, const float* part,
                                                             int nparts, __nv_bfloat16* f16) {
    pdl_wait();
    pdl_trigger();
    const int F4 = p.F / 4;
    const size_t pst = (size_t)p.B * 2 * p.F;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < p.B * F4; idx += gridDim.x * blockDim.x) {
        const int b = idx / F4, c = (idx - b * F4) * 4;
        if (!L.act_fwd()[b]) continue;
        const float* pb = part + (size_t)b * 2 * p.F + c;
        float u[4] = {0.0f, 0.0f, 0.0f, 0.0f}, gt[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int r = 0; r < kBdMaxParts; r++)
            if (r < nparts) {
                const float4 a = __ldcg(reinterpret_cast<const float4*>(pb + r * pst));
                const float4 z = __ldcg(reinterpret_cast<const float4*>(pb + r * pst + p.F));
                u[0] += a.x; u[1] += a.y; u[2] += a.z; u[3] += a.w;
                gt[0] += z.x; gt[1] += z.y; gt[2] += z.z; gt[3] += z.w;
            }
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; j++) v[j] = (gt[j] / (1.0f + expf(-gt[j]))) * u[j];
        *reinterpret_cast<float4*>(p.f + (size_t)b * p.F + c) = make_float4(v[0], v[1], v[2], v[3]);
        if (f16)
#pragma unroll
            for (int j = 0; j < 4; j++) bf16_split_store(f16 + (size_t)b * p.F + c + j, (size_t)p.Bcap * p.F, v[j]);
    }
}

// Sampling and bookkeeping of the head sequences (the token loop's phase).
template <typename WT>
__global__ void __launch_bounds__(kThreads, 1) bd_sample_kernel(const LoopParams<WT> p, BdLists L, int nparts) {
    extern __shared__ __align__(16) float smem_f[];
    pdl_wait();
    pdl_trigger();
    LoopSmem sm = bd_smem(smem_f, p.Bcap);
    const int nh = L.base[1], t = L.base[2];
    for (int i = threadIdx.x; i < nh; i += blockDim.x) sm.head[i] = L.head()[i];
    __syncthreads();
    if (nh > 0) phase_sample<WT>(p, t, sm, nh, nparts);
    if (p.stamps && t + 1 == p.T && blockIdx.x == 0 && threadIdx.x == 0) p.stamps[p.T] = globaltimer_ns();
}

template <typename WT>
__global__ void __launch_bounds__(kThreads) bd_prologue_kernel(const LoopParams<WT> p) {
    pdl_wait();
    pdl_trigger();
    loop_prologue(p);
}

}  // namespace mc

// mc_cluster_loop.cuh — cluster-resident decode token loop for sm_100a.
//
// For models whose per-layer weights are small (the Minima default decoder:
// 0.98 MB per layer, 15.4 MB tied lm_head) the grid-barrier loop is bound by
// synchronisation latency, not bandwidth: a grid barrier costs ~2 us on
// B200, a cluster barrier ~0.24 us.  This loop therefore splits the GPU in
// two roles inside one launch of CS-CTA clusters:
//
//  * layer cluster (cluster 0): runs every transformer layer of every step
//    for the whole batch.  Each CTA owns a fixed row slice of every layer
//    matrix; the slices of upcoming layers stream from L2/HBM into shared
//    memory with TMA bulk copies (cp.async.bulk, one destination CTA) tracked by
//    mbarriers, kStages layers ahead.  Activations are replicated in every
//    CTA's shared memory and exchanged through distributed shared memory;
//    the five phases of a layer (forward_one, generate.c:97-185) are
//    separated by hardware cluster barriers.
//  * head clusters (all others): each CTA holds a slice of the tied
//    lm_head (tok_emb rows) resident in shared memory for the whole launch,
//    computes its logits for every sequence that needs them
//    (generate.c:187-191), applies the sampler's value transform and
//    returns per-CTA argmax partials.
//
// The two roles hand off through a release/acquire counter pair in global
// memory (two grid-level handoffs per decode step instead of ~42 grid
// barriers).  Sampling here is greedy (top_k == 1, generate.c:447-460 with
// its tie and NaN rules) with all penalties, bans and stop sequences; other
// sampling settings use the grid-barrier loop.  Every wait is bounded by a
// %globaltimer deadline that sets the status word and unwinds.
#pragma once

#include <cooperative_groups.h>

#include "mc_device.cuh"
#include "mc_sampler.cuh"
#include "mc_token_loop.cuh"

namespace mc {

namespace cg = cooperative_groups;

constexpr int kStages = 2;          // layers of weights in flight per CTA
constexpr unsigned kExit = 0x7fffffffu;
constexpr unsigned kHcEmbOffset = 2048;   // head CTA: byte offset of the lm_head slice
constexpr unsigned kLcHeader = 1024;      // layer CTA: mbarriers, ints, red scratch

struct CSlice {
    int q0, q1, p0, p1, f0, f1;     // rows: qkv [q0,q1), proj/down [p0,p1), up/gate [f0,f1)
};

// Row slice of CTA `c` in a cluster of `cs`.  Slices are whole groups of 4
// rows (Q, D and F are multiples of 4 here), so each CTA's results can be
// pushed to the other CTAs as float4 chunks; qkv slices keep RoPE pairs.
__host__ __device__ inline CSlice cluster_slice(int c, int cs, int Q, int D, int F) {
    CSlice s;
    const int qpc = 4 * ((Q / 4 + cs - 1) / cs);
    s.q0 = min(c * qpc, Q);
    s.q1 = min((c + 1) * qpc, Q);
    const int rpc = 4 * ((D / 4 + cs - 1) / cs);
    s.p0 = min(c * rpc, D);
    s.p1 = min((c + 1) * rpc, D);
    const int fpc = 4 * ((F / 4 + cs - 1) / cs);
    s.f0 = min(c * fpc, F);
    s.f1 = min((c + 1) * fpc, F);
    return s;
}

__host__ __device__ inline size_t slice_floats(const CSlice& s, int D, int F) {
    return (size_t)(s.q1 - s.q0) * D + (size_t)(s.p1 - s.p0) * D + 2 * (size_t)(s.f1 - s.f0) * D +
           (size_t)(s.p1 - s.p0) * F;
}

struct ClusterParams {
    LoopParams<float> lp;       // model, buffers, sequences, sampling (greedy)
    int cs;                     // CTAs per cluster
    int n_clusters;
    // layer-cluster shared-memory plan (byte offsets)
    unsigned off_x, off_xn, off_qkv, off_attp, off_att, off_f, off_sc, off_kv, off_stage;
    unsigned off_rmsf, off_rope;
    unsigned stage_floats;      // floats per weight stage (slice + rms1 + rms2)
    int n_split;                // attention splits per (sequence, KV head)
    int kv_tile;                // keys staged per attention tile
    // head clusters
    int hc_rows;                // tok_emb rows per head CTA
    unsigned hc_ld;             // padded row stride (floats) of the resident slice
    unsigned off_hc_x;          // byte offset of the normalised-x copy
    float* xfin;                // [Bcap][D] rmsnorm(x, rms_final), layer -> head
    int* hgen;                  // [Bcap] sampler step of each sequence in this head phase, -1 = none
    unsigned* go;               // head phases issued (or kExit)
    unsigned* hdone;            // head CTA arrivals
    float* hpv;                 // [Bcap][n_head_ctas][2] best transformed value (bans, no bans)
    int* hpi;                   // [Bcap][n_head_ctas][2] its id
};

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ unsigned smem_addr(const void* p) {
    return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// 1-D bulk copy global -> this CTA's own shared memory (single destination).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes,
                                         unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Wait for phase `parity` of `bar`, bounded by the deadline; false on expiry.
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, unsigned parity,
                                          unsigned long long timeout_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer_ns() - t0 > timeout_ns) return false;
    return true;
}

__device__ __forceinline__ void st_release_u32(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ------------------------------------------------------------ layer cluster
struct LcState {
    float* x;      // [B][D]
    float* xn;     // [B][D]
    float* qkv;    // [B][Q]
    float* attp;   // [B][H][n_split][hd + 2]
    float* att;    // [B][D]
    float* f;      // [B][F]
    float* sc;     // [G][kv_tile]
    float* kv;     // [2][kv_tile][hd + 4]
    float* stage;  // [kStages][stage_floats]
    float* rmsf;   // [D] final RMSNorm scale
    float2* rope;  // [hd/2] (cos, sin) at the current position
    unsigned long long* bar;  // [kStages]
    int* ints;     // [64]: 0..15 fwd list, 16..31 head list, 32.. scalars,
                   //       36/37 cluster error slots, 38 this CTA saw an error
    float* red;    // [64]
    struct SeqMirror* seq;    // [kBCMax] sequence table mirrored in shared memory
    int epoch;     // cluster barriers passed (identical in every CTA of the cluster)
};

// The sequence table in shared memory: the layer cluster reads it every
// step, so it is kept here (identical in every layer CTA; rank 0 updates it
// and broadcasts) and written back to global memory once, at exit.
struct SeqMirror {
    int P, nnew, gen, done, tok, result, final_pos, pad;
    unsigned long long rng;
};

// Flag a failure seen by this CTA; the next lc_sync makes it cluster-wide.
__device__ __forceinline__ void lc_fail(LcState& S, int* status, int code) {
    atomicMax(status, code);
    S.ints[38] = 1;
}

// Issue the TMA bulk copies of layer `l`'s weight slice into stage `s`.
__device__ void lc_issue_layer(const ClusterParams& cp, const CSlice& sl, LcState& S, int l, int s) {
    const LoopParams<float>& p = cp.lp;
    const size_t D = p.D, F = p.F;
    float* dst = S.stage + (size_t)s * cp.stage_floats;
    const unsigned nq = sl.q1 - sl.q0, np = sl.p1 - sl.p0, nf = sl.f1 - sl.f0;
    // slice rows, then this layer's rms1 and rms2 scales (D floats each)
    const unsigned bytes = (unsigned)((nq * D + np * D + 2 * nf * D + np * F + 2 * D) * 4);
    mbar_expect_tx(&S.bar[s], bytes);
    float* scales = dst + slice_floats(sl, p.D, p.F);
    bulk_g2s(scales, p.rms1 + (size_t)l * D, D * 4, &S.bar[s]);
    bulk_g2s(scales + D, p.rms2 + (size_t)l * D, D * 4, &S.bar[s]);
    if (nq) bulk_g2s(dst, p.w_qkv + ((size_t)l * p.Q + sl.q0) * D, nq * D * 4, &S.bar[s]);
    dst += nq * D;
    if (np) bulk_g2s(dst, p.w_proj + ((size_t)l * p.D + sl.p0) * D, np * D * 4, &S.bar[s]);
    dst += np * D;
    if (nf) bulk_g2s(dst, p.w_up + ((size_t)l * p.F + sl.f0) * D, nf * D * 4, &S.bar[s]);
    dst += nf * D;
    if (nf) bulk_g2s(dst, p.w_gate + ((size_t)l * p.F + sl.f0) * D, nf * D * 4, &S.bar[s]);
    dst += nf * D;
    if (np) bulk_g2s(dst, p.w_down + ((size_t)l * p.D + sl.p0) * F, np * F * 4, &S.bar[s]);
}

// x_b * inv_rms * scale for the sequences in `list` (generate.c:57-63).
__device__ void lc_norm(const float* x, float* xn, const float* scale, const int* list, int n,
                        int D, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = warp; i < n; i += kWarps) {
        const float* xr = x + list[i] * D;
        float ss = 0.0f;
        for (int k = lane; k < D; k += 32) ss += xr[k] * xr[k];
        ss = warp_sum(ss);
        if (lane == 0) red[i] = 1.0f / sqrtf(ss / (float)D + 1e-5f);
    }
    __syncthreads();
    for (int i = 0; i < n; i++) {
        const int b = list[i];
        for (int k = threadIdx.x; k < D; k += blockDim.x) xn[b * D + k] = x[b * D + k] * red[i] * scale[k];
    }
    __syncthreads();
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Start async copies of cached K/V rows [a0, a0+n) of one (sequence, KV
// head) into the staging tile; row t is produced this step and is filled
// from shared memory separately.
__device__ __forceinline__ void att_issue(const float* kg, const float* vg, float* ks, float* vs,
                                          int a0, int n, int t, int hd, int ldk) {
    const int q4 = hd / 4;
    for (int e = threadIdx.x; e < n * q4; e += blockDim.x) {
        const int j = e / q4, c4 = (e % q4) * 4, pos = a0 + j;
        if (pos == t) continue;
        cp_async16(ks + j * ldk + c4, kg + (size_t)pos * hd + c4);
        cp_async16(vs + j * ldk + c4, vg + (size_t)pos * hd + c4);
    }
}

// 32 per-lane partial sums -> lane l ends with the complete sum of value l
// (a transposed butterfly: 16+8+4+2+1 shuffles instead of 5 per value).
__device__ __forceinline__ float transpose_reduce32(float (&v)[32]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int m = 16, n = 32; m >= 1; m >>= 1, n >>= 1) {
        const bool upper = lane & m;
#pragma unroll
        for (int j = 0; j < n / 2; j++) {
            const float send = upper ? v[j] : v[j + n / 2];
            const float keep = upper ? v[j + n / 2] : v[j];
            v[j] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
    }
    return v[0];
}

// Four shared-memory rows of length `len` against the activation rows of the
// sequences in `list` (n <= kBCMax).  Lanes split each row in float4 chunks;
// lane l returns the full dot product of row (l >> 3) with sequence
// list[l & 7] (0 for slots past n).
__device__ __forceinline__ float lc_gemv4(const float* r0, const float* r1, const float* r2,
                                          const float* r3, int len, const float* xs, int ld,
                                          const int* list, int n) {
    const int lane = threadIdx.x & 31;
    const float* xb[kBCMax];
#pragma unroll
    for (int i = 0; i < kBCMax; i++) xb[i] = xs + (i < n ? list[i] : 0) * ld;
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; i++) acc[i] = 0.0f;
    for (int k = lane * 4; k < len; k += 128) {
        const float4 w0 = *reinterpret_cast<const float4*>(r0 + k);
        const float4 w1 = *reinterpret_cast<const float4*>(r1 + k);
        const float4 w2 = *reinterpret_cast<const float4*>(r2 + k);
        const float4 w3 = *reinterpret_cast<const float4*>(r3 + k);
#pragma unroll
        for (int i = 0; i < kBCMax; i++) {
            if (i < n) {
                const float4 x = *reinterpret_cast<const float4*>(xb[i] + k);
                acc[0 * 8 + i] += w0.x * x.x + w0.y * x.y + w0.z * x.z + w0.w * x.w;
                acc[1 * 8 + i] += w1.x * x.x + w1.y * x.y + w1.z * x.z + w1.w * x.w;
                acc[2 * 8 + i] += w2.x * x.x + w2.y * x.y + w2.z * x.z + w2.w * x.w;
                acc[3 * 8 + i] += w3.x * x.x + w3.y * x.y + w3.z * x.z + w3.w * x.w;
            }
        }
    }
    return transpose_reduce32(acc);
}

// Dot of `nr` (<= 2) shared-memory rows of length `len` with the activation
// rows xs[b] for every b in list; lanes split the row (float4).  Returns the
// sums in acc[r][i] on every lane.
__device__ __forceinline__ void lc_dot2(const float* r0, const float* r1, int len, const float* xs,
                                        int ld, const int* list, int n, float (&acc)[2][kBCMax]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < kBCMax; i++) { acc[0][i] = 0.0f; acc[1][i] = 0.0f; }
    for (int k = lane * 4; k < len; k += 128) {
        const float4 w0 = *reinterpret_cast<const float4*>(r0 + k);
        const float4 w1 = *reinterpret_cast<const float4*>(r1 + k);
#pragma unroll
        for (int i = 0; i < kBCMax; i++) {
            if (i < n) {
                const float4 xv = *reinterpret_cast<const float4*>(xs + list[i] * ld + k);
                acc[0][i] += w0.x * xv.x + w0.y * xv.y + w0.z * xv.z + w0.w * xv.w;
                acc[1][i] += w1.x * xv.x + w1.y * xv.y + w1.z * xv.z + w1.w * xv.w;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < kBCMax; i++)
        if (i < n) { acc[0][i] = warp_sum(acc[0][i]); acc[1][i] = warp_sum(acc[1][i]); }
}

// Copy rows [r0, r1) of buf[b][ld] for the sequences in `list` from this
// CTA's shared memory into the same place in every other CTA of the
// cluster, as float4 stores (remote-store cost is per transaction, so 16-byte
// chunks move four times the data of scalar stores for the same cost).
// Caller: all threads, after the rows are written locally and a CTA barrier.
__device__ __forceinline__ void push_rows(cg::cluster_group& cl, float* buf, int ld, int r0, int r1,
                                          const int* list, int n, int cs, int crank) {
    const int n4 = (r1 - r0) >> 2, per_rank = n * n4;
    for (int e = threadIdx.x; e < per_rank * cs; e += blockDim.x) {
        const int r = e / per_rank;
        if (r == crank) continue;
        const int w = e - r * per_rank, i = w / n4, c = w - i * n4;
        const int off = list[i] * ld + r0 + 4 * c;
        const float4 v = *reinterpret_cast<const float4*>(buf + off);
        *reinterpret_cast<float4*>(cl.map_shared_rank(buf, r) + off) = v;
    }
}

// Copy floats [off, off + len) (len % 4 == 0, off % 4 == 0) to every other CTA.
__device__ __forceinline__ void push_block(cg::cluster_group& cl, float* buf, int off, int len, int cs,
                                           int crank) {
    const int n4 = len >> 2;
    for (int e = threadIdx.x; e < n4 * cs; e += blockDim.x) {
        const int r = e / n4;
        if (r == crank) continue;
        const int o = off + 4 * (e - r * n4);
        *reinterpret_cast<float4*>(cl.map_shared_rank(buf, r) + o) =
            *reinterpret_cast<const float4*>(buf + o);
    }
}

// Cluster barrier plus a cluster-uniform error decision: a CTA that sees a
// failure before arriving sets the flag of this barrier's epoch in every
// CTA; after the barrier all CTAs read the same flag, so they all leave at
// the same barrier.  Flags alternate between two slots so that a flag meant
// for the next barrier cannot be seen by a CTA still reading this one.
// Failures are raised by the CTA that sees them (lc_fail), so no global
// memory is read here.
__device__ bool lc_sync(cg::cluster_group& cl, LcState& S, int cs) {
    const int slot = 36 + (S.epoch & 1);
    __syncthreads();
    if (threadIdx.x == 0 && S.ints[38])
        for (int r = 0; r < cs; r++) cl.map_shared_rank(S.ints, r)[slot] = 1;
    cl.sync();
    const bool ok = S.ints[slot] == 0;
    S.epoch++;
    return ok;
}

// One layer for the sequences in the fwd list at position t.
__device__ bool lc_layer(const ClusterParams& cp, const CSlice& sl, LcState& S,
                         cg::cluster_group& cl, int crank, int l, int t, const int* fl, int nf,
                         const float* w) {
    const LoopParams<float>& p = cp.lp;
    const int D = p.D, Q = p.Q, F = p.F, hd = p.hd, K = p.K, G = p.G, H = p.H;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cs = cp.cs;
    const float* wq = w;
    const float* wp = wq + (size_t)(sl.q1 - sl.q0) * D;
    const float* wu = wp + (size_t)(sl.p1 - sl.p0) * D;
    const float* wg = wu + (size_t)(sl.f1 - sl.f0) * D;
    const float* wd = wg + (size_t)(sl.f1 - sl.f0) * D;
    const float* rms1 = w + slice_floats(sl, D, F);
    const float* rms2 = rms1 + D;

    // Attention geometry; the first tile of this CTA's first unit is fetched
    // now so that its L2 latency overlaps the QKV phase.
    const int ns = cp.n_split;
    const int units = nf * K * ns;
    const int ldk = hd + 4;
    float* ks = S.kv;
    float* vs = S.kv + cp.kv_tile * ldk;
    if (crank < units) {
        const int u = crank, s = u % ns, g = (u / ns) % K, b = fl[u / (ns * K)];
        const int per = (t + 1 + ns - 1) / ns;
        const int j0 = min(s * per, t + 1), j1 = min(j0 + per, t + 1);
        const size_t cbase = (((size_t)l * p.Bcap + b) * K + g) * p.cap;
        att_issue(p.kc + cbase * hd, p.vc + cbase * hd, ks, vs, j0, min(cp.kv_tile, j1 - j0), t, hd, ldk);
    }

    // ---- QKV + RoPE + K/V append (generate.c:99-119)
    lc_norm(S.x, S.xn, rms1, fl, nf, D, S.red);
    for (int r0 = sl.q0 + 4 * warp; r0 < sl.q1; r0 += 4 * kWarps) {
        const float* w0 = wq + (size_t)(r0 - sl.q0) * D;
        const float val = lc_gemv4(w0, w0 + D, w0 + 2 * D, w0 + 3 * D, D, S.xn, D, fl, nf);
        // lane: row r0 + (lane >> 3), sequence slot lane & 7; the RoPE partner
        // row (2p <-> 2p+1) sits in lane ^ 8
        const float other = __shfl_xor_sync(0xffffffffu, val, 8);
        const int r = r0 + (lane >> 3), i = lane & 7;
        const int slot = r / hd, d = r % hd;
        float out = val;
        if (slot < H + K) {
            const float2 rr = S.rope[d / 2];
            out = (d & 1) ? other * rr.y + val * rr.x     // z' = a s + z c
                          : val * rr.x - other * rr.y;    // a' = a c - z s
        }
        if (i < nf) {
            const int b = fl[i];
            S.qkv[b * Q + r] = out;
            if (slot >= H) {
                const bool isk = slot < H + K;
                const int g = isk ? slot - H : slot - H - K;
                (isk ? p.kc : p.vc)[((((size_t)l * p.Bcap + b) * K + g) * p.cap + t) * hd + d] = out;
            }
        }
    }
    __syncthreads();
    push_rows(cl, S.qkv, Q, sl.q0, sl.q1, fl, nf, cs, crank);
    __threadfence();   // K/V rows are read from global by other CTAs in later steps
    if (!lc_sync(cl, S, cs)) return false;

    // ---- attention, split over the cluster (generate.c:121-156)
    const float scale = 1.0f / sqrtf((float)hd);
    for (int u = crank; u < units; u += cs) {
        const int s = u % ns, g = (u / ns) % K, b = fl[u / (ns * K)];
        const int nkeys = t + 1;
        const int per = (nkeys + ns - 1) / ns;
        const int j0 = min(s * per, nkeys), j1 = min(j0 + per, nkeys);
        const size_t cbase = (((size_t)l * p.Bcap + b) * K + g) * p.cap;
        const float* kg = p.kc + cbase * hd;
        const float* vg = p.vc + cbase * hd;
        const float* q = S.qkv + b * Q + g * G * hd;
        // running softmax state per head: m, l in red[2h], red[2h+1]; o accumulates in att scratch
        float* o = S.sc + G * cp.kv_tile;          // [G][hd]
        for (int i = threadIdx.x; i < G * hd; i += blockDim.x) o[i] = 0.0f;
        if (threadIdx.x < G) { S.red[2 * threadIdx.x] = -INFINITY; S.red[2 * threadIdx.x + 1] = 0.0f; }
        for (int a0 = j0; a0 < j1; a0 += cp.kv_tile) {
            const int n = min(cp.kv_tile, j1 - a0);
            __syncthreads();
            // stage K/V rows [a0, a0+n) (the first tile of the first unit is
            // already in flight); the row at t comes from this step's qkv
            if (!(u == crank && a0 == j0)) att_issue(kg, vg, ks, vs, a0, n, t, hd, ldk);
            if (t >= a0 && t < a0 + n) {
                const int j = t - a0;
                for (int c = threadIdx.x; c < hd; c += blockDim.x) {
                    ks[j * ldk + c] = S.qkv[b * Q + D + g * hd + c];
                    vs[j * ldk + c] = S.qkv[b * Q + D + p.kvd + g * hd + c];
                }
            }
            cp_async_wait_all();
            __syncthreads();
            for (int e = threadIdx.x; e < G * n; e += blockDim.x) {
                const int h = e / n, j = e % n;
                const float* qh = q + h * hd;
                const float* kr = ks + j * ldk;
                float dot = 0.0f;
                for (int d = 0; d < hd; d += 4) {
                    const float4 kk = *reinterpret_cast<const float4*>(kr + d);
                    dot += qh[d] * kk.x + qh[d + 1] * kk.y + qh[d + 2] * kk.z + qh[d + 3] * kk.w;
                }
                S.sc[h * cp.kv_tile + j] = dot * scale;
            }
            __syncthreads();
            for (int h = warp; h < G; h += kWarps) {
                float m = -INFINITY;
                for (int j = lane; j < n; j += 32) m = fmaxf(m, S.sc[h * cp.kv_tile + j]);
                m = warp_max(m);
                const float mold = S.red[2 * h], mnew = fmaxf(mold, m);
                float ls = 0.0f;
                for (int j = lane; j < n; j += 32) {
                    const float e = expf(S.sc[h * cp.kv_tile + j] - mnew);
                    S.sc[h * cp.kv_tile + j] = e;
                    ls += e;
                }
                ls = warp_sum(ls);
                __syncwarp();
                if (lane == 0) {
                    const float corr = expf(mold - mnew);
                    S.red[2 * h] = mnew;
                    S.red[2 * h + 1] = S.red[2 * h + 1] * corr + ls;
                    S.red[32 + h] = corr;
                }
            }
            __syncthreads();
            for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
                const int h = i / hd, d = i % hd;
                float acc = o[i] * S.red[32 + h];
                for (int j = 0; j < n; j++) acc += S.sc[h * cp.kv_tile + j] * vs[j * ldk + d];
                o[i] = acc;
            }
        }
        __syncthreads();
        // partial (o, m, l) of the unit's G heads: one contiguous block of
        // G rows of pw = hd + 4 floats, written locally and pushed
        const int pw = hd + 4;
        const int blk = (((b * K + g) * ns + s) * G) * pw;
        for (int i = threadIdx.x; i < G * pw; i += blockDim.x) {
            const int h = i / pw, e = i % pw;
            S.attp[blk + i] = e < hd ? o[h * hd + e] : (e < hd + 2 ? S.red[2 * h + (e - hd)] : 0.0f);
        }
        __syncthreads();
        push_block(cl, S.attp, blk, G * pw, cs, crank);
        __syncthreads();   // o and red are reused by this CTA's next unit
    }
    if (!lc_sync(cl, S, cs)) return false;

    // ---- combine splits (every CTA), then PROJ + residual (generate.c:158-163)
    {
        const int pw = hd + 4;
        for (int e = threadIdx.x; e < nf * H * hd; e += blockDim.x) {
            const int i = e / (H * hd), h = (e / hd) % H, d = e % hd, b = fl[i];
            const int g = h / G, hh = h % G;
            const float* pp = S.attp + ((size_t)((b * K + g) * ns) * G + hh) * pw;  // split stride G*pw
            float M = -INFINITY;
            for (int s2 = 0; s2 < ns; s2++) M = fmaxf(M, pp[s2 * G * pw + hd]);
            float num = 0.0f, den = 0.0f;
            for (int s2 = 0; s2 < ns; s2++) {
                const float* q2 = pp + s2 * G * pw;
                const float ls = q2[hd + 1];
                if (ls > 0.0f) {
                    const float wgt = expf(q2[hd] - M);
                    den += wgt * ls;
                    num += wgt * q2[d];
                }
            }
            S.att[b * D + h * hd + d] = num / den;
        }
        __syncthreads();
    }
    for (int r0 = sl.p0 + 4 * warp; r0 < sl.p1; r0 += 4 * kWarps) {
        const float* w0 = wp + (size_t)(r0 - sl.p0) * D;
        const float val = lc_gemv4(w0, w0 + D, w0 + 2 * D, w0 + 3 * D, D, S.att, D, fl, nf);
        const int i = lane & 7;
        if (i < nf) S.x[fl[i] * D + r0 + (lane >> 3)] += val;
    }
    __syncthreads();
    push_rows(cl, S.x, D, sl.p0, sl.p1, fl, nf, cs, crank);
    if (!lc_sync(cl, S, cs)) return false;

    // ---- FFN up/gate + SwiGLU (generate.c:165-179)
    lc_norm(S.x, S.xn, rms2, fl, nf, D, S.red);
    for (int j = sl.f0 + 2 * warp; j < sl.f1; j += 2 * kWarps) {
        // rows: up j, up j+1, gate j, gate j+1 -> the gate of lane's up row is in lane ^ 16
        const float* u0 = wu + (size_t)(j - sl.f0) * D;
        const float* g0 = wg + (size_t)(j - sl.f0) * D;
        const float val = lc_gemv4(u0, u0 + D, g0, g0 + D, D, S.xn, D, fl, nf);
        const float gate = __shfl_xor_sync(0xffffffffu, val, 16);
        const int i = lane & 7;
        if (lane < 16 && i < nf) {
            const float sv = gate / (1.0f + expf(-gate));
            S.f[fl[i] * F + j + (lane >> 3)] = sv * val;
        }
    }
    __syncthreads();
    push_rows(cl, S.f, F, sl.f0, sl.f1, fl, nf, cs, crank);
    if (!lc_sync(cl, S, cs)) return false;

    // ---- down + residual (generate.c:181-184)
    for (int r0 = sl.p0 + 4 * warp; r0 < sl.p1; r0 += 4 * kWarps) {
        const float* w0 = wd + (size_t)(r0 - sl.p0) * F;
        const float val = lc_gemv4(w0, w0 + F, w0 + 2 * F, w0 + 3 * F, F, S.f, F, fl, nf);
        const int i = lane & 7;
        if (i < nf) S.x[fl[i] * D + r0 + (lane >> 3)] += val;
    }
    __syncthreads();
    push_rows(cl, S.x, D, sl.p0, sl.p1, fl, nf, cs, crank);
    return lc_sync(cl, S, cs);
}

// Greedy choice from the head partials for sequence b (generate.c:469-478,
// 510): returns the id and whether the reference draws from the RNG.
__device__ void lc_choose(const ClusterParams& cp, int b, int nhc, float* red, int* ints,
                          int& id, bool& draws) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float bv[2] = {-INFINITY, -INFINITY};
    int bi[2] = {0x7fffffff, 0x7fffffff};
    for (int c = threadIdx.x; c < nhc; c += blockDim.x)
        for (int k = 0; k < 2; k++) {
            const size_t at = ((size_t)b * nhc + c) * 2 + k;
            const float v = ldcg(cp.hpv + at);
            const int i = __ldcg(cp.hpi + at);
            if (better(v, i, bv[k], bi[k])) { bv[k] = v; bi[k] = i; }
        }
    for (int k = 0; k < 2; k++) warp_argmax(bv[k], bi[k]);
    __syncthreads();
    if (lane == 0) {
        red[warp] = bv[0]; ints[40 + warp] = bi[0];
        red[16 + warp] = bv[1]; ints[48 + warp] = bi[1];
    }
    __syncthreads();
    float v0 = red[0], v1 = red[16];
    int i0 = ints[40], i1 = ints[48];
    for (int w = 1; w < kWarps; w++) {
        if (better(red[w], ints[40 + w], v0, i0)) { v0 = red[w]; i0 = ints[40 + w]; }
        if (better(red[16 + w], ints[48 + w], v1, i1)) { v1 = red[16 + w]; i1 = ints[48 + w]; }
    }
    if (i0 == 0x7fffffff) i0 = 0;
    if (i1 == 0x7fffffff) i1 = 0;
    __syncthreads();
    if (isfinite(v0)) { id = i0; draws = true; }
    else if (cp.lp.s.ngram > 0) { id = i1; draws = isfinite(v1); }
    else { id = i0; draws = false; }
}

__device__ void lc_main(const ClusterParams& cp, unsigned char* smem, cg::cluster_group& cl,
                        int crank) {
    const LoopParams<float>& p = cp.lp;
    LcState S;
    S.bar = reinterpret_cast<unsigned long long*>(smem);
    S.ints = reinterpret_cast<int*>(smem + 64);
    S.red = reinterpret_cast<float*>(smem + 64 + 64 * 4);
    S.x = reinterpret_cast<float*>(smem + cp.off_x);
    S.xn = reinterpret_cast<float*>(smem + cp.off_xn);
    S.qkv = reinterpret_cast<float*>(smem + cp.off_qkv);
    S.attp = reinterpret_cast<float*>(smem + cp.off_attp);
    S.att = reinterpret_cast<float*>(smem + cp.off_att);
    S.f = reinterpret_cast<float*>(smem + cp.off_f);
    S.sc = reinterpret_cast<float*>(smem + cp.off_sc);
    S.kv = reinterpret_cast<float*>(smem + cp.off_kv);
    S.stage = reinterpret_cast<float*>(smem + cp.off_stage);
    S.rmsf = reinterpret_cast<float*>(smem + cp.off_rmsf);
    S.rope = reinterpret_cast<float2*>(smem + cp.off_rope);
    S.seq = reinterpret_cast<SeqMirror*>(smem + 576);
    const CSlice sl = cluster_slice(crank, cp.cs, p.Q, p.D, p.F);
    const int nhc = (cp.n_clusters - 1) * cp.cs;
    int* fl = S.ints;        // [16]
    int* hl = S.ints + 16;   // [16]
    int* toks = S.ints + 40; // [8] ids fed at this step

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) mbar_init(&S.bar[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.ints[38] = 0;
    }
    for (int b = threadIdx.x; b < p.B; b += blockDim.x) {
        const SeqState& g = p.seq[b];
        SeqMirror& m = S.seq[b];
        m.P = g.P; m.nnew = g.nnew; m.gen = g.gen; m.done = g.done; m.tok = g.tok;
        m.result = g.result; m.final_pos = g.final_pos; m.rng = g.rng;
    }
    for (int k = threadIdx.x; k < p.D; k += blockDim.x) S.rmsf[k] = __ldg(p.rmsf + k);
    __syncthreads();
    // prologue: prompts into the history, penalty counts, first bans (CTA b)
    for (int b = crank; b < p.B; b += cp.cs) {
        const SeqState* st = p.seq + b;
        if (st->done) continue;
        const int P = st->P;
        uint16_t* out = p.out_ids + (size_t)b * p.out_cap;
        for (int i = threadIdx.x; i < P; i += blockDim.x) out[i] = p.prompts[(size_t)b * p.prompt_stride + i];
        if (p.s.pen_active) {
            unsigned* cnt = p.counts + (size_t)b * p.V;
            for (int v = threadIdx.x; v < p.V; v += blockDim.x) cnt[v] = 0u;
            __syncthreads();
            for (int i = threadIdx.x; i < P; i += blockDim.x) {
                const int id = p.prompts[(size_t)b * p.prompt_stride + i];
                if (id < p.V) atomicAdd(&cnt[id], 1u);
            }
        }
        __syncthreads();
        if (p.s.ngram > 0) compute_bans(p, b, P);
    }
    __threadfence();
    unsigned layer_count = 0;      // layers issued so far (ring position)
    if (threadIdx.x == 0)
        for (int s = 0; s < kStages; s++) lc_issue_layer(cp, sl, S, s % p.L, s);
    unsigned issued = kStages;
    unsigned heads = 0;
    S.epoch = 0;
    if (threadIdx.x == 0) { S.ints[36] = 0; S.ints[37] = 0; }
    cl.sync();   // error slots are zero everywhere before anyone can set one
    bool ok = lc_sync(cl, S, cp.cs);

    for (int t = p.t0; ok && t < p.T; t++) {
        if (threadIdx.x == 0) {
            int nf = 0, nh = 0;
            for (int b = 0; b < p.B; b++) {
                const SeqMirror& m = S.seq[b];
                if (m.done || t >= m.P + m.nnew - 1) continue;
                fl[nf++] = b;
                if (t >= m.P - 1) hl[nh++] = b;
            }
            S.ints[32] = nf;
            S.ints[33] = nh;
            if (crank == 0 && p.stamps) p.stamps[t] = globaltimer_ns();
        }
        __syncthreads();
        const int nf = S.ints[32], nh = S.ints[33];
        if (nf == 0) break;
        // ids fed at position t and this position's RoPE row, in one round trip
        if (threadIdx.x < nf) {
            const int b = fl[threadIdx.x];
            const SeqMirror& m = S.seq[b];
            int tok = t < m.P ? (int)p.prompts[(size_t)b * p.prompt_stride + t] : m.tok;
            if (tok < 0 || tok >= p.V) {
                lc_fail(S, p.status, ST_DEVICE);
                tok = 0;
            }
            toks[threadIdx.x] = tok;
        }
        for (int j = threadIdx.x; j < p.hd / 2; j += blockDim.x)
            S.rope[j] = p.rope[(size_t)t * (p.hd / 2) + j];
        __syncthreads();
        // embedding of the token at position t (generate.c:86-88)
        for (int e = threadIdx.x; e < nf * p.D; e += blockDim.x) {
            const int i = e / p.D, k = e % p.D;
            S.x[fl[i] * p.D + k] = __ldg(p.tok_emb + (size_t)toks[i] * p.D + k);
        }
        __syncthreads();
        for (int l = 0; ok && l < p.L; l++) {
            const int s = layer_count % kStages;
            const unsigned parity = (layer_count / kStages) & 1u;
            // On expiry the status is set; the layer still runs (on stale
            // shared memory) so that every CTA meets the same cluster
            // barriers, and the next barrier turns the status into a
            // cluster-wide exit.
            if (!mbar_wait(&S.bar[s], parity, p.timeout_ns)) lc_fail(S, p.status, ST_TIMEOUT);
            ok = lc_layer(cp, sl, S, cl, crank, l, t, fl, nf, S.stage + (size_t)s * cp.stage_floats);
            layer_count++;
            // every thread of this CTA is past the stage: refill it kStages layers ahead
            if (threadIdx.x == 0 && ok) {
                lc_issue_layer(cp, sl, S, issued % p.L, s);
                issued++;
            }
        }
        if (!ok) break;
        if (nh == 0) continue;

        // ---- hand the final norm to the head CTAs (generate.c:187-191)
        lc_norm(S.x, S.xn, S.rmsf, hl, nh, p.D, S.red);
        {
            const int cols = (p.D + cp.cs - 1) / cp.cs, c0 = crank * cols, c1 = min(p.D, c0 + cols);
            for (int e = threadIdx.x; e < nh * (c1 - c0); e += blockDim.x) {
                const int b = hl[e / (c1 - c0)], k = c0 + e % (c1 - c0);
                cp.xfin[(size_t)b * p.D + k] = S.xn[b * p.D + k];
            }
            if (crank == 0)
                for (int b = threadIdx.x; b < p.B; b += blockDim.x) {
                    int g = -1;
                    for (int i = 0; i < nh; i++)
                        if (hl[i] == b) g = S.seq[b].gen;
                    cp.hgen[b] = g;
                }
        }
        __threadfence();
        ok = lc_sync(cl, S, cp.cs);
        if (!ok) break;
        heads++;
        if (crank == 0) {
            // ---- release the head CTAs, wait for all of them, choose the next ids
            if (threadIdx.x == 0) {
                st_release_u32(cp.go, heads);
                const unsigned target = heads * ((unsigned)nhc + p.extra_arrivals);
                const unsigned long long t0 = globaltimer_ns();
                while ((int)(ld_acquire_u32(cp.hdone) - target) < 0) {
                    if (globaltimer_ns() - t0 > p.timeout_ns) {
                        lc_fail(S, p.status, ST_TIMEOUT);
                        break;
                    }
                }
            }
            __syncthreads();
            for (int i = 0; i < nh; i++) {
                const int b = hl[i];
                int id;
                bool draws;
                lc_choose(cp, b, nhc, S.red, S.ints, id, draws);
                if (threadIdx.x == 0) {
                    SeqMirror& m = S.seq[b];
                    if (draws) (void)rng_f32(m.rng);
                    const int P = m.P, g = m.gen, nnew = m.nnew;
                    uint16_t* out = p.out_ids + (size_t)b * p.out_cap;
                    out[P + g] = (uint16_t)id;
                    if (p.s.pen_active) p.counts[(size_t)b * p.V + id] += 1u;
                    const int generated = g + 1;
                    m.gen = generated;
                    bool stop = false;
                    if (p.s.stop_len > 0 && generated >= p.s.min_new && generated >= p.s.stop_len) {
                        stop = true;
                        const int s0 = P + generated - p.s.stop_len;
                        for (int k = 0; k < p.s.stop_len; k++)
                            if (ld_u16_cg(out + s0 + k) != (int)p.s.stop_ids[k]) { stop = false; break; }
                    }
                    if (stop) {
                        m.result = P + generated - p.s.stop_len;
                        m.final_pos = P + g;
                        m.done = 1;
                    } else if (generated >= nnew) {
                        m.result = P + nnew;
                        m.final_pos = P + nnew;
                        m.done = 1;
                    } else {
                        m.tok = id;
                    }
                    S.ints[34] = m.done;
                    S.ints[35] = m.gen;
                }
                __syncthreads();
                if (p.s.ngram > 0 && !S.ints[34]) compute_bans(p, b, S.seq[b].P + S.ints[35]);
                __syncthreads();
            }
            // the other layer CTAs get the updated table before the barrier
            const int words = p.B * (int)(sizeof(SeqMirror) / 4);
            for (int e = threadIdx.x; e < words * cp.cs; e += blockDim.x) {
                const int r = e / words, w = e % words;
                if (r == 0) continue;
                int* dst = reinterpret_cast<int*>(cl.map_shared_rank(S.seq, r));
                dst[w] = reinterpret_cast<const int*>(S.seq)[w];
            }
            __threadfence();
        }
        ok = lc_sync(cl, S, cp.cs);
    }
    // release the head CTAs, publish the sequence table, drain bulk copies
    if (crank == 0) {
        for (int b = threadIdx.x; b < p.B; b += blockDim.x) {
            const SeqMirror& m = S.seq[b];
            SeqState& g = p.seq[b];
            g.gen = m.gen; g.done = m.done; g.tok = m.tok; g.result = m.result;
            g.final_pos = m.final_pos; g.rng = m.rng;
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) st_release_u32(cp.go, kExit);
    }
    if (threadIdx.x == 0 && crank == 0 && p.stamps) p.stamps[p.T] = globaltimer_ns();
    for (unsigned k = layer_count; k < issued; k++) {
        const int s = k % kStages;
        if (!mbar_wait(&S.bar[s], (k / kStages) & 1u, p.timeout_ns)) {
            atomicMax(p.status, (int)ST_TIMEOUT);
            break;
        }
    }
    __syncthreads();
    cl.sync();   // no CTA leaves while others may still write its shared memory
}

// ------------------------------------------------------------- head CTAs
__device__ void hc_main(const ClusterParams& cp, unsigned char* smem, int hc) {
    const LoopParams<float>& p = cp.lp;
    const int D = p.D;
    const int r0 = hc * cp.hc_rows, r1 = min(p.V, r0 + cp.hc_rows), nr = max(0, r1 - r0);
    // [0,8) mbarrier | [64,1088) 256 ints | [1088,1856) 192 floats | [2048,...) lm_head slice
    unsigned long long* bar = reinterpret_cast<unsigned long long*>(smem);
    int* ints = reinterpret_cast<int*>(smem + 64);
    float* red = reinterpret_cast<float*>(smem + 1088);
    float* emb = reinterpret_cast<float*>(smem + kHcEmbOffset);
    float* xs = reinterpret_cast<float*>(smem + cp.off_hc_x);
    const int nhc = (cp.n_clusters - 1) * cp.cs;
    const int nwords = (p.V + 31) >> 5;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // resident lm_head slice, rows padded to hc_ld floats (conflict-free reads)
    if (threadIdx.x == 0 && nr > 0) {
        mbar_expect_tx(bar, (unsigned)(nr * D * 4));
        for (int r = 0; r < nr; r++)
            bulk_g2s(emb + (size_t)r * cp.hc_ld, p.tok_emb + (size_t)(r0 + r) * D, D * 4, bar);
    }
    bool ok = nr == 0 || mbar_wait(bar, 0, p.timeout_ns);
    if (!ok) atomicMax(p.status, (int)ST_TIMEOUT);
    unsigned seen = 0;
    while (ok) {
        if (threadIdx.x == 0) {
            const unsigned long long t0 = globaltimer_ns();
            unsigned g;
            while ((g = ld_acquire_u32(cp.go)) == seen) {
                if (globaltimer_ns() - t0 > p.timeout_ns || ld_volatile_i32(p.status) != ST_OK) {
                    atomicMax(p.status, (int)ST_TIMEOUT);
                    g = kExit;
                    break;
                }
            }
            ints[0] = (int)g;
        }
        __syncthreads();
        const unsigned g = (unsigned)ints[0];
        if (g == kExit) break;
        seen = g;
        // which sequences need logits, and all normalised rows, in one round trip
        int* hg = ints + 16;   // [kBCMax] sampler step per sequence, -1 = none
        for (int b = threadIdx.x; b < p.B; b += blockDim.x) hg[b] = __ldcg(cp.hgen + b);
        for (int e = threadIdx.x; e < p.B * D; e += blockDim.x) xs[e] = ldcg(cp.xfin + e);
        __syncthreads();
        if (threadIdx.x == 0) {
            int nh = 0;
            for (int b = 0; b < p.B; b++)
                if (hg[b] >= 0) ints[8 + nh++] = b;
            ints[1] = nh;
        }
        __syncthreads();
        const int nh = ints[1];
        const int* hl = ints + 8;
        // thread per row: full dot products from the resident slice
        float bv[2][kBCMax];
        int bi[2][kBCMax];
#pragma unroll
        for (int i = 0; i < kBCMax; i++) {
            bv[0][i] = bv[1][i] = -INFINITY;
            bi[0][i] = bi[1][i] = 0x7fffffff;
        }
        const float* xb[kBCMax];
#pragma unroll
        for (int i = 0; i < kBCMax; i++) xb[i] = xs + (i < nh ? hl[i] : 0) * D;
        for (int r = threadIdx.x; r < nr; r += blockDim.x) {
            const float* __restrict__ er = emb + (size_t)r * cp.hc_ld;
            float acc[kBCMax];
#pragma unroll
            for (int i = 0; i < kBCMax; i++) acc[i] = 0.0f;
#pragma unroll 4
            for (int k = 0; k < D; k += 4) {
                const float4 w = *reinterpret_cast<const float4*>(er + k);
#pragma unroll
                for (int i = 0; i < kBCMax; i++)
                    if (i < nh) {
                        const float4 xv = *reinterpret_cast<const float4*>(xb[i] + k);
                        acc[i] = fmaf(w.x, xv.x, acc[i]);
                        acc[i] = fmaf(w.y, xv.y, acc[i]);
                        acc[i] = fmaf(w.z, xv.z, acc[i]);
                        acc[i] = fmaf(w.w, xv.w, acc[i]);
                    }
            }
            const int v = r0 + r;
            // static indices only: the per-sequence state stays in registers
#pragma unroll
            for (int i = 0; i < kBCMax; i++) {
                if (i >= nh) continue;
                const int b = hl[i];
                const float lg = v < 4 ? -INFINITY : acc[i];
                if (p.trace) {
                    const int gi = hg[b];
                    if (gi < p.trace_steps) p.trace[((size_t)b * p.trace_steps + gi) * p.V + v] = lg;
                }
                const unsigned cnt = p.s.pen_active ? __ldcg(p.counts + (size_t)b * p.V + v) : 0u;
                const bool ban = p.s.ngram > 0 &&
                                 ((__ldcg(p.banned + (size_t)b * nwords + (v >> 5)) >> (v & 31)) & 1u);
                const float tv = transform_value(lg, cnt, ban, p.s);
                if (better(tv, v, bv[0][i], bi[0][i])) { bv[0][i] = tv; bi[0][i] = v; }
                if (p.s.ngram > 0) {
                    const float tn = transform_value(lg, cnt, false, p.s);
                    if (better(tn, v, bv[1][i], bi[1][i])) { bv[1][i] = tn; bi[1][i] = v; }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kBCMax; i++) {
            if (i >= nh) continue;
#pragma unroll
            for (int k = 0; k < 2; k++) {
                float v = bv[k][i];
                int id = bi[k][i];
                warp_argmax(v, id);
                if (lane == 0) { red[(k * kBCMax + i) * kWarps + warp] = v; ints[64 + (k * kBCMax + i) * kWarps + warp] = id; }
            }
        }
        __syncthreads();
        if (threadIdx.x < 2 * nh) {
            const int k = threadIdx.x / nh, i = threadIdx.x % nh;
            const int base = (k * kBCMax + i) * kWarps;
            float v = red[base];
            int id = ints[64 + base];
            for (int w = 1; w < kWarps; w++)
                if (better(red[base + w], ints[64 + base + w], v, id)) { v = red[base + w]; id = ints[64 + base + w]; }
            const size_t at = ((size_t)hl[i] * nhc + hc) * 2 + k;
            cp.hpv[at] = v;
            cp.hpi[at] = id;
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) red_release_add_u32(cp.hdone, 1u);
    }
}

__global__ void __launch_bounds__(kThreads, 1) cluster_loop_kernel(const ClusterParams cp) {
    extern __shared__ __align__(128) unsigned char smem_c[];
    cg::cluster_group cl = cg::this_cluster();
    const int cid = blockIdx.x / cp.cs;
    if (cid == 0) {
        lc_main(cp, smem_c, cl, (int)cl.block_rank());
    } else {
        hc_main(cp, smem_c, blockIdx.x - cp.cs);
    }
}

}  // namespace mc

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
constexpr int kAttMaxG = 4;               // query heads per KV head (attention unit)
constexpr int kAttMaxND = 2;              // head_dim / 32, rounded up
constexpr int kAttMaxO = kAttMaxG * kAttMaxND;
constexpr int kAttMaxQ4 = 8 * kAttMaxND;      // head_dim / 4
constexpr int kAttMaxTile = 8 * 32;       // keys per tile: a run of 32 per warp

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
    unsigned off_x, off_xn, off_qkv, off_att, off_attp, off_f, off_sc, off_kv, off_stage;
    unsigned off_rope, off_pages;
    unsigned stage_floats;      // floats per weight stage (slice + rms1 + rms2)
    int kv_tile;                // keys staged per attention tile
    // head clusters
    int hc_rows;                // tok_emb rows per head CTA
    unsigned hc_ld;             // padded row stride (floats) of the resident slice
    unsigned off_hc_x;          // byte offset of the normalised-x copy
    // two-phase layer loop (mc_cluster_loop2.cuh)
    int v2;                     // 0: five-phase loop; 1: two-phase loop, cluster barriers
                                // between phases; 2: two-phase loop, partials exchanged by
                                // bulk copies onto the receivers' mbarriers (dataflow)
    unsigned off_wb;            // phase B weight buffer (off_stage: phase A buffer)
    unsigned off_pair;          // a unit's second key range: merged attention state
    int fpc;                    // up/gate rows (ffn_down columns) per CTA, padded
    int dp_b;                   // sequence stride of the ffn_down partials
    const float* proj_h;        // [L][K][D][G hd] attn_proj column blocks per KV head
    const float* down_s;        // [L][cs][D][fpc] ffn_down column blocks per CTA
    float* xfin;                // [Bcap][D] rmsnorm(x, rms_final), layer -> head
    int* hgen;                  // [Bcap] sampler step of each sequence in this head phase, -1 = none
    unsigned* go;               // head phases issued (or kExit)
    unsigned* hdone;            // head CTA arrivals
    unsigned long long* hkey;   // [2][Bcap][2] best (bans, no bans) over the head CTAs as
                                // hc_key(value, id), 0 = none; head phase h uses buffer h & 1,
                                // which CTA 0 zeroes when it releases phase h (every layer CTA
                                // read it, at phase h - 2, before the last step barrier)
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

// 1-D bulk copy of `bytes` (a multiple of 16, 16-byte aligned) from this
// CTA's shared memory to the same offset in CTA `rank` of the cluster; the
// bytes complete on that CTA's mbarrier at `bar`'s offset.
__device__ __forceinline__ void bulk_s2peer(const void* src, unsigned bytes, unsigned long long* bar,
                                            unsigned rank) {
    unsigned dst, rbar;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(dst) : "r"(smem_addr(src)), "r"(rank));
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(smem_addr(bar)), "r"(rank));
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(dst),
        "r"(smem_addr(src)), "r"(bytes), "r"(rbar)
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
    float* att;    // [B][D]
    float* attp;   // [units][G * hd + 2 G, padded to 4] merged states of split units
    float* f;      // [B][F]
    float* sc;     // [kWarps][G * hd + 2 G] per-warp attention states, [kWarps][kAttMaxG][32] probabilities
    float* kv;     // [K, V][kv_tile][hd]
    float* stage;  // [kStages][stage_floats] (two-phase loop: the phase A buffer)
    float* wb;     // two-phase loop: the phase B weight buffer
    float* dp;     // two-phase loop: ffn_down partials [cs][kBCMax][D] (shares kv's bytes)
    float2* rope;  // [hd/2] (cos, sin) at the current position
    unsigned long long* bar;  // [kStages]
    unsigned long long* kvbar;  // K/V tile copies
    int* pages;    // [kBCMax][pps] the sequences' page tables, copied at launch
    int* ints;     // [64]: 0..15 fwd list, 16..31 head list, 32.. scalars,
                   //       34 dataflow exchange stopped after a failed wait,
                   //       36/37 cluster error slots, 38 this CTA saw an error,
                   //       39 a K/V tile wait failed (thread 0)
    float* red;    // [64]
    struct SeqMirror* seq;    // [kBCMax] sequence table mirrored in shared memory
    int epoch;     // cluster barriers passed (identical in every CTA of the cluster)
    unsigned kvph;      // thread 0: phase of kvbar awaited next
    int kvpend;         // thread 0: a copy into the K/V tile is outstanding
    // dataflow exchange of the two-phase loop (all threads hold the same values)
    unsigned long long* atbar;   // attn_proj partials of every unit have landed
    unsigned long long* dpbar;   // [2] ffn_down partials of every CTA have landed (layer parity)
    unsigned atph;               // phase of atbar awaited next
    unsigned dpph;               // bit p: phase of dpbar[p] awaited next
    int nlayer;                  // layers run in this launch (selects the dpbar / partial buffer)
    unsigned long long* pairbar; // a unit's second key range: its merged state has landed
    float* pair;                 // [G hd + 2 G, padded to 4] that state (sent / received)
    unsigned prph;               // phase of pairbar awaited next
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
__device__ __forceinline__ void lc_norm(const float* x, float* xn, const float* scale, const int* list, int n,
                                        int D, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // a warp per sequence: sum of squares, then that sequence's row, so one
    // CTA barrier closes the phase
    for (int i = warp; i < n; i += kWarps) {
        const float* xr = x + list[i] * D;
        float* xo = xn + list[i] * D;
        float ss = 0.0f;
        for (int k = lane; k < D; k += 32) ss += xr[k] * xr[k];
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)D + 1e-5f);
        for (int k = lane; k < D; k += 32) xo[k] = xr[k] * inv * scale[k];
    }
    (void)red;
    __syncthreads();
}

// Copy cached K/V rows [a0, a0 + n) of one (sequence, KV head) into the
// K/V tile with two bulk copies that complete on kvbar.  The row at position
// t is produced in this step and is read from the qkv buffer instead, so the
// copies stop below it.  Thread 0 only; after a failed wait no further
// copies are issued (the cluster leaves at its next barrier).
// Keys [a0, a0 + rows) of (layer l, sequence b, KV head g) are contiguous
// within a page only, so the tile arrives as one K and one V copy per page
// it touches (row t, written in this step, is never copied).
__device__ __forceinline__ void att_issue_tile(const ClusterParams& cp, LcState& S, int l, int b, int g,
                                               int a0, int n, int t, int hd) {
    if (S.ints[39]) return;
    const LoopParams<float>& p = cp.lp;
    const int rows = min(n, t - a0);
    const unsigned bytes = rows > 0 ? (unsigned)(rows * hd * 4) : 0u;
    mbar_expect_tx(S.kvbar, 2 * bytes);
    const int plen = 1 << p.pg.shift;
    for (int r = 0; r < rows;) {
        const int j = a0 + r;
        const int seg = min(rows - r, plen - (j & (plen - 1)));
        const size_t row =
            kv_row_at(S.pages[b * p.pg.pps + (j >> p.pg.shift)], p.pg.shift, p.L, p.K, l, g, j);
        const unsigned sb = (unsigned)(seg * hd * 4);
        bulk_g2s(S.kv + (size_t)r * hd, p.kc + row * hd, sb, S.kvbar);
        bulk_g2s(S.kv + (size_t)(cp.kv_tile + r) * hd, p.vc + row * hd, sb, S.kvbar);
        r += seg;
    }
    S.kvpend = 1;
}

// Thread 0: wait (bounded) for the copies into the K/V tile.
__device__ __forceinline__ void att_wait_tile(const LoopParams<float>& p, LcState& S) {
    if (!S.kvpend || S.ints[39]) return;
    if (mbar_wait(S.kvbar, S.kvph, p.timeout_ns)) {
        S.kvph ^= 1u;
        S.kvpend = 0;
    } else {
        S.ints[39] = 1;
        lc_fail(S, p.status, ST_TIMEOUT);
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

// lc_sync in two halves, so that work can run between the arrival and the
// wait: lc_arrive publishes this CTA's failure flag of the epoch and
// arrives (release); lc_wait waits (acquire) and takes the cluster-wide
// decision.  A CTA arrives exactly once between two waits.
__device__ __forceinline__ void lc_arrive(cg::cluster_group& cl, LcState& S, int cs) {
    const int slot = 36 + (S.epoch & 1);
    __syncthreads();
    if (threadIdx.x == 0 && S.ints[38])
        for (int r = 0; r < cs; r++) cl.map_shared_rank(S.ints, r)[slot] = 1;
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ bool lc_wait(LcState& S) {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    const bool ok = S.ints[36 + (S.epoch & 1)] == 0;
    S.epoch++;
    return ok;
}

// Attention unit u: sequence fl[u / (ns K)], KV head (u / ns) mod K, keys
// [j0, j1) of split u mod ns.
struct AttUnit {
    int b, g, j0, j1;
};
__device__ __forceinline__ AttUnit att_unit(int u, int K, int ns, int per, int nkeys, const int* fl) {
    AttUnit a;
    const int s = u % ns;
    a.g = (u / ns) % K;
    a.b = fl[u / (ns * K)];
    a.j0 = min(s * per, nkeys);
    a.j1 = min(a.j0 + per, nkeys);
    return a;
}

// One run of up to 32 keys (a warp) for all G heads of a KV head: lane j
// scores key j against every head, then owns output dims lane + 32 i in
// P.V; (mrun, lrun, o) is the warp's running state per head.  Rows past the
// run may be read: their scores are masked and the V rows there are zero
// (the tile loop clears them).  HD > 0 fixes head_dim at compile time; 0 =
// any multiple of 4 up to 32 kAttMaxND.
template <int HD>
__device__ __forceinline__ void att_run(const float* kr0, const float* vr0, const float* q, float* pb,
                                        int kn, int hd_rt, int G, float scale,
                                        float (&mrun)[kAttMaxG], float (&lrun)[kAttMaxG],
                                        float (&o)[kAttMaxG][kAttMaxND]) {
    const int hd = HD > 0 ? HD : hd_rt;
    const int q4 = hd / 4;
    const int lane = threadIdx.x & 31;
    // scores; lane j starts at chunk (j mod hd/4) so that the rows the lanes
    // read fall in different banks
    const float* kr = kr0 + lane * hd;
    const int r = lane % q4;
    float dd[kAttMaxG];
#pragma unroll
    for (int h = 0; h < kAttMaxG; h++) dd[h] = 0.0f;
#pragma unroll 8
    for (int c = 0; c < (HD > 0 ? HD / 4 : kAttMaxQ4); c++)
        if (HD > 0 || c < q4) {
            const int cc = r + c < q4 ? r + c : r + c - q4;
            const float4 kk = *reinterpret_cast<const float4*>(kr + 4 * cc);
#pragma unroll
            for (int h = 0; h < kAttMaxG; h++)
                if (h < G) {
                    const float4 qq = *reinterpret_cast<const float4*>(q + h * hd + 4 * cc);
                    dd[h] = fmaf(qq.x, kk.x, dd[h]);
                    dd[h] = fmaf(qq.y, kk.y, dd[h]);
                    dd[h] = fmaf(qq.z, kk.z, dd[h]);
                    dd[h] = fmaf(qq.w, kk.w, dd[h]);
                }
        }
    const bool valid = lane < kn;
    float corr[kAttMaxG];
#pragma unroll
    for (int h = 0; h < kAttMaxG; h++) {
        corr[h] = 1.0f;
        if (h < G) {
            const float sv = valid ? dd[h] * scale : -INFINITY;
            const float mnew = fmaxf(mrun[h], warp_max(sv));
            const float e = valid ? expf(sv - mnew) : 0.0f;
            corr[h] = expf(mrun[h] - mnew);
            lrun[h] = lrun[h] * corr[h] + warp_sum(e);
            mrun[h] = mnew;
            pb[h * 32 + lane] = e;
        }
    }
    __syncwarp();
    // P.V, four keys at a time; V loads are shared by the heads
    float acc[kAttMaxG][kAttMaxND][2];
#pragma unroll
    for (int h = 0; h < kAttMaxG; h++)
#pragma unroll
        for (int i = 0; i < kAttMaxND; i++) acc[h][i][0] = acc[h][i][1] = 0.0f;
    const float* vr = vr0 + lane;
#pragma unroll 2
    for (int kk = 0; kk < 32; kk += 4) {
#pragma unroll
        for (int i = 0; i < kAttMaxND; i++)
            if (32 * i < hd && lane + 32 * i < hd) {
                const float* v = vr + kk * hd + 32 * i;
                const float v0 = v[0], v1 = v[hd], v2 = v[2 * hd], v3 = v[3 * hd];
#pragma unroll
                for (int h = 0; h < kAttMaxG; h++)
                    if (h < G) {
                        const float4 p4 = *reinterpret_cast<const float4*>(pb + h * 32 + kk);
                        acc[h][i][0] = fmaf(p4.x, v0, acc[h][i][0]);
                        acc[h][i][1] = fmaf(p4.y, v1, acc[h][i][1]);
                        acc[h][i][0] = fmaf(p4.z, v2, acc[h][i][0]);
                        acc[h][i][1] = fmaf(p4.w, v3, acc[h][i][1]);
                    }
            }
    }
    __syncwarp();   // pb is rewritten by this warp's next run
#pragma unroll
    for (int h = 0; h < kAttMaxG; h++)
#pragma unroll
        for (int i = 0; i < kAttMaxND; i++) o[h][i] = o[h][i] * corr[h] + (acc[h][i][0] + acc[h][i][1]);
}

// Attention phase of one layer at position t (generate.c:121-156), ending
// with the cluster barrier; false when the cluster must leave.  A unit
// stages its keys in tiles of kv_tile (bulk copies; the first tile of a
// CTA's first unit was requested before the QKV phase); the warps take the
// tile's runs of 32 keys.  The warps' states are merged per unit; split
// units exchange their merged states and every CTA combines them.
template <int HD>
__device__ bool lc_attention(const ClusterParams& cp, LcState& S, cg::cluster_group& cl, int crank,
                             int l, int t, const int* fl, int nf, int ns, int per, int units,
                             bool wrote_kv) {
    const LoopParams<float>& p = cp.lp;
    const int D = p.D, Q = p.Q, hd = HD > 0 ? HD : p.hd, K = p.K, G = p.G, H = p.H;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cs = cp.cs, nkeys = t + 1;
    const float scale = 1.0f / sqrtf((float)hd);
    const int ghd = G * hd, nd = (hd + 31) / 32;
    const int pw = ghd + 2 * G;                        // outputs, then (max, sum) per head
    const int pwp = (pw + 3) & ~3;                     // exchanged state stride (float4 pushes)
    float* part = S.sc;                                // [kWarps][pw]
    float* pb = S.sc + kWarps * pw + warp * 32 * kAttMaxG;   // this warp's probabilities
    float* ks = S.kv;
    float* vs = S.kv + (size_t)cp.kv_tile * hd;
    for (int u = crank; u < units; u += cs) {
        const AttUnit a = att_unit(u, K, ns, per, nkeys, fl);
        const float* q = S.qkv + a.b * Q + a.g * ghd;
        const float* kq = S.qkv + a.b * Q + D + a.g * hd;          // row t of K
        const float* vq = kq + p.kvd;                              // row t of V
        float mrun[kAttMaxG], lrun[kAttMaxG], o[kAttMaxG][kAttMaxND];
#pragma unroll
        for (int h = 0; h < kAttMaxG; h++) {
            mrun[h] = -INFINITY;
            lrun[h] = 0.0f;
#pragma unroll
            for (int i = 0; i < kAttMaxND; i++) o[h][i] = 0.0f;
        }
        for (int a0 = a.j0; a0 < a.j1; a0 += cp.kv_tile) {
            const int n = min(cp.kv_tile, a.j1 - a0);
            // every warp is past the previous tile (the barrier closing it,
            // or the merge of the previous unit): the tile buffer is free
            if (threadIdx.x == 0 && (u != crank || a0 != a.j0))
                att_issue_tile(cp, S, l, a.b, a.g, a0, n, t, hd);
            // Row t is produced in this step: the copies stop below it and its
            // slot is filled from the qkv buffer.  V rows from n up to the next
            // multiple of 32 are cleared for the unmasked P.V.  The copies
            // write neither range.
            if (t >= a0 && t < a0 + n)
                for (int c = threadIdx.x; c < 2 * hd; c += blockDim.x) {
                    if (c < hd) ks[(t - a0) * hd + c] = kq[c];
                    else vs[(t - a0) * hd + c - hd] = vq[c - hd];
                }
            const int pad = ((n + 31) & ~31) - n;
            for (int c = threadIdx.x; c < pad * hd; c += blockDim.x) vs[n * hd + c] = 0.0f;
            if (threadIdx.x == 0) att_wait_tile(p, S);
            __syncthreads();
            for (int rr = warp; rr * 32 < n; rr += kWarps)
                att_run<HD>(ks + (size_t)rr * 32 * hd, vs + (size_t)rr * 32 * hd, q, pb,
                            min(32, n - rr * 32), hd, G, scale, mrun, lrun, o);
            __syncthreads();
        }
        // merge the warps' states: (m, l) per head, then the outputs
#pragma unroll
        for (int h = 0; h < kAttMaxG; h++)
            if (h < G) {
                if (lane == 0) {
                    part[warp * pw + ghd + 2 * h] = mrun[h];
                    part[warp * pw + ghd + 2 * h + 1] = lrun[h];
                }
#pragma unroll
                for (int i = 0; i < kAttMaxND; i++) {
                    const int d = lane + 32 * i;
                    if (i < nd && d < hd) part[warp * pw + h * hd + d] = o[h][i];
                }
            }
        __syncthreads();
        float* dst = ns == 1 ? S.att + a.b * D + a.g * ghd : S.attp + (size_t)u * pwp;
        for (int i = threadIdx.x; i < ghd; i += blockDim.x) {
            const int h = i / hd;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kWarps; w++) M = fmaxf(M, part[w * pw + ghd + 2 * h]);
            float num = 0.0f, den = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; w++) {
                const float mw = part[w * pw + ghd + 2 * h];
                const float c = mw == -INFINITY ? 0.0f : expf(mw - M);   // a warp may see no keys
                den += c * part[w * pw + ghd + 2 * h + 1];
                num += c * part[w * pw + i];
            }
            if (ns == 1) {
                dst[i] = num / den;
            } else {
                dst[i] = num;
                if (i % hd == 0) {
                    dst[ghd + 2 * h] = M;
                    dst[ghd + 2 * h + 1] = den;
                }
            }
        }
        __syncthreads();
        if (ns == 1) push_block(cl, S.att, a.b * D + a.g * ghd, ghd, cs, crank);
        else push_block(cl, S.attp, u * pwp, pwp, cs, crank);
        __syncthreads();   // part is rewritten by this CTA's next unit
    }
    // K/V rows written in this step are read by later steps' bulk copies
    // (async proxy) in other CTAs: order them before the cluster barrier
    if (wrote_kv) asm volatile("fence.proxy.async.global;" ::: "memory");
    if (!lc_sync(cl, S, cs)) return false;
    // combine the splits (every CTA): per (sequence, head) the split weights
    // exp(m_s - M) and 1 / sum, then every output element
    if (ns > 1) {
        // ns > 1 implies nf K <= cs / 2, so nf H <= G cs / 2 <= 32 pairs and nf H ns <= 64
        float* wgt = S.sc;                                         // [pairs][ns]
        float* rden = S.sc + 64;                                   // [pairs]
        int* src = reinterpret_cast<int*>(S.sc + 96);              // [pairs] attp offset
        int* dsto = reinterpret_cast<int*>(S.sc + 128);            // [pairs] att offset
        for (int pr = threadIdx.x; pr < nf * H; pr += blockDim.x) {
            const int i = pr / H, h = pr - i * H, g = h / G, hh = h - g * G;
            const float* pp = S.attp + (size_t)((i * K + g) * ns) * pwp + ghd + 2 * hh;
            float M = -INFINITY;
            for (int s2 = 0; s2 < ns; s2++) M = fmaxf(M, pp[s2 * pwp]);
            float den = 0.0f;
            for (int s2 = 0; s2 < ns; s2++) {
                const float ms = pp[s2 * pwp];
                const float c = ms == -INFINITY ? 0.0f : expf(ms - M);   // a split may see no keys
                wgt[pr * ns + s2] = c;
                den += c * pp[s2 * pwp + 1];
            }
            rden[pr] = den;
            src[pr] = ((i * K + g) * ns) * pwp + hh * hd;
            dsto[pr] = fl[i] * D + h * hd;
        }
        __syncthreads();
        for (int e = threadIdx.x; e < nf * H * hd; e += blockDim.x) {
            const int pr = e / hd, d = e - pr * hd;
            const float* ps = S.attp + src[pr] + d;
            float num = 0.0f;
            for (int s2 = 0; s2 < ns; s2++) num += wgt[pr * ns + s2] * ps[s2 * pwp];
            S.att[dsto[pr] + d] = num / rden[pr];
        }
        __syncthreads();
    }
    return true;
}

// One layer for the sequences in the fwd list at position t.
__device__ bool lc_layer(const ClusterParams& cp, const CSlice& sl, LcState& S,
                         cg::cluster_group& cl, int crank, int l, int t, const int* fl, int nf,
                         const float* w) {
    const LoopParams<float>& p = cp.lp;
    const int D = p.D, Q = p.Q, F = p.F, hd = p.hd, K = p.K, H = p.H;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cs = cp.cs;
    const float* wq = w;
    const float* wp = wq + (size_t)(sl.q1 - sl.q0) * D;
    const float* wu = wp + (size_t)(sl.p1 - sl.p0) * D;
    const float* wg = wu + (size_t)(sl.f1 - sl.f0) * D;
    const float* wd = wg + (size_t)(sl.f1 - sl.f0) * D;
    const float* rms1 = w + slice_floats(sl, D, F);
    const float* rms2 = rms1 + D;

    // Attention units are (sequence, KV head, key split).  A unit's warps
    // take its keys 32 at a time, so keys are split over CTAs only past
    // kWarps * 32 keys per unit (and only while there are idle CTAs): below
    // that a split adds a merge after the cluster barrier and saves nothing.
    // The first K/V tile of this CTA's first unit is requested now so that
    // its transfer overlaps the QKV phase.
    const int nkeys = t + 1;
    const int ns = min(max(1, cs / (nf * K)), (nkeys + kWarps * 32 - 1) / (kWarps * 32));
    const int per = (nkeys + ns - 1) / ns;
    const int units = nf * K * ns;
    if (crank < units && threadIdx.x == 0) {
        const AttUnit a = att_unit(crank, K, ns, per, nkeys, fl);
        if (a.j1 > a.j0) att_issue_tile(cp, S, l, a.b, a.g, a.j0, min(cp.kv_tile, a.j1 - a.j0), t, hd);
    }

    // ---- QKV + RoPE + K/V append (generate.c:99-119)
    lc_norm(S.x, S.xn, rms1, fl, nf, D, S.red);
    bool wrote_kv = false;
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
                (isk ? p.kc : p.vc)[kv_row_at(S.pages[b * p.pg.pps + (t >> p.pg.shift)], p.pg.shift, p.L, K,
                                              l, g, t) * hd + d] = out;
                wrote_kv = true;
            }
        }
    }
    __syncthreads();
    push_rows(cl, S.qkv, Q, sl.q0, sl.q1, fl, nf, cs, crank);
    if (!lc_sync(cl, S, cs)) return false;

    // ---- attention (generate.c:121-156)
    bool ok;
    switch (hd) {
    case 16: ok = lc_attention<16>(cp, S, cl, crank, l, t, fl, nf, ns, per, units, wrote_kv); break;
    case 32: ok = lc_attention<32>(cp, S, cl, crank, l, t, fl, nf, ns, per, units, wrote_kv); break;
    case 64: ok = lc_attention<64>(cp, S, cl, crank, l, t, fl, nf, ns, per, units, wrote_kv); break;
    default: ok = lc_attention<0>(cp, S, cl, crank, l, t, fl, nf, ns, per, units, wrote_kv); break;
    }
    if (!ok) return false;

    // ---- PROJ + residual (generate.c:158-163)
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
    // With fewer 4-row groups than warps, each group's F-long rows are split
    // into nks slices over nks warps and the partial sums meet in shared
    // memory (S.sc is free after the attention phase).
    const int ngroups = (sl.p1 - sl.p0) >> 2;
    const int nks = ngroups > 0 ? kWarps / ngroups : 1;
    if (nks >= 2 && F % (4 * nks) == 0) {
        const int grp = warp % ngroups, ks = warp / ngroups, kl = F / nks;
        if (ks < nks) {
            const int k0 = ks * kl;
            const float* w0 = wd + (size_t)(4 * grp) * F + k0;
            S.sc[warp * 32 + lane] = lc_gemv4(w0, w0 + F, w0 + 2 * F, w0 + 3 * F, kl, S.f + k0, F, fl, nf);
        }
        __syncthreads();
        if (ks == 0) {
            float val = 0.0f;
            for (int s2 = 0; s2 < nks; s2++) val += S.sc[(s2 * ngroups + grp) * 32 + lane];
            const int i = lane & 7;
            if (i < nf) S.x[fl[i] * D + sl.p0 + 4 * grp + (lane >> 3)] += val;
        }
    } else {
        for (int r0 = sl.p0 + 4 * warp; r0 < sl.p1; r0 += 4 * kWarps) {
            const float* w0 = wd + (size_t)(r0 - sl.p0) * F;
            const float val = lc_gemv4(w0, w0 + F, w0 + 2 * F, w0 + 3 * F, F, S.f, F, fl, nf);
            const int i = lane & 7;
            if (i < nf) S.x[fl[i] * D + r0 + (lane >> 3)] += val;
        }
    }
    __syncthreads();
    push_rows(cl, S.x, D, sl.p0, sl.p1, fl, nf, cs, crank);
    return lc_sync(cl, S, cs);
}

// Greedy choice for head sequence b from the head CTAs' partials
// (generate.c:447-460 with top_k == 1: NaN never wins, ties go to the lowest
// id, and with every id banned the unbanned values decide) and its
// bookkeeping (generate.c:560-595): history, penalty counts, stop sequence,
// length.  One warp; lane 0 updates the mirrored table entry m and leaves
// done / generated in ints[40 + slot] / ints[48 + slot].
// Layer CTA 0: the residual rows of the sequences in hl (nh of them) and
// each sequence's sampler step (-1 = no logits this phase) for the head
// CTAs, and key buffer kb zeroed for their maxima; ends with a CTA barrier
// (the caller's release of `go` follows).
__device__ __forceinline__ void lc_publish_rows(const ClusterParams& cp, const LcState& S, const int* hl, int nh,
                                                int kb) {
    const LoopParams<float>& p = cp.lp;
    for (int i = threadIdx.x; i < 2 * p.Bcap; i += blockDim.x) cp.hkey[(size_t)kb * 2 * p.Bcap + i] = 0ull;
    for (int e = threadIdx.x; e < nh * p.D; e += blockDim.x) {
        const int b = hl[e / p.D], k = e % p.D;
        cp.xfin[(size_t)b * p.D + k] = S.x[b * p.D + k];
    }
    for (int b = threadIdx.x; b < p.B; b += blockDim.x) {
        int g = -1;
        for (int i = 0; i < nh; i++)
            if (hl[i] == b) g = S.seq[b].gen;
        cp.hgen[b] = g;
    }
    __syncthreads();
}

// Greedy selection key: for values that are not NaN, a > b between keys is
// better() between (value, id) pairs (larger value; equal values, +0 and
// -0 included, keep the lower id), and every key is nonzero.
__device__ __forceinline__ unsigned long long hc_key(float v, int id) {
    return ((unsigned long long)order_key(v) << 32) | (unsigned)~(unsigned)id;
}
// (value, id) of a key; 0 (no candidate) gives (-inf, 0x7fffffff).
__device__ __forceinline__ void hc_unkey(unsigned long long k, float& v, int& id) {
    if (k == 0ull) {
        v = -INFINITY;
        id = 0x7fffffff;
        return;
    }
    const unsigned o = (unsigned)(k >> 32);
    v = __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
    id = (int)~(unsigned)k;
}

// The next id of sequence b from the head CTAs' keys (buffer kb) and its
// bookkeeping in the mirror m (generate.c:447-468 and the loop around it).
// The leader also writes the id and the penalty count; the others only
// update their own mirror, which therefore stays identical to the leader's
// (the stop check reads earlier ids from out_ids and takes this one from
// here).
__device__ void lc_choose(const ClusterParams& cp, SeqMirror& m, int b, int slot, int* ints, int kb,
                          bool leader) {
    const LoopParams<float>& p = cp.lp;
    const int lane = threadIdx.x & 31;
    const bool twok = p.s.ngram > 0;
    if (lane != 0) return;
    float bv0, bv1 = -INFINITY;
    int bi0, bi1 = 0x7fffffff;
    const unsigned long long* key = cp.hkey + ((size_t)kb * p.Bcap + b) * 2;
    hc_unkey(__ldcg(key), bv0, bi0);
    if (twok) hc_unkey(__ldcg(key + 1), bv1, bi1);
    if (bi0 == 0x7fffffff) bi0 = 0;
    if (bi1 == 0x7fffffff) bi1 = 0;
    int id;
    bool draws;
    if (isfinite(bv0)) { id = bi0; draws = true; }
    else if (twok) { id = bi1; draws = isfinite(bv1); }
    else { id = bi0; draws = false; }
    if (draws) (void)rng_f32(m.rng);
    const int P = m.P, g = m.gen, nnew = m.nnew;
    uint16_t* out = p.out_ids + (size_t)b * p.out_cap;
    if (leader) {
        out[P + g] = (uint16_t)id;
        if (p.s.pen_active) p.counts[(size_t)b * p.V + id] += 1u;
    }
    const int generated = g + 1;
    m.gen = generated;
    bool stop = false;
    if (p.s.stop_len > 0 && generated >= p.s.min_new && generated >= p.s.stop_len) {
        stop = true;
        const int s0 = P + generated - p.s.stop_len;
        for (int k = 0; k < p.s.stop_len; k++) {
            const int have = s0 + k == P + g ? id : ld_u16_cg(out + s0 + k);
            if (have != (int)p.s.stop_ids[k]) { stop = false; break; }
        }
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
    ints[40 + slot] = m.done;
    ints[48 + slot] = m.gen;
}

__device__ void lc_main(const ClusterParams& cp, unsigned char* smem, cg::cluster_group& cl,
                        int crank) {
    const LoopParams<float>& p = cp.lp;
    LcState S;
    S.bar = reinterpret_cast<unsigned long long*>(smem);
    S.kvbar = S.bar + kStages;
    S.ints = reinterpret_cast<int*>(smem + 64);
    S.red = reinterpret_cast<float*>(smem + 64 + 64 * 4);
    S.x = reinterpret_cast<float*>(smem + cp.off_x);
    S.xn = reinterpret_cast<float*>(smem + cp.off_xn);
    S.qkv = reinterpret_cast<float*>(smem + cp.off_qkv);
    S.att = reinterpret_cast<float*>(smem + cp.off_att);
    S.attp = reinterpret_cast<float*>(smem + cp.off_attp);
    S.f = reinterpret_cast<float*>(smem + cp.off_f);
    S.sc = reinterpret_cast<float*>(smem + cp.off_sc);
    S.kv = reinterpret_cast<float*>(smem + cp.off_kv);
    S.stage = reinterpret_cast<float*>(smem + cp.off_stage);
    S.rope = reinterpret_cast<float2*>(smem + cp.off_rope);
    S.pages = reinterpret_cast<int*>(smem + cp.off_pages);
    S.seq = reinterpret_cast<SeqMirror*>(smem + 576);
    const CSlice sl = cluster_slice(crank, cp.cs, p.Q, p.D, p.F);
    const int nhc = (cp.n_clusters - 1) * cp.cs;
    int* fl = S.ints;        // [16]
    int* hl = S.ints + 16;   // [16]
    int* toks = S.ints + 40; // [8] ids fed at this step
    const int warp = threadIdx.x >> 5;
    for (int e = threadIdx.x; e < p.B * p.pg.pps; e += blockDim.x) S.pages[e] = __ldg(p.pg.table + e);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) mbar_init(&S.bar[s], 1);
        mbar_init(S.kvbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.ints[38] = 0;
        S.ints[39] = 0;
    }
    S.kvph = 0u;
    S.kvpend = 0;
    for (int b = threadIdx.x; b < p.B; b += blockDim.x) {
        const SeqState& g = p.seq[b];
        SeqMirror& m = S.seq[b];
        m.P = g.P; m.nnew = g.nnew; m.gen = g.gen; m.done = g.done; m.tok = g.tok;
        m.result = g.result; m.final_pos = g.final_pos; m.rng = g.rng;
    }
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

        heads++;
        if (crank == 0) {
            // ---- hand the sampling sequences' residual rows to the head CTAs
            // (which apply the final rmsnorm, generate.c:187-191), release
            // them, wait for all of them, choose the next ids
            lc_publish_rows(cp, S, hl, nh, (int)(heads & 1u));
            if (threadIdx.x == 0) {
                __threadfence();
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
            // one warp per head sequence; bans need the whole CTA afterwards
            if (warp < nh) lc_choose(cp, S.seq[hl[warp]], hl[warp], warp, S.ints, (int)(heads & 1u), true);
            __syncthreads();
            if (p.s.ngram > 0)
                for (int i = 0; i < nh; i++)
                    if (!S.ints[40 + i]) compute_bans(p, hl[i], S.seq[hl[i]].P + S.ints[48 + i]);
            __syncthreads();
            // the other layer CTAs get the updated table before the barrier
            const int words = p.B * (int)(sizeof(SeqMirror) / 4);
            for (int e = threadIdx.x; e < words * cp.cs; e += blockDim.x) {
                const int r = e / words, w = e % words;
                if (r == 0) continue;
                int* dst = reinterpret_cast<int*>(cl.map_shared_rank(S.seq, r));
                dst[w] = reinterpret_cast<const int*>(S.seq)[w];
            }
            // (the cluster barrier's release / acquire orders these stores)
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
    // a K/V tile still in flight after a failed wait
    if (threadIdx.x == 0 && S.kvpend && !mbar_wait(S.kvbar, S.kvph, p.timeout_ns))
        atomicMax(p.status, (int)ST_TIMEOUT);
    __syncthreads();
    cl.sync();   // no CTA leaves while others may still write its shared memory
}

// Logits of this head CTA's rows for the head sequences (generate.c:187-191)
// and the sampler's greedy choice among them.  A lane owns one row per
// round (a warp: 32 consecutive rows, conflict-free float4 reads when
// D % 32 == 0 since rows are padded to hc_ld = D + 4 floats) and runs its
// whole dot products with the nh <= NHP normalised rows (broadcast reads).
// Each lane keeps the best transformed value per slot; the warp's best per
// slot lands in red / ints (k = 0: with bans, k = 1: without, only when bans
// are active).
template <int NHP>
__device__ __forceinline__ void hc_rows(const ClusterParams& cp, const float* emb, const float* xs,
                                        const int* hl, const int* hg, int nh, int r0, int nr,
                                        float* red, int* ints) {
    constexpr int HR = 1;    // rows per lane and round (more measured slower)
    const LoopParams<float>& p = cp.lp;
    const int D = p.D;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwords = (p.V + 31) >> 5;
    const bool twok = p.s.ngram > 0;
    float bv0[NHP], bv1[NHP];
    int bi0[NHP], bi1[NHP];
    const float* xq[NHP];
#pragma unroll
    for (int q = 0; q < NHP; q++) {
        bv0[q] = bv1[q] = -INFINITY;
        bi0[q] = bi1[q] = 0x7fffffff;
        xq[q] = xs + (q < nh ? hl[q] : hl[0]) * D;
    }
    for (int blk = 32 * HR * warp; blk < nr; blk += 32 * HR * kWarps) {
        const float* er[HR];
#pragma unroll
        for (int j = 0; j < HR; j++) {
            const int row = blk + lane + 32 * j;
            er[j] = emb + (size_t)(row < nr ? row : 0) * cp.hc_ld;
        }
        float acc[HR][NHP];
#pragma unroll
        for (int j = 0; j < HR; j++)
#pragma unroll
            for (int q = 0; q < NHP; q++) acc[j][q] = 0.0f;
#pragma unroll 4
        for (int k = 0; k < D; k += 4) {
            float4 w[HR];
#pragma unroll
            for (int j = 0; j < HR; j++) w[j] = *reinterpret_cast<const float4*>(er[j] + k);
#pragma unroll
            for (int q = 0; q < NHP; q++) {
                if (q < nh) {
                    const float4 x = *reinterpret_cast<const float4*>(xq[q] + k);
#pragma unroll
                    for (int j = 0; j < HR; j++) {
                        acc[j][q] = fmaf(w[j].x, x.x, acc[j][q]);
                        acc[j][q] = fmaf(w[j].y, x.y, acc[j][q]);
                        acc[j][q] = fmaf(w[j].z, x.z, acc[j][q]);
                        acc[j][q] = fmaf(w[j].w, x.w, acc[j][q]);
                    }
                }
            }
        }
#pragma unroll
        for (int j = 0; j < HR; j++) {
            const int row = blk + lane + 32 * j;
            if (row >= nr) continue;
            const int vid = r0 + row;
#pragma unroll
            for (int q = 0; q < NHP; q++) {
                if (q >= nh) continue;
                const int b = hl[q];
                const float lg = vid < 4 ? -INFINITY : acc[j][q];
                if (p.trace) {
                    const int gi = hg[b];
                    if (gi < p.trace_steps) p.trace[((size_t)b * p.trace_steps + gi) * p.V + vid] = lg;
                }
                const unsigned cnt = p.s.pen_active ? __ldcg(p.counts + (size_t)b * p.V + vid) : 0u;
                const bool ban =
                    twok && ((__ldcg(p.banned + (size_t)b * nwords + (vid >> 5)) >> (vid & 31)) & 1u);
                const float tv = transform_value(lg, cnt, ban, p.s);
                if (better(tv, vid, bv0[q], bi0[q])) { bv0[q] = tv; bi0[q] = vid; }
                if (twok) {
                    const float tn = transform_value(lg, cnt, false, p.s);
                    if (better(tn, vid, bv1[q], bi1[q])) { bv1[q] = tn; bi1[q] = vid; }
                }
            }
        }
    }
    // the warp's best per slot
#pragma unroll
    for (int q = 0; q < NHP; q++) {
        if (q >= nh) continue;
        warp_argmax(bv0[q], bi0[q]);
        if (twok) warp_argmax(bv1[q], bi1[q]);
        if (lane == 0) {
            red[q * kWarps + warp] = bv0[q];
            ints[64 + q * kWarps + warp] = bi0[q];
            if (twok) {
                red[(kBCMax + q) * kWarps + warp] = bv1[q];
                ints[64 + (kBCMax + q) * kWarps + warp] = bi1[q];
            }
        }
    }
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
        // the final rmsnorm of each sampling sequence (generate.c:187-189),
        // in place: warp b normalises row b (B <= kBCMax <= kWarps)
        static_assert(kBCMax <= kWarps, "a warp per sequence");
        {
            const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
            if (w < p.B && hg[w] >= 0) {
                float* xr = xs + w * D;
                float ss = 0.0f;
                for (int k = lane; k < D; k += 32) ss += xr[k] * xr[k];
                ss = warp_sum(ss);
                const float inv = 1.0f / sqrtf(ss / (float)D + 1e-5f);
                for (int k = lane; k < D; k += 32) xr[k] = xr[k] * inv * __ldg(p.rmsf + k);
            }
        }
        __syncthreads();
        const int nh = ints[1];
        const int* hl = ints + 8;
        switch (nh <= 1 ? 1 : nh <= 2 ? 2 : nh <= 4 ? 4 : 8) {
        case 1: hc_rows<1>(cp, emb, xs, hl, hg, nh, r0, nr, red, ints); break;
        case 2: hc_rows<2>(cp, emb, xs, hl, hg, nh, r0, nr, red, ints); break;
        case 4: hc_rows<4>(cp, emb, xs, hl, hg, nh, r0, nr, red, ints); break;
        default: hc_rows<8>(cp, emb, xs, hl, hg, nh, r0, nr, red, ints); break;
        }
        __syncthreads();
        if (threadIdx.x < (p.s.ngram > 0 ? 2 : 1) * nh) {
            const int k = threadIdx.x / nh, i = threadIdx.x % nh;
            const int base = (k * kBCMax + i) * kWarps;
            float v = red[base];
            int id = ints[64 + base];
            for (int w = 1; w < kWarps; w++)
                if (better(red[base + w], ints[64 + base + w], v, id)) { v = red[base + w]; id = ints[64 + base + w]; }
            // this CTA's best into the sequence's maximum over all head CTAs
            // (no candidate: every value was NaN, nothing to publish)
            if (id != 0x7fffffff) atomicMax(cp.hkey + ((size_t)(g & 1) * p.Bcap + hl[i]) * 2 + k, hc_key(v, id));
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) red_release_add_u32(cp.hdone, 1u);
    }
}

}  // namespace mc

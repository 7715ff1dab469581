// mc_cluster_loop2.cuh — the two-phase layer loop of the cluster-resident
// token loop (used when every (sequence, KV head) pair of the batch gets a
// CTA of the layer cluster; the five-phase loop of mc_cluster_loop.cuh
// serves the other shapes).  Head CTAs, the hand-off and the sampler are
// those of mc_cluster_loop.cuh.
//
// One layer of forward_one (generate.c:97-185) for the sequences fed at
// position t, in two phases separated by cluster barriers:
//
//  A. unit phase: CTA u < nf K owns sequence fl[u / K] and KV head u % K.
//     It normalises that sequence's residual (rms1), computes the Q rows of
//     the head group's G query heads and the K and V rows of its KV head
//     (+RoPE, K/V appended to the paged cache), attends over keys 0..t for
//     the G heads, and multiplies the G heads' outputs by their columns of
//     attn_proj: a D-long partial of x += W_proj . attn, pushed to every CTA.
//  B. FFN phase: every CTA adds the K partials of each sequence to its
//     residual (KV head order), normalises (rms2), computes its slice of
//     up/gate rows and the SwiGLU product, and multiplies that slice by its
//     columns of ffn_down: a D-long partial per sequence, pushed to every
//     CTA.  The next layer (or the hand-off to the head CTAs, which apply
//     the final norm) starts by adding the cs partials in CTA order.
// At D = 128 the RMSNorms of both phases run in the registers of each warp
// that computes rows (lane j: elements 4j .. 4j + 3), without a phase of
// their own.
//
// Every CTA therefore keeps the whole residual stream of every sequence,
// updated by the same additions in the same order (identical everywhere).
// The column blocks of attn_proj per KV head and of ffn_down per CTA are
// contiguous, transposed copies made by cl2_relayout_kernel when the
// weights change ([input][output]: a thread per output reads consecutive
// addresses across the warp).
// Each phase's weights (A: Q/K/V rows of the CTA's KV head, its attn_proj
// block, rms1; B: its up/gate rows, its ffn_down block, rms2) stream into a
// single buffer per phase by bulk copies issued as soon as the phase is
// done with the previous layer's, so a copy has the other phase's duration
// to land.  The down partials share their shared memory with the K/V tile:
// they are summed before the tile's first copy is issued and written by
// other CTAs only after the barrier that ends the attention.
//
// Dataflow exchange (plan v2 == 2): instead of remote stores closed by a
// cluster barrier, each CTA sends its partial with one bulk copy per peer
// (shared::cta -> shared::cluster) that completes on the receiver's
// mbarrier, and a receiver waits only for the bytes it sums:
//  * atbar: the nf K units' attn_proj partials (single buffer).  A unit
//    writes layer n+1's partial only after it summed every CTA's layer-n
//    down partials, each sent after that CTA had summed layer n's attn_proj
//    partials, so no copy lands on a buffer still being read, and the
//    sender's own slot has been read by every receiver.
//  * dpbar[n & 1]: the cs CTAs' ffn_down partials of layer n, in two
//    buffers by layer parity (a CTA that is not a unit may still be summing
//    layer n's while a fast peer already sends layer n+1's; layer n+2's
//    needs its layer n+1 partial first).  Both buffers share the K/V
//    tile's bytes: layer n's is summed before the tile of layer n+1 is
//    requested, and no layer n+1 partial exists before every unit has
//    finished that layer's attention.
// Arrivals may precede the receiver's expect_tx (tx-count goes negative in
// between, as the mbarrier allows); the chains above keep every phase
// complete before bytes of the next one of the same barrier are sent.  One
// cluster barrier per step remains, split into an arrival after the layers
// and a wait once every layer CTA has chosen the next ids into its own copy
// of the sequence table: it orders the K/V rows written in the step before
// later steps' bulk reads and makes failures cluster-wide.
// After a failed wait a CTA stops arming, waiting and sending for the rest
// of the launch (its peers' waits then expire too) and every CTA leaves at
// that step's barrier; a launch that failed this way lets in-flight copies
// land before its CTAs exit.
#pragma once

#include "mc_cluster_loop.cuh"

namespace mc {

// The thread that issues and awaits the K/V tile copies (its LcState holds
// the tile's mbarrier phase): lane 0 of the last warp, so that warp 0 is
// free for the RMSNorm that follows the first request.
constexpr int kTileThread = kThreads - 32;

// proj_h[l][g][c][i] = W_proj[l][i][g G hd + c]; down_s[l][s][j][i] =
// W_down[l][i][s fpc + j] (0 past F).
__global__ void cl2_relayout_kernel(const float* __restrict__ w_proj, const float* __restrict__ w_down,
                                    float* __restrict__ proj_h, float* __restrict__ down_s, int L, int D,
                                    int F, int K, int ghd, int cs, int fpc) {
    const size_t n1 = (size_t)L * K * D * ghd, n2 = (size_t)L * cs * D * fpc;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n1 + n2;
         e += (size_t)gridDim.x * blockDim.x) {
        if (e < n1) {
            const size_t i = e % D, c = (e / D) % ghd, g = (e / ((size_t)D * ghd)) % K, l = e / ((size_t)D * ghd * K);
            proj_h[e] = w_proj[(l * D + i) * D + g * ghd + c];
        } else {
            const size_t f = e - n1;
            const size_t i = f % D, j = (f / D) % fpc, c = (f / ((size_t)D * fpc)) % cs, l = f / ((size_t)D * fpc * cs);
            const size_t col = c * fpc + j;
            down_s[f] = col < (size_t)F ? w_down[(l * D + i) * F + col] : 0.0f;
        }
    }
}

// Phase A weights of layer l for KV head g: Q rows of heads g G .. g G +
// G - 1, the K and V rows of KV head g, the attn_proj block of g, rms1.
__device__ void cl2_issue_a(const ClusterParams& cp, LcState& S, int l, int g) {
    const LoopParams<float>& p = cp.lp;
    const size_t D = p.D;
    const int G = p.G, hd = p.hd, ghd = G * hd;
    float* dst = S.stage;
    const unsigned qb = (unsigned)(ghd * D * 4), kb = (unsigned)(hd * D * 4), pb = (unsigned)(D * ghd * 4);
    mbar_expect_tx(&S.bar[0], qb + 2 * kb + pb + (unsigned)(D * 4));
    const float* wl = p.w_qkv + (size_t)l * p.Q * D;
    bulk_g2s(dst, wl + (size_t)g * ghd * D, qb, &S.bar[0]);
    bulk_g2s(dst + (size_t)ghd * D, wl + (D + (size_t)g * hd) * D, kb, &S.bar[0]);
    bulk_g2s(dst + (size_t)(ghd + hd) * D, wl + (D + (size_t)p.kvd + (size_t)g * hd) * D, kb, &S.bar[0]);
    bulk_g2s(dst + (size_t)(ghd + 2 * hd) * D, cp.proj_h + ((size_t)l * p.K + g) * D * ghd, pb, &S.bar[0]);
    bulk_g2s(dst + (size_t)(ghd + 2 * hd) * D + D * ghd, p.rms1 + (size_t)l * D, (unsigned)(D * 4), &S.bar[0]);
}

// Phase B weights of layer l for this CTA: up and gate rows [f0, f1), its
// ffn_down block [fpc][D], rms2.
__device__ void cl2_issue_b(const ClusterParams& cp, const CSlice& sl, LcState& S, int l, int crank) {
    const LoopParams<float>& p = cp.lp;
    const size_t D = p.D, fpc = cp.fpc;
    const unsigned nfr = (unsigned)(sl.f1 - sl.f0);
    float* dst = S.wb;
    const unsigned ub = (unsigned)(nfr * D * 4), db = (unsigned)(D * fpc * 4);
    mbar_expect_tx(&S.bar[1], 2 * ub + db + (unsigned)(D * 4));
    if (nfr) {
        bulk_g2s(dst, p.w_up + ((size_t)l * p.F + sl.f0) * D, ub, &S.bar[1]);
        bulk_g2s(dst + fpc * D, p.w_gate + ((size_t)l * p.F + sl.f0) * D, ub, &S.bar[1]);
    }
    bulk_g2s(dst + 2 * fpc * D, cp.down_s + ((size_t)l * cp.cs + crank) * D * fpc, db, &S.bar[1]);
    bulk_g2s(dst + 2 * fpc * D + D * fpc, p.rms2 + (size_t)l * D, (unsigned)(D * 4), &S.bar[1]);
}

// 32 rows of length len (row stride ld) against one vector: lane j returns
// the dot product of row r0 + j (0 past nrows).  Lanes read 16-byte chunks
// of each row (a warp reads 512 contiguous bytes), then a transposed
// reduction.  len % 4 == 0.
__device__ __forceinline__ float cl2_dot32(const float* rows, int ld, int r0, int nrows, int len,
                                           const float* xv) {
    const int lane = threadIdx.x & 31;
    float acc[32];
#pragma unroll
    for (int j = 0; j < 32; j++) acc[j] = 0.0f;
    for (int k = 4 * lane; k < len; k += 128) {
        const float4 x = *reinterpret_cast<const float4*>(xv + k);
#pragma unroll
        for (int j = 0; j < 32; j++) {
            if (r0 + j < nrows) {
                const float4 w = *reinterpret_cast<const float4*>(rows + (size_t)(r0 + j) * ld + k);
                acc[j] += w.x * x.x + w.y * x.y + w.z * x.z + w.w * x.w;
            }
        }
    }
    return transpose_reduce32(acc);
}

// RMSNorm (generate.c:57-63) of one D = 128 row, in registers: lane j of
// the calling warp returns elements 4j .. 4j + 3 of x * inv_rms * scale.
__device__ __forceinline__ float4 cl2_norm128(const float* x, const float* scale) {
    const int lane = threadIdx.x & 31;
    const float4 v = *reinterpret_cast<const float4*>(x + 4 * lane);
    float ss = v.x * v.x;
    ss += v.y * v.y;
    ss += v.z * v.z;
    ss += v.w * v.w;
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / 128.0f + 1e-5f);
    const float4 sc = *reinterpret_cast<const float4*>(scale + 4 * lane);
    return make_float4(v.x * inv * sc.x, v.y * inv * sc.y, v.z * inv * sc.z, v.w * inv * sc.w);
}

// cl2_dot32 for rows of length 128 against a vector held in registers as
// cl2_norm128 returns it.
__device__ __forceinline__ float cl2_dot32_r(const float* rows, int ld, int r0, int nrows, float4 x) {
    const int lane = threadIdx.x & 31;
    float acc[32];
#pragma unroll
    for (int j = 0; j < 32; j++) {
        acc[j] = 0.0f;
        if (r0 + j < nrows) {
            const float4 w = *reinterpret_cast<const float4*>(rows + (size_t)(r0 + j) * ld + 4 * lane);
            acc[j] = w.x * x.x + w.y * x.y + w.z * x.z + w.w * x.w;
        }
    }
    return transpose_reduce32(acc);
}

// Up/gate rows [f0, f1) of this CTA's slice and their SwiGLU
// (generate.c:165-179) at D = 128, for nf <= NFP sequences normalised in
// registers (xr[q]: sequence fl[q], as cl2_norm128 returns it).  A warp
// takes H = 16 / NFP F indices per round: rows up j .. j + H - 1, then gate
// j .. j + H - 1, lane r NFP + q holding row r against sequence q after the
// transposed reduction, so the gate of an up value sits in lane ^ 16.  Rows
// are read up to the next multiple of H past f1 (inside the weight buffer
// when the slice is a multiple of 16 rows; those results are not stored).
template <int NFP>
__device__ __forceinline__ void cl2_upgate(const float* wu, const float* wg, const float4 (&xr)[kBCMax],
                                           const int* fl, int nf, int f0, int f1, int fpc, float* f) {
    constexpr int R = 32 / NFP, H = R / 2;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int j = f0 + H * warp; j < f1; j += H * kWarps) {
        float acc[32];
#pragma unroll
        for (int r = 0; r < R; r++) {
            const float* row = r < H ? wu + (size_t)(j - f0 + r) * 128 : wg + (size_t)(j - f0 + r - H) * 128;
            const float4 w = *reinterpret_cast<const float4*>(row + 4 * lane);
#pragma unroll
            for (int q = 0; q < NFP; q++) {
                const float4 x = xr[q];
                acc[r * NFP + q] = q < nf ? w.x * x.x + w.y * x.y + w.z * x.z + w.w * x.w : 0.0f;
            }
        }
        const float val = transpose_reduce32(acc);
        const float gate = __shfl_xor_sync(0xffffffffu, val, 16);
        const int q = lane % NFP, r = lane / NFP;
        if (lane < 16 && q < nf && j + r < f1) {
            const float sv = gate / (1.0f + expf(-gate));
            f[fl[q] * fpc + (j - f0) + r] = sv * val;
        }
    }
}

// x[fl[i]] += sum over the cs CTAs' ffn_down partials (CTA order; partial
// of CTA c for the i-th fed sequence at dp[(c dp_b + i) D]): a thread per
// element, all cs loads issued before the additions.  All threads; ends
// with a CTA barrier.
__device__ __forceinline__ void cl2_add_down(const ClusterParams& cp, LcState& S, const float* dp,
                                             const int* fl, int nf) {
    const int D = cp.lp.D, cs = cp.cs;
    const size_t cstride = (size_t)cp.dp_b * D;
    for (int e = threadIdx.x; e < nf * D; e += blockDim.x) {
        const int i = e / D, k = e % D, b = fl[i];
        const float* src = dp + (size_t)i * D + k;
        float v[16];
#pragma unroll
        for (int c = 0; c < 16; c++) v[c] = c < cs ? src[c * cstride] : 0.0f;
        float s = 0.0f;
#pragma unroll
        for (int c = 0; c < 16; c++) s += v[c];
        S.x[b * D + k] += s;
    }
    __syncthreads();
}

// Thread 0: wait (bounded) for the phase `ph` of a dataflow mbarrier.  A
// failure stops the exchange for the rest of the launch (ints[34]).
__device__ __forceinline__ void df_wait(const LoopParams<float>& p, LcState& S, unsigned long long* bar,
                                        unsigned ph) {
    if (!S.ints[34] && !mbar_wait(bar, ph, p.timeout_ns)) {
        S.ints[34] = 1;
        lc_fail(S, p.status, ST_TIMEOUT);
    }
}

// One layer (two phases).  pa / pb: parities of the phase buffers' next
// copies; `first`: the residual is the embedding.  DF: partials move by
// bulk copies onto the receivers' mbarriers and the layer ends with the
// ffn_down partials summed; otherwise by remote stores, each phase closed
// by a cluster barrier, and the next layer starts with that sum.
// HD / DC / FC / GC > 0 fix head_dim, dim, the F slice and the query heads
// per KV head at compile time (the default model's 32 / 128 / 32 / 2), so
// that the short loops of every phase have constant trip counts and their
// loads issue ahead of the arithmetic; 0 = read them from the parameters.
template <int HD, int DC, int FC, int GC, bool DF>
__device__ __forceinline__ bool cl2_layer(const ClusterParams& cp, const CSlice& sl, LcState& S, cg::cluster_group& cl,
                          int crank, int l, int t, const int* fl, int nf, bool first, unsigned& pa,
                          unsigned& pbp) {
    const LoopParams<float>& p = cp.lp;
    const int D = DC > 0 ? DC : p.D, K = p.K, G = GC > 0 ? GC : p.G, hd = HD > 0 ? HD : p.hd, cs = cp.cs;
    const int ghd = G * hd, rows_a = ghd + 2 * hd, fpc = FC > 0 ? FC : cp.fpc;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nd = (hd + 31) / 32;
    if (!DF && !first) cl2_add_down(cp, S, S.dp, fl, nf);
    const int nu = nf * K;
    const bool unit = crank < nu;
    // this layer's attn_proj partials: one from each unit but this CTA
    if (DF && threadIdx.x == 0 && !S.ints[34])
        mbar_expect_tx(S.atbar, (unsigned)(nu - (unit ? 1 : 0)) * (unsigned)(D * 4));

    // ------------------------------------------------ phase A: unit crank
    if (!mbar_wait(&S.bar[0], pa, p.timeout_ns)) lc_fail(S, p.status, ST_TIMEOUT);
    pa ^= 1u;
    const int nkeys = t + 1;
    // DF, when a unit's keys need more than one tile and the cluster has a
    // CTA to spare for every unit: CTA nu + u (the second of unit u: same
    // sequence and KV head, since nu is a multiple of K) attends over keys
    // [kv_tile, t] and sends its merged state to u, which covers
    // [0, kv_tile) and merges the two (the same online-softmax merge as its
    // warps').  The second computes the Q/K/V rows itself (row t is in its
    // range) but leaves the cache append to the unit.
    const bool split = DF && 2 * nu <= cs && nkeys > cp.kv_tile;
    const bool second = split && crank >= nu && crank < 2 * nu;
    const bool attends = unit || second;
    const int key0 = second ? cp.kv_tile : 0;
    const int key1 = unit && split ? cp.kv_tile : nkeys;
    const unsigned pair_bytes = (unsigned)(((ghd + 2 * G + 3) & ~3) * 4);
    if (split && unit && threadIdx.x == 0 && !S.ints[34]) mbar_expect_tx(S.pairbar, pair_bytes);
    const int g = crank % K;
    const int b = attends ? fl[(second ? crank - nu : crank) / K] : 0;
    bool wrote_kv = false;
    // DF: this layer's FFN weights are requested here, behind the first K/V
    // tile, which the unit phase waits on first (the barrier variant
    // requests them at the end of the previous layer)
    if (DF && !attends && threadIdx.x == kTileThread) cl2_issue_b(cp, sl, S, l, crank);
    if (attends) {
        // the first K/V tile is requested by the last warp (warp 0 normalises)
        if (threadIdx.x == kTileThread) {
            att_issue_tile(cp, S, l, b, g, key0, min(cp.kv_tile, key1 - key0), t, hd);
            if (DF) cl2_issue_b(cp, sl, S, l, crank);
        }
        const float* wa = S.stage;
        const float* rms1 = wa + (size_t)(rows_a + ghd) * D;
        // rmsnorm of sequence b (generate.c:57-63): at D = 128 each warp that
        // computes rows normalises in registers; otherwise one warp sums and
        // the CTA scales
        float4 xn4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float* xn = S.xn + b * D;
        if constexpr (DC == 128) {
            if (32 * warp < rows_a) xn4 = cl2_norm128(S.x + b * D, rms1);
        } else {
            if (warp == 0) {
                float ss = 0.0f;
                for (int k = lane; k < D; k += 32) ss += S.x[b * D + k] * S.x[b * D + k];
                ss = warp_sum(ss);
                if (lane == 0) S.red[0] = 1.0f / sqrtf(ss / (float)D + 1e-5f);
            }
            __syncthreads();
            const float inv = S.red[0];
            for (int k = threadIdx.x; k < D; k += blockDim.x) xn[k] = S.x[b * D + k] * inv * rms1[k];
            __syncthreads();
        }
        // Q rows of the G heads, K and V rows of KV head g (generate.c:99-119)
        for (int r0 = 32 * warp; r0 < rows_a; r0 += 32 * kWarps) {
            const float val =
                DC == 128 ? cl2_dot32_r(wa, D, r0, rows_a, xn4) : cl2_dot32(wa, D, r0, rows_a, D, xn);
            const float other = __shfl_xor_sync(0xffffffffu, val, 1);    // RoPE partner (2p <-> 2p+1)
            const int r = r0 + lane;
            if (r < rows_a) {
                const bool isq = r < ghd, isk = !isq && r < ghd + hd;
                const int d = isq ? r % hd : isk ? r - ghd : r - ghd - hd;
                float out = val;
                if (isq || isk) {
                    const float2 rr = S.rope[d / 2];
                    out = (d & 1) ? other * rr.y + val * rr.x : val * rr.x - other * rr.y;
                }
                S.qkv[r] = out;
                if (!isq && unit) {
                    const int page = S.pages[b * p.pg.pps + (t >> p.pg.shift)];
                    (isk ? p.kc : p.vc)[kv_row_at(page, p.pg.shift, p.L, K, l, g, t) * hd + d] = out;
                    wrote_kv = true;
                }
            }
        }
        __syncthreads();
        // attention of the G heads over keys 0..t (generate.c:121-156)
        const float scale = 1.0f / sqrtf((float)hd);
        const int pw = ghd + 2 * G;
        float* part = S.sc;                                       // [kWarps][pw]
        float* pbuf = S.sc + kWarps * pw + warp * 32 * kAttMaxG;   // this warp's probabilities
        float* ks = S.kv;
        float* vs = S.kv + (size_t)cp.kv_tile * hd;
        const float* q = S.qkv;
        const float* kq = S.qkv + ghd;
        const float* vq = kq + hd;
        float mrun[kAttMaxG], lrun[kAttMaxG], o[kAttMaxG][kAttMaxND];
#pragma unroll
        for (int h = 0; h < kAttMaxG; h++) {
            mrun[h] = -INFINITY;
            lrun[h] = 0.0f;
#pragma unroll
            for (int i = 0; i < kAttMaxND; i++) o[h][i] = 0.0f;
        }
        for (int a0 = key0; a0 < key1; a0 += cp.kv_tile) {
            const int n = min(cp.kv_tile, key1 - a0);
            if (threadIdx.x == kTileThread && a0 != key0) att_issue_tile(cp, S, l, b, g, a0, n, t, hd);
            if (t >= a0 && t < a0 + n)
                for (int c = threadIdx.x; c < 2 * hd; c += blockDim.x) {
                    if (c < hd) ks[(t - a0) * hd + c] = kq[c];
                    else vs[(t - a0) * hd + c - hd] = vq[c - hd];
                }
            const int pad = ((n + 31) & ~31) - n;
            for (int c = threadIdx.x; c < pad * hd; c += blockDim.x) vs[n * hd + c] = 0.0f;
            if (threadIdx.x == kTileThread) att_wait_tile(p, S);
            __syncthreads();
            for (int rr = warp; rr * 32 < n; rr += kWarps)
                att_run<HD>(ks + (size_t)rr * 32 * hd, vs + (size_t)rr * 32 * hd, q, pbuf, min(32, n - rr * 32),
                            hd, G, scale, mrun, lrun, o);
            __syncthreads();
        }
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
        if (second) {
            // this range's state merged over the warps, unnormalised:
            // pair[i < G hd] = sum_w c_w o_w, pair[G hd + 2h] = max_w m_w,
            // pair[G hd + 2h + 1] = sum_w c_w l_w (c_w = exp(m_w - max))
            for (int i = threadIdx.x; i < ghd + 2 * G; i += blockDim.x) {
                const int h = i < ghd ? i / hd : (i - ghd) / 2;
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < kWarps; w++) M = fmaxf(M, part[w * pw + ghd + 2 * h]);
                float acc = 0.0f;
                const int src = i < ghd ? i : ghd + 2 * h + 1;
#pragma unroll
                for (int w = 0; w < kWarps; w++) {
                    const float mw = part[w * pw + ghd + 2 * h];
                    const float c = mw == -INFINITY ? 0.0f : expf(mw - M);
                    acc += c * part[w * pw + src];
                }
                S.pair[i] = (i >= ghd && ((i - ghd) & 1) == 0) ? M : acc;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
            if (threadIdx.x == 0 && !S.ints[34]) bulk_s2peer(S.pair, pair_bytes, S.pairbar, (unsigned)(crank - nu));
        } else {
            if (split) {
                if (threadIdx.x == 0) df_wait(p, S, S.pairbar, S.prph);
                S.prph ^= 1u;
                __syncthreads();
            }
            for (int i = threadIdx.x; i < ghd; i += blockDim.x) {
                const int h = i / hd;
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < kWarps; w++) M = fmaxf(M, part[w * pw + ghd + 2 * h]);
                if (split) M = fmaxf(M, S.pair[ghd + 2 * h]);
                float num = 0.0f, den = 0.0f;
#pragma unroll
                for (int w = 0; w < kWarps; w++) {
                    const float mw = part[w * pw + ghd + 2 * h];
                    const float c = mw == -INFINITY ? 0.0f : expf(mw - M);   // a warp may see no keys
                    den += c * part[w * pw + ghd + 2 * h + 1];
                    num += c * part[w * pw + i];
                }
                if (split) {   // the second range always holds key t: its maximum is finite
                    const float c = expf(S.pair[ghd + 2 * h] - M);
                    den += c * S.pair[ghd + 2 * h + 1];
                    num += c * S.pair[i];
                }
                S.att[i] = num / den;
            }
            __syncthreads();
            // this head group's share of attn_proj (generate.c:158-163): a thread
            // per output over the block's [G hd][D] (transposed) columns
            const float* wp = wa + (size_t)rows_a * D;
            for (int i = threadIdx.x; i < D; i += blockDim.x) {
                float a0 = 0.0f, a1 = 0.0f;
                int c = 0;
#pragma unroll
                for (; c + 1 < ghd; c += 2) {
                    a0 = fmaf(wp[(size_t)c * D + i], S.att[c], a0);
                    a1 = fmaf(wp[(size_t)(c + 1) * D + i], S.att[c + 1], a1);
                }
                if (c < ghd) a0 = fmaf(wp[(size_t)c * D + i], S.att[c], a0);
                S.attp[crank * D + i] = a0 + a1;
            }
            // DF: this thread's shared-memory writes (the partial, and the K/V
            // tile that later partials overwrite) before the async proxy's copies
            if (DF) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
            if (!DF) push_block(cl, S.attp, crank * D, D, cs, crank);
            else if (warp == 0 && lane < cs && lane != crank && !S.ints[34])
                bulk_s2peer(S.attp + (size_t)crank * D, (unsigned)(D * 4), S.atbar, (unsigned)lane);
        }
    }
    // K/V rows written in this step are read by later steps' bulk copies
    // (async proxy) in other CTAs: order them before the cluster barrier
    if (wrote_kv) asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) cl2_issue_a(cp, S, (l + 1) % p.L, g);
    if (DF) {
        if (threadIdx.x == 0) df_wait(p, S, S.atbar, S.atph);
        S.atph ^= 1u;
        __syncthreads();
    } else if (!lc_sync(cl, S, cs)) {
        return false;
    }

    // ------------------------------------------------ phase B: FFN slice
    const int par = DF ? (S.nlayer & 1) : 0;
    float* dpb = S.dp + (size_t)par * cs * cp.dp_b * D;
    // this layer's ffn_down partials: one from every other CTA
    if (DF && threadIdx.x == 0 && !S.ints[34])
        mbar_expect_tx(&S.dpbar[par], (unsigned)((cs - 1) * nf * D * 4));
    for (int e = threadIdx.x; e < nf * D; e += blockDim.x) {
        const int i = e / D, k = e % D;
        float s = 0.0f;
        for (int gg = 0; gg < K; gg++) s += S.attp[(i * K + gg) * D + k];
        S.x[fl[i] * D + k] += s;
    }
    if (!mbar_wait(&S.bar[1], pbp, p.timeout_ns)) lc_fail(S, p.status, ST_TIMEOUT);
    pbp ^= 1u;
    __syncthreads();
    const float* wu = S.wb;
    const float* wg = S.wb + (size_t)fpc * D;
    const float* wd = S.wb + 2 * (size_t)fpc * D;
    const float* rms2 = wd + (size_t)D * fpc;
    // rmsnorm of every fed sequence (generate.c:57-63): at D = 128 in the
    // registers of each warp that computes rows, otherwise a warp per sequence
    if constexpr (DC == 128 && FC % 16 == 0) {
        // FC % 16 == 0: every round's rows stay inside the up/gate buffer
        float4 xr[kBCMax];
#pragma unroll
        for (int i = 0; i < kBCMax; i++)
            xr[i] = i < nf ? cl2_norm128(S.x + fl[i] * D, rms2) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        // four sequence slots per round at nf <= 4 (a 32-row slice is one
        // round of the 8 warps; fewer slots would leave warps idle), else eight
        if (nf <= 4) cl2_upgate<4>(wu, wg, xr, fl, nf, sl.f0, sl.f1, fpc, S.f);
        else cl2_upgate<8>(wu, wg, xr, fl, nf, sl.f0, sl.f1, fpc, S.f);
    } else {
        lc_norm(S.x, S.xn, rms2, fl, nf, D, S.red);
        // up/gate rows [f0, f1) and SwiGLU (generate.c:165-179)
        for (int j = sl.f0 + 2 * warp; j < sl.f1; j += 2 * kWarps) {
            // rows: up j, up j+1, gate j, gate j+1 -> the gate of lane's up row is in lane ^ 16
            const float* u0 = wu + (size_t)(j - sl.f0) * D;
            const float* g0 = wg + (size_t)(j - sl.f0) * D;
            const float val = lc_gemv4(u0, u0 + D, g0, g0 + D, D, S.xn, D, fl, nf);
            const float gate = __shfl_xor_sync(0xffffffffu, val, 16);
            const int i = lane & 7;
            if (lane < 16 && i < nf) {
                const float sv = gate / (1.0f + expf(-gate));
                S.f[fl[i] * fpc + (j - sl.f0) + (lane >> 3)] = sv * val;
            }
        }
    }
    __syncthreads();
    // this slice's share of ffn_down (generate.c:181-184), into this CTA's
    // slot of the partials
    // a thread per (output, sequence) over the block's [fpc][D] (transposed)
    // columns; the SwiGLU values are broadcast reads
    // all fpc columns: past this CTA's rows the SwiGLU values and the block
    // are zero, so the extra terms add exact zeros
    float* mine = dpb + (size_t)crank * cp.dp_b * D;
    for (int e = threadIdx.x; e < D * nf; e += blockDim.x) {
        const int i = e % D, s = e / D;
        const float* fr = S.f + fl[s] * fpc;
        float a0 = 0.0f, a1 = 0.0f;
        int j = 0;
#pragma unroll
        for (; j + 1 < fpc; j += 2) {
            a0 = fmaf(wd[(size_t)j * D + i], fr[j], a0);
            a1 = fmaf(wd[(size_t)(j + 1) * D + i], fr[j + 1], a1);
        }
        if (j < fpc) a0 = fmaf(wd[(size_t)j * D + i], fr[j], a0);
        mine[s * D + i] = a0 + a1;
    }
    if (DF) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (DF) {
        if (warp == 0 && lane < cs && lane != crank && !S.ints[34])
            bulk_s2peer(mine, (unsigned)(nf * D * 4), &S.dpbar[par], (unsigned)lane);
    } else {
        const int n4 = D >> 2, per_rank = nf * n4;
        for (int e = threadIdx.x; e < per_rank * cs; e += blockDim.x) {
            const int r = e / per_rank;
            if (r == crank) continue;
            const int off = 4 * (e - r * per_rank);
            const float4 v = *reinterpret_cast<const float4*>(mine + off);
            *reinterpret_cast<float4*>(cl.map_shared_rank(mine, r) + off) = v;
        }
        __syncthreads();
    }
    if (!DF && threadIdx.x == 0) cl2_issue_b(cp, sl, S, (l + 1) % p.L, crank);
    if (!DF) return lc_sync(cl, S, cs);
    if (threadIdx.x == 0) df_wait(p, S, &S.dpbar[par], (S.dpph >> par) & 1u);
    S.dpph ^= 1u << par;
    S.nlayer++;
    __syncthreads();
    cl2_add_down(cp, S, dpb, fl, nf);
    return true;
}

// Layer l through the specialisation for this model's dims.
template <bool DF>
__device__ __forceinline__ bool cl2_layer_any(const ClusterParams& cp, const CSlice& sl, LcState& S,
                                              cg::cluster_group& cl, int crank, int l, int t, const int* fl,
                                              int nf, unsigned& pa, unsigned& pbp) {
    const LoopParams<float>& p = cp.lp;
    const bool first = l == 0;
    if (p.hd == 32 && p.D == 128 && cp.fpc == 32 && p.G == 2)    // the default model (config.h)
        return cl2_layer<32, 128, 32, 2, DF>(cp, sl, S, cl, crank, l, t, fl, nf, first, pa, pbp);
    switch (p.hd) {
    case 16: return cl2_layer<16, 0, 0, 0, DF>(cp, sl, S, cl, crank, l, t, fl, nf, first, pa, pbp);
    case 32: return cl2_layer<32, 0, 0, 0, DF>(cp, sl, S, cl, crank, l, t, fl, nf, first, pa, pbp);
    case 64: return cl2_layer<64, 0, 0, 0, DF>(cp, sl, S, cl, crank, l, t, fl, nf, first, pa, pbp);
    default: return cl2_layer<0, 0, 0, 0, DF>(cp, sl, S, cl, crank, l, t, fl, nf, first, pa, pbp);
    }
}

template <bool DF>
__device__ void cl2_main(const ClusterParams& cp, unsigned char* smem, cg::cluster_group& cl, int crank) {
    const LoopParams<float>& p = cp.lp;
    LcState S;
    S.bar = reinterpret_cast<unsigned long long*>(smem);   // [0] phase A, [1] phase B
    S.kvbar = S.bar + 2;
    S.atbar = S.bar + 3;
    S.dpbar = S.bar + 4;                                   // [2]
    S.pairbar = S.bar + 6;
    S.pair = reinterpret_cast<float*>(smem + cp.off_pair);
    constexpr bool df = DF;
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
    S.dp = S.kv;                                           // shared with the K/V tile
    S.stage = reinterpret_cast<float*>(smem + cp.off_stage);
    S.wb = reinterpret_cast<float*>(smem + cp.off_wb);
    S.rope = reinterpret_cast<float2*>(smem + cp.off_rope);
    S.pages = reinterpret_cast<int*>(smem + cp.off_pages);
    S.seq = reinterpret_cast<SeqMirror*>(smem + 576);
    const CSlice sl = cluster_slice(crank, cp.cs, p.Q, p.D, p.F);
    const int nhc = (cp.n_clusters - 1) * cp.cs;
    int* fl = S.ints;        // [16]
    int* hl = S.ints + 16;   // [16]
    const int warp = threadIdx.x >> 5;

    if (threadIdx.x == 0) {
        mbar_init(&S.bar[0], 1);
        mbar_init(&S.bar[1], 1);
        mbar_init(S.kvbar, 1);
        mbar_init(S.atbar, 1);
        mbar_init(&S.dpbar[0], 1);
        mbar_init(&S.dpbar[1], 1);
        mbar_init(S.pairbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.ints[34] = 0;
        S.ints[38] = 0;
        S.ints[39] = 0;
    }
    S.kvph = 0u;
    S.kvpend = 0;
    S.atph = 0u;
    S.dpph = 0u;
    S.prph = 0u;
    S.nlayer = 0;
    for (int b = threadIdx.x; b < p.B; b += blockDim.x) {
        const SeqState& g = p.seq[b];
        SeqMirror& m = S.seq[b];
        m.P = g.P; m.nnew = g.nnew; m.gen = g.gen; m.done = g.done; m.tok = g.tok;
        m.result = g.result; m.final_pos = g.final_pos; m.rng = g.rng;
    }
    for (int e = threadIdx.x; e < p.B * p.pg.pps; e += blockDim.x) S.pages[e] = __ldg(p.pg.table + e);
    // the SwiGLU slice is read past f1 - f0 by nobody, but keep it finite
    for (int e = threadIdx.x; e < cp.dp_b * cp.fpc; e += blockDim.x) S.f[e] = 0.0f;
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
    unsigned pa = 0u, pbp = 0u;
    if (threadIdx.x == 0) {
        cl2_issue_a(cp, S, 0, crank % p.K);
        if (!DF) cl2_issue_b(cp, sl, S, 0, crank);
    }
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
        // this position's RoPE row and the embedding of the id fed at t
        // (generate.c:86-88), in one round trip once decoding (a generated id
        // is in the sequence table; a prompt id is read first)
        for (int j = threadIdx.x; j < p.hd / 2; j += blockDim.x)
            S.rope[j] = p.rope[(size_t)t * (p.hd / 2) + j];
        for (int e = threadIdx.x; e < nf * p.D; e += blockDim.x) {
            const int i = e / p.D, k = e % p.D, b = fl[i];
            const SeqMirror& m = S.seq[b];
            int tok = t < m.P ? (int)p.prompts[(size_t)b * p.prompt_stride + t] : m.tok;
            if (tok < 0 || tok >= p.V) {
                if (k == 0) lc_fail(S, p.status, ST_DEVICE);
                tok = 0;
            }
            S.x[b * p.D + k] = __ldg(p.tok_emb + (size_t)tok * p.D + k);
        }
        __syncthreads();
        for (int l = 0; ok && l < p.L; l++)
            ok = cl2_layer_any<DF>(cp, sl, S, cl, crank, l, t, fl, nf, pa, pbp);
        if (!ok) break;
        if constexpr (DF) {
            // The dataflow layers have no cluster barrier of their own; the
            // step's one (ordering its K/V rows before later bulk reads,
            // making a failure cluster-wide) is split: the arrival here, the
            // wait once the next ids are chosen, so the hand-off hides it.
            // Every layer CTA waits for the head CTAs and chooses the ids
            // into its own mirror (the same update everywhere); CTA 0 alone
            // also releases the heads and writes ids, counts and bans.
            lc_arrive(cl, S, cp.cs);
            if (nh > 0) {
                heads++;
                if (crank == 0) {
                    lc_publish_rows(cp, S, hl, nh, (int)(heads & 1u));
                    if (threadIdx.x == 0) {
                        __threadfence();
                        st_release_u32(cp.go, heads);
                    }
                }
                if (threadIdx.x == 0) {
                    const unsigned target = heads * ((unsigned)nhc + p.extra_arrivals);
                    const unsigned long long t0 = globaltimer_ns();
                    while ((int)(ld_acquire_u32(cp.hdone) - target) < 0) {
                        if (globaltimer_ns() - t0 > p.timeout_ns) {
                            lc_fail(S, p.status, ST_TIMEOUT);   // cluster-wide at the next arrival
                            break;
                        }
                    }
                }
                __syncthreads();
                if (warp < nh)
                    lc_choose(cp, S.seq[hl[warp]], hl[warp], warp, S.ints, (int)(heads & 1u), crank == 0);
                __syncthreads();
                if (crank == 0 && p.s.ngram > 0)
                    for (int i = 0; i < nh; i++)
                        if (!S.ints[40 + i]) compute_bans(p, hl[i], S.seq[hl[i]].P + S.ints[48 + i]);
            }
            ok = lc_wait(S);
            continue;
        }
        if (nh == 0) continue;
        cl2_add_down(cp, S, S.dp, fl, nf);

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
            if (warp < nh) lc_choose(cp, S.seq[hl[warp]], hl[warp], warp, S.ints, (int)(heads & 1u), true);
            __syncthreads();
            if (p.s.ngram > 0)
                for (int i = 0; i < nh; i++)
                    if (!S.ints[40 + i]) compute_bans(p, hl[i], S.seq[hl[i]].P + S.ints[48 + i]);
            __syncthreads();
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
    // one copy per phase buffer is always in flight (issued for the next
    // layer; DF: only the unit phase's, the FFN weights being requested in
    // their own layer), and possibly a K/V tile after a failed wait
    if (threadIdx.x == 0) {
        if (!mbar_wait(&S.bar[0], pa, p.timeout_ns)) atomicMax(p.status, (int)ST_TIMEOUT);
        if (!DF && !mbar_wait(&S.bar[1], pbp, p.timeout_ns)) atomicMax(p.status, (int)ST_TIMEOUT);
    }
    if (threadIdx.x == kTileThread && S.kvpend && !mbar_wait(S.kvbar, S.kvph, p.timeout_ns))
        atomicMax(p.status, (int)ST_TIMEOUT);
    __syncthreads();
    cl.sync();   // no CTA leaves while others may still write its shared memory
    if (df && !ok) {
        // after a failed dataflow wait, copies already issued to a CTA that
        // stopped waiting may still be in flight: let them land first
        const unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 50000ull) {
        }
        cl.sync();
    }
}

// One instantiation per layer loop (V2 == cp.v2), so that each is
// register-allocated on its own.
template <int V2>
__global__ void __launch_bounds__(kThreads, 1) cluster_loop_kernel(const ClusterParams cp) {
    extern __shared__ __align__(128) unsigned char smem_c[];
    cg::cluster_group cl = cg::this_cluster();
    const int cid = blockIdx.x / cp.cs;
    if (cid == 0) {
        if constexpr (V2 == 0) lc_main(cp, smem_c, cl, (int)cl.block_rank());
        else cl2_main<V2 == 2>(cp, smem_c, cl, (int)cl.block_rank());
    } else {
        hc_main(cp, smem_c, blockIdx.x - cp.cs);
    }
}
template __global__ void cluster_loop_kernel<0>(const ClusterParams);
template __global__ void cluster_loop_kernel<1>(const ClusterParams);
template __global__ void cluster_loop_kernel<2>(const ClusterParams);

}  // namespace mc

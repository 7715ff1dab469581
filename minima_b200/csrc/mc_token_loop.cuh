// mc_token_loop.cuh — the persistent decode token loop for sm_100a.
//
// One cooperative launch runs every step of generate_with_options
// (generate.c:522-602) for a batch of independent sequences: prompt
// positions are fed teacher-forced, then each step samples on device and
// feeds the sampled id back, so the host is not involved per token.
//
// Per step and per layer the work is split into five grid-wide phases
// separated by deadline-bounded grid barriers (forward_one, generate.c:
// 76-194):
//   QKV   rmsnorm(x, rms1) -> W_qkv rows -> RoPE (rotary.h:9-40) -> q, and
//         K/V appended to the cache at position t          (generate.c:99-119)
//   ATT   split-K flash decode over positions 0..t per (sequence, KV head),
//         combined by the last split to finish               (generate.c:121-156)
//   PROJ  x += W_proj . att                                  (generate.c:158-163)
//   UPG   f = silu(W_gate . h) * (W_up . h), h = rmsnorm(x, rms2) (generate.c:165-179)
//   DOWN  x += W_down . f                                    (generate.c:181-184)
// then
//   HEAD  logits = tok_emb . rmsnorm(x, rms_final), ids 0..3 -> -inf
//         (generate.c:187-191, 580-581), plus per-CTA argmax partials
//   SAMP  one CTA per sequence: sample, stop-sequence check, bookkeeping
//         (generate.c:582-598)
// Every sequence is at position t during step t, so ragged prompts need no
// padding: a sequence is teacher-forced while t < its prompt length.
#pragma once

#include "mc_device.cuh"
#include "mc_sampler.cuh"

namespace mc {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kBCMax = 8;          // sequences per GEMV chunk
constexpr int kSplitLen = 64;      // keys per attention split

struct SeqState {
    int P;          // prompt length
    int nnew;       // new-token budget after generate.c:554-556 clamps (0 = idle)
    int gen;        // ids sampled so far
    int done;
    int result;     // value generate_with_options returns
    int final_pos;  // cache->pos the reference would leave
    int tok;        // sampled id to feed next
    int pad;
    unsigned long long rng;
};

template <typename WT>
struct LoopParams {
    int V, D, L, H, K, hd, kvd, Q, F, G;
    const WT* tok_emb;
    const WT* w_qkv;
    const WT* w_proj;
    const WT* w_up;
    const WT* w_gate;
    const WT* w_down;
    const float* rms1;
    const float* rms2;
    const float* rmsf;
    const float2* rope;   // [rope_len][hd/2] (cos, sin) computed on the host
    int rope_len;
    float* kc;            // K pages [n_pages][L][K][page_len][hd] (KvPages)
    float* vc;            // V pages, same layout
    KvPages pg;           // page table of the sequences
    int cap;
    int Bcap;
    float* x;             // [Bcap][D] residual stream
    float* q;             // [Bcap][D] rotated queries
    float* att;           // [Bcap][D] attention output
    float* f;             // [Bcap][F]
    float* logits;        // [Bcap][V]
    float* part_o;        // [Bcap][H][max_split][hd]
    float* part_m;        // [Bcap][H][max_split]
    float* part_l;
    unsigned* att_cnt;    // [Bcap][K]
    float* amax_v;        // [Bcap][grid]
    int* amax_i;
    unsigned* counts;     // [Bcap][V]
    unsigned* banned;     // [Bcap][ceil(V/32)]
    int max_split;
    int B;
    SeqState* seq;
    const uint16_t* prompts;
    int prompt_stride;
    uint16_t* out_ids;
    int out_cap;
    SamplingArgs s;
    int T;                // forward steps to run
    int t0;               // first position (earlier ones were prefilled)
    int all_logits;       // teacher-forced logits mode (no sampling)
    float* trace;         // [B][trace_steps][V] or null
    int trace_steps;
    unsigned* bar;
    int* status;
    unsigned long long timeout_ns;
    unsigned long long* stamps;   // [T+1] %globaltimer at each step start, or null
    unsigned extra_arrivals;      // test hook: arrivals a wait expects beyond the real ones
    int bc;               // GEMV chunk (<= kBCMax)
    int xs_ld;            // row stride of the chunk buffer in smem (floats)
};

// ---------------------------------------------------------------- GEMV core
// NR weight rows against bc (<= kBCMax) activation vectors held in shared
// memory; one warp; result summed across lanes (every lane holds it).
template <typename WT, int NR, bool VEC>
__device__ __forceinline__ void warp_dot(const WT* const* rows, int len, const float* xs,
                                         int ldx, int bc, float (&acc)[NR][kBCMax]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
        for (int c = 0; c < kBCMax; c++) acc[r][c] = 0.0f;
    if constexpr (VEC) {
        constexpr int N = WVec<WT>::N;
        for (int k = lane * N; k < len; k += 32 * N) {
            float w[NR][N];
#pragma unroll
            for (int r = 0; r < NR; r++) WVec<WT>::load(rows[r] + k, w[r]);
#pragma unroll
            for (int c = 0; c < kBCMax; c++) {
                if (c < bc) {
                    const float4* xp = reinterpret_cast<const float4*>(xs + c * ldx + k);
#pragma unroll
                    for (int e4 = 0; e4 < N / 4; e4++) {
                        const float4 xv = xp[e4];
#pragma unroll
                        for (int r = 0; r < NR; r++) {
                            acc[r][c] += w[r][4 * e4 + 0] * xv.x;
                            acc[r][c] += w[r][4 * e4 + 1] * xv.y;
                            acc[r][c] += w[r][4 * e4 + 2] * xv.z;
                            acc[r][c] += w[r][4 * e4 + 3] * xv.w;
                        }
                    }
                }
            }
        }
    } else {
        for (int k = lane; k < len; k += 32) {
            float w[NR];
#pragma unroll
            for (int r = 0; r < NR; r++) w[r] = wload1(rows[r] + k);
#pragma unroll
            for (int c = 0; c < kBCMax; c++)
                if (c < bc) {
                    const float xv = xs[c * ldx + k];
#pragma unroll
                    for (int r = 0; r < NR; r++) acc[r][c] += w[r] * xv;
                }
        }
    }
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
        for (int c = 0; c < kBCMax; c++)
            if (c < bc) acc[r][c] = warp_sum(acc[r][c]);
}

// ------------------------------------------------------------ shared state
struct LoopSmem {
    float* red;        // [64]
    int* fwd;          // [Bcap] sequences that run a forward this step
    int* head;         // [Bcap] sequences that need logits this step
    int* ints;         // [32] scalars
    float* xs;         // phase region (GEMV chunk, attention, sampler)
};

__host__ __device__ inline size_t loop_fixed_bytes(int Bcap) {
    size_t b = 64 * 4 + (size_t)Bcap * 4 * 2 + 32 * 4;
    return (b + 15) & ~(size_t)15;
}

// Row-normalised chunk: xs[c][0..D) = x_b * inv_rms * scale (generate.c:57-63).
// src_emb != nullptr: x_b is the embedding row of token tok[c] (layer 0).
template <typename WT>
__device__ void load_norm_chunk(const LoopParams<WT>& p, const int* bl, int bc, const float* src,
                                int src_ld, const float* scale, bool normalize, int len,
                                float* xs, int ldx, float* red, const int* toks, bool write_x) {
    for (int c = 0; c < bc; c++) {
        const int b = bl[c];
        for (int i = threadIdx.x; i < len; i += blockDim.x) {
            float v;
            if (toks) v = wload1(p.tok_emb + (size_t)toks[c] * len + i);
            else v = ldcg(src + (size_t)b * src_ld + i);
            xs[c * ldx + i] = v;
            if (write_x) p.x[(size_t)b * p.D + i] = v;
        }
    }
    __syncthreads();
    if (!normalize) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int c = warp; c < bc; c += kWarps) {
        float ss = 0.0f;
        for (int i = lane; i < len; i += 32) {
            const float v = xs[c * ldx + i];
            ss += v * v;
        }
        ss = warp_sum(ss);
        if (lane == 0) red[c] = 1.0f / sqrtf(ss / (float)len + 1e-5f);
    }
    __syncthreads();
    for (int c = 0; c < bc; c++) {
        const float inv = red[c];
        for (int i = threadIdx.x; i < len; i += blockDim.x)
            xs[c * ldx + i] = xs[c * ldx + i] * inv * scale[i];
    }
    __syncthreads();
}

// ------------------------------------------------------------------ phases
template <typename WT, bool VEC>
__device__ void phase_qkv(const LoopParams<WT>& p, int l, int t, LoopSmem& sm, int nfwd) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = warp * gridDim.x + blockIdx.x, tw = gridDim.x * kWarps;
    const int ph = (p.hd + 1) / 2;                 // row pairs per head
    const int units = (p.H + 2 * p.K) * ph;
    const WT* W = p.w_qkv + (size_t)l * p.Q * p.D;
    int* toks = sm.ints + 4;  // up to kBCMax token ids (ints[4..12))
    for (int c0 = 0; c0 < nfwd; c0 += p.bc) {
        const int bc = min(p.bc, nfwd - c0);
        const int* bl = sm.fwd + c0;
        if (l == 0) {
            if (threadIdx.x < bc) {
                const int b = bl[threadIdx.x];
                const SeqState* ss = p.seq + b;
                const int P = ld_volatile_i32(&ss->P);
                int tok = t < P ? (int)p.prompts[(size_t)b * p.prompt_stride + t]
                                : ld_volatile_i32(&ss->tok);
                if (tok < 0 || tok >= p.V) {  // never index past tok_emb
                    atomicMax(p.status, (int)ST_DEVICE);
                    tok = 0;
                }
                toks[threadIdx.x] = tok;
            }
            __syncthreads();
        }
        load_norm_chunk(p, bl, bc, p.x, p.D, p.rms1 + (size_t)l * p.D, true, p.D, sm.xs, p.xs_ld,
                        sm.red, l == 0 ? toks : nullptr, l == 0 && blockIdx.x == 0);
        for (int u = gw; u < units; u += tw) {
            const int slot = u / ph, pr = u % ph;
            const int r0 = slot * p.hd + 2 * pr;
            const bool has1 = 2 * pr + 1 < p.hd;
            const WT* rows[2] = {W + (size_t)r0 * p.D, W + (size_t)(has1 ? r0 + 1 : r0) * p.D};
            float acc[2][kBCMax];
            warp_dot<WT, 2, VEC>(rows, p.D, sm.xs, p.xs_ld, bc, acc);
            if (lane == 0) {
                const bool rotate = has1 && slot < p.H + p.K;
                float cs = 1.0f, sn = 0.0f;
                if (rotate) {
                    const float2 r = p.rope[(size_t)t * (p.hd / 2) + pr];
                    cs = r.x; sn = r.y;
                }
                for (int c = 0; c < bc; c++) {
                    const int b = bl[c];
                    float a = acc[0][c], z = acc[1][c];
                    if (rotate) {
                        const float a2 = a * cs - z * sn;
                        const float z2 = a * sn + z * cs;
                        a = a2; z = z2;
                    }
                    const int d = 2 * pr;
                    if (slot < p.H) {
                        float* qd = p.q + (size_t)b * p.D + slot * p.hd + d;
                        qd[0] = a;
                        if (has1) qd[1] = z;
                    } else {
                        const bool isk = slot < p.H + p.K;
                        const int g = isk ? slot - p.H : slot - p.H - p.K;
                        float* base = (isk ? p.kc : p.vc) + kv_row(p.pg, p.L, p.K, l, b, g, t) * p.hd + d;
                        base[0] = a;
                        if (has1) base[1] = z;
                    }
                }
            }
        }
        __syncthreads();
    }
}

// Shared memory of the attention phase: queries [G][hd], scores
// [G][kSplitLen], and the split's K and V rows staged [kSplitLen][hd] each.
__host__ __device__ inline size_t att_phase_bytes(int G, int hd) {
    return ((size_t)G * hd + (size_t)G * kSplitLen + 2 * (size_t)kSplitLen * hd) * 4;
}

template <typename WT>
__device__ void phase_att(const LoopParams<WT>& p, int l, int t, LoopSmem& sm, int nfwd) {
    const int nkeys = t + 1;
    const int nsplit = (nkeys + kSplitLen - 1) / kSplitLen;
    const int units = nfwd * p.K * nsplit;
    const int G = p.G, hd = p.hd, q4 = hd / 4;
    const float scale = 1.0f / sqrtf((float)hd);
    float* qs = sm.xs;                       // [G][hd]
    float* sc = sm.xs + G * hd;              // [G][kSplitLen]
    float* ks = sc + G * kSplitLen;          // [kSplitLen][hd]
    float* vs = ks + kSplitLen * hd;         // [kSplitLen][hd]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool combine = nsplit > 1 || G > 32;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int s = u % nsplit;
        const int g = (u / nsplit) % p.K;
        const int b = sm.fwd[u / (nsplit * p.K)];
        const int j0 = s * kSplitLen, j1 = min(nkeys, j0 + kSplitLen), n = j1 - j0;
        // the split's kSplitLen (64) keys start 64-aligned: one page
        const size_t row0 = kv_row(p.pg, p.L, p.K, l, b, g, j0);
        const float* kb = p.kc + row0 * hd;
        const float* vb = p.vc + row0 * hd;
        // stage q, and the split's K and V rows, with coalesced L2 reads
        // (rows written by other CTAs earlier in this launch)
        for (int i = threadIdx.x; i < G * hd; i += blockDim.x)
            qs[i] = ldcg(p.q + (size_t)b * p.D + (size_t)g * G * hd + i);
        if ((hd & 3) == 0) {
            for (int e = threadIdx.x; e < n * q4; e += blockDim.x) {
                reinterpret_cast<float4*>(ks)[e] = ldcg4(kb + 4 * e);
                reinterpret_cast<float4*>(vs)[e] = ldcg4(vb + 4 * e);
            }
        } else {
            for (int e = threadIdx.x; e < n * hd; e += blockDim.x) {
                ks[e] = ldcg(kb + e);
                vs[e] = ldcg(vb + e);
            }
        }
        __syncthreads();
        // scores: a thread per (head, key); its key row is read starting at
        // element (j mod hd) so that neighbouring keys fall in different banks
        for (int e = threadIdx.x; e < G * n; e += blockDim.x) {
            const int h = e / n, j = e - h * n;
            const float* kr = ks + j * hd;
            const float* qh = qs + h * hd;
            float part = 0.0f;
            if ((hd & 3) == 0) {
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
            sc[h * kSplitLen + j] = part * scale;
        }
        __syncthreads();
        // local softmax statistics per head
        for (int h = warp; h < G; h += kWarps) {
            float m = -INFINITY;
            for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[h * kSplitLen + j]);
            m = warp_max(m);
            float lsum = 0.0f;
            for (int j = lane; j < n; j += 32) {
                const float e = expf(sc[h * kSplitLen + j] - m);
                sc[h * kSplitLen + j] = e;
                lsum += e;
            }
            lsum = warp_sum(lsum);
            if (lane == 0) {
                const size_t pi = ((size_t)b * p.H + g * G + h) * p.max_split + s;
                if (combine) { p.part_m[pi] = m; p.part_l[pi] = lsum; }
                else sm.red[h] = lsum;
            }
        }
        __syncthreads();
        // P.V
        for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
            const int h = i / hd, d = i % hd;
            float o = 0.0f;
#pragma unroll 8
            for (int j = 0; j < n; j++) o += sc[h * kSplitLen + j] * vs[j * hd + d];
            if (!combine) {
                p.att[(size_t)b * p.D + (g * G + h) * hd + d] = o / sm.red[h];
            } else {
                p.part_o[(((size_t)b * p.H + g * G + h) * p.max_split + s) * hd + d] = o;
            }
        }
        if (combine) {
            // last split to finish combines (flash-decoding reduction)
            __threadfence();
            __syncthreads();
            if (threadIdx.x == 0) {
                const unsigned prev = atomicAdd(&p.att_cnt[b * p.K + g], 1u);
                sm.ints[0] = (prev == (unsigned)nsplit - 1);
            }
            __syncthreads();
            if (sm.ints[0]) {
                __threadfence();
                for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
                    const int h = i / hd, d = i % hd;
                    const size_t pb = ((size_t)b * p.H + g * G + h) * p.max_split;
                    float M = -INFINITY;
                    for (int s2 = 0; s2 < nsplit; s2++) M = fmaxf(M, ldcg(p.part_m + pb + s2));
                    float num = 0.0f, den = 0.0f;
                    for (int s2 = 0; s2 < nsplit; s2++) {
                        const float w = expf(ldcg(p.part_m + pb + s2) - M);
                        den += w * ldcg(p.part_l + pb + s2);
                        num += w * ldcg(p.part_o + (pb + s2) * hd + d);
                    }
                    p.att[(size_t)b * p.D + (g * G + h) * hd + d] = num / den;
                }
                if (threadIdx.x == 0) p.att_cnt[b * p.K + g] = 0u;
            }
        }
        __syncthreads();
    }
}

// x[b][j] += W[j] . xs[c] for D output rows (PROJ: W_proj over att; DOWN:
// W_down over f).
template <typename WT, bool VEC>
__device__ void phase_residual(const LoopParams<WT>& p, const WT* W, int len, const float* src,
                               int src_ld, LoopSmem& sm, int nfwd) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = warp * gridDim.x + blockIdx.x, tw = gridDim.x * kWarps;
    const int units = (p.D + 1) / 2;
    for (int c0 = 0; c0 < nfwd; c0 += p.bc) {
        const int bc = min(p.bc, nfwd - c0);
        const int* bl = sm.fwd + c0;
        load_norm_chunk(p, bl, bc, src, src_ld, nullptr, false, len, sm.xs, p.xs_ld, sm.red,
                        nullptr, false);
        for (int u = gw; u < units; u += tw) {
            const int r0 = 2 * u;
            const bool has1 = r0 + 1 < p.D;
            const WT* rows[2] = {W + (size_t)r0 * len, W + (size_t)(has1 ? r0 + 1 : r0) * len};
            float acc[2][kBCMax];
            warp_dot<WT, 2, VEC>(rows, len, sm.xs, p.xs_ld, bc, acc);
            if (lane == 0) {
                for (int c = 0; c < bc; c++) {
                    float* xr = p.x + (size_t)bl[c] * p.D + r0;
                    xr[0] = ldcg(xr) + acc[0][c];
                    if (has1) xr[1] = ldcg(xr + 1) + acc[1][c];
                }
            }
        }
        __syncthreads();
    }
}

template <typename WT, bool VEC>
__device__ void phase_upgate(const LoopParams<WT>& p, int l, LoopSmem& sm, int nfwd) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = warp * gridDim.x + blockIdx.x, tw = gridDim.x * kWarps;
    const WT* Wu = p.w_up + (size_t)l * p.F * p.D;
    const WT* Wg = p.w_gate + (size_t)l * p.F * p.D;
    for (int c0 = 0; c0 < nfwd; c0 += p.bc) {
        const int bc = min(p.bc, nfwd - c0);
        const int* bl = sm.fwd + c0;
        load_norm_chunk(p, bl, bc, p.x, p.D, p.rms2 + (size_t)l * p.D, true, p.D, sm.xs, p.xs_ld,
                        sm.red, nullptr, false);
        for (int j = gw; j < p.F; j += tw) {
            const WT* rows[2] = {Wu + (size_t)j * p.D, Wg + (size_t)j * p.D};
            float acc[2][kBCMax];
            warp_dot<WT, 2, VEC>(rows, p.D, sm.xs, p.xs_ld, bc, acc);
            if (lane == 0) {
                for (int c = 0; c < bc; c++) {
                    const float up = acc[0][c], g = acc[1][c];
                    const float s = g / (1.0f + expf(-g));
                    p.f[(size_t)bl[c] * p.F + j] = s * up;
                }
            }
        }
        __syncthreads();
    }
}

template <typename WT, bool VEC>
__device__ void phase_head(const LoopParams<WT>& p, int t, LoopSmem& sm, int nhead) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = warp * gridDim.x + blockIdx.x, tw = gridDim.x * kWarps;
    const int units = (p.V + 1) / 2;
    const bool greedy = !p.all_logits && p.s.top_k == 1;
    float* wv = sm.red;                                   // [kWarps][kBCMax] best values
    int* wi = reinterpret_cast<int*>(sm.xs + p.bc * p.xs_ld);  // [kWarps][kBCMax] best ids
    const int nwords = (p.V + 31) >> 5;
    for (int c0 = 0; c0 < nhead; c0 += p.bc) {
        const int bc = min(p.bc, nhead - c0);
        const int* bl = sm.head + c0;
        load_norm_chunk(p, bl, bc, p.x, p.D, p.rmsf, true, p.D, sm.xs, p.xs_ld, sm.red, nullptr,
                        false);
        float bv[kBCMax];
        int bi[kBCMax];
#pragma unroll
        for (int c = 0; c < kBCMax; c++) { bv[c] = -INFINITY; bi[c] = 0x7fffffff; }
        for (int u = gw; u < units; u += tw) {
            const int r0 = 2 * u;
            const bool has1 = r0 + 1 < p.V;
            const WT* rows[2] = {p.tok_emb + (size_t)r0 * p.D,
                                 p.tok_emb + (size_t)(has1 ? r0 + 1 : r0) * p.D};
            float acc[2][kBCMax];
            warp_dot<WT, 2, VEC>(rows, p.D, sm.xs, p.xs_ld, bc, acc);
            if (lane == 0) {
                for (int c = 0; c < bc; c++) {
                    const int b = bl[c];
                    for (int r = 0; r < (has1 ? 2 : 1); r++) {
                        const int v = r0 + r;
                        // forward_one's logits are raw; generate masks ids 0..3
                        const float lg = (v < 4 && !p.all_logits) ? -INFINITY : acc[r][c];
                        if (p.all_logits) {
                            p.trace[((size_t)b * p.trace_steps + t) * p.V + v] = lg;
                        } else {
                            p.logits[(size_t)b * p.V + v] = lg;
                            if (greedy) {
                                const unsigned cnt =
                                    p.s.pen_active ? __ldcg(p.counts + (size_t)b * p.V + v) : 0u;
                                const bool ban =
                                    p.s.ngram > 0 &&
                                    ((__ldcg(p.banned + (size_t)b * nwords + (v >> 5)) >> (v & 31)) & 1u);
                                const float tv = transform_value(lg, cnt, ban, p.s);
                                if (better(tv, v, bv[c], bi[c])) { bv[c] = tv; bi[c] = v; }
                            }
                        }
                    }
                }
            }
        }
        if (greedy) {
            __syncthreads();  // xs no longer read; wi may alias beyond it
            if (lane == 0)
                for (int c = 0; c < bc; c++) { wv[warp * kBCMax + c] = bv[c]; wi[warp * kBCMax + c] = bi[c]; }
            __syncthreads();
            if (threadIdx.x < bc) {
                const int c = threadIdx.x;
                float v = wv[c];
                int i = wi[c];
                for (int w = 1; w < kWarps; w++)
                    if (better(wv[w * kBCMax + c], wi[w * kBCMax + c], v, i)) {
                        v = wv[w * kBCMax + c];
                        i = wi[w * kBCMax + c];
                    }
                p.amax_v[(size_t)bl[c] * gridDim.x + blockIdx.x] = v;
                p.amax_i[(size_t)bl[c] * gridDim.x + blockIdx.x] = i;
            }
        }
        __syncthreads();
    }
}

// n-gram bans for the next draw of sequence b (mark_repeated_ngrams,
// generate.c:394-412) from history out_ids[b][0..hlen).
template <typename WT>
__device__ void compute_bans(const LoopParams<WT>& p, int b, int hlen) {
    const int nwords = (p.V + 31) >> 5;
    unsigned* bw = p.banned + (size_t)b * nwords;
    const uint16_t* hist = p.out_ids + (size_t)b * p.out_cap;
    for (int w = threadIdx.x; w < nwords; w += blockDim.x) bw[w] = 0u;
    __syncthreads();
    const int n = p.s.ngram;
    if (n == 1) {
        for (int i = threadIdx.x; i < hlen; i += blockDim.x) {
            const int id = ld_u16_cg(hist + i);
            if (id < p.V) atomicOr(&bw[id >> 5], 1u << (id & 31));
        }
    } else if (n > 1) {
        const int pl = n - 1;
        if (hlen >= pl) {
            const int cur = hlen - pl;
            for (int st = threadIdx.x; st + pl < hlen; st += blockDim.x) {
                bool eq = true;
                for (int k = 0; k < pl && eq; k++)
                    eq = ld_u16_cg(hist + st + k) == ld_u16_cg(hist + cur + k);
                if (eq) {
                    const int id = ld_u16_cg(hist + st + pl);
                    if (id < p.V) atomicOr(&bw[id >> 5], 1u << (id & 31));
                }
            }
        }
    }
    __syncthreads();
}

template <typename WT>
__device__ void phase_sample(const LoopParams<WT>& p, int t, LoopSmem& sm, int nhead, int nparts) {
    SamplerSmem ss = sampler_carve(sm.xs, p.V);
    const int nwords = (p.V + 31) >> 5;
    for (int i = blockIdx.x; i < nhead; i += gridDim.x) {
        const int b = sm.head[i];
        SeqState* st = p.seq + b;
        const int P = ld_volatile_i32(&st->P), g = ld_volatile_i32(&st->gen);
        const int nnew = ld_volatile_i32(&st->nnew);
        const float* lg = p.logits + (size_t)b * p.V;
        if (p.trace && g < p.trace_steps)
            for (int v = threadIdx.x; v < p.V; v += blockDim.x)
                p.trace[((size_t)b * p.trace_steps + g) * p.V + v] = ldcg(lg + v);
        unsigned long long rng = ld_volatile_u64(&st->rng);
        int id = 0;
        if (p.s.top_k == 1) {
            // the best of the nparts greedy partials: better() is a total
            // order, so the parallel reduction picks the same (value, id)
            {
                float v = -INFINITY;
                int best = 0x7fffffff;
                for (int c = threadIdx.x; c < nparts; c += blockDim.x) {
                    const float cv = ldcg(p.amax_v + (size_t)b * nparts + c);
                    const int ci = __ldcg(p.amax_i + (size_t)b * nparts + c);
                    if (better(cv, ci, v, best)) { v = cv; best = ci; }
                }
                warp_argmax(v, best);
                const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
                if (lane == 0) { sm.red[warp] = v; sm.ints[16 + warp] = best; }
                __syncthreads();
                if (threadIdx.x == 0) {
                    for (int w = 1; w < kWarps; w++)
                        if (better(sm.red[w], sm.ints[16 + w], v, best)) { v = sm.red[w]; best = sm.ints[16 + w]; }
                    if (best == 0x7fffffff) { best = 0; }
                    sm.red[0] = v;
                    sm.ints[1] = best;
                }
            }
            __syncthreads();
            float v = sm.red[0];
            id = sm.ints[1];
            if (!isfinite(v) && p.s.ngram > 0) {
                // all candidates banned: redo without bans (generate.c:472-476)
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                for (int vv = threadIdx.x; vv < p.V; vv += blockDim.x) {
                    const unsigned cnt = p.s.pen_active ? __ldcg(p.counts + (size_t)b * p.V + vv) : 0u;
                    const float tv = transform_value(ldcg(lg + vv), cnt, false, p.s);
                    if (better(tv, vv, bv, bi)) { bv = tv; bi = vv; }
                }
                warp_argmax(bv, bi);
                const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
                __syncthreads();
                if (lane == 0) { sm.red[warp] = bv; sm.ints[16 + warp] = bi; }
                __syncthreads();
                if (threadIdx.x == 0) {
                    float fv = sm.red[0];
                    int fi = sm.ints[16];
                    for (int w = 1; w < kWarps; w++)
                        if (better(sm.red[w], sm.ints[16 + w], fv, fi)) { fv = sm.red[w]; fi = sm.ints[16 + w]; }
                    sm.red[32] = fv;
                    sm.ints[1] = fi == 0x7fffffff ? 0 : fi;
                }
                __syncthreads();
                v = sm.red[32];
                id = sm.ints[1];
            }
            if (isfinite(v)) (void)rng_f32(rng);  // the draw of generate.c:510
        } else {
            const int k = min(min(p.s.top_k, p.V), MC_MAX_TOPK_DEV);
            bool use_bans = p.s.ngram > 0;
            for (int attempt = 0; attempt < 2; attempt++) {
                const bool has_nan = sampler_fill(lg, p.counts + (size_t)b * p.V,
                                                  p.banned + (size_t)b * nwords, use_bans, p.V, p.s, ss);
                int n = k;
                bool fast = !has_nan && topk_fast(p.V, k, ss);
                if (!fast) {
                    __syncthreads();
                    topk_replay(p.V, k, ss, n);
                }
                __syncthreads();
                if (threadIdx.x == 0) {
                    bool retry = false;
                    const int r = sampler_tail(n, p.s, ss, rng, retry, use_bans);
                    sm.ints[1] = r;
                    sm.ints[2] = retry;
                }
                __syncthreads();
                id = sm.ints[1];
                if (!sm.ints[2]) break;
                use_bans = false;
                __syncthreads();
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            if (id < 0 || id >= p.V) {
                atomicMax(p.status, (int)ST_DEVICE);
            } else {
                uint16_t* out = p.out_ids + (size_t)b * p.out_cap;
                out[P + g] = (uint16_t)id;
                if (p.s.pen_active) p.counts[(size_t)b * p.V + id] += 1u;
                const int generated = g + 1;
                st->gen = generated;
                st->rng = rng;
                bool stop = false;
                if (p.s.stop_len > 0 && generated >= p.s.min_new && generated >= p.s.stop_len) {
                    stop = true;
                    const int s0 = P + generated - p.s.stop_len;
                    for (int k = 0; k < p.s.stop_len; k++)
                        if (ld_u16_cg(out + s0 + k) != (int)p.s.stop_ids[k]) { stop = false; break; }
                }
                if (stop) {
                    st->result = P + generated - p.s.stop_len;
                    st->final_pos = P + g;
                    st->done = 1;
                } else if (generated >= nnew) {
                    st->result = P + nnew;
                    st->final_pos = P + nnew;
                    st->done = 1;
                } else {
                    st->tok = id;
                }
                sm.ints[3] = st->done;
            }
        }
        __syncthreads();
        if (p.s.ngram > 0 && !sm.ints[3]) compute_bans(p, b, P + g + 1);
        __syncthreads();
    }
}

// Prologue of a generate call: one CTA per sequence copies the prompt into
// its history, seeds penalty counts and first-draw n-gram bans.
template <typename WT>
__device__ void loop_prologue(const LoopParams<WT>& p) {
    for (int b = blockIdx.x; b < p.B; b += gridDim.x) {
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
}

// ------------------------------------------------------------------ kernel
template <typename WT, bool VEC>
__global__ void __launch_bounds__(kThreads, 1) token_loop_kernel(const LoopParams<WT> p) {
    extern __shared__ __align__(16) float smem_f[];
    LoopSmem sm;
    sm.red = smem_f;
    sm.fwd = reinterpret_cast<int*>(smem_f + 64);
    sm.head = sm.fwd + p.Bcap;
    sm.ints = sm.head + p.Bcap;
    sm.xs = smem_f + loop_fixed_bytes(p.Bcap) / 4;
    GridSync gs{p.bar, p.status, gridDim.x + p.extra_arrivals, 0u, p.timeout_ns};

    if (!p.all_logits) loop_prologue(p);
    if (!gs.sync()) return;

    for (int t = p.t0; t < p.T; t++) {
        // Sequence lists for this step (identical in every CTA).
        if (threadIdx.x == 0) {
            int nf = 0, nh = 0;
            for (int b = 0; b < p.B; b++) {
                const SeqState* st = p.seq + b;
                if (ld_volatile_i32(&st->done)) continue;
                const int P = ld_volatile_i32(&st->P);
                const int nnew = ld_volatile_i32(&st->nnew);
                const int Tb = p.all_logits ? P : P + nnew - 1;
                if (t >= Tb) continue;
                sm.fwd[nf++] = b;
                if (p.all_logits || t >= P - 1) sm.head[nh++] = b;
            }
            sm.ints[12] = nf;
            sm.ints[13] = nh;
        }
        __syncthreads();
        const int nf = sm.ints[12], nh = sm.ints[13];
        if (p.stamps && blockIdx.x == 0 && threadIdx.x == 0) p.stamps[t] = globaltimer_ns();
        if (nf == 0) break;
        for (int l = 0; l < p.L; l++) {
            phase_qkv<WT, VEC>(p, l, t, sm, nf);
            if (!gs.sync()) return;
            phase_att<WT>(p, l, t, sm, nf);
            if (!gs.sync()) return;
            phase_residual<WT, VEC>(p, p.w_proj + (size_t)l * p.D * p.D, p.D, p.att, p.D, sm, nf);
            if (!gs.sync()) return;
            phase_upgate<WT, VEC>(p, l, sm, nf);
            if (!gs.sync()) return;
            phase_residual<WT, VEC>(p, p.w_down + (size_t)l * p.D * p.F, p.F, p.f, p.F, sm, nf);
            if (!gs.sync()) return;
        }
        if (nh > 0) {
            phase_head<WT, VEC>(p, t, sm, nh);
            if (!gs.sync()) return;
            if (!p.all_logits) {
                phase_sample<WT>(p, t, sm, nh, (int)gridDim.x);
                if (!gs.sync()) return;
            }
        }
    }
    if (p.stamps && blockIdx.x == 0 && threadIdx.x == 0) p.stamps[p.T] = globaltimer_ns();
}

}  // namespace mc

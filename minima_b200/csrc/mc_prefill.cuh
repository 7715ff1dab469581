// mc_prefill.cuh — batched prefill of prompt positions for sm_100a.
//
// generate_with_options feeds the prompt one position at a time
// (generate.c:575-578); every position's forward is independent of the
// sampler, so positions [0, Pf) of all sequences (Pf = shortest prompt - 1)
// run here as one causal batched forward (the arithmetic of model_forward,
// forward.c:176-274, restricted to the layers) on M = B * Pf rows:
//   norm -> QKV GEMM (+RoPE, K/V into the cache) -> causal attention ->
//   proj GEMM (+residual) -> norm -> up/gate GEMM (+SwiGLU) -> down GEMM
//   (+residual)
// The tied lm_head is not applied: no logits of those positions are read.
// The token loop then continues at position Pf.  GEMMs are fp32 on CUDA
// cores (64x64 tiles, 4x4 per thread, k-major shared tiles).
#pragma once

#include "mc_device.cuh"

namespace mc {

struct PrefillArgs {
    int V, D, L, H, K, hd, kvd, Q, F, G;
    int B, Bcap, cap;          // sequences, cache batch stride, cache capacity
    int c0, c1;                // positions of this chunk
    int chunk;                 // rows per sequence in the work buffers (>= c1 - c0)
    const uint16_t* prompts;
    int prompt_stride;
    const float2* rope;
    float* kc;                 // K / V pages (KvPages)
    float* vc;
    KvPages pg;
    float* X;                  // [B*chunk][D] residual
    float* XN;                 // [B*chunk][D]
    float* QB;                 // [B*chunk][D] rotated queries
    float* ATT;                // [B*chunk][D]
    float* FH;                 // [B*chunk][F]
    // bf16 copies of the GEMM inputs for the tensor-core path with bf16
    // weights (kind::f16 needs both operands in bf16); null otherwise
    __nv_bfloat16* XN16;
    __nv_bfloat16* ATT16;
    __nv_bfloat16* FH16;
    // model_forward's per-layer caches (forward.h:17-23): when set, the
    // SwiGLU epilogue also stores the up and gate projections [B*chunk][F]
    float* UP;
    float* GATE;
    int* status;
};

__device__ __forceinline__ int pf_rows(const PrefillArgs& a) { return a.B * (a.c1 - a.c0); }
// row m <-> (sequence b, position t)
__device__ __forceinline__ void pf_row(const PrefillArgs& a, int m, int& b, int& t) {
    const int n = a.c1 - a.c0;
    b = m / n;
    t = a.c0 + m % n;
}

// X = embedding (layer 0 only), XN = rmsnorm(X, scale) (generate.c:57-63,
// 86-88); one warp per row.
template <typename WT>
__global__ void __launch_bounds__(256) pf_norm_kernel(PrefillArgs a, const WT* tok_emb,
                                                      const float* scale, int embed) {
    const int lane = threadIdx.x & 31;
    const int m = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (m >= pf_rows(a)) return;
    int b, t;
    pf_row(a, m, b, t);
    float* x = a.X + (size_t)m * a.D;
    if (embed) {
        int tok = a.prompts[(size_t)b * a.prompt_stride + t];
        if (tok >= a.V) {
            if (lane == 0) atomicMax(a.status, (int)ST_DEVICE);
            tok = 0;
        }
        for (int k = lane; k < a.D; k += 32) x[k] = wload1(tok_emb + (size_t)tok * a.D + k);
        __syncwarp();
    }
    float ss = 0.0f;
    for (int k = lane; k < a.D; k += 32) ss += x[k] * x[k];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)a.D + 1e-5f);
    for (int k = lane; k < a.D; k += 32) {
        const float v = x[k] * inv * scale[k];
        a.XN[(size_t)m * a.D + k] = v;
        if (a.XN16) a.XN16[(size_t)m * a.D + k] = __float2bfloat16_rn(v);
    }
}

enum PfEpi { EPI_QKV = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_STORE = 3 };

constexpr int GBM = 64, GBN = 64, GBK = 32;
constexpr int kPfMaxSplit = 8;   // K slices of one output tile (gridDim.z)

// C[M][N] = A[M][K] . W[N][K]^T with a fused epilogue.  For EPI_SWIGLU, W2 is
// the gate matrix and the output is silu(A.W2) * (A.W); EPI_STORE writes
// C as is (the lm_head of model_forward).  K % 4 == 0.
//
// The next K tile is read from global memory into registers while the
// current one is multiplied.  With gridDim.z = ks > 1 (small M, where the
// tiles alone leave most SMs idle) the K blocks are split in ks contiguous
// slices: each CTA stores its partial tile in `part`, and the last CTA of a
// tile to arrive (counter `cnt`, left at zero again for the next launch)
// sums the slices in slice order 0..ks-1, so the result does not depend on
// the arrival order, and applies the epilogue.
template <typename WT, int EPI>
__global__ void __launch_bounds__(256, 1) pf_gemm_kernel(PrefillArgs a, const float* A, int M, int N,
                                                      int Kd, const WT* W, const WT* W2, float* C,
                                                      int ldc, int layer, float* part, unsigned* cnt) {
    constexpr int DUAL = EPI == EPI_SWIGLU ? 2 : 1;
    __shared__ __align__(16) float As[GBK][GBM + 4];
    __shared__ __align__(16) float Ws[DUAL][GBK][GBN + 4];
    __shared__ unsigned s_last;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * GBM, n0 = blockIdx.x * GBN;
    const int nk = (Kd + GBK - 1) / GBK, ks = gridDim.z, z = blockIdx.z;
    const int kb0 = (int)((long long)nk * z / ks), kb1 = (int)((long long)nk * (z + 1) / ks);
    float acc[DUAL][4][4];
#pragma unroll
    for (int d = 0; d < DUAL; d++)
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[d][i][j] = 0.0f;
    // tiles: 64 rows x 32 k = 512 float4, two per thread, stored k-major
    float4 ra[2];
    float rw[DUAL][2][4];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int e = threadIdx.x + 256 * u;
            const int r = e / (GBK / 4), kq = (e % (GBK / 4)) * 4;
            const int gm = m0 + r, gk = k0 + kq;
            ra[u] = gm < M && gk < Kd ? *reinterpret_cast<const float4*>(A + (size_t)gm * Kd + gk)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int d = 0; d < DUAL; d++) {
                const WT* Wd = d == 0 ? W : W2;
                const int gn = n0 + r;
#pragma unroll
                for (int q = 0; q < 4; q++) rw[d][u][q] = 0.0f;
                if (gn < N && gk < Kd) {
                    const WT* src = Wd + (size_t)gn * Kd + gk;
#pragma unroll
                    for (int q = 0; q < 4; q++) rw[d][u][q] = wload1(src + q);
                }
            }
        }
    };
    if (kb0 < kb1) fetch(kb0 * GBK);
    for (int kb = kb0; kb < kb1; kb++) {
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int e = threadIdx.x + 256 * u;
            const int r = e / (GBK / 4), kq = (e % (GBK / 4)) * 4;
            As[kq + 0][r] = ra[u].x; As[kq + 1][r] = ra[u].y; As[kq + 2][r] = ra[u].z; As[kq + 3][r] = ra[u].w;
#pragma unroll
            for (int d = 0; d < DUAL; d++)
#pragma unroll
                for (int q = 0; q < 4; q++) Ws[d][kq + q][r] = rw[d][u][q];
        }
        __syncthreads();
        if (kb + 1 < kb1) fetch((kb + 1) * GBK);   // in flight during the FMAs below
#pragma unroll 8
        for (int kk = 0; kk < GBK; kk++) {
            const float4 av = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
            const float ar[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
            for (int d = 0; d < DUAL; d++) {
                const float4 wv = *reinterpret_cast<const float4*>(&Ws[d][kk][tx * 4]);
                const float wr[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[d][i][j] = fmaf(ar[i], wr[j], acc[d][i][j]);
            }
        }
        __syncthreads();
    }
    if (ks > 1) {
        // partial tiles thread-major: each thread writes and later reads its own 16 * DUAL floats
        const int tile = blockIdx.y * gridDim.x + blockIdx.x, ntiles = gridDim.x * gridDim.y;
        float4* mine = reinterpret_cast<float4*>(part) +
                       (((size_t)z * ntiles + tile) * 256 + threadIdx.x) * (4 * DUAL);
#pragma unroll
        for (int d = 0; d < DUAL; d++)
#pragma unroll
            for (int i = 0; i < 4; i++)
                mine[d * 4 + i] = make_float4(acc[d][i][0], acc[d][i][1], acc[d][i][2], acc[d][i][3]);
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s_last = atomicAdd(cnt + tile, 1u) == (unsigned)(ks - 1);
        __syncthreads();
        if (!s_last) return;
        __threadfence();
#pragma unroll
        for (int d = 0; d < DUAL; d++)
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[d][i][j] = 0.0f;
        for (int sl = 0; sl < ks; sl++) {
            const float4* ps = reinterpret_cast<const float4*>(part) +
                               (((size_t)sl * ntiles + tile) * 256 + threadIdx.x) * (4 * DUAL);
#pragma unroll
            for (int d = 0; d < DUAL; d++)
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float4 v = __ldcg(ps + d * 4 + i);
                    acc[d][i][0] += v.x; acc[d][i][1] += v.y; acc[d][i][2] += v.z; acc[d][i][3] += v.w;
                }
        }
        if (threadIdx.x == 0) cnt[tile] = 0u;
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = m0 + ty * 4 + i;
        if (m >= M) continue;
        if constexpr (EPI == EPI_QKV) {
            int b, t;
            pf_row(a, m, b, t);
#pragma unroll
            for (int j = 0; j < 4; j += 2) {
                const int n = n0 + tx * 4 + j;      // even; n and n+1 are a RoPE pair
                if (n >= N) continue;
                float v0 = acc[0][i][j], v1 = acc[0][i][j + 1];
                const int slot = n / a.hd, dd = n % a.hd;
                if (slot < a.H + a.K) {
                    const float2 r = a.rope[(size_t)t * (a.hd / 2) + dd / 2];
                    const float x0 = v0 * r.x - v1 * r.y, x1 = v0 * r.y + v1 * r.x;
                    v0 = x0; v1 = x1;
                }
                if (slot < a.H) {
                    a.QB[(size_t)m * a.D + n] = v0;
                    a.QB[(size_t)m * a.D + n + 1] = v1;
                } else {
                    const bool isk = slot < a.H + a.K;
                    const int g = isk ? slot - a.H : slot - a.H - a.K;
                    float* dst = (isk ? a.kc : a.vc) + kv_row(a.pg, a.L, a.K, layer, b, g, t) * a.hd + dd;
                    dst[0] = v0;
                    dst[1] = v1;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int n = n0 + tx * 4 + j;
                if (n >= N) continue;
                if constexpr (EPI == EPI_RESID) {
                    C[(size_t)m * ldc + n] += acc[0][i][j];
                } else if constexpr (EPI == EPI_STORE) {
                    C[(size_t)m * ldc + n] = acc[0][i][j];
                } else {
                    const float up = acc[0][i][j], g = acc[DUAL - 1][i][j];
                    C[(size_t)m * ldc + n] = (g / (1.0f + expf(-g))) * up;
                    if (a.UP) {
                        a.UP[(size_t)m * ldc + n] = up;
                        a.GATE[(size_t)m * ldc + n] = g;
                    }
                }
            }
        }
    }
}

// The rows of model_forward's qkv cache (forward.c:224-227: the QKV
// projection after RoPE) for the chunk: Q from QB, K and V from the KV
// cache, laid out [row][Q heads | K heads | V heads].  One CTA per row.
__global__ void __launch_bounds__(256) pf_gather_qkv_kernel(PrefillArgs a, int layer, float* out) {
    const int m = blockIdx.x;
    if (m >= pf_rows(a)) return;
    int b, t;
    pf_row(a, m, b, t);
    float* row = out + (size_t)m * a.Q;
    for (int n = threadIdx.x; n < a.Q; n += blockDim.x) {
        float v;
        if (n < a.D) {
            v = a.QB[(size_t)m * a.D + n];
        } else {
            const bool isk = n < a.D + a.kvd;
            const int c = isk ? n - a.D : n - a.D - a.kvd;
            const int g = c / a.hd, dd = c % a.hd;
            v = (isk ? a.kc : a.vc)[kv_row(a.pg, a.L, a.K, layer, b, g, t) * a.hd + dd];
        }
        row[n] = v;
    }
}

// Causal attention for the chunk's queries over cached keys [0, t]
// (generate.c:121-156 per position).  Block = (query tile, KV head,
// sequence); rows = G heads x QT positions, 16 rows per warp; keys staged
// 64 at a time; online softmax.
constexpr int PF_KT = 64;

__global__ void __launch_bounds__(256) pf_attention_kernel(PrefillArgs a, int layer, int QT) {
    extern __shared__ __align__(16) float pfs[];
    const int hd = a.hd, G = a.G, n = a.c1 - a.c0;
    const int qt0 = a.c0 + blockIdx.x * QT;           // first query position of the tile
    const int g = blockIdx.y, b = blockIdx.z;
    if (qt0 >= a.c1) return;
    const int qt1 = min(a.c1, qt0 + QT);
    const int rows = G * QT;
    float* Qs = pfs;                                  // [rows][hd]
    float* Ks = Qs + rows * hd;                       // [KT][hd+1]
    float* Vs = Ks + PF_KT * (hd + 1);                // [KT][hd]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float scale = 1.0f / sqrtf((float)hd);
    for (int e = threadIdx.x; e < rows * hd; e += blockDim.x) {
        const int r = e / hd, d = e % hd, h = r / QT, qi = r % QT;
        const int t = qt0 + qi;
        Qs[e] = t < qt1 ? a.QB[((size_t)b * n + (t - a.c0)) * a.D + (g * G + h) * hd + d] : 0.0f;
    }
    // per-row state: rows handled by this warp are r = warp + 8 * k
    constexpr int RPW = 16;
    float m_run[RPW], l_run[RPW], o_acc[RPW][2];
#pragma unroll
    for (int k = 0; k < RPW; k++) { m_run[k] = -INFINITY; l_run[k] = 0.0f; o_acc[k][0] = o_acc[k][1] = 0.0f; }
    for (int k0 = 0; k0 < qt1; k0 += PF_KT) {
        const int kn = min(PF_KT, qt1 - k0);
        // PF_KT (64) keys from a multiple of 64: one page
        const size_t row0 = kv_row(a.pg, a.L, a.K, layer, b, g, k0);
        const float* kg = a.kc + row0 * hd;
        const float* vg = a.vc + row0 * hd;
        __syncthreads();
        for (int e = threadIdx.x; e < kn * hd; e += blockDim.x) {
            const int j = e / hd, d = e % hd;
            Ks[j * (hd + 1) + d] = ldcg(kg + (size_t)j * hd + d);
            Vs[j * hd + d] = ldcg(vg + (size_t)j * hd + d);
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < RPW; k++) {
            const int r = warp + 8 * k;
            if (r >= rows) break;
            const int t = qt0 + r % QT;
            if (t >= qt1 || k0 > t) continue;           // padded row / no visible key
            const float* q = Qs + r * hd;
            float s0 = -INFINITY, s1 = -INFINITY;
            const int j0 = lane, j1 = lane + 32;
            if (j0 < kn && k0 + j0 <= t) {
                float dot = 0.0f;
                for (int d = 0; d < hd; d++) dot += q[d] * Ks[j0 * (hd + 1) + d];
                s0 = dot * scale;
            }
            if (j1 < kn && k0 + j1 <= t) {
                float dot = 0.0f;
                for (int d = 0; d < hd; d++) dot += q[d] * Ks[j1 * (hd + 1) + d];
                s1 = dot * scale;
            }
            const float mt = warp_max(fmaxf(s0, s1));
            const float mnew = fmaxf(m_run[k], mt);
            const float p0 = s0 == -INFINITY ? 0.0f : expf(s0 - mnew);
            const float p1 = s1 == -INFINITY ? 0.0f : expf(s1 - mnew);
            const float corr = m_run[k] == -INFINITY ? 0.0f : expf(m_run[k] - mnew);
            l_run[k] = l_run[k] * corr + warp_sum(p0 + p1);
            m_run[k] = mnew;
            float o0 = o_acc[k][0] * corr, o1 = o_acc[k][1] * corr;
            for (int j = 0; j < kn; j++) {
                const float pj = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
                // lanes past head_dim own no output (and row kn - 1 + lane
                // would fall past the tile when head_dim < 32)
                if (lane < hd) o0 += pj * Vs[j * hd + lane];
                if (lane + 32 < hd) o1 += pj * Vs[j * hd + lane + 32];
            }
            o_acc[k][0] = o0;
            o_acc[k][1] = o1;
        }
    }
#pragma unroll
    for (int k = 0; k < RPW; k++) {
        const int r = warp + 8 * k;
        if (r >= rows) break;
        const int h = r / QT, t = qt0 + r % QT;
        if (t >= qt1) continue;
        const size_t off = ((size_t)b * n + (t - a.c0)) * a.D + (g * G + h) * hd;
        float* dst = a.ATT + off;
        const float inv = 1.0f / l_run[k];
        const float v0 = o_acc[k][0] * inv, v1 = o_acc[k][1] * inv;
        if (lane < hd) dst[lane] = v0;
        if (lane + 32 < hd) dst[lane + 32] = v1;
        if (a.ATT16) {
            if (lane < hd) a.ATT16[off + lane] = __float2bfloat16_rn(v0);
            if (lane + 32 < hd) a.ATT16[off + lane + 32] = __float2bfloat16_rn(v1);
        }
    }
}

// The same causal attention with register tiles, for head_dim 16, 32 or 64
// and G * QT <= 128 query rows per block.  256 threads as 16 x 16: thread
// (tr, tc) holds rows tr + 16 i (i < 8) and, per 64-key tile, keys
// tc + 16 j (j < 4) of the scores, and the same rows x dimensions
// [HD/16 tc, HD/16 (tc + 1)) of the output, so a score costs one FMA per
// dimension against float4 shared-memory reads shared by 4 x 8 products.
// Row r is head r / QT of the block's KV head at position qt0 + r % QT.
// Per key tile: scores, a per-row online softmax (the 16 threads of a row
// reduce with shuffles), P through shared memory, then P.V.
constexpr int PF_RT = 128;                    // rows per block
constexpr int PF_PLD = PF_KT + 4;             // row stride of the probability tile

template <int HD>
__global__ void __launch_bounds__(256) pf_attention_tile_kernel(PrefillArgs a, int layer, int QT) {
    constexpr int E = HD / 16;                // output dimensions per thread
    constexpr int LD = HD + 4;                // padded row stride of the Q and K tiles
    extern __shared__ __align__(16) float pfs[];
    float* Qs = pfs;                          // [PF_RT][LD]
    float* Ks = Qs + PF_RT * LD;              // [PF_KT][LD]
    float* Vs = Ks + PF_KT * LD;              // [PF_KT][HD]
    float* Ps = Vs + PF_KT * HD;              // [PF_RT][PF_PLD]
    const int G = a.G, n = a.c1 - a.c0;
    const int qt0 = a.c0 + blockIdx.x * QT;
    const int g = blockIdx.y, b = blockIdx.z;
    if (qt0 >= a.c1) return;
    const int qt1 = min(a.c1, qt0 + QT);
    const int rows = G * QT;
    const int tr = threadIdx.x >> 4, tc = threadIdx.x & 15;
    const float scale = 1.0f / sqrtf((float)HD);
    // queries (zero rows past the block's)
    for (int e = threadIdx.x; e < PF_RT * (HD / 4); e += blockDim.x) {
        const int r = e / (HD / 4), c = e - r * (HD / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < rows) {
            const int h = r / QT, t = qt0 + r % QT;
            if (t < qt1)
                v = *reinterpret_cast<const float4*>(a.QB + ((size_t)b * n + (t - a.c0)) * a.D +
                                                     (g * G + h) * HD + 4 * c);
        }
        *reinterpret_cast<float4*>(Qs + r * LD + 4 * c) = v;
    }
    int pos[8];                               // position of each row, -1 past the block
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int r = tr + 16 * i;
        const int t = qt0 + r % QT;
        pos[i] = (r < rows && t < qt1) ? t : -1;
    }
    float m_run[8], l_run[8], o[8][E];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        m_run[i] = -INFINITY;
        l_run[i] = 0.0f;
#pragma unroll
        for (int e = 0; e < E; e++) o[i][e] = 0.0f;
    }
    for (int k0 = 0; k0 < qt1; k0 += PF_KT) {
        const int kn = min(PF_KT, qt1 - k0);
        // PF_KT (64) keys from a multiple of 64: one page
        const size_t row0 = kv_row(a.pg, a.L, a.K, layer, b, g, k0);
        const float* kg = a.kc + row0 * HD;
        const float* vg = a.vc + row0 * HD;
        __syncthreads();                      // the previous tile's readers are done
        for (int e = threadIdx.x; e < PF_KT * (HD / 4); e += blockDim.x) {
            const int j = e / (HD / 4), c = e - j * (HD / 4);
            float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
            if (j < kn) {
                kv4 = ldcg4(kg + (size_t)j * HD + 4 * c);
                vv4 = ldcg4(vg + (size_t)j * HD + 4 * c);
            }
            *reinterpret_cast<float4*>(Ks + j * LD + 4 * c) = kv4;
            *reinterpret_cast<float4*>(Vs + j * HD + 4 * c) = vv4;
        }
        __syncthreads();
        // scores of rows tr + 16 i against keys tc + 16 j
        float sacc[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) sacc[i][j] = 0.0f;
#pragma unroll 4
        for (int c = 0; c < HD / 4; c++) {
            float4 kk[4];
#pragma unroll
            for (int j = 0; j < 4; j++) kk[j] = *reinterpret_cast<const float4*>(Ks + (tc + 16 * j) * LD + 4 * c);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float4 q = *reinterpret_cast<const float4*>(Qs + (tr + 16 * i) * LD + 4 * c);
#pragma unroll
                for (int j = 0; j < 4; j++)
                    sacc[i][j] += q.x * kk[j].x + q.y * kk[j].y + q.z * kk[j].z + q.w * kk[j].w;
            }
        }
        // causal mask, online softmax per row (the 16 threads of a row are
        // lanes of one half-warp)
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int key = k0 + tc + 16 * j;
                const bool ok = tc + 16 * j < kn && pos[i] >= 0 && key <= pos[i];
                sacc[i][j] = ok ? sacc[i][j] * scale : -INFINITY;
                mx = fmaxf(mx, sacc[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mnew = fmaxf(m_run[i], mx);
            const float corr = m_run[i] == -INFINITY ? 0.0f : expf(m_run[i] - mnew);
            float ls = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float pj = sacc[i][j] == -INFINITY ? 0.0f : expf(sacc[i][j] - mnew);
                Ps[(tr + 16 * i) * PF_PLD + tc + 16 * j] = pj;
                ls += pj;
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
            l_run[i] = l_run[i] * corr + ls;
            m_run[i] = mnew;
#pragma unroll
            for (int e = 0; e < E; e++) o[i][e] *= corr;
        }
        __syncthreads();
        // P.V: rows tr + 16 i, dimensions E tc .. E tc + E - 1
#pragma unroll 2
        for (int j = 0; j < PF_KT; j += 4) {
            float vv[4][E];
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const float* vr = Vs + (j + jj) * HD + E * tc;
                if constexpr (E == 4) {
                    const float4 v4 = *reinterpret_cast<const float4*>(vr);
                    vv[jj][0] = v4.x; vv[jj][1] = v4.y; vv[jj][2] = v4.z; vv[jj][3] = v4.w;
                } else if constexpr (E == 2) {
                    const float2 v2 = *reinterpret_cast<const float2*>(vr);
                    vv[jj][0] = v2.x; vv[jj][1] = v2.y;
                } else {
#pragma unroll
                    for (int e = 0; e < E; e++) vv[jj][e] = vr[e];
                }
            }
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float4 p4 = *reinterpret_cast<const float4*>(Ps + (tr + 16 * i) * PF_PLD + j);
#pragma unroll
                for (int e = 0; e < E; e++)
                    o[i][e] += p4.x * vv[0][e] + p4.y * vv[1][e] + p4.z * vv[2][e] + p4.w * vv[3][e];
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        if (pos[i] < 0) continue;
        const int r = tr + 16 * i, h = r / QT;
        const size_t off = ((size_t)b * n + (pos[i] - a.c0)) * a.D + (g * G + h) * HD + E * tc;
        const float inv = 1.0f / l_run[i];
#pragma unroll
        for (int e = 0; e < E; e++) {
            a.ATT[off + e] = o[i][e] * inv;
            if (a.ATT16) a.ATT16[off + e] = __float2bfloat16_rn(o[i][e] * inv);
        }
    }
}

__host__ inline size_t pf_attention_tile_smem(int hd) {
    return ((size_t)PF_RT * (hd + 4) + (size_t)PF_KT * (hd + 4) + (size_t)PF_KT * hd + (size_t)PF_RT * PF_PLD) * 4;
}

__host__ inline size_t pf_attention_smem(int hd, int G, int QT) {
    return ((size_t)G * QT * hd + (size_t)PF_KT * (hd + 1) + (size_t)PF_KT * hd) * 4;
}

}  // namespace mc

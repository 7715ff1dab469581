// mc_tcgen05.cuh — tensor-core GEMMs for sm_100a: TMA-fed shared-memory
// tiles, tcgen05.mma with the accumulator in tensor memory (TMEM), and the
// prefill's fused epilogues applied straight out of TMEM.
//
//   C[M][N] = A[M][K] . B[N][K]^T      (A: activations, B: a weight matrix in
//                                       the reference's [out][in] layout)
//
// One CTA per 128 x BN output tile (BN = 64, 128 or 256), 128 threads:
//   thread 0   issues the TMA loads of a STAGES-deep ring (A tiles of 128 rows,
//              B tiles of BN rows, 128 bytes of K each, 128-byte swizzle),
//   thread 32  issues tcgen05.mma (kind::tf32 for fp32 operands, kind::f16
//              for bf16 operands; M = 128, N = BN, 32 bytes of K per
//              instruction) and frees each stage with tcgen05.commit,
//   all 4 warps then drain TMEM with tcgen05.ld (warp w owns lanes
//              32w..32w+31 = output rows) and apply the epilogue.
// For SwiGLU the up and gate tiles share the A tile and accumulate into two
// TMEM column ranges.
//
// Split K (decode GEMMs: a few dozen rows against a whole weight matrix):
// with ksplit > 1 the grid holds ksplit CTAs per output tile, CTA r
// accumulating the r-th slice of K and storing its partial tile with plain
// stores to C + r * M * ldc (EPI_PART); the kernel that next reads the
// result sums the partials in slice order.  Every wait is bounded by the caller's deadline; a
// wait that expires sets the status word, stops the pipeline, drains the
// copies in flight and still frees TMEM.
//
// Numerics: kind::tf32 multiplies with 10-bit mantissas (fp32 accumulate),
// kind::f16 with bf16 operands; both are looser than the fp32 CUDA-core
// path, and the prefill uses them only when asked to.
#pragma once

#include <cuda.h>

#include "mc_device.cuh"
#include "mc_cluster_loop.cuh"
#include "mc_prefill.cuh"

namespace mc {

constexpr int TC_BM = 128;                  // output rows per CTA (TMEM lanes)
constexpr int TC_BKB = 128;                 // bytes of K per stage (one swizzle row)
constexpr int TC_STAGES = 4;                // ring depth of the prefill / mc_gemm launches
constexpr int TC_THREADS = 128;
constexpr int TC_GROUP_M = 8;               // tile rows per rasterization group (L2 reuse)
constexpr uint32_t TC_TILE = TC_BM * TC_BKB;   // 16 KB: A tile; a B tile is BN x 128 B
enum TcKind { TC_TF32 = 0, TC_BF16 = 1 };
constexpr int TCE_STORE = EPI_STORE;        // plain C = A.B^T
constexpr int EPI_PART = 4;                 // partial tile of K slice r at C + r * M * ldc
constexpr int EPI_PART2 = 5;                // the same for a matrix pair: [0, N) and [N, 2N) of a row

struct TcArgs {
    int M, N, K;               // problem
    int layer;                 // z coordinate of the weight tensor maps
    float* C;
    int ldc;
    PrefillArgs pa;            // rows <-> (sequence, position) for the QKV epilogue
    // decode mode (batched token loop): row m is sequence m at the position
    // *tpos; rows whose act[m] is 0 are not written.  act == null: prefill.
    const int* act;
    const int* tpos;
    int* status;
    unsigned long long timeout_ns;
    int ksplit;                // CTAs splitting K per tile (<= 1: no split; EPI_PART only)
    int x_lo_row;              // decode, bf16: first row of the lo halves in the X map
    // decode lm_head (tc_dec_kernel with TCE_STORE and head != 0): ids 0..3
    // are stored as -inf (generate.c:580-581) and, for greedy sampling, each
    // (sequence, 128-id tile)'s best transformed value and its id
    // (generate.c:438-460) go to amax_v/amax_i at [sequence][tile]
    int head;
    SamplingArgs sa;
    const unsigned* counts;    // [B][N] ids sampled so far (penalties)
    const unsigned* banned;    // [B][ceil(N/32)] n-gram bans
    float* amax_v;
    int* amax_i;
};

// Dynamic shared memory of a launch with `btiles` B tiles of `bn` rows per
// stage (1, or 2 for SwiGLU) and `stages` stages: alignment slack, the
// ring, barriers and control words.
__host__ __device__ constexpr size_t tc_smem_bytes(int btiles, int bn, int stages) {
    return 1024 + (size_t)stages * (TC_TILE + (size_t)btiles * bn * TC_BKB) + 256;
}

// Shared-memory matrix descriptor of a K-major tile of 8-row groups of
// 128-byte rows with the 128-byte swizzle (sm_100 format: start >> 4 at
// [0,14), leading offset [16,30) unused for swizzled K-major, stride offset
// 1024 B >> 4 at [32,46), version 1 at [46,48), layout 2 = SWIZZLE_128B at
// [61,64)).
__device__ __forceinline__ uint64_t tc_sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}

// Instruction descriptor: fp32 accumulate, A/B format (tf32 = 2, bf16 = 1),
// both K-major, N >> 3 at [17,23), M >> 4 at [24,29).
template <int KIND, int BN>
__device__ __forceinline__ uint32_t tc_idesc() {
    constexpr uint32_t fmt = KIND == TC_TF32 ? 2u : 1u;
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BN >> 3) << 17) |
           ((uint32_t)(TC_BM >> 4) << 24);
}

__device__ __forceinline__ void tc_tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                          uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tc_tma_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                          uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

template <int KIND>
__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    if constexpr (KIND == TC_TF32) {
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
    } else {
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
    }
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive TMEM columns of this warp's 32 lanes: lane l gets row
// (32 w + l), columns [col, col + 32).
__device__ __forceinline__ void tc_tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
        "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
        "%30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tc_tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Epilogue of W consecutive columns [n, n + W) of row m (m < M; n, W even;
// in decode mode the caller has checked that row m runs).
template <int EPI, int W>
__device__ __forceinline__ void tc_epilogue(const TcArgs& g, int m, int n, const float (&u)[W],
                                            const float (&gt)[W], int split) {
    if constexpr (EPI == EPI_QKV) {
        const PrefillArgs& a = g.pa;
        int b, t;
        if (g.act) {
            b = m;
            t = *g.tpos;
        } else {
            pf_row(a, m, b, t);
        }
#pragma unroll
        for (int j = 0; j < W; j += 2) {
            const int c = n + j;                 // even: c, c + 1 are a RoPE pair
            if (c >= g.N) break;
            float v0 = u[j], v1 = u[j + 1];
            const int slot = c / a.hd, dd = c - slot * a.hd;
            if (slot < a.H + a.K) {
                const float2 r = a.rope[(size_t)t * (a.hd / 2) + dd / 2];
                const float x0 = v0 * r.x - v1 * r.y, x1 = v0 * r.y + v1 * r.x;
                v0 = x0;
                v1 = x1;
            }
            if (slot < a.H) {
                a.QB[(size_t)m * a.D + c] = v0;
                a.QB[(size_t)m * a.D + c + 1] = v1;
            } else {
                const bool isk = slot < a.H + a.K;
                const int gk = isk ? slot - a.H : slot - a.H - a.K;
                float* dst = (isk ? a.kc : a.vc) + kv_row(a.pg, a.L, a.K, g.layer, b, gk, t) * a.hd + dd;
                dst[0] = v0;
                dst[1] = v1;
            }
        }
    } else if constexpr (EPI == EPI_PART || EPI == EPI_PART2) {
        float* crow = g.C + ((size_t)split * g.M + m) * g.ldc;
#pragma unroll
        for (int j = 0; j < W; j++) {
            if (n + j >= g.N) break;
            crow[n + j] = u[j];
            if constexpr (EPI == EPI_PART2) crow[g.N + n + j] = gt[j];
        }
    } else {
        float* crow = g.C + (size_t)m * g.ldc;
#pragma unroll
        for (int j = 0; j < W; j++) {
            const int c = n + j;
            if (c >= g.N) break;
            if constexpr (EPI == EPI_RESID) {
                crow[c] += u[j];
            } else if constexpr (EPI == EPI_SWIGLU) {
                const float v = (gt[j] / (1.0f + expf(-gt[j]))) * u[j];
                crow[c] = v;
                if (g.pa.FH16) g.pa.FH16[(size_t)m * g.ldc + c] = __float2bfloat16_rn(v);
            } else {
                crow[c] = u[j];
            }
        }
    }
}

template <int KIND, int EPI, int BN, int STAGES>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmB2, const TcArgs g) {
    constexpr int DUAL = EPI == EPI_SWIGLU ? 2 : 1;
    constexpr int ES = KIND == TC_TF32 ? 4 : 2;
    constexpr int BKE = TC_BKB / ES;                       // K elements per stage
    constexpr uint32_t BTILE = (uint32_t)BN * TC_BKB;      // bytes of one B tile
    constexpr uint32_t STAGE = TC_TILE + DUAL * BTILE;
    static_assert(DUAL * BN <= 512, "TMEM holds 512 fp32 columns");
    constexpr int TLD = DUAL * BN + 4;                     // epilogue tile row stride (floats)
    static_assert((size_t)TC_BM * TLD * 4 <= (size_t)STAGES * STAGE, "epilogue tile fits the ring");
    static_assert((2 * STAGES + 1) * 8 + 16 <= 256, "barriers and control words fit the tail");
    static_assert(tc_smem_bytes(DUAL, BN, STAGES) <= 232448, "ring fits 227 KB of shared memory");
    extern __shared__ unsigned char tc_smem_raw[];
    unsigned char* base =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned long long* full = reinterpret_cast<unsigned long long*>(base + STAGES * STAGE);
    unsigned long long* empty = full + STAGES;
    unsigned long long* done = empty + STAGES;
    volatile int* ctl = reinterpret_cast<volatile int*>(done + 1);   // 0 tmem, 1 error, 2 issued, 3 consumed
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = g.ksplit > 1 ? g.ksplit : 1;
    const int split = blockIdx.x % ks;                     // slice of K
    // tiles in groups of TC_GROUP_M tile rows, column-major inside a group,
    // so that the CTAs resident at one time share their A and B tiles in L2
    int m0, n0;
    {
        const int tiles_m = (g.M + TC_BM - 1) / TC_BM, tiles_n = (g.N + BN - 1) / BN;
        const int t = blockIdx.x / ks, per_group = TC_GROUP_M * tiles_n;
        const int first = (t / per_group) * TC_GROUP_M, rows = min(tiles_m - first, TC_GROUP_M);
        const int r = t % per_group;
        m0 = (first + r % rows) * TC_BM;
        n0 = (r / rows) * BN;
    }
    const int nk_all = (g.K + BKE - 1) / BKE;
    // this CTA's K blocks [kb0, kb0 + nk); non-empty while ksplit <= nk_all
    const int kb0 = (int)((long long)split * nk_all / ks);
    const int nk = (int)((long long)(split + 1) * nk_all / ks) - kb0;

    // the ring and the control words must lie inside the dynamic shared
    // memory this launch received; nothing is touched otherwise
    uint32_t dyn = 0;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
    const unsigned char* ctl_end = reinterpret_cast<const unsigned char*>(const_cast<int*>(ctl) + 4);
    if ((size_t)(ctl_end - tc_smem_raw) > dyn || smem_addr(ctl_end) >= (1u << 18)) {
        if (threadIdx.x == 0) atomicMax(g.status, (int)ST_DEVICE);
        return;
    }

    if (threadIdx.x == 0) {
        // descriptors into the TMA unit's cache while the prologue runs
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
        if constexpr (DUAL == 2)
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB2)) : "memory");
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        ctl[1] = 0;
        ctl[2] = 0;
        ctl[3] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();                                  // tcgen05.alloc is warp-collective
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr((const void*)ctl)),
                     "r"(DUAL * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = (uint32_t)ctl[0];
    // an allocation is lane 0 and a column range inside the 512 columns
    const bool tmem_ok = (tmem >> 16) == 0 && (tmem & 0xFFFFu) + DUAL * BN <= 512;
    if (!tmem_ok) {
        if (threadIdx.x == 0) {
            ctl[1] = 1;
            atomicMax(g.status, (int)ST_DEVICE);
        }
        __syncthreads();
        return;
    }

    if (threadIdx.x == 0) {
        // ---- producer: TMA ring
        int issued = 0;
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % STAGES;
            if (kb >= STAGES &&
                !mbar_wait(&empty[s], (uint32_t)((kb / STAGES) - 1) & 1u, g.timeout_ns)) {
                ctl[1] = 1;
                atomicMax(g.status, (int)ST_TIMEOUT);
                break;
            }
            if (ctl[1]) break;
            const uint32_t st = smem_addr(base + (size_t)s * STAGE);
            mbar_expect_tx(&full[s], STAGE);
            const uint32_t fb = smem_addr(&full[s]);
            const int kx = (kb0 + kb) * BKE;
            tc_tma_2d(st, &tmA, kx, m0, fb);
            tc_tma_3d(st + TC_TILE, &tmB, kx, n0, g.layer, fb);
            if constexpr (DUAL == 2) tc_tma_3d(st + TC_TILE + BTILE, &tmB2, kx, n0, g.layer, fb);
            issued++;
        }
        ctl[2] = issued;
    } else if (threadIdx.x == 32) {
        // ---- MMA issuer
        const uint32_t idesc = tc_idesc<KIND, BN>();
        int consumed = 0;
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % STAGES;
            if (!mbar_wait(&full[s], (uint32_t)(kb / STAGES) & 1u, g.timeout_ns)) {
                ctl[1] = 1;
                atomicMax(g.status, (int)ST_TIMEOUT);
                break;
            }
            consumed++;
            tc_fence_after();
            const uint32_t a_addr = smem_addr(base + (size_t)s * STAGE);
#pragma unroll
            for (int k = 0; k < TC_BKB / 32; k++) {
                const uint64_t ad = tc_sw128_desc(a_addr + 32 * k);
                const uint32_t acc = (kb | k) != 0;
                tc_mma<KIND>(tmem, ad, tc_sw128_desc(a_addr + TC_TILE + 32 * k), idesc, acc);
                if constexpr (DUAL == 2)
                    tc_mma<KIND>(tmem + BN, ad, tc_sw128_desc(a_addr + TC_TILE + BTILE + 32 * k), idesc,
                                 acc);
            }
            tc_commit(smem_addr(&empty[s]));     // the stage is free once these MMAs are done
        }
        ctl[3] = consumed;
        tc_commit(smem_addr(done));              // every MMA issued above has completed
    }
    __syncwarp();
    // ---- epilogue: TMEM -> registers -> global
    const bool finished = mbar_wait(done, 0, g.timeout_ns);
    if (!finished) atomicMax(g.status, (int)ST_TIMEOUT);
    tc_fence_after();
    // block-uniform decision: tcgen05.ld is warp-collective
    const bool store = __syncthreads_and(finished) && ctl[1] == 0 && nk > 0;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    // TMEM -> registers -> the ring, now idle, as a row-major tile (row
    // stride TLD keeps the float4 writes of 8 consecutive rows in distinct
    // banks); then a warp per row applies the epilogue to column pairs, so
    // every global access of a warp covers consecutive addresses
    float* tile = reinterpret_cast<float*>(base);
    float* trow_s = tile + (size_t)(warp * 32 + lane) * TLD;
#pragma unroll 1
    for (int c0 = 0; c0 < DUAL * BN; c0 += 32) {
        if (!store) break;                                 // block-uniform
        float u[32];
        tc_tmem_ld32(trow + c0, u);
        tc_tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(trow_s + c0 + j) = make_float4(u[j], u[j + 1], u[j + 2], u[j + 3]);
    }
    __syncthreads();
    for (int r = warp; r < TC_BM && store; r += TC_THREADS / 32) {
        const int m = m0 + r;
        if (m >= g.M) break;                               // rows ascend: warp-uniform
        if (g.act && !g.act[m]) continue;
        const float* src = tile + (size_t)r * TLD;
#pragma unroll 1
        for (int c = 2 * lane; c < BN; c += 64) {
            if (n0 + c >= g.N) break;
            const float2 uv = *reinterpret_cast<const float2*>(src + c);
            const float u[2] = {uv.x, uv.y};
            float gt[2] = {0.0f, 0.0f};
            if constexpr (DUAL == 2) {
                const float2 gv = *reinterpret_cast<const float2*>(src + BN + c);
                gt[0] = gv.x;
                gt[1] = gv.y;
            }
            tc_epilogue<EPI, 2>(g, m, n0 + c, u, gt, split);
        }
    }
    // ---- drain copies still in flight (only after a failed wait), free TMEM
    if (threadIdx.x == 0)
        for (int kb = ctl[3]; kb < ctl[2]; kb++)
            if (!mbar_wait(&full[kb % STAGES], (uint32_t)(kb / STAGES) & 1u, g.timeout_ns)) break;
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(DUAL * BN));
}

// ---------------------------------------------------------------------------
// Decode GEMM with the operands swapped: C[M][N] = X[M][K] . W[N][K]^T where
// M (sequences, at most a few dozen to a few hundred) is small.  The MMA's
// 128-row operand is a tile of 128 weight rows (output features) and the
// N = BN operand a tile of BN sequences, so no MMA row is spent on padding
// and the tensor pipe reads each weight byte once per BN sequences.  The
// accumulator is feature-major in TMEM (lane = feature, column = sequence);
// the epilogue turns it sequence-major through shared memory and applies
// the same per-row epilogues as the prefill kernel.  With ksplit > 1 (only
// for the partial epilogues) CTA r of a tile accumulates the r-th K slice.
// For a matrix pair (EPI_PART2: up and gate) two weight tiles share the
// sequence tile and accumulate into two TMEM column ranges.
template <int KIND, int EPI, int BN, int STAGES>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_dec_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                  const __grid_constant__ CUtensorMap tmW2, const TcArgs g) {
    constexpr int DUAL = EPI == EPI_PART2 ? 2 : 1;
    constexpr int ES = KIND == TC_TF32 ? 4 : 2;
    constexpr int BKE = TC_BKB / ES;                       // K elements per stage
    constexpr uint32_t XTILE = (uint32_t)BN * TC_BKB;      // bytes of the sequence tile
    // bf16: the activations come as hi and lo tiles (rows s0 and
    // g.x_lo_row + s0 of X), both multiplied into the same accumulator
    constexpr int XS = KIND == TC_BF16 ? 2 : 1;
    constexpr uint32_t STAGE = DUAL * TC_TILE + XS * XTILE;
    constexpr int TLD = DUAL * TC_BM + 4;                  // epilogue tile row stride (floats)
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "N of an M = 128 MMA");
    static_assert(DUAL * BN <= 512 && (DUAL * BN & (DUAL * BN - 1)) == 0 && DUAL * BN >= 32,
                  "TMEM allocation: a power of two from 32 to 512 columns");
    static_assert(STAGE % 1024 == 0, "stages stay 1024-byte aligned for the 128-byte swizzle");
    static_assert((size_t)BN * TLD * 4 <= (size_t)STAGES * STAGE, "epilogue tile fits the ring");
    static_assert((2 * STAGES + 1) * 8 + 16 <= 256, "barriers and control words fit the tail");
    static_assert(1024 + (size_t)STAGES * STAGE + 256 <= 232448, "ring fits 227 KB of shared memory");
    extern __shared__ unsigned char tc_smem_raw[];
    unsigned char* base =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned long long* full = reinterpret_cast<unsigned long long*>(base + STAGES * STAGE);
    unsigned long long* empty = full + STAGES;
    unsigned long long* done = empty + STAGES;
    volatile int* ctl = reinterpret_cast<volatile int*>(done + 1);   // 0 tmem, 1 error, 2 issued, 3 consumed
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = g.ksplit > 1 ? g.ksplit : 1;
    const int split = blockIdx.x % ks;                     // slice of K
    const int tiles_f = (g.N + TC_BM - 1) / TC_BM;
    const int tile = blockIdx.x / ks;
    const int f0 = (tile % tiles_f) * TC_BM;               // first feature (weight row)
    const int s0 = (tile / tiles_f) * BN;                  // first sequence
    const int nk_all = (g.K + BKE - 1) / BKE;
    const int kb0 = (int)((long long)split * nk_all / ks);
    const int nk = (int)((long long)(split + 1) * nk_all / ks) - kb0;

    uint32_t dyn = 0;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
    const unsigned char* ctl_end = reinterpret_cast<const unsigned char*>(const_cast<int*>(ctl) + 4);
    if ((size_t)(ctl_end - tc_smem_raw) > dyn || smem_addr(ctl_end) >= (1u << 18)) {
        if (threadIdx.x == 0) atomicMax(g.status, (int)ST_DEVICE);
        return;
    }
    if (threadIdx.x == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
        if constexpr (DUAL == 2)
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW2)) : "memory");
        for (int st = 0; st < STAGES; st++) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], 1);
        }
        mbar_init(done, 1);
        ctl[1] = 0;
        ctl[2] = 0;
        ctl[3] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr((const void*)ctl)),
                     "r"(DUAL * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = (uint32_t)ctl[0];
    const bool tmem_ok = (tmem >> 16) == 0 && (tmem & 0xFFFFu) + DUAL * BN <= 512;
    if (!tmem_ok) {
        if (threadIdx.x == 0) {
            ctl[1] = 1;
            atomicMax(g.status, (int)ST_DEVICE);
        }
        __syncthreads();
        return;
    }

    // weights are constant: the first ring's worth of weight tiles is
    // requested before waiting for the kernel that produces X
    const int pre = min(nk, STAGES);
    if (threadIdx.x == 0)
        for (int kb = 0; kb < pre; kb++) {
            const uint32_t sa = smem_addr(base + (size_t)kb * STAGE);
            mbar_expect_tx(&full[kb], STAGE);
            const int kx = (kb0 + kb) * BKE;
            tc_tma_3d(sa, &tmW, kx, f0, g.layer, smem_addr(&full[kb]));
            if constexpr (DUAL == 2) tc_tma_3d(sa + TC_TILE, &tmW2, kx, f0, g.layer, smem_addr(&full[kb]));
        }
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) {
        // ---- producer: weight tile(s) and the sequence tile of each K block
        int issued = 0;
        for (int kb = 0; kb < nk; kb++) {
            const int st = kb % STAGES;
            if (kb >= STAGES &&
                !mbar_wait(&empty[st], (uint32_t)((kb / STAGES) - 1) & 1u, g.timeout_ns)) {
                ctl[1] = 1;
                atomicMax(g.status, (int)ST_TIMEOUT);
                break;
            }
            if (kb >= pre && ctl[1]) break;      // pre-issued stages always get their X tile
            const uint32_t sa = smem_addr(base + (size_t)st * STAGE);
            const uint32_t fb = smem_addr(&full[st]);
            const int kx = (kb0 + kb) * BKE;
            if (kb >= pre) {
                mbar_expect_tx(&full[st], STAGE);
                tc_tma_3d(sa, &tmW, kx, f0, g.layer, fb);
                if constexpr (DUAL == 2) tc_tma_3d(sa + TC_TILE, &tmW2, kx, f0, g.layer, fb);
            }
            tc_tma_2d(sa + DUAL * TC_TILE, &tmX, kx, s0, fb);
            if constexpr (XS == 2) tc_tma_2d(sa + DUAL * TC_TILE + XTILE, &tmX, kx, g.x_lo_row + s0, fb);
            issued++;
        }
        ctl[2] = issued;
    } else if (threadIdx.x == 32) {
        // ---- MMA issuer: D[feature][sequence] += W . X^T
        const uint32_t idesc = tc_idesc<KIND, BN>();
        int consumed = 0;
        for (int kb = 0; kb < nk; kb++) {
            const int st = kb % STAGES;
            if (!mbar_wait(&full[st], (uint32_t)(kb / STAGES) & 1u, g.timeout_ns)) {
                ctl[1] = 1;
                atomicMax(g.status, (int)ST_TIMEOUT);
                break;
            }
            consumed++;
            tc_fence_after();
            const uint32_t sa = smem_addr(base + (size_t)st * STAGE);
#pragma unroll
            for (int k = 0; k < TC_BKB / 32; k++) {
#pragma unroll
                for (int x = 0; x < XS; x++) {
                    const uint64_t xd = tc_sw128_desc(sa + DUAL * TC_TILE + x * XTILE + 32 * k);
                    const uint32_t acc = (kb | k | x) != 0;
                    tc_mma<KIND>(tmem, tc_sw128_desc(sa + 32 * k), xd, idesc, acc);
                    if constexpr (DUAL == 2)
                        tc_mma<KIND>(tmem + BN, tc_sw128_desc(sa + TC_TILE + 32 * k), xd, idesc, acc);
                }
            }
            tc_commit(smem_addr(&empty[st]));
        }
        ctl[3] = consumed;
        tc_commit(smem_addr(done));
    }
    __syncwarp();
    const bool finished = mbar_wait(done, 0, g.timeout_ns);
    if (!finished) atomicMax(g.status, (int)ST_TIMEOUT);
    tc_fence_after();
    const bool store = __syncthreads_and(finished) && ctl[1] == 0 && nk > 0;
    // TMEM (lane = feature, column = sequence) -> a sequence-major tile in
    // the idle ring: a warp's 32 lanes write 32 consecutive features of one
    // sequence per store, so neither side has bank conflicts
    const uint32_t tlane = tmem + ((uint32_t)(warp * 32) << 16);
    float* tilep = reinterpret_cast<float*>(base);
    const int fl = warp * 32 + lane;
#pragma unroll 1
    for (int c0 = 0; c0 < DUAL * BN; c0 += 32) {
        if (!store) break;                                 // block-uniform
        float v[32];
        tc_tmem_ld32(tlane + c0, v);
        tc_tmem_wait_ld();
        const int part = c0 / BN, sq = c0 - part * BN;     // which matrix, first sequence
#pragma unroll
        for (int j = 0; j < 32; j++) tilep[(size_t)(sq + j) * TLD + part * TC_BM + fl] = v[j];
    }
    __syncthreads();
    bool row_epilogue = true;
    if constexpr (EPI == TCE_STORE) {
        if (g.head) {
            // lm_head: a thread per (sequence, 32-id chunk) of the tile
            // (float4 reads of its row, conflict-free for 8 consecutive
            // sequences), then the chunks' greedy partials are combined per
            // sequence; better() is a total order, so the result does not
            // depend on how the ids are grouped
            row_epilogue = false;
            constexpr int NQ = TC_BM / 32;
            static_assert((size_t)BN * TLD * 4 + (size_t)NQ * BN * 8 <= (size_t)STAGES * STAGE,
                          "tile and chunk partials fit the ring");
            float* bestv = tilep + (size_t)BN * TLD;
            int* besti = reinterpret_cast<int*>(bestv + NQ * BN);
            const bool greedy = g.sa.top_k == 1;
            const int nwords = (g.N + 31) >> 5;
            for (int it = threadIdx.x; it < NQ * BN; it += TC_THREADS) {
                const int r = it % BN, q = it / BN;
                const int m = s0 + r;
                const int n0 = f0 + 32 * q;
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                if (store && m < g.M && (!g.act || g.act[m]) && n0 < g.N) {
                    const float* src = tilep + (size_t)r * TLD + 32 * q;
                    float* crow = g.C + (size_t)m * g.ldc;
                    const unsigned bw = greedy && g.sa.ngram > 0 ? __ldg(g.banned + (size_t)m * nwords + (n0 >> 5)) : 0u;
#pragma unroll
                    for (int j4 = 0; j4 < 32; j4 += 4) {
                        const float4 v4 = *reinterpret_cast<const float4*>(src + j4);
                        float x[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            if (n0 + j4 + j < 4) x[j] = -INFINITY;   // generate.c:580-581
                        if (n0 + j4 + 3 < g.N && (g.ldc & 3) == 0) {
                            *reinterpret_cast<float4*>(crow + n0 + j4) = make_float4(x[0], x[1], x[2], x[3]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 4; j++)
                                if (n0 + j4 + j < g.N) crow[n0 + j4 + j] = x[j];
                        }
                        if (greedy) {
#pragma unroll
                            for (int j = 0; j < 4; j++) {
                                const int n = n0 + j4 + j;
                                if (n >= g.N) break;
                                const unsigned cnt = g.sa.pen_active ? __ldg(g.counts + (size_t)m * g.N + n) : 0u;
                                const bool ban = (bw >> (n & 31)) & 1u;
                                const float tv = transform_value(x[j], cnt, ban, g.sa);
                                if (better(tv, n, bv, bi)) {
                                    bv = tv;
                                    bi = n;
                                }
                            }
                        }
                    }
                }
                bestv[q * BN + r] = bv;
                besti[q * BN + r] = bi;
            }
            __syncthreads();
            if (greedy && store)
                for (int r = threadIdx.x; r < BN; r += TC_THREADS) {
                    const int m = s0 + r;
                    if (m >= g.M || (g.act && !g.act[m])) continue;
                    float bv = bestv[r];
                    int bi = besti[r];
                    for (int q = 1; q < NQ; q++)
                        if (better(bestv[q * BN + r], besti[q * BN + r], bv, bi)) {
                            bv = bestv[q * BN + r];
                            bi = besti[q * BN + r];
                        }
                    g.amax_v[(size_t)m * tiles_f + f0 / TC_BM] = bv;
                    g.amax_i[(size_t)m * tiles_f + f0 / TC_BM] = bi;
                }
        }
    }
    // a warp per sequence, lanes over feature pairs
    for (int r = warp; r < BN && store && row_epilogue; r += TC_THREADS / 32) {
        const int m = s0 + r;
        if (m >= g.M) break;                               // sequences ascend: warp-uniform
        if (g.act && !g.act[m]) continue;
        const float* src = tilep + (size_t)r * TLD;
#pragma unroll
        for (int c = 2 * lane; c < TC_BM; c += 64) {
            if (f0 + c >= g.N) break;
            const float2 uv = *reinterpret_cast<const float2*>(src + c);
            const float u[2] = {uv.x, uv.y};
            float gt[2] = {0.0f, 0.0f};
            if constexpr (DUAL == 2) {
                const float2 gv = *reinterpret_cast<const float2*>(src + TC_BM + c);
                gt[0] = gv.x;
                gt[1] = gv.y;
            }
            tc_epilogue<EPI, 2>(g, m, f0 + c, u, gt, split);
        }
    }
    if (threadIdx.x == 0)
        for (int kb = ctl[3]; kb < ctl[2]; kb++)
            if (!mbar_wait(&full[kb % STAGES], (uint32_t)(kb / STAGES) & 1u, g.timeout_ns)) break;
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(DUAL * BN));
}

}  // namespace mc

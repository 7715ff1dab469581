// minima_cuda.cu — C ABI (include/minima_cuda.h) over the sm_100a decode
// token loop: weight upload, device KV cache / work buffers, and the single
// cooperative launch that runs a whole generate_with_options batch.
#include "minima_cuda.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <type_traits>
#include <vector>

#include "mc_token_loop.cuh"
#include "mc_cluster_loop2.cuh"
#include "mc_prefill.cuh"
#include "mc_checkpoint.cuh"
#include "mc_tcgen05.cuh"
#include "mc_batched.cuh"
#include "mc_stats.cuh"
#include "mc_matmul.cuh"

#include <cudaTypedefs.h>

namespace {

thread_local char g_err[512] = "";

mc_status fail(mc_status st, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return st;
}

#define MC_CUDA(call)                                                                  \
    do {                                                                               \
        cudaError_t e_ = (call);                                                       \
        if (e_ != cudaSuccess)                                                         \
            return fail(e_ == cudaErrorMemoryAllocation ? MC_ERR_NOMEM : MC_ERR_CUDA,   \
                        "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_),        \
                        __FILE__, __LINE__);                                           \
    } while (0)

int kv_head_count(int n_heads) {  // model.c:34-40
    if (n_heads <= 1) return 1;
    for (int kv = n_heads / 2; kv >= 1; kv--)
        if (n_heads % kv == 0) return kv;
    return 1;
}

uint16_t bf16_rne(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    if ((u & 0x7F800000u) == 0x7F800000u) return (uint16_t)(u >> 16);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace

struct mc_model {
    int device;
    int V, D, L, H, K, hd, kvd, Q, F, max_seq;
    int dtype;
    void* wblock;              // all weight matrices
    float* norms;              // rms1 [L*D], rms2 [L*D], rms_final [D]
    float2* rope;              // [max_seq][hd/2]
    size_t off[6];             // byte offsets of the six matrices in wblock
    size_t weight_bytes;
    unsigned version;          // bumped whenever the weights are (re)written
};

struct mc_session {
    mc_model* m;
    int Bcap, cap;
    cudaStream_t stream;
    cudaEvent_t ev0, ev1;
    int grid;
    size_t smem;
    int bc, xs_ld, max_split;
    // device buffers
    float *kc, *vc, *x, *q, *att, *f, *logits, *part_o, *part_m, *part_l, *amax_v;
    // paged KV cache (mc::KvPages): pools kc / vc of kv_pages pages of
    // 2^kv_shift positions, table [Bcap][kv_pps] on the device and its host
    // copy; a paged session (kv_paged) hands out pages per call from
    // kv_order, other sessions keep the identity table
    int* kv_table;
    int kv_pps, kv_shift, kv_pages;
    bool kv_paged;
    std::vector<int> kv_host, kv_order;
    int* amax_i;
    unsigned *att_cnt, *counts, *banned;
    unsigned* bar;
    int* status;
    mc::SeqState* seq;
    uint16_t* prompts;         // [Bcap][cap] staging for host prompts
    uint16_t* out;             // [Bcap][cap] staging for host outputs
    uint16_t* stop;            // [MC_MAX_STOP]
    float* trace;
    size_t trace_bytes;
    unsigned long long* stamps;   // [cap + 1]
    int last_T;
    float last_ms;
    int last_launches;
    // cluster-resident loop (greedy fp32 decode of small models)
    bool cl_ok;                   // plan fits this device
    int cl_cs, cl_nc;             // CTAs per cluster, clusters
    size_t cl_smem;
    mc::ClusterParams cl_plan;    // shared-memory offsets and geometry
    float *cl_proj_h, *cl_down_s; // two-phase loop: column blocks of attn_proj / ffn_down
    unsigned cl2_version;         // model version those blocks were made from
    float* xfin;
    int* hgen;
    unsigned* hsync;              // [0] go, [32] hdone (separate lines)
    unsigned long long* hkey;     // [2][Bcap][2] head CTAs' greedy maxima (by head-phase parity)
    int last_path;                // 0 grid loop, 1 cluster loop
    // batched prefill work buffers (allocated on first use)
    float *pf_x, *pf_xn, *pf_q, *pf_att, *pf_f;
    size_t pf_rows;               // rows the buffers hold
    bool pf_tc;                   // prefill GEMMs on tcgen05 (tf32 / bf16), MINIMA_CUDA_PREFILL=tcgen05
    bool pf_maps_ok;              // tensor maps below match the current buffers
    CUtensorMap pf_map[3];        // A operands of the prefill GEMMs: xn, att, f
    bool w_maps_ok;
    CUtensorMap w_map[6];         // B operands: qkv, proj, up, gate, down, tok_emb
    // batched decode on tcgen05 (mc_batched.cuh), MINIMA_CUDA_DECODE=tcgen05
    bool bd_tc;
    int* bd_lists;
    float* bd_xn;                 // [Bcap][D]
    __nv_bfloat16 *bd_xn16, *bd_att16, *bd_f16;
    bool bd_maps_ok;
    CUtensorMap bd_map[3];        // A operands: xn, att, f ([Bcap] rows)
    CUtensorMap bd_wmap[6];       // weights as 128-row boxes (the MMA's M side in decode)
    CUtensorMap bd_xmap[3];       // xn, att, f as 64-row boxes (the MMA's N side in decode)
    float* bd_part;               // K-slice partials of the decode GEMMs
    size_t bd_part_floats;
    float* pf_logits;             // [Bcap x kPrefillChunk][V] lm_head scratch of mc_model_forward
    float* pf_part;               // K-slice partial tiles of the CUDA-core prefill GEMMs
    size_t pf_part_floats;
    unsigned* pf_cnt;             // per-tile arrival counters of those GEMMs (kept at zero)
    __nv_bfloat16 *pf_xn16, *pf_att16, *pf_f16;   // bf16 GEMM inputs (tensor cores, bf16 weights)
    cudaEvent_t ev_mid;           // end of prefill
    mc_token_stats* stats;   // result of mc_next_token_stats (allocated on first use)
    float *pf_cap_qkv, *pf_cap_up, *pf_cap_gate;   // model_forward cache staging (on first use)
    size_t pf_cap_rows;
    int last_prefill_pos;         // positions prefilled by the last call
    float last_prefill_ms;
};

namespace {

template <typename WT, bool VEC>
cudaError_t prepare_kernel(size_t smem) {
    return cudaFuncSetAttribute(mc::token_loop_kernel<WT, VEC>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

template <typename WT, bool VEC>
cudaError_t launch_loop(const mc::LoopParams<WT>& p, int grid, size_t smem, cudaStream_t st) {
    void* args[] = {const_cast<mc::LoopParams<WT>*>(&p)};
    return cudaLaunchCooperativeKernel((const void*)mc::token_loop_kernel<WT, VEC>, dim3(grid),
                                       dim3(mc::kThreads), args, smem, st);
}

bool vec_ok(const mc_model* m) {
    const int n = m->dtype == MC_WEIGHTS_BF16 ? 8 : 4;
    return m->D % n == 0 && m->F % n == 0;
}

// Every device-side wait gives up after this deadline (default 1 s) and
// reports MC_ERR_TIMEOUT.  MINIMA_CUDA_WAIT_NS shortens it and
// MINIMA_CUDA_TEST_STALL=1 makes each wait expect one arrival that never
// comes: test hooks for the failure path, off unless set.
template <typename WT>
void wait_hooks(mc::LoopParams<WT>& p) {
    const char* wait_ns = getenv("MINIMA_CUDA_WAIT_NS");
    p.timeout_ns = wait_ns ? strtoull(wait_ns, nullptr, 10) : 1000ull * 1000ull * 1000ull;
    const char* stall = getenv("MINIMA_CUDA_TEST_STALL");
    p.extra_arrivals = (stall && stall[0] == '1') ? 1u : 0u;
}

template <typename WT>
void fill_params(mc::LoopParams<WT>& p, const mc_session* s) {
    const mc_model* m = s->m;
    const char* wb = static_cast<const char*>(m->wblock);
    p.V = m->V; p.D = m->D; p.L = m->L; p.H = m->H; p.K = m->K; p.hd = m->hd;
    p.kvd = m->kvd; p.Q = m->Q; p.F = m->F; p.G = m->H / m->K;
    p.tok_emb = reinterpret_cast<const WT*>(wb + m->off[0]);
    p.w_qkv = reinterpret_cast<const WT*>(wb + m->off[1]);
    p.w_proj = reinterpret_cast<const WT*>(wb + m->off[2]);
    p.w_up = reinterpret_cast<const WT*>(wb + m->off[3]);
    p.w_gate = reinterpret_cast<const WT*>(wb + m->off[4]);
    p.w_down = reinterpret_cast<const WT*>(wb + m->off[5]);
    p.rms1 = m->norms;
    p.rms2 = m->norms + (size_t)m->L * m->D;
    p.rmsf = m->norms + 2 * (size_t)m->L * m->D;
    p.rope = m->rope;
    p.rope_len = m->max_seq;
    p.kc = s->kc; p.vc = s->vc; p.cap = s->cap; p.Bcap = s->Bcap;
    p.pg = mc::KvPages{s->kv_table, s->kv_pps, s->kv_shift};
    p.x = s->x; p.q = s->q; p.att = s->att; p.f = s->f; p.logits = s->logits;
    p.part_o = s->part_o; p.part_m = s->part_m; p.part_l = s->part_l;
    p.att_cnt = s->att_cnt; p.amax_v = s->amax_v; p.amax_i = s->amax_i;
    p.counts = s->counts; p.banned = s->banned; p.max_split = s->max_split;
    p.seq = s->seq;
    p.bar = s->bar; p.status = s->status;
    wait_hooks(p);
    p.bc = s->bc; p.xs_ld = s->xs_ld;
}

// The cluster loop's instantiation for a plan's layer loop (ClusterParams::v2).
using ClusterKernel = void (*)(const mc::ClusterParams);
ClusterKernel cluster_kernel(int v2) {
    return v2 == 2 ? mc::cluster_loop_kernel<2> : v2 == 1 ? mc::cluster_loop_kernel<1> : mc::cluster_loop_kernel<0>;
}

cudaError_t launch_cluster(const mc::ClusterParams& cp, int cs, int nc, size_t smem,
                           cudaStream_t st, bool cooperative) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nc * cs);
    cfg.blockDim = dim3(mc::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cooperative ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, cluster_kernel(cp.v2), cp);
}

// Plan of the cluster-resident loop (mc_cluster_loop.cuh, and its
// two-phase layer loop in mc_cluster_loop2.cuh) for this model on this
// device: shared-memory offsets, cluster size and count such that every
// cluster is co-resident.  The two-phase loop is chosen when every
// (sequence, KV head) pair of the session's batch gets a CTA of the layer
// cluster and its buffers fit, with its dataflow exchange when the two
// buffers of ffn_down partials fit too (MINIMA_CUDA_LOOP=cluster2 keeps
// the cluster barriers, cluster1 the five-phase loop).  Returns false when
// none applies; the grid-barrier loop then serves every call.
bool plan_cluster(mc_session* s, const cudaDeviceProp& prop) {
    const mc_model* m = s->m;
    if (m->dtype != MC_WEIGHTS_F32) return false;
    const int G = m->H / m->K;
    // attention units hold G heads x hd/32 outputs per lane in registers
    if (m->hd % 4 || m->D % 4 || m->F % 4 || m->Q % 2 || G > mc::kAttMaxG ||
        m->hd > 32 * mc::kAttMaxND)
        return false;
    const char* env = getenv("MINIMA_CUDA_LOOP");
    if (env && strcmp(env, "grid") == 0) return false;
    const int max_v2 = env && strcmp(env, "cluster1") == 0 ? 0 : env && strcmp(env, "cluster2") == 0 ? 1 : 2;
    const size_t optin = prop.sharedMemPerBlockOptin;
    for (int v = 0; v <= 2; v++)
        if (cudaFuncSetAttribute(cluster_kernel(v), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)optin) !=
                cudaSuccess ||
            cudaFuncSetAttribute(cluster_kernel(v), cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
                cudaSuccess) {
            cudaGetLastError();
            return false;
        }
    const int B8 = std::min(s->Bcap, mc::kBCMax);    // activation rows held per CTA
    const int hd = m->hd, ghd = G * hd, D = m->D, F = m->F;
    for (int v2 = max_v2; v2 >= 0; v2--) {
        for (int cs : {16, 8}) {
            if (v2 && B8 * m->K > cs) continue;
            mc::ClusterParams cp{};
            cp.cs = cs;
            cp.v2 = v2;
            size_t off = mc::kLcHeader;
            auto take = [&](size_t floats, size_t align) {
                off = align_up(off, align);
                const size_t o = off;
                off += floats * 4;
                return (unsigned)o;
            };
            size_t stage_f = 0, wb_f = 0, sc_f = 0, union_min = 0;
            if (v2) {
                const mc::CSlice s0 = mc::cluster_slice(0, cs, m->Q, D, F);
                cp.fpc = s0.f1 - s0.f0;
                cp.dp_b = B8;
                stage_f = (size_t)(ghd + 2 * hd) * D + (size_t)D * ghd + D;
                wb_f = 2 * (size_t)cp.fpc * D + (size_t)D * cp.fpc + D;
                if (stage_f * 4 >= (1u << 20) || wb_f * 4 >= (1u << 20)) continue;   // mbarrier tx-count limit
                cp.off_x = take((size_t)B8 * D, 16);
                cp.off_xn = take((size_t)B8 * D, 16);
                cp.off_qkv = take((size_t)ghd + 2 * hd, 16);
                cp.off_att = take((size_t)ghd, 16);
                cp.off_attp = take((size_t)B8 * m->K * D, 16);
                cp.off_f = take((size_t)B8 * cp.fpc, 16);
                cp.off_rope = take((size_t)std::max(hd, 2), 16);
                cp.off_pages = take((size_t)B8 * s->kv_pps, 16);
                cp.off_pair = take((size_t)((ghd + 2 * G + 3) & ~3), 16);
                sc_f = (size_t)mc::kWarps * (ghd + 2 * G + 32 * mc::kAttMaxG);
                cp.off_sc = take(sc_f, 16);
                cp.off_stage = take(stage_f, 128);
                cp.off_wb = take(wb_f, 128);
                // ffn_down partials (two buffers for the dataflow exchange,
                // whose per-phase byte count must stay well inside the
                // mbarrier's tx-count range)
                union_min = (size_t)(v2 == 2 ? 2 : 1) * cs * B8 * D;
                if (v2 == 2 && (size_t)(cs - 1) * B8 * D * 4 * 2 >= (1u << 20)) continue;
            } else {
                const mc::CSlice s0 = mc::cluster_slice(0, cs, m->Q, D, F);
                // weight slice plus this layer's rms1 / rms2 scales
                stage_f = align_up(mc::slice_floats(s0, D, F) + 2 * (size_t)D, 32);
                if (stage_f * 4 >= (1u << 20)) continue;           // mbarrier tx-count limit
                cp.off_x = take((size_t)B8 * D, 16);
                cp.off_xn = take((size_t)B8 * D, 16);
                cp.off_qkv = take((size_t)B8 * m->Q, 16);
                cp.off_att = take((size_t)B8 * D, 16);
                // merged states of split attention units: at most max(cs, B K) units
                cp.off_attp = take((size_t)std::max(cs, B8 * m->K) * ((ghd + 2 * G + 3) & ~3), 16);
                cp.off_f = take((size_t)B8 * F, 16);
                cp.off_rope = take((size_t)std::max(hd, 2), 16);
                cp.off_pages = take((size_t)B8 * s->kv_pps, 16);
                sc_f = (size_t)mc::kWarps * (ghd + 2 * G + 32 * mc::kAttMaxG);
            }
            const size_t fixed = off;
            // the K/V tile (v2: sharing its bytes with the ffn_down partials),
            // then, for the five-phase loop, the weight stages
            int tile = mc::kAttMaxTile;
            for (; tile >= 32; tile /= 2) {
                size_t o2 = align_up(fixed, 16);
                if (!v2) o2 += sc_f * 4;
                o2 = align_up(o2, 16) + std::max(2 * (size_t)tile * hd, union_min) * 4;
                if (!v2) o2 = align_up(o2, 128) + mc::kStages * stage_f * 4;
                if (o2 <= optin) break;
            }
            if (tile < 32) continue;
            cp.kv_tile = tile;
            if (!v2) cp.off_sc = take(sc_f, 16);
            cp.off_kv = take(std::max(2 * (size_t)tile * hd, union_min), 16);
            if (!v2) cp.off_stage = take(mc::kStages * stage_f, 128);
            cp.stage_floats = (unsigned)stage_f;
            const size_t lc_bytes = off;
            for (int nc = prop.multiProcessorCount / cs; nc >= 2; nc--) {
                const int nhc = (nc - 1) * cs;
                const int rows = (m->V + nhc - 1) / nhc;
                const size_t ld = (size_t)D + 4;
                if ((size_t)rows * D * 4 >= (1u << 20)) break;
                const size_t hc_x = align_up(mc::kHcEmbOffset + (size_t)rows * ld * 4, 16);
                const size_t hc_bytes = hc_x + (size_t)B8 * D * 4;
                const size_t smem = align_up(std::max(lc_bytes, hc_bytes), 128);
                if (smem > optin) break;
                cudaLaunchConfig_t cfg = {};
                cfg.gridDim = dim3(nc * cs);
                cfg.blockDim = dim3(mc::kThreads);
                cfg.dynamicSmemBytes = smem;
                cudaLaunchAttribute attr[1];
                attr[0].id = cudaLaunchAttributeClusterDimension;
                attr[0].val.clusterDim.x = cs;
                attr[0].val.clusterDim.y = 1;
                attr[0].val.clusterDim.z = 1;
                cfg.attrs = attr;
                cfg.numAttrs = 1;
                int maxc = 0;
                if (cudaOccupancyMaxActiveClusters(&maxc, (void*)cluster_kernel(v2), &cfg) != cudaSuccess) {
                    cudaGetLastError();
                    break;
                }
                if (maxc >= nc) {
                    cp.n_clusters = nc;
                    cp.hc_rows = rows;
                    cp.hc_ld = (unsigned)ld;
                    cp.off_hc_x = (unsigned)hc_x;
                    s->cl_cs = cs;
                    s->cl_nc = nc;
                    s->cl_smem = smem;
                    s->cl_plan = cp;
                    return true;
                }
            }
        }
    }
    return false;
}

mc_status validate_dims(const mc_model_desc* d) {
    if (!d) return fail(MC_ERR_INVALID, "null model description");
    if (d->vocab_size < 5 || d->vocab_size > MC_MAX_VOCAB || d->dim <= 0 || d->dim > MC_MAX_DIM ||
        d->n_layers <= 0 || d->n_layers > MC_MAX_LAYERS || d->n_heads <= 0 ||
        d->n_heads > MC_MAX_HEADS || d->dim % d->n_heads != 0 || d->dim / d->n_heads < 2 ||
        d->dim / d->n_heads > MC_MAX_HEAD_DIM || d->ffn_dim <= 0 || d->ffn_dim > MC_MAX_FFN ||
        d->max_seq <= 0 || d->max_seq > MC_MAX_SEQ)
        return fail(MC_ERR_INVALID, "model dimensions outside the supported envelope");
    const int K = kv_head_count(d->n_heads), hd = d->dim / d->n_heads;
    if (d->head_dim != hd || d->n_kv_heads != K || d->kv_dim != K * hd ||
        d->qkv_dim != d->dim + 2 * K * hd)
        return fail(MC_ERR_INVALID, "derived model dimensions inconsistent (model.c:55-89)");
    return MC_OK;
}

mc_status validate_desc(const mc_model_desc* d) {
    const mc_status st = validate_dims(d);
    if (st) return st;
    if (!d->tok_emb || !d->attn_qkv || !d->attn_proj || !d->ffn_up || !d->ffn_gate ||
        !d->ffn_down || !d->rms1_scale || !d->rms2_scale || !d->rms_final_scale)
        return fail(MC_ERR_INVALID, "null weight pointer");
    return MC_OK;
}

mc_status upload_weights(mc_model* m, const mc_model_desc* d) {
    const size_t V = m->V, D = m->D, L = m->L, Q = m->Q, F = m->F;
    const size_t counts[6] = {V * D, L * Q * D, L * D * D, L * F * D, L * F * D, L * D * F};
    const float* src[6] = {d->tok_emb, d->attn_qkv, d->attn_proj, d->ffn_up, d->ffn_gate, d->ffn_down};
    const size_t es = m->dtype == MC_WEIGHTS_BF16 ? 2 : 4;
    char* wb = static_cast<char*>(m->wblock);
    std::vector<uint16_t> tmp;
    for (int i = 0; i < 6; i++) {
        if (m->dtype == MC_WEIGHTS_BF16) {
            tmp.resize(counts[i]);
            for (size_t k = 0; k < counts[i]; k++) tmp[k] = bf16_rne(src[i][k]);
            MC_CUDA(cudaMemcpy(wb + m->off[i], tmp.data(), counts[i] * es, cudaMemcpyHostToDevice));
        } else {
            MC_CUDA(cudaMemcpy(wb + m->off[i], src[i], counts[i] * es, cudaMemcpyHostToDevice));
        }
    }
    MC_CUDA(cudaMemcpy(m->norms, d->rms1_scale, L * D * 4, cudaMemcpyHostToDevice));
    MC_CUDA(cudaMemcpy(m->norms + L * D, d->rms2_scale, L * D * 4, cudaMemcpyHostToDevice));
    MC_CUDA(cudaMemcpy(m->norms + 2 * L * D, d->rms_final_scale, D * 4, cudaMemcpyHostToDevice));
    m->version++;
    return MC_OK;
}

}  // namespace

extern "C" {

const char* mc_last_error(void) { return g_err; }

// The drop-in calls mc_init on every generate call, so the device check is
// made once per device and with single attribute queries: a full
// cudaGetDeviceProperties takes about 2.5 ms on B200.
static std::atomic<bool> g_device_checked[64];

mc_status mc_init(int device) {
    int n = 0;
    MC_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return fail(MC_ERR_INVALID, "device %d of %d", device, n);
    MC_CUDA(cudaSetDevice(device));
    const bool cache = device < 64;
    if (cache && g_device_checked[device].load(std::memory_order_acquire)) return MC_OK;
    int major = 0, minor = 0, coop = 0;
    MC_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    MC_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
    MC_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device));
    if (major != 10)
        return fail(MC_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", device,
                    major, minor);
    if (!coop) return fail(MC_ERR_UNSUPPORTED, "no cooperative launch");
    if (cache) g_device_checked[device].store(true, std::memory_order_release);
    return MC_OK;
}

}  // extern "C"

namespace {

// Device buffers and RoPE table of a model with d's dimensions (weights not
// yet written).
mc_status model_alloc(const mc_model_desc* d, int dtype, mc_model** out) {
    if (dtype != MC_WEIGHTS_F32 && dtype != MC_WEIGHTS_BF16)
        return fail(MC_ERR_INVALID, "unknown weight dtype %d", dtype);
    mc_model* m = new mc_model();
    MC_CUDA(cudaGetDevice(&m->device));
    m->V = d->vocab_size; m->D = d->dim; m->L = d->n_layers; m->H = d->n_heads;
    m->K = d->n_kv_heads; m->hd = d->head_dim; m->kvd = d->kv_dim; m->Q = d->qkv_dim;
    m->F = d->ffn_dim; m->max_seq = d->max_seq; m->dtype = dtype;
    const size_t V = m->V, D = m->D, L = m->L, Q = m->Q, F = m->F;
    const size_t counts[6] = {V * D, L * Q * D, L * D * D, L * F * D, L * F * D, L * D * F};
    const size_t es = dtype == MC_WEIGHTS_BF16 ? 2 : 4;
    size_t off = 0;
    for (int i = 0; i < 6; i++) {
        m->off[i] = off;
        off = align_up(off + counts[i] * es, 256);
    }
    m->weight_bytes = off;
    cudaError_t e = cudaMalloc(&m->wblock, off);
    if (e == cudaSuccess) e = cudaMalloc(&m->norms, (2 * L * D + D) * 4);
    const int half = m->hd / 2;
    if (e == cudaSuccess) e = cudaMalloc(&m->rope, (size_t)m->max_seq * std::max(half, 1) * sizeof(float2));
    if (e != cudaSuccess) {
        mc_model_destroy(m);
        return fail(MC_ERR_NOMEM, "weight allocation (%zu bytes): %s", off, cudaGetErrorString(e));
    }
    // RoPE table with the reference's float expression (rotary.h:19-24),
    // evaluated by the host libm exactly as the reference evaluates it.
    if (half > 0) {
        std::vector<float2> rope((size_t)m->max_seq * half);
        for (int pair = 0; pair < half; pair++) {
            const float exponent = (2.0f * (float)pair) / (float)m->hd;
            const float base = ::powf(10000.0f, -exponent);
            for (int pos = 0; pos < m->max_seq; pos++) {
                const float angle = (float)pos * base;
                rope[(size_t)pos * half + pair] = make_float2(::cosf(angle), ::sinf(angle));
            }
        }
        e = cudaMemcpy(m->rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            mc_model_destroy(m);
            return fail(MC_ERR_CUDA, "rope upload: %s", cudaGetErrorString(e));
        }
    }
    *out = m;
    return MC_OK;
}

}  // namespace

extern "C" {

mc_status mc_model_create(const mc_model_desc* d, int dtype, mc_model** out) {
    if (!out) return fail(MC_ERR_INVALID, "null output handle");
    *out = nullptr;
    mc_status st = validate_desc(d);
    if (st) return st;
    mc_model* m = nullptr;
    st = model_alloc(d, dtype, &m);
    if (st) return st;
    st = upload_weights(m, d);
    if (st) {
        mc_model_destroy(m);
        return st;
    }
    *out = m;
    return MC_OK;
}

mc_status mc_model_update(mc_model* m, const mc_model_desc* d) {
    if (!m) return fail(MC_ERR_INVALID, "null model");
    mc_status st = validate_desc(d);
    if (st) return st;
    if (d->vocab_size != m->V || d->dim != m->D || d->n_layers != m->L || d->n_heads != m->H ||
        d->ffn_dim != m->F)
        return fail(MC_ERR_INVALID, "mc_model_update: dimensions differ from the uploaded model");
    return upload_weights(m, d);
}

mc_status mc_model_destroy(mc_model* m) {
    if (!m) return MC_OK;
    cudaFree(m->wblock);
    cudaFree(m->norms);
    cudaFree(m->rope);
    delete m;
    return MC_OK;
}

mc_status mc_session_destroy(mc_session* s) {
    if (!s) return MC_OK;
    void* bufs[] = {s->kv_table, s->kc, s->vc, s->x, s->q, s->att, s->f, s->logits, s->part_o, s->part_m,
                    s->part_l, s->amax_v, s->amax_i, s->att_cnt, s->counts, s->banned, s->bar,
                    s->status, s->seq, s->prompts, s->out, s->stop, s->trace, s->stamps,
                    s->xfin, s->hgen, s->hsync, s->hkey,
                    s->pf_x, s->pf_xn, s->pf_q, s->pf_att, s->pf_f, s->pf_logits,
                    s->pf_xn16, s->pf_att16, s->pf_f16, s->pf_part, s->pf_cnt, s->bd_lists, s->bd_xn,
                    s->bd_xn16, s->bd_att16, s->bd_f16, s->bd_part, s->stats,
                    s->pf_cap_qkv, s->pf_cap_up, s->pf_cap_gate, s->cl_proj_h, s->cl_down_s};
    for (void* b : bufs) cudaFree(b);
    if (s->ev_mid) cudaEventDestroy(s->ev_mid);
    if (s->ev0) cudaEventDestroy(s->ev0);
    if (s->ev1) cudaEventDestroy(s->ev1);
    if (s->stream) cudaStreamDestroy(s->stream);
    delete s;
    return MC_OK;
}

}  // extern "C"

namespace {

// page_len 0: the identity table over max_batch * ceil(max_seq / 64) pages
// of 64 positions (every sequence owns max_seq positions, as kvcache_init
// reserves them); otherwise a pool of n_pages pages of page_len positions
// handed out per call.
mc_status session_create(mc_model* m, int max_batch, int max_seq, int page_len, int n_pages,
                         mc_session** out) {
    if (!out) return fail(MC_ERR_INVALID, "null output handle");
    *out = nullptr;
    if (!m) return fail(MC_ERR_INVALID, "null model");
    if (max_batch <= 0 || max_batch > MC_MAX_BATCH || max_seq <= 0 || max_seq > m->max_seq)
        return fail(MC_ERR_INVALID, "session batch %d / max_seq %d outside [1,%d] / [1,%d]",
                    max_batch, max_seq, MC_MAX_BATCH, m->max_seq);
    const bool paged = page_len != 0;
    if (paged && (page_len < MC_MIN_PAGE_LEN || (page_len & (page_len - 1)) || page_len > MC_MAX_SEQ ||
                  n_pages <= 0))
        return fail(MC_ERR_INVALID, "page_len %d (a power of two >= %d) / n_pages %d", page_len,
                    MC_MIN_PAGE_LEN, n_pages);
    if (!paged) page_len = MC_MIN_PAGE_LEN;
    int shift = 0;
    while ((1 << shift) < page_len) shift++;
    const int pps = (max_seq + page_len - 1) / page_len;
    if (!paged) n_pages = max_batch * pps;
    mc_session* s = new mc_session();
    s->kv_paged = paged;
    s->kv_shift = shift;
    s->kv_pps = pps;
    s->kv_pages = n_pages;
    s->kv_host.assign((size_t)max_batch * pps, 0);
    if (paged) {
        // handed out from the top of the pool down, so that consecutive
        // positions of a sequence never sit in consecutive pages
        for (int i = n_pages - 1; i >= 0; i--) s->kv_order.push_back(i);
    } else {
        for (size_t i = 0; i < s->kv_host.size(); i++) s->kv_host[i] = (int)i;
    }
    {
        const char* pe = getenv("MINIMA_CUDA_PREFILL");
        s->pf_tc = pe && std::strcmp(pe, "tcgen05") == 0;
        const char* de = getenv("MINIMA_CUDA_DECODE");
        s->bd_tc = de && std::strcmp(de, "tcgen05") == 0;
    }
    s->m = m;
    s->Bcap = max_batch;
    s->cap = max_seq;
    cudaDeviceProp prop;
    MC_CUDA(cudaGetDeviceProperties(&prop, m->device));
    s->max_split = (max_seq + mc::kSplitLen - 1) / mc::kSplitLen;

    // Shared-memory plan: fixed lists + one phase region sized for the
    // largest of GEMV chunk, attention split and sampler.
    const int G = m->H / m->K;
    s->xs_ld = (int)align_up((size_t)std::max(m->D, m->F), 4);
    const size_t att_bytes = mc::att_phase_bytes(G, m->hd);
    const size_t samp_bytes = mc::sampler_smem_bytes(m->V);
    const size_t limit = (size_t)prop.sharedMemPerBlockOptin;
    const size_t fixed = mc::loop_fixed_bytes(max_batch);
    const size_t wi_bytes = mc::kWarps * mc::kBCMax * 4;
    size_t phase = std::max(att_bytes, samp_bytes);
    const size_t row_bytes = (size_t)s->xs_ld * 4;
    int bc = mc::kBCMax;
    while (bc > 1 && fixed + std::max(phase, bc * row_bytes + wi_bytes) > limit) bc--;
    s->bc = bc;
    phase = std::max(phase, bc * row_bytes + wi_bytes);
    s->smem = align_up(fixed + phase, 16);
    if (s->smem > limit) {
        delete s;
        return fail(MC_ERR_UNSUPPORTED, "shared memory plan %zu B exceeds %zu B", fixed + phase, limit);
    }
    // The attribute is a per-function limit shared by every session on the
    // device, so it is raised to the device maximum rather than to this plan.
    cudaError_t e;
    if (m->dtype == MC_WEIGHTS_BF16)
        e = vec_ok(m) ? prepare_kernel<__nv_bfloat16, true>(limit)
                      : prepare_kernel<__nv_bfloat16, false>(limit);
    else
        e = vec_ok(m) ? prepare_kernel<float, true>(limit) : prepare_kernel<float, false>(limit);
    if (e != cudaSuccess) {
        delete s;
        return fail(MC_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    }
    int per_sm = 0;
    if (m->dtype == MC_WEIGHTS_BF16)
        e = vec_ok(m) ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                            &per_sm, mc::token_loop_kernel<__nv_bfloat16, true>, mc::kThreads, s->smem)
                      : cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                            &per_sm, mc::token_loop_kernel<__nv_bfloat16, false>, mc::kThreads, s->smem);
    else
        e = vec_ok(m) ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                            &per_sm, mc::token_loop_kernel<float, true>, mc::kThreads, s->smem)
                      : cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                            &per_sm, mc::token_loop_kernel<float, false>, mc::kThreads, s->smem);
    if (e != cudaSuccess || per_sm < 1) {
        delete s;
        return fail(MC_ERR_UNSUPPORTED, "token loop kernel cannot be resident (%s)",
                    cudaGetErrorString(e));
    }
    s->grid = prop.multiProcessorCount;

    const size_t B = max_batch, L = m->L, K = m->K, hd = m->hd, D = m->D, F = m->F, V = m->V;
    const size_t H = m->H, cap = max_seq, ms = s->max_split;
    const size_t page_floats = L * K * ((size_t)1 << shift) * hd;
    struct Alloc { void** p; size_t bytes; } allocs[] = {
        {(void**)&s->kc, (size_t)n_pages * page_floats * 4},
        {(void**)&s->vc, (size_t)n_pages * page_floats * 4},
        {(void**)&s->kv_table, s->kv_host.size() * 4},
        {(void**)&s->x, B * D * 4},
        {(void**)&s->q, B * D * 4},
        {(void**)&s->att, B * D * 4},
        {(void**)&s->f, B * F * 4},
        {(void**)&s->logits, B * V * 4},
        {(void**)&s->part_o, B * H * ms * hd * 4},
        {(void**)&s->part_m, B * H * ms * 4},
        {(void**)&s->part_l, B * H * ms * 4},
        // greedy partials: one per CTA of the grid loop, or per 128-id tile
        // of the batched decode's lm_head
        {(void**)&s->amax_v, B * std::max<size_t>(s->grid, (V + 127) / 128) * 4},
        {(void**)&s->amax_i, B * std::max<size_t>(s->grid, (V + 127) / 128) * 4},
        {(void**)&s->att_cnt, B * K * 4},
        {(void**)&s->counts, B * V * 4},
        {(void**)&s->banned, B * ((V + 31) / 32) * 4},
        {(void**)&s->bar, 256},
        {(void**)&s->status, 256},
        {(void**)&s->seq, B * sizeof(mc::SeqState)},
        {(void**)&s->prompts, B * cap * 2},
        {(void**)&s->out, B * cap * 2},
        {(void**)&s->stop, MC_MAX_STOP * 2},
        {(void**)&s->stamps, (cap + 2) * 8},
    };
    for (auto& a : allocs) {
        e = cudaMalloc(a.p, a.bytes);
        if (e != cudaSuccess) {
            mc_session_destroy(s);
            return fail(MC_ERR_NOMEM, "session allocation of %zu bytes: %s", a.bytes,
                        cudaGetErrorString(e));
        }
    }
    s->cl_ok = plan_cluster(s, prop);
    if (s->cl_ok) {
        const mc::ClusterParams& cpl = s->cl_plan;
        const size_t G = m->H / m->K;
        struct Alloc cl_allocs[] = {
            {(void**)&s->cl_proj_h, cpl.v2 ? L * K * D * G * hd * 4 : 0},
            {(void**)&s->cl_down_s, cpl.v2 ? L * (size_t)s->cl_cs * D * cpl.fpc * 4 : 0},
            {(void**)&s->xfin, B * D * 4},
            {(void**)&s->hgen, B * 4},
            {(void**)&s->hsync, 64 * 4},
            {(void**)&s->hkey, 2 * B * 2 * 8},
        };
        s->cl2_version = ~0u;
        for (auto& a : cl_allocs) {
            if (!a.bytes) continue;
            e = cudaMalloc(a.p, a.bytes);
            if (e != cudaSuccess) {
                mc_session_destroy(s);
                return fail(MC_ERR_NOMEM, "session allocation of %zu bytes: %s", a.bytes,
                            cudaGetErrorString(e));
            }
        }
    }
    e = cudaMemset(s->att_cnt, 0, B * K * 4);
    if (e == cudaSuccess)
        e = cudaMemcpy(s->kv_table, s->kv_host.data(), s->kv_host.size() * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreate(&s->ev0);
    if (e == cudaSuccess) e = cudaEventCreate(&s->ev_mid);
    if (e == cudaSuccess) e = cudaEventCreate(&s->ev1);
    if (e != cudaSuccess) {
        mc_session_destroy(s);
        return fail(MC_ERR_CUDA, "session setup: %s", cudaGetErrorString(e));
    }
    *out = s;
    return MC_OK;
}

}  // namespace

extern "C" {

mc_status mc_session_create(mc_model* m, int max_batch, int max_seq, mc_session** out) {
    return session_create(m, max_batch, max_seq, 0, 0, out);
}

mc_status mc_session_create_paged(mc_model* m, int max_batch, int max_seq, int page_len, int n_pages,
                                  mc_session** out) {
    if (page_len == 0) return fail(MC_ERR_INVALID, "page_len 0");
    return session_create(m, max_batch, max_seq, page_len, n_pages, out);
}

}  // extern "C"

namespace {

// Pages for positions [0, positions[b]) of sequences b < batch of a paged
// session, from the pool in kv_order (a call starts every sequence at
// position 0, so the whole pool is free at each call).  Unassigned table
// entries repeat the sequence's last page.  Identity sessions: nothing to do.
mc_status assign_pages(mc_session* s, int batch, const int* positions) {
    if (!s->kv_paged) return MC_OK;
    const int plen = 1 << s->kv_shift;
    size_t next = 0;
    for (int b = 0; b < batch; b++) {
        const int need = std::max(1, (positions[b] + plen - 1) / plen);
        if (need > s->kv_pps || next + need > s->kv_order.size())
            return fail(MC_ERR_NOMEM, "paged KV cache: %d sequences need more than the pool's %d pages of %d "
                        "positions", batch, s->kv_pages, plen);
        int* row = s->kv_host.data() + (size_t)b * s->kv_pps;
        for (int i = 0; i < s->kv_pps; i++) row[i] = s->kv_order[next + std::min(i, need - 1)];
        next += need;
    }
    MC_CUDA(cudaMemcpyAsync(s->kv_table, s->kv_host.data(), (size_t)batch * s->kv_pps * 4,
                            cudaMemcpyHostToDevice, s->stream));
    // the host copy is reused by the next call: wait until this one is read
    MC_CUDA(cudaStreamSynchronize(s->stream));
    return MC_OK;
}

mc_status ensure_trace(mc_session* s, size_t bytes) {
    if (bytes <= s->trace_bytes) return MC_OK;
    if (s->trace) cudaFree(s->trace);
    s->trace = nullptr;
    s->trace_bytes = 0;
    MC_CUDA(cudaMalloc(&s->trace, bytes));
    s->trace_bytes = bytes;
    return MC_OK;
}

// Launch the token loop with the per-call fields already in p.
template <typename WT>
mc_status run_loop(mc_session* s, mc::LoopParams<WT>& p) {
    fill_params(p, s);
    p.stamps = s->stamps;
    s->last_T = p.T;
    MC_CUDA(cudaMemsetAsync(s->stamps, 0, ((size_t)p.T + 1) * 8, s->stream));
    MC_CUDA(cudaMemsetAsync(s->bar, 0, 256, s->stream));
    MC_CUDA(cudaMemsetAsync(s->status, 0, 256, s->stream));
    MC_CUDA(cudaMemsetAsync(s->att_cnt, 0, (size_t)s->Bcap * s->m->K * 4, s->stream));
    cudaError_t e = vec_ok(s->m) ? launch_loop<WT, true>(p, s->grid, s->smem, s->stream)
                                 : launch_loop<WT, false>(p, s->grid, s->smem, s->stream);
    if (e != cudaSuccess) return fail(MC_ERR_CUDA, "token loop launch: %s", cudaGetErrorString(e));
    MC_CUDA(cudaEventRecord(s->ev1, s->stream));
    s->last_launches = 1;
    s->last_path = 0;
    int status = 0;
    MC_CUDA(cudaMemcpyAsync(&status, s->status, 4, cudaMemcpyDeviceToHost, s->stream));
    MC_CUDA(cudaStreamSynchronize(s->stream));
    MC_CUDA(cudaEventElapsedTime(&s->last_ms, s->ev0, s->ev1));
    if (status == mc::ST_TIMEOUT)
        return fail(MC_ERR_TIMEOUT, "token loop: a grid barrier passed its deadline");
    if (status != 0) return fail(MC_ERR_DEVICE, "token loop reported status %d", status);
    return MC_OK;
}

// Launch the cluster-resident loop (greedy, fp32, batch <= kBCMax).
mc_status run_cluster(mc_session* s, mc::LoopParams<float>& p) {
    fill_params(p, s);
    p.stamps = s->stamps;
    s->last_T = p.T;
    mc::ClusterParams cp = s->cl_plan;
    cp.lp = p;
    cp.xfin = s->xfin;
    cp.hgen = s->hgen;
    cp.go = s->hsync;
    cp.hdone = s->hsync + 32;
    cp.hkey = s->hkey;
    cp.proj_h = s->cl_proj_h;
    cp.down_s = s->cl_down_s;
    int relayouts = 0;
    if (cp.v2 && s->cl2_version != s->m->version) {
        // the column blocks of attn_proj / ffn_down, from the current weights
        const mc_model* m = s->m;
        const char* wb = static_cast<const char*>(m->wblock);
        mc::cl2_relayout_kernel<<<4 * 148, 256, 0, s->stream>>>(
            reinterpret_cast<const float*>(wb + m->off[2]), reinterpret_cast<const float*>(wb + m->off[5]),
            s->cl_proj_h, s->cl_down_s, m->L, m->D, m->F, m->K, (m->H / m->K) * m->hd, s->cl_cs, cp.fpc);
        MC_CUDA(cudaGetLastError());
        s->cl2_version = m->version;
        relayouts = 1;
    }
    MC_CUDA(cudaMemsetAsync(s->stamps, 0, ((size_t)p.T + 1) * 8, s->stream));
    MC_CUDA(cudaMemsetAsync(s->status, 0, 256, s->stream));
    MC_CUDA(cudaMemsetAsync(s->hsync, 0, 64 * 4, s->stream));
    MC_CUDA(cudaMemsetAsync(s->hkey, 0, 2 * (size_t)s->Bcap * 2 * 8, s->stream));
    // MINIMA_CUDA_CLUSTER_NONCOOP=1 skips the cooperative attribute (kernel
    // profilers that cannot instrument cooperative cluster launches)
    const char* noncoop = getenv("MINIMA_CUDA_CLUSTER_NONCOOP");
    const bool coop = !(noncoop && noncoop[0] == '1');
    cudaError_t e = launch_cluster(cp, s->cl_cs, s->cl_nc, s->cl_smem, s->stream, coop);
    if (e != cudaSuccess && coop) {
        // cooperative scheduling of clusters unsupported: the plan already
        // checked that every cluster can be resident, and every wait is bounded
        cudaGetLastError();
        e = launch_cluster(cp, s->cl_cs, s->cl_nc, s->cl_smem, s->stream, false);
    }
    if (e != cudaSuccess) return fail(MC_ERR_CUDA, "cluster loop launch: %s", cudaGetErrorString(e));
    MC_CUDA(cudaEventRecord(s->ev1, s->stream));
    s->last_launches = 1 + relayouts;
    s->last_path = 1;
    int status = 0;
    MC_CUDA(cudaMemcpyAsync(&status, s->status, 4, cudaMemcpyDeviceToHost, s->stream));
    MC_CUDA(cudaStreamSynchronize(s->stream));
    MC_CUDA(cudaEventElapsedTime(&s->last_ms, s->ev0, s->ev1));
    if (status == mc::ST_TIMEOUT)
        return fail(MC_ERR_TIMEOUT, "cluster loop: a device-side wait passed its deadline");
    if (status != 0) return fail(MC_ERR_DEVICE, "cluster loop reported status %d", status);
    return MC_OK;
}

// Shapes the batched prefill kernels handle (float4 GEMM tiles, RoPE pairs
// inside a thread's columns, two head dimensions per lane in attention).
bool prefill_ok(const mc_model* m) {
    return m->D % 4 == 0 && m->F % 4 == 0 && m->hd % 2 == 0 && m->hd <= 64 && m->H / m->K <= 128;
}

constexpr int kPrefillChunk = 256;   // positions per prefill pass (CUDA-core GEMMs, logits)
constexpr int kPfTcRows = 8192;      // tensor-core prefill: rows per pass it aims for

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime.
PFN_cuTensorMapEncodeTiled_v12000 tc_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

// Tensor map of a row-major [layers][rows][inner] array (layers == 0: 2-D)
// read as box_rows-row x 128-byte boxes with the 128-byte swizzle.  The
// caller guarantees a 16-byte aligned base and inner * es % 16 == 0.
mc_status tc_map(CUtensorMap* map, const void* base, int es, uint64_t inner, uint64_t rows,
                 uint64_t layers, uint32_t box_rows = mc::TC_BM) {
    auto enc = tc_encoder();
    if (!enc) return fail(MC_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[3] = {inner, rows, layers ? layers : 1};
    const cuuint64_t strides[2] = {inner * es, inner * rows * es};
    const cuuint32_t box[3] = {(cuuint32_t)(mc::TC_BKB / es), box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = enc(map, es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                           layers ? 3 : 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MC_ERR_INVALID, "tensor map encode failed (%d)", (int)r);
    return MC_OK;
}

// B maps must be built with box_rows == BN.
template <int KIND, int EPI, int BN = 128, int STAGES = mc::TC_STAGES>
cudaError_t tc_launch(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& b2,
                      const mc::TcArgs& g, cudaStream_t st) {
    const size_t smem = mc::tc_smem_bytes(EPI == mc::EPI_SWIGLU ? 2 : 1, BN, STAGES);
    static unsigned long long attr_set = 0;    // one bit per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !((attr_set >> dev) & 1ull)) {
        e = cudaFuncSetAttribute(mc::tc_gemm_kernel<KIND, EPI, BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return e;
        attr_set |= 1ull << dev;
    }
    const unsigned tiles = (unsigned)((g.N + BN - 1) / BN) * (unsigned)((g.M + mc::TC_BM - 1) / mc::TC_BM);
    // split K only for partial-tile launches: ksplit CTAs per tile
    const unsigned ks = g.ksplit > 1 ? (unsigned)g.ksplit : 1u;
    if (ks > 1 && EPI != mc::EPI_PART) return cudaErrorInvalidValue;
    mc::tc_gemm_kernel<KIND, EPI, BN, STAGES><<<tiles * ks, mc::TC_THREADS, smem, st>>>(a, b, b2, g);
    return cudaGetLastError();
}

// CTAs splitting K for a decode GEMM of `tiles` output tiles and nk K
// blocks: about one CTA per SM in all, at most 8 partials per element and
// at least one K block each.
// Launch with programmatic stream serialization: the kernel may start while
// the previous one in the stream finishes (its pdl_wait orders the rest).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Decode GEMM launch (tc_dec_kernel): X maps with BN-row boxes, weight maps
// with 128-row boxes; ksplit CTAs per (128 features x BN sequences) tile.
template <int KIND, int EPI, int BN, int STAGES>
cudaError_t tc_dec_launch(const CUtensorMap& x, const CUtensorMap& w, const CUtensorMap& w2,
                          const mc::TcArgs& g, cudaStream_t st) {
    constexpr int DUAL = EPI == mc::EPI_PART2 ? 2 : 1;
    constexpr int XS = KIND == mc::TC_BF16 ? 2 : 1;      // bf16: hi and lo activation tiles
    const size_t smem = 1024 + (size_t)STAGES * (DUAL * mc::TC_TILE + (size_t)XS * BN * mc::TC_BKB) + 256;
    static unsigned long long attr_set = 0;    // one bit per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !((attr_set >> dev) & 1ull)) {
        e = cudaFuncSetAttribute(mc::tc_dec_kernel<KIND, EPI, BN, STAGES>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr_set |= 1ull << dev;
    }
    const unsigned ks = g.ksplit > 1 ? (unsigned)g.ksplit : 1u;
    if (ks > 1 && EPI != mc::EPI_PART && EPI != mc::EPI_PART2) return cudaErrorInvalidValue;
    const unsigned tiles = (unsigned)((g.N + mc::TC_BM - 1) / mc::TC_BM) * (unsigned)((g.M + BN - 1) / BN);
    return launch_pdl(mc::tc_dec_kernel<KIND, EPI, BN, STAGES>, dim3(tiles * ks), dim3(mc::TC_THREADS), smem, st,
                      x, w, w2, g);
}

constexpr int kMaxKSplit = mc::kBdMaxParts;
int tc_ksplit(int tiles, int nk, int sms) {
    int ks = sms / std::max(tiles, 1);
    ks = std::min(ks, kMaxKSplit);
    ks = std::min(ks, nk);
    return std::max(ks, 1);
}

// Tensor maps of the weight matrices: fp32 operands (kind::tf32) for fp32
// weights, bf16 operands (kind::f16) for bf16 weights.  Single-matrix GEMMs
// run 128 x 256 tiles, the SwiGLU pair 128 x 128.
mc_status tc_weight_maps(mc_session* s) {
    if (s->w_maps_ok) return MC_OK;
    const mc_model* m = s->m;
    const char* wb = static_cast<const char*>(m->wblock);
    const uint64_t D = m->D, F = m->F, Q = m->Q, L = m->L;
    const int es = m->dtype == MC_WEIGHTS_BF16 ? 2 : 4;
    mc_status st = MC_OK;
    if (!st) st = tc_map(&s->w_map[0], wb + m->off[1], es, D, Q, L, 256);
    if (!st) st = tc_map(&s->w_map[1], wb + m->off[2], es, D, D, L, 256);
    if (!st) st = tc_map(&s->w_map[2], wb + m->off[3], es, D, F, L, 128);
    if (!st) st = tc_map(&s->w_map[3], wb + m->off[4], es, D, F, L, 128);
    if (!st) st = tc_map(&s->w_map[4], wb + m->off[5], es, F, D, L, 256);
    if (!st) st = tc_map(&s->w_map[5], wb + m->off[0], es, D, m->V, 1, 256);
    s->w_maps_ok = st == MC_OK;
    return st;
}

// A-operand maps of the prefill buffers (their bf16 copies for bf16 weights).
mc_status pf_tc_maps(mc_session* s) {
    const mc_model* m = s->m;
    const uint64_t R = s->pf_rows, D = m->D, F = m->F;
    const bool b16 = m->dtype == MC_WEIGHTS_BF16;
    const int es = b16 ? 2 : 4;
    const void* xn = b16 ? (const void*)s->pf_xn16 : (const void*)s->pf_xn;
    const void* att = b16 ? (const void*)s->pf_att16 : (const void*)s->pf_att;
    const void* fh = b16 ? (const void*)s->pf_f16 : (const void*)s->pf_f;
    mc_status st = tc_weight_maps(s);
    if (!st) st = tc_map(&s->pf_map[0], xn, es, D, R, 0);
    if (!st) st = tc_map(&s->pf_map[1], att, es, D, R, 0);
    if (!st) st = tc_map(&s->pf_map[2], fh, es, F, R, 0);
    s->pf_maps_ok = st == MC_OK;
    return st;
}

// Batched forward of positions [0, Pf) of every sequence (mc_prefill.cuh):
// fills the KV cache so that the token loop can start at position Pf.
// With `logits` set (mc_model_forward), every chunk also applies the final
// norm and the tied lm_head (forward.c:253-270) and copies the chunk's rows
// to logits[b][t][V] (sequence length S, host or device memory).
template <typename WT>
mc_status run_prefill(mc_session* s, int batch, const uint16_t* prompts, int stride, int Pf,
                      int& launches, float* logits = nullptr, bool logits_dev = false, int S = 0,
                      const mc_forward_caches* caps = nullptr) {
    const mc_model* m = s->m;
    constexpr bool kB16 = std::is_same<WT, __nv_bfloat16>::value;
    constexpr int KD = kB16 ? mc::TC_BF16 : mc::TC_TF32;
    // bf16 operands need rows of a multiple of 8 elements (16-byte strides)
    // (the cache capture of model_forward runs the fp32 CUDA-core GEMMs)
    const bool tc = s->pf_tc && !caps && (!kB16 || (m->D % 8 == 0 && m->F % 8 == 0));
    // positions per pass: kPrefillChunk, or on the tensor-core path (without
    // logits) up to four times that, so that a small batch of long prompts
    // still gives each GEMM about kPfTcRows rows: 128-row tiles for every SM
    int chunk = kPrefillChunk;
    if (tc && !logits)
        chunk = std::max(chunk, std::min(4 * kPrefillChunk, (kPfTcRows / std::max(1, s->Bcap) + 63) / 64 * 64));
    chunk = std::min(chunk, s->cap);
    const size_t rows = (size_t)s->Bcap * chunk;
    if (s->pf_rows < rows) {
        float** bufs[] = {&s->pf_x, &s->pf_xn, &s->pf_q, &s->pf_att, &s->pf_f};
        for (float** b : bufs) { cudaFree(*b); *b = nullptr; }
        s->pf_rows = 0;
        const size_t D = m->D, F = m->F;
        MC_CUDA(cudaMalloc(&s->pf_x, rows * D * 4));
        MC_CUDA(cudaMalloc(&s->pf_xn, rows * D * 4));
        MC_CUDA(cudaMalloc(&s->pf_q, rows * D * 4));
        MC_CUDA(cudaMalloc(&s->pf_att, rows * D * 4));
        MC_CUDA(cudaMalloc(&s->pf_f, rows * F * 4));
        s->pf_rows = rows;
        s->pf_maps_ok = false;
        cudaFree(s->pf_logits);
        s->pf_logits = nullptr;
        for (__nv_bfloat16** b : {&s->pf_xn16, &s->pf_att16, &s->pf_f16}) {
            cudaFree(*b);
            *b = nullptr;
        }
    }
    if (caps && (!s->pf_cap_qkv || s->pf_cap_rows < s->pf_rows)) {
        for (float** b : {&s->pf_cap_qkv, &s->pf_cap_up, &s->pf_cap_gate}) {
            cudaFree(*b);
            *b = nullptr;
        }
        const size_t R = s->pf_rows;
        if (cudaMalloc(&s->pf_cap_qkv, R * m->Q * 4) != cudaSuccess ||
            cudaMalloc(&s->pf_cap_up, R * m->F * 4) != cudaSuccess ||
            cudaMalloc(&s->pf_cap_gate, R * m->F * 4) != cudaSuccess) {
            cudaGetLastError();
            s->pf_cap_rows = 0;
            return fail(MC_ERR_NOMEM, "model_forward: cache staging buffers");
        }
        s->pf_cap_rows = R;
    }
    if (tc && kB16 && !s->pf_xn16) {
        const size_t D = m->D, F = m->F, R = s->pf_rows;
        if (cudaMalloc(&s->pf_xn16, R * D * 2) != cudaSuccess || cudaMalloc(&s->pf_att16, R * D * 2) != cudaSuccess ||
            cudaMalloc(&s->pf_f16, R * F * 2) != cudaSuccess) {
            cudaGetLastError();
            return fail(MC_ERR_NOMEM, "prefill bf16 buffers");
        }
        s->pf_maps_ok = false;
    }
    if (logits && !s->pf_logits) {
        // logits passes are kPrefillChunk positions (chunk above)
        const size_t bytes = (size_t)s->Bcap * std::min(kPrefillChunk, s->cap) * (size_t)m->V * 4;
        if (cudaMalloc(&s->pf_logits, bytes) != cudaSuccess) {
            cudaGetLastError();
            return fail(MC_ERR_NOMEM, "model_forward: lm_head scratch (%zu bytes)", bytes);
        }
    }
    if (tc && !s->pf_maps_ok) {
        const mc_status st = pf_tc_maps(s);
        if (st) return st;
    }
    mc::PrefillArgs a{};
    a.V = m->V; a.D = m->D; a.L = m->L; a.H = m->H; a.K = m->K; a.hd = m->hd; a.kvd = m->kvd;
    a.Q = m->Q; a.F = m->F; a.G = m->H / m->K;
    a.B = batch; a.Bcap = s->Bcap; a.cap = s->cap;
    a.prompts = prompts; a.prompt_stride = stride;
    a.rope = m->rope; a.kc = s->kc; a.vc = s->vc;
    a.pg = mc::KvPages{s->kv_table, s->kv_pps, s->kv_shift};
    a.X = s->pf_x; a.XN = s->pf_xn; a.QB = s->pf_q; a.ATT = s->pf_att; a.FH = s->pf_f;
    if (tc && kB16) {
        a.XN16 = s->pf_xn16;
        a.ATT16 = s->pf_att16;
        a.FH16 = s->pf_f16;
    }
    a.status = s->status;
    if (caps) {
        a.UP = s->pf_cap_up;
        a.GATE = s->pf_cap_gate;
    }
    const char* wb = static_cast<const char*>(m->wblock);
    const WT* emb = reinterpret_cast<const WT*>(wb + m->off[0]);
    const WT* wqkv = reinterpret_cast<const WT*>(wb + m->off[1]);
    const WT* wproj = reinterpret_cast<const WT*>(wb + m->off[2]);
    const WT* wup = reinterpret_cast<const WT*>(wb + m->off[3]);
    const WT* wgate = reinterpret_cast<const WT*>(wb + m->off[4]);
    const WT* wdown = reinterpret_cast<const WT*>(wb + m->off[5]);
    const float* rms1 = m->norms;
    const float* rms2 = m->norms + (size_t)m->L * m->D;
    const int QT = std::max(1, 128 / a.G);
    // register-tiled attention for head_dim 16/32/64, else the row-per-warp kernel
    const bool att_tile = m->hd == 16 || m->hd == 32 || m->hd == 64;
    const size_t att_smem = att_tile ? mc::pf_attention_tile_smem(m->hd) : mc::pf_attention_smem(m->hd, a.G, QT);
    if (att_tile)
        MC_CUDA(cudaFuncSetAttribute(m->hd == 16 ? mc::pf_attention_tile_kernel<16>
                                     : m->hd == 32 ? mc::pf_attention_tile_kernel<32>
                                                   : mc::pf_attention_tile_kernel<64>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)att_smem));
    else
        MC_CUDA(cudaFuncSetAttribute(mc::pf_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)att_smem));
    cudaStream_t st = s->stream;
    const cudaStream_t st_ = st;
    // Copy `width` floats per chunk row from the device buffer src to the
    // host array dst laid out as model_forward's caches: [layers][batch*S]
    // rows, row b*S + t (the chunk's rows of sequence b are contiguous).
    auto capture = [&](float* dst, int layer, const float* src, int width) -> cudaError_t {
        if (!dst) return cudaSuccess;
        const size_t w = (size_t)width, n = (size_t)a.chunk;
        float* d0 = dst + ((size_t)layer * batch * S + a.c0) * w;
        return cudaMemcpy2DAsync(d0, (size_t)S * w * 4, src, n * w * 4, n * w * 4, batch,
                                 cudaMemcpyDeviceToHost, st);
    };
    auto attention = [&](int l) {
        const dim3 grid((a.chunk + QT - 1) / QT, m->K, batch);
        switch (att_tile ? m->hd : 0) {
        case 16: mc::pf_attention_tile_kernel<16><<<grid, 256, att_smem, st_>>>(a, l, QT); break;
        case 32: mc::pf_attention_tile_kernel<32><<<grid, 256, att_smem, st_>>>(a, l, QT); break;
        case 64: mc::pf_attention_tile_kernel<64><<<grid, 256, att_smem, st_>>>(a, l, QT); break;
        default: mc::pf_attention_kernel<<<grid, 256, att_smem, st_>>>(a, l, QT); break;
        }
    };
    const size_t D = m->D, F = m->F, Q = m->Q;
    auto grid2 = [](int N, int M) { return dim3((N + mc::GBN - 1) / mc::GBN, (M + mc::GBM - 1) / mc::GBM); };
    // CUDA-core GEMMs whose tiles leave SMs idle (few prompt rows) split K
    // into up to kPfMaxSplit slices of at least two K blocks each.
    auto with_split = [&](dim3 g, int Kd) {
        const int tiles = (int)(g.x * g.y), nk = (Kd + mc::GBK - 1) / mc::GBK;
        g.z = (unsigned)std::max(1, std::min({mc::kPfMaxSplit, nk / 2, (s->grid + tiles - 1) / tiles}));
        return g;
    };
    if (!tc) {
        size_t need = 0;
        for (int c0 = 0; c0 < Pf; c0 += kPrefillChunk) {
            const int M = batch * (std::min(Pf, c0 + kPrefillChunk) - c0);
            const struct { int N, Kd, dual; } gemms[4] = {
                {m->Q, m->D, 1}, {m->D, m->D, 1}, {m->F, m->D, 2}, {m->D, m->F, 1}};
            for (const auto& g : gemms) {
                const dim3 gr = with_split(grid2(g.N, M), g.Kd);
                if (gr.z > 1) need = std::max(need, (size_t)gr.z * gr.x * gr.y * 256 * 16 * g.dual);
            }
        }
        if (need > s->pf_part_floats) {
            cudaFree(s->pf_part);
            s->pf_part = nullptr;
            s->pf_part_floats = 0;
            MC_CUDA(cudaMalloc(&s->pf_part, need * 4));
            s->pf_part_floats = need;
        }
        if (need > 0 && !s->pf_cnt) {
            MC_CUDA(cudaMalloc(&s->pf_cnt, 1024 * sizeof(unsigned)));
            MC_CUDA(cudaMemsetAsync(s->pf_cnt, 0, 1024 * sizeof(unsigned), st));
        }
    }
    for (int c0 = 0; c0 < Pf; c0 += chunk) {
        a.c0 = c0;
        a.c1 = std::min(Pf, c0 + chunk);
        a.chunk = a.c1 - a.c0;
        const int M = batch * a.chunk;
        for (int l = 0; l < m->L; l++) {
            mc::pf_norm_kernel<WT><<<(M + 7) / 8, 256, 0, st>>>(a, emb, rms1 + l * D, l == 0);
            if (tc) {
                mc::TcArgs g{};
                g.M = M;
                g.layer = l;
                g.pa = a;
                g.status = s->status;
                g.timeout_ns = 1000ull * 1000ull * 1000ull;
                const CUtensorMap* mp = s->pf_map;
                const CUtensorMap* wm = s->w_map;
                cudaError_t e;
                g.N = m->Q; g.K = m->D; g.C = nullptr; g.ldc = 0;
                e = tc_launch<KD, mc::EPI_QKV, 256>(mp[0], wm[0], wm[0], g, st);
                if (e != cudaSuccess) return fail(MC_ERR_CUDA, "tcgen05 prefill: %s", cudaGetErrorString(e));
                attention(l);
                g.N = m->D; g.K = m->D; g.C = a.X; g.ldc = m->D;
                e = tc_launch<KD, mc::EPI_RESID, 256>(mp[1], wm[1], wm[1], g, st);
                if (e != cudaSuccess) return fail(MC_ERR_CUDA, "tcgen05 prefill: %s", cudaGetErrorString(e));
                mc::pf_norm_kernel<WT><<<(M + 7) / 8, 256, 0, st>>>(a, emb, rms2 + l * D, 0);
                g.N = m->F; g.K = m->D; g.C = a.FH; g.ldc = m->F;
                e = tc_launch<KD, mc::EPI_SWIGLU>(mp[0], wm[2], wm[3], g, st);
                if (e != cudaSuccess) return fail(MC_ERR_CUDA, "tcgen05 prefill: %s", cudaGetErrorString(e));
                g.N = m->D; g.K = m->F; g.C = a.X; g.ldc = m->D;
                e = tc_launch<KD, mc::EPI_RESID, 256>(mp[2], wm[4], wm[4], g, st);
                if (e != cudaSuccess) return fail(MC_ERR_CUDA, "tcgen05 prefill: %s", cudaGetErrorString(e));
                launches += 7;
                continue;
            }
            if (caps) MC_CUDA(capture(caps->resid_attn, l, a.X, m->D));
            mc::pf_gemm_kernel<WT, mc::EPI_QKV><<<with_split(grid2(m->Q, M), m->D), 256, 0, st>>>(
                a, a.XN, M, m->Q, m->D, wqkv + l * Q * D, nullptr, nullptr, 0, l, s->pf_part, s->pf_cnt);
            if (caps && caps->qkv) {
                mc::pf_gather_qkv_kernel<<<M, 256, 0, st>>>(a, l, s->pf_cap_qkv);
                MC_CUDA(capture(caps->qkv, l, s->pf_cap_qkv, m->Q));
                launches++;
            }
            attention(l);
            if (caps) MC_CUDA(capture(caps->attn_out, l, a.ATT, m->D));
            mc::pf_gemm_kernel<WT, mc::EPI_RESID><<<with_split(grid2(m->D, M), m->D), 256, 0, st>>>(
                a, a.ATT, M, m->D, m->D, wproj + l * D * D, nullptr, a.X, m->D, l, s->pf_part, s->pf_cnt);
            if (caps) MC_CUDA(capture(caps->resid_ffn, l, a.X, m->D));
            mc::pf_norm_kernel<WT><<<(M + 7) / 8, 256, 0, st>>>(a, emb, rms2 + l * D, 0);
            mc::pf_gemm_kernel<WT, mc::EPI_SWIGLU><<<with_split(grid2(m->F, M), m->D), 256, 0, st>>>(
                a, a.XN, M, m->F, m->D, wup + l * F * D, wgate + l * F * D, a.FH, m->F, l, s->pf_part,
                s->pf_cnt);
            if (caps) {
                MC_CUDA(capture(caps->up_buf, l, a.UP, m->F));
                MC_CUDA(capture(caps->gate_buf, l, a.GATE, m->F));
                MC_CUDA(capture(caps->ffn_buf, l, a.FH, m->F));
            }
            mc::pf_gemm_kernel<WT, mc::EPI_RESID><<<with_split(grid2(m->D, M), m->F), 256, 0, st>>>(
                a, a.FH, M, m->D, m->F, wdown + l * D * F, nullptr, a.X, m->D, l, s->pf_part, s->pf_cnt);
            launches += 7;
        }
        if (caps && !logits && (caps->x || caps->x_norm)) {
            const float* rmsf = m->norms + 2 * (size_t)m->L * m->D;
            mc::pf_norm_kernel<WT><<<(M + 7) / 8, 256, 0, st>>>(a, emb, rmsf, 0);
            launches++;
        }
        if (caps) MC_CUDA(capture(caps->x, 0, a.X, m->D));
        if (caps && !logits) MC_CUDA(capture(caps->x_norm, 0, a.XN, m->D));
        if (logits) {
            const float* rmsf = m->norms + 2 * (size_t)m->L * m->D;
            mc::pf_norm_kernel<WT><<<(M + 7) / 8, 256, 0, st>>>(a, emb, rmsf, 0);
            if (tc) {
                mc::TcArgs g{};
                g.M = M; g.N = m->V; g.K = m->D; g.layer = 0; g.C = s->pf_logits; g.ldc = m->V;
                g.pa = a;
                g.status = s->status;
                g.timeout_ns = 1000ull * 1000ull * 1000ull;
                const cudaError_t e = tc_launch<KD, mc::TCE_STORE, 256>(s->pf_map[0], s->w_map[5],
                                                                                 s->w_map[5], g, st);
                if (e != cudaSuccess) return fail(MC_ERR_CUDA, "tcgen05 lm_head: %s", cudaGetErrorString(e));
            } else {
                mc::pf_gemm_kernel<WT, mc::EPI_STORE><<<grid2(m->V, M), 256, 0, st>>>(
                    a, a.XN, M, m->V, m->D, emb, nullptr, s->pf_logits, m->V, 0, nullptr, nullptr);
            }
            launches += 2;
            if (caps) MC_CUDA(capture(caps->x_norm, 0, a.XN, m->D));
            // rows of sequence b are contiguous in the chunk and in the output
            const size_t n = a.chunk, V = m->V;
            for (int b = 0; b < batch; b++)
                MC_CUDA(cudaMemcpyAsync(logits + ((size_t)b * S + a.c0) * V, s->pf_logits + (size_t)b * n * V,
                                        n * V * 4, logits_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                                        st));
        }
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MC_ERR_CUDA, "prefill launch: %s", cudaGetErrorString(e));
    return MC_OK;
}

// Shapes the batched tensor-core decode handles: TMA rows of 16 bytes
// (bf16: multiples of 8 elements) and the attention phase's limits.
bool batched_ok(const mc_model* m) {
    const int mult = m->dtype == MC_WEIGHTS_BF16 ? 8 : 4;
    const int G = m->H / m->K;
    return m->D % mult == 0 && m->F % mult == 0 && G * m->hd <= mc::kBdAttMaxO * mc::kBdAttThreads &&
           G <= mc::kBdAttThreads && m->D <= 4 * mc::kBdNormCols * mc::kThreads;
}

// The token loop as one launch sequence per step with every matrix product
// a batch-wide tcgen05 GEMM (mc_batched.cuh).
template <typename WT>
mc_status run_batched(mc_session* s, mc::LoopParams<WT>& p) {
    const mc_model* m = s->m;
    constexpr bool kB16 = std::is_same<WT, __nv_bfloat16>::value;
    constexpr int KD = kB16 ? mc::TC_BF16 : mc::TC_TF32;
    constexpr int BN = 64;                       // sequences per decode GEMM tile
    // ring stages: the bf16 stages carry two activation tiles
    constexpr int ST1 = kB16 ? 6 : 8, ST2 = kB16 ? 4 : 5;
    fill_params(p, s);
    p.stamps = s->stamps;
    s->last_T = p.T;
    const size_t Bc = s->Bcap, D = m->D, F = m->F, Q = m->Q;
    int dev = 0, optin = 0, sms = 0;
    MC_CUDA(cudaGetDevice(&dev));
    MC_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    MC_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    // K splits: about one CTA per SM for every GEMM but the lm_head, whose
    // V/128 feature tiles fill the GPU by themselves
    const int bke = mc::TC_BKB / (kB16 ? 2 : 4), tsq = (p.B + BN - 1) / BN;
    auto tiles = [&](size_t n) { return tsq * (int)((n + mc::TC_BM - 1) / mc::TC_BM); };
    auto nkb = [&](size_t k) { return (int)((k + bke - 1) / bke); };
    const int ks_qkv = tc_ksplit(tiles(Q), nkb(D), sms);
    const int ks_proj = tc_ksplit(tiles(D), nkb(D), sms);
    const int ks_up = tc_ksplit(tiles(F), nkb(D), sms);
    const int ks_down = tc_ksplit(tiles(D), nkb(F), sms);
    const size_t part_need = std::max({(size_t)ks_qkv * p.B * Q, (size_t)ks_proj * p.B * D,
                                       (size_t)ks_up * p.B * 2 * F, (size_t)ks_down * p.B * D});
    if (!s->bd_lists) {
        bool ok = cudaMalloc(&s->bd_lists, mc::bd_lists_ints(s->Bcap) * 4) == cudaSuccess &&
                  cudaMalloc(&s->bd_xn, Bc * D * 4) == cudaSuccess;
        // bf16 operands: rows [0, Bc) hi halves, rows [Bc, 2 Bc) lo halves
        if (ok && kB16)
            ok = cudaMalloc(&s->bd_xn16, 2 * Bc * D * 2) == cudaSuccess &&
                 cudaMalloc(&s->bd_att16, 2 * Bc * D * 2) == cudaSuccess &&
                 cudaMalloc(&s->bd_f16, 2 * Bc * F * 2) == cudaSuccess;
        if (!ok) {
            cudaGetLastError();
            return fail(MC_ERR_NOMEM, "batched decode buffers");
        }
        s->bd_maps_ok = false;
    }
    if (s->bd_part_floats < part_need) {
        cudaFree(s->bd_part);
        s->bd_part = nullptr;
        s->bd_part_floats = 0;
        if (cudaMalloc(&s->bd_part, part_need * 4) != cudaSuccess) {
            cudaGetLastError();
            return fail(MC_ERR_NOMEM, "batched decode partials (%zu B)", part_need * 4);
        }
        s->bd_part_floats = part_need;
    }
    if (!s->bd_maps_ok) {
        const int es = kB16 ? 2 : 4;
        mc_status st = MC_OK;
        const uint64_t xrows = kB16 ? 2 * Bc : Bc;
        if (!st) st = tc_map(&s->bd_xmap[0], kB16 ? (const void*)s->bd_xn16 : (const void*)s->bd_xn, es, D, xrows, 0, BN);
        if (!st) st = tc_map(&s->bd_xmap[1], kB16 ? (const void*)s->bd_att16 : (const void*)s->att, es, D, xrows, 0, BN);
        if (!st) st = tc_map(&s->bd_xmap[2], kB16 ? (const void*)s->bd_f16 : (const void*)s->f, es, F, xrows, 0, BN);
        const char* wb = static_cast<const char*>(m->wblock);
        const uint64_t L = m->L;
        if (!st) st = tc_map(&s->bd_wmap[0], wb + m->off[1], es, D, Q, L, mc::TC_BM);
        if (!st) st = tc_map(&s->bd_wmap[1], wb + m->off[2], es, D, D, L, mc::TC_BM);
        if (!st) st = tc_map(&s->bd_wmap[2], wb + m->off[3], es, D, F, L, mc::TC_BM);
        if (!st) st = tc_map(&s->bd_wmap[3], wb + m->off[4], es, D, F, L, mc::TC_BM);
        if (!st) st = tc_map(&s->bd_wmap[4], wb + m->off[5], es, F, D, L, mc::TC_BM);
        if (!st) st = tc_map(&s->bd_wmap[5], wb + m->off[0], es, D, m->V, 1, mc::TC_BM);
        if (st) return st;
        s->bd_maps_ok = true;
    }
    // attention: a lane per key for head_dim 32/64 and G <= kBdWMaxG, else
    // the shared-memory tile kernel
    const int G = m->H / m->K;
    const bool att_lane = (m->hd == 32 || m->hd == 64) && G <= mc::kBdWMaxG;
    const size_t att_smem = att_lane ? mc::bd_attw_smem(G, m->hd) : mc::bd_att_smem(G, m->hd);
    const int att_warps = mc::kBdWWarps;
    if (att_smem > (size_t)optin)
        return fail(MC_ERR_UNSUPPORTED, "batched attention needs %zu B of shared memory", att_smem);
    cudaStream_t st = s->stream;
    MC_CUDA(cudaMemsetAsync(s->stamps, 0, ((size_t)p.T + 1) * 8, st));
    MC_CUDA(cudaMemsetAsync(s->status, 0, 256, st));
    MC_CUDA(cudaMemsetAsync(s->att_cnt, 0, (size_t)s->Bcap * m->K * 4, st));
    MC_CUDA(cudaMemsetAsync(s->bd_lists + 3, 0, 4, st));
    static unsigned long long attr_set = 0;     // dynamic shared memory limits, per device
    if (dev < 64 && !((attr_set >> dev) & 1ull)) {
        // the device maximum, shared by every session on the device
        MC_CUDA(cudaFuncSetAttribute(mc::bd_att_kernel<WT>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
        MC_CUDA(cudaFuncSetAttribute(mc::bd_attw_kernel<WT, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
        MC_CUDA(cudaFuncSetAttribute(mc::bd_attw_kernel<WT, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
        MC_CUDA(cudaFuncSetAttribute(mc::bd_sample_kernel<WT>, cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
        attr_set |= 1ull << dev;
    }
    const mc::BdLists L{s->bd_lists, s->Bcap};
    mc::TcArgs g{};
    g.M = p.B;
    g.x_lo_row = kB16 ? (int)Bc : 0;
    g.act = L.base + 4 + 2 * (size_t)s->Bcap;      // act_fwd
    g.tpos = L.base + 2;
    g.status = s->status;
    g.timeout_ns = p.timeout_ns;
    g.C = s->bd_part;
    const CUtensorMap* xm = s->bd_xmap;
    const CUtensorMap* wm = s->bd_wmap;
    const float* rmsf = m->norms + 2 * (size_t)m->L * m->D;
    const unsigned swiglu_blocks = (unsigned)std::max(1, std::min(4 * sms, (int)((p.B * F / 4 + 255) / 256)));
    // resident attention CTAs per SM (lane-per-key kernel), for the split choice below
    int att_per_sm = 1;
    if (att_lane) {
        const cudaError_t oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &att_per_sm, m->hd == 32 ? mc::bd_attw_kernel<WT, 32> : mc::bd_attw_kernel<WT, 64>, att_warps * 32,
            att_smem);
        if (oe != cudaSuccess || att_per_sm < 1) {
            cudaGetLastError();
            att_per_sm = 1;
        }
    }
    __nv_bfloat16* xn16 = kB16 ? s->bd_xn16 : nullptr;
    __nv_bfloat16* f16 = kB16 ? s->bd_f16 : nullptr;
    int launches = 0;
    mc::bd_prologue_kernel<WT><<<s->grid, mc::kThreads, 0, st>>>(p);
    launches++;
    cudaError_t e = cudaSuccess;
    for (int t = p.t0; t < p.T && e == cudaSuccess; t++) {
        if ((e = launch_pdl(mc::bd_lists_kernel<WT>, dim3(1), dim3(1024), 0, st, p, L, (int)(t == p.t0))) !=
            cudaSuccess)
            break;
        launches++;
        // attention units: (sequence, KV head) pairs, each split into
        // klen-key pieces only when the pairs alone would not fill the GPU
        // twice over (the device's position is t too)
        const int pairs = p.B * m->K, nkeys = t + 1;
        // (a multiple of the tile, and at least kSplitLen keys so that the
        // splits fit the max_split partial slots)
        auto klen_of = [&](int want) {
            return std::max(mc::kSplitLen, ((nkeys + want - 1) / want + mc::kBdTile - 1) / mc::kBdTile * mc::kBdTile);
        };
        int klen = klen_of(std::max(1, (2 * sms + pairs - 1) / pairs));
        if (att_lane) {
            // lane-per-key kernel: the split count with the fewest (waves of
            // resident CTAs) x (32-key chunks per warp), one chunk's worth
            // added for the merge of split units
            const long slots = (long)att_per_sm * sms;
            long best = -1;
            for (int want = 1; want <= p.max_split; want++) {
                const int kl = klen_of(want), ns = (nkeys + kl - 1) / kl;
                if (want > 1 && ns == (nkeys + klen_of(want - 1) - 1) / klen_of(want - 1)) continue;
                const long waves = ((long)pairs * ns + slots - 1) / slots;
                const long per_warp = ((kl + 31) / 32 + att_warps - 1) / att_warps;
                const long cost = waves * per_warp + (ns > 1 ? 1 : 0);
                if (best < 0 || cost < best) {
                    best = cost;
                    klen = kl;
                }
                if (ns >= nkeys / mc::kSplitLen) break;
            }
        }
        const unsigned att_units = (unsigned)pairs * (unsigned)((nkeys + klen - 1) / klen);
        // every GEMM leaves K-slice partials in bd_part; the kernel after it
        // sums them in slice order (norm: residual; attention: q and the
        // new K/V row with RoPE; swiglu: f)
        for (int l = 0; l < m->L; l++) {
            if ((e = launch_pdl(mc::bd_norm_kernel<WT>, dim3(p.B), dim3(mc::kThreads), 0, st, p, L, 0,
                                m->norms + (size_t)l * D, (int)(l == 0), s->bd_xn, xn16, s->bd_part,
                                l == 0 ? 0 : ks_down)) != cudaSuccess)
                break;
            g.layer = l;
            g.N = m->Q; g.K = m->D; g.ldc = m->Q; g.ksplit = ks_qkv;
            if ((e = tc_dec_launch<KD, mc::EPI_PART, BN, ST1>(xm[0], wm[0], wm[0], g, st)) != cudaSuccess) break;
            // (bf16: the attention also writes the hi/lo operand of the proj GEMM)
            __nv_bfloat16* att16 = kB16 ? s->bd_att16 : nullptr;
            if (att_lane)
                e = launch_pdl(m->hd == 32 ? mc::bd_attw_kernel<WT, 32> : mc::bd_attw_kernel<WT, 64>,
                               dim3(att_units), dim3(mc::kBdWWarps * 32), att_smem, st, p, L, l, t, klen,
                               (const float*)s->bd_part, ks_qkv, att16);
            else
                e = launch_pdl(mc::bd_att_kernel<WT>, dim3(att_units), dim3(mc::kBdAttThreads), att_smem, st, p,
                               L, l, t, klen, (const float*)s->bd_part, ks_qkv, att16);
            if (e != cudaSuccess) break;
            g.N = m->D; g.K = m->D; g.ldc = m->D; g.ksplit = ks_proj;
            if ((e = tc_dec_launch<KD, mc::EPI_PART, BN, ST1>(xm[1], wm[1], wm[1], g, st)) != cudaSuccess) break;
            if ((e = launch_pdl(mc::bd_norm_kernel<WT>, dim3(p.B), dim3(mc::kThreads), 0, st, p, L, 0,
                                m->norms + ((size_t)m->L + l) * D, 0, s->bd_xn, xn16, s->bd_part, ks_proj)) !=
                cudaSuccess)
                break;
            g.N = m->F; g.K = m->D; g.ldc = 2 * m->F; g.ksplit = ks_up;
            if ((e = tc_dec_launch<KD, mc::EPI_PART2, BN, ST2>(xm[0], wm[2], wm[3], g, st)) != cudaSuccess) break;
            if ((e = launch_pdl(mc::bd_swiglu_kernel<WT>, dim3(swiglu_blocks), dim3(mc::kThreads), 0, st, p, L,
                                (const float*)s->bd_part, ks_up, f16)) != cudaSuccess)
                break;
            g.N = m->D; g.K = m->F; g.ldc = m->D; g.ksplit = ks_down;
            if ((e = tc_dec_launch<KD, mc::EPI_PART, BN, ST1>(xm[2], wm[4], wm[4], g, st)) != cudaSuccess) break;
            launches += 8;
        }
        if (e != cudaSuccess) break;
        if ((e = launch_pdl(mc::bd_norm_kernel<WT>, dim3(p.B), dim3(mc::kThreads), 0, st, p, L, 1, rmsf, 0,
                            s->bd_xn, xn16, s->bd_part, ks_down)) != cudaSuccess)
            break;
        // lm_head for the sequences that sample, with the reserved-id mask and
        // the greedy partials in its epilogue
        mc::TcArgs gh = g;
        gh.act = L.base + 4 + 3 * (size_t)s->Bcap;     // act_head
        gh.N = m->V; gh.K = m->D; gh.C = s->logits; gh.ldc = m->V; gh.layer = 0; gh.ksplit = 1;
        gh.head = 1; gh.sa = p.s; gh.counts = s->counts; gh.banned = s->banned;
        gh.amax_v = s->amax_v; gh.amax_i = s->amax_i;
        if ((e = tc_dec_launch<KD, mc::TCE_STORE, BN, ST1>(xm[0], wm[5], wm[5], gh, st)) != cudaSuccess) break;
        if ((e = launch_pdl(mc::bd_sample_kernel<WT>, dim3(s->grid), dim3(mc::kThreads), s->smem, st, p, L,
                            (int)((m->V + mc::TC_BM - 1) / mc::TC_BM))) != cudaSuccess)
            break;
        launches += 3;
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return fail(MC_ERR_CUDA, "batched decode launch: %s", cudaGetErrorString(e));
    MC_CUDA(cudaEventRecord(s->ev1, st));
    s->last_launches = launches;
    s->last_path = 2;
    int status = 0;
    MC_CUDA(cudaMemcpyAsync(&status, s->status, 4, cudaMemcpyDeviceToHost, st));
    MC_CUDA(cudaStreamSynchronize(st));
    MC_CUDA(cudaEventElapsedTime(&s->last_ms, s->ev0, s->ev1));
    if (status == mc::ST_TIMEOUT) return fail(MC_ERR_TIMEOUT, "batched decode: a pipeline wait passed its deadline");
    if (status != 0) {
        int check = 0;
        MC_CUDA(cudaMemcpy(&check, s->bd_lists + 3, 4, cudaMemcpyDeviceToHost));
        return fail(MC_ERR_DEVICE, "batched decode reported status %d (check %d)", status, check);
    }
    return MC_OK;
}

bool options_valid(const mc_sampling* o) {  // generate.c:528-541
    return o && o->max_new_tokens >= 0 && std::isfinite(o->temperature) && o->temperature > 0.0f &&
           std::isfinite(o->top_p) && o->top_p > 0.0f && o->top_p <= 1.0f &&
           std::isfinite(o->repetition_penalty) && o->repetition_penalty >= 1.0f &&
           std::isfinite(o->min_p) && o->min_p >= 0.0f && o->min_p <= 1.0f &&
           std::isfinite(o->frequency_penalty) && o->frequency_penalty >= -2.0f &&
           o->frequency_penalty <= 2.0f && std::isfinite(o->presence_penalty) &&
           o->presence_penalty >= -2.0f && o->presence_penalty <= 2.0f &&
           o->no_repeat_ngram_size >= 0 && o->no_repeat_ngram_size <= 16 &&
           o->min_new_tokens >= 0 && o->min_new_tokens <= 512 &&
           o->min_new_tokens <= o->max_new_tokens && o->stop_sequence_len >= 0 &&
           o->stop_sequence_len <= MC_MAX_STOP &&
           !(o->stop_sequence_len > 0 && !o->stop_sequence_ids);
}

template <typename WT>
mc_status generate_t(mc_session* s, int batch, const uint16_t* prompts, int prompt_stride,
                     const int* prompt_lens, uint16_t* out_ids, int out_cap, const mc_sampling* o,
                     uint64_t* rng_states, int* out_counts, int* final_pos, unsigned flags,
                     float* trace_logits, int trace_steps) {
    const mc_model* m = s->m;
    const bool dev = flags & MC_DEVICE_POINTERS;
    // Per-sequence bookkeeping exactly as generate.c:553-564.
    std::vector<mc::SeqState> seq(batch);
    int T = 0;
    for (int b = 0; b < batch; b++) {
        const int P = prompt_lens[b];
        if (P <= 0 || P > out_cap || P > s->cap || P > prompt_stride)
            return fail(MC_ERR_INVALID, "prompt %d: length %d outside [1, min(out_cap, max_seq)]", b, P);
        int nnew = o->max_new_tokens;
        nnew = std::min(nnew, out_cap - P);
        nnew = std::min(nnew, s->cap - P);
        mc::SeqState& q = seq[b];
        memset(&q, 0, sizeof(q));
        q.P = P;
        q.nnew = std::max(nnew, 0);
        q.done = nnew <= 0;
        q.result = P;
        q.final_pos = 0;
        if (!dev) q.rng = rng_states[b];
        if (nnew > 0) T = std::max(T, P + nnew - 1);
    }
    if (!dev) {
        for (int b = 0; b < batch; b++)
            for (int i = 0; i < prompt_lens[b]; i++)
                if (prompts[(size_t)b * prompt_stride + i] >= m->V)
                    return fail(MC_ERR_INVALID, "prompt %d holds id %d >= vocab", b,
                                (int)prompts[(size_t)b * prompt_stride + i]);
    }
    for (int i = 0; i < o->stop_sequence_len; i++)
        if (o->stop_sequence_ids[i] >= m->V) return fail(MC_ERR_INVALID, "stop id >= vocab");
    if (s->kv_paged) {
        // positions a sequence feeds: its prompt and all but its last new id
        std::vector<int> need(batch);
        for (int b = 0; b < batch; b++) need[b] = seq[b].nnew > 0 ? seq[b].P + seq[b].nnew - 1 : 0;
        const mc_status st = assign_pages(s, batch, need.data());
        if (st) return st;
    }

    mc::LoopParams<WT> p{};
    p.B = batch;
    p.out_cap = dev ? out_cap : s->cap;
    p.out_ids = dev ? out_ids : s->out;
    p.prompt_stride = dev ? prompt_stride : s->cap;
    p.prompts = dev ? prompts : s->prompts;
    p.s.temperature = o->temperature;
    p.s.top_p = o->top_p;
    p.s.rep = o->repetition_penalty;
    p.s.min_p = o->min_p;
    p.s.freq = o->frequency_penalty;
    p.s.pres = o->presence_penalty;
    int top_k = o->top_k;
    top_k = std::max(top_k, 1);
    top_k = std::min(top_k, m->V);
    top_k = std::min(top_k, MC_MAX_TOPK);
    p.s.top_k = top_k;
    p.s.min_new = o->min_new_tokens;
    p.s.ngram = o->no_repeat_ngram_size;
    p.s.stop_ids = s->stop;
    p.s.stop_len = o->stop_sequence_len;
    p.s.pen_active = o->repetition_penalty > 1.0f || o->frequency_penalty != 0.0f ||
                     o->presence_penalty != 0.0f;
    p.T = T;
    p.all_logits = 0;
    p.trace_steps = trace_logits ? trace_steps : 0;
    if (p.trace_steps > 0) {
        mc_status st = ensure_trace(s, (size_t)batch * p.trace_steps * m->V * 4);
        if (st) return st;
        MC_CUDA(cudaMemsetAsync(s->trace, 0, (size_t)batch * p.trace_steps * m->V * 4, s->stream));
        p.trace = s->trace;
    }
    if (o->stop_sequence_len > 0)
        MC_CUDA(cudaMemcpyAsync(s->stop, o->stop_sequence_ids, o->stop_sequence_len * 2,
                                cudaMemcpyHostToDevice, s->stream));
    if (!dev) {
        size_t maxP = 0;
        for (int b = 0; b < batch; b++) maxP = std::max(maxP, (size_t)prompt_lens[b]);
        MC_CUDA(cudaMemcpy2DAsync(s->prompts, (size_t)s->cap * 2, prompts, (size_t)prompt_stride * 2,
                                  maxP * 2, batch, cudaMemcpyHostToDevice, s->stream));
    } else {
        // RNG states live on the device: gather them into the sequence table.
        for (int b = 0; b < batch; b++) seq[b].rng = 0;
    }
    MC_CUDA(cudaMemcpyAsync(s->seq, seq.data(), batch * sizeof(mc::SeqState),
                            cudaMemcpyHostToDevice, s->stream));
    if (dev) {
        for (int b = 0; b < batch; b++)
            MC_CUDA(cudaMemcpyAsync(&s->seq[b].rng, rng_states + b, 8, cudaMemcpyDeviceToDevice,
                                    s->stream));
    }
    if (T > 0) {
        // positions every sequence feeds before its first sampled id
        int Pf = s->cap;
        for (int b = 0; b < batch; b++) Pf = std::min(Pf, seq[b].P - 1);
        if (!prefill_ok(m)) Pf = 0;
        MC_CUDA(cudaEventRecord(s->ev0, s->stream));
        int pf_launches = 0;
        if (Pf > 0) {
            mc_status st = run_prefill<WT>(s, batch, p.prompts, p.prompt_stride, Pf, pf_launches);
            if (st) return st;
        }
        MC_CUDA(cudaEventRecord(s->ev_mid, s->stream));
        p.t0 = Pf;
        mc_status st;
        if (s->bd_tc && batched_ok(m)) {
            st = run_batched<WT>(s, p);
        } else if constexpr (std::is_same<WT, float>::value) {
            if (s->cl_ok && p.s.top_k == 1 && batch <= mc::kBCMax) st = run_cluster(s, p);
            else st = run_loop<WT>(s, p);
        } else {
            st = run_loop<WT>(s, p);
        }
        if (st) return st;
        s->last_launches += pf_launches;
        s->last_prefill_pos = Pf;
        MC_CUDA(cudaEventElapsedTime(&s->last_prefill_ms, s->ev0, s->ev_mid));
    } else {
        s->last_ms = 0.0f;
        s->last_launches = 0;
    }
    // Results.
    if (dev) {
        for (int b = 0; b < batch; b++) {
            MC_CUDA(cudaMemcpyAsync(rng_states + b, &s->seq[b].rng, 8, cudaMemcpyDeviceToDevice, s->stream));
            MC_CUDA(cudaMemcpyAsync(out_counts + b, &s->seq[b].result, 4, cudaMemcpyDeviceToDevice, s->stream));
            if (final_pos)
                MC_CUDA(cudaMemcpyAsync(final_pos + b, &s->seq[b].final_pos, 4, cudaMemcpyDeviceToDevice,
                                        s->stream));
            if (seq[b].nnew <= 0)  // generate.c:557-559: prompt copied, nothing else
                MC_CUDA(cudaMemcpyAsync(out_ids + (size_t)b * out_cap, prompts + (size_t)b * prompt_stride,
                                        (size_t)seq[b].P * 2, cudaMemcpyDeviceToDevice, s->stream));
        }
        MC_CUDA(cudaStreamSynchronize(s->stream));
        return MC_OK;
    }
    MC_CUDA(cudaMemcpyAsync(seq.data(), s->seq, batch * sizeof(mc::SeqState), cudaMemcpyDeviceToHost,
                            s->stream));
    int maxR = 0;
    for (int b = 0; b < batch; b++) maxR = std::max(maxR, prompt_lens[b] + seq[b].nnew);
    MC_CUDA(cudaStreamSynchronize(s->stream));
    if (T > 0)
        MC_CUDA(cudaMemcpy2DAsync(out_ids, (size_t)out_cap * 2, s->out, (size_t)s->cap * 2,
                                  (size_t)maxR * 2, batch, cudaMemcpyDeviceToHost, s->stream));
    if (trace_logits && p.trace_steps > 0)
        MC_CUDA(cudaMemcpyAsync(trace_logits, s->trace, (size_t)batch * p.trace_steps * m->V * 4,
                                cudaMemcpyDeviceToHost, s->stream));
    MC_CUDA(cudaStreamSynchronize(s->stream));
    for (int b = 0; b < batch; b++) {
        if (seq[b].nnew <= 0) {
            memcpy(out_ids + (size_t)b * out_cap, prompts + (size_t)b * prompt_stride,
                   (size_t)seq[b].P * 2);
            out_counts[b] = seq[b].P;
            if (final_pos) final_pos[b] = 0;
        } else {
            out_counts[b] = seq[b].result;
            if (final_pos) final_pos[b] = seq[b].final_pos;
        }
        rng_states[b] = seq[b].rng;
    }
    return MC_OK;
}

// Teacher-forced forward of tokens[b*n .. b*n+n) (host ids), one position
// at a time; leaves the logits of every position in s->trace on the device.
template <typename WT>
mc_status forward_logits_dev(mc_session* s, int batch, const uint16_t* tokens, int n) {
    const mc_model* m = s->m;
    for (size_t i = 0; i < (size_t)batch * n; i++)
        if (tokens[i] >= m->V) return fail(MC_ERR_INVALID, "token id %d >= vocab", (int)tokens[i]);
    std::vector<mc::SeqState> seq(batch);
    for (int b = 0; b < batch; b++) {
        memset(&seq[b], 0, sizeof(mc::SeqState));
        seq[b].P = n;
        seq[b].nnew = 1;
    }
    mc_status st = ensure_trace(s, (size_t)batch * n * m->V * 4);
    if (st) return st;
    if (s->kv_paged) {
        std::vector<int> need(batch, n);
        st = assign_pages(s, batch, need.data());
        if (st) return st;
    }
    mc::LoopParams<WT> p{};
    p.B = batch;
    p.prompts = s->prompts;
    p.prompt_stride = s->cap;
    p.out_ids = s->out;
    p.out_cap = s->cap;
    p.s.top_k = 1;
    p.s.temperature = 1.0f;
    p.T = n;
    p.all_logits = 1;
    p.trace = s->trace;
    p.trace_steps = n;
    MC_CUDA(cudaMemcpy2DAsync(s->prompts, (size_t)s->cap * 2, tokens, (size_t)n * 2, (size_t)n * 2,
                              batch, cudaMemcpyHostToDevice, s->stream));
    MC_CUDA(cudaMemcpyAsync(s->seq, seq.data(), batch * sizeof(mc::SeqState), cudaMemcpyHostToDevice,
                            s->stream));
    MC_CUDA(cudaEventRecord(s->ev0, s->stream));
    p.t0 = 0;
    st = run_loop<WT>(s, p);
    if (st) return st;
    s->last_prefill_pos = 0;
    s->last_prefill_ms = 0.0f;
    return MC_OK;
}

template <typename WT>
mc_status forward_logits_t(mc_session* s, int batch, const uint16_t* tokens, int n, float* out) {
    const mc_status st = forward_logits_dev<WT>(s, batch, tokens, n);
    if (st) return st;
    MC_CUDA(cudaMemcpy(out, s->trace, (size_t)batch * n * s->m->V * 4, cudaMemcpyDeviceToHost));
    return MC_OK;
}

}  // namespace

extern "C" {

mc_status mc_generate(mc_session* s, int batch, const uint16_t* prompts, int prompt_stride,
                      const int* prompt_lens, uint16_t* out_ids, int out_cap, const mc_sampling* o,
                      uint64_t* rng_states, int* out_counts, int* final_pos, unsigned flags,
                      float* trace_logits, int trace_steps) {
    if (!s) return fail(MC_ERR_INVALID, "null session");
    if (batch <= 0 || batch > s->Bcap)
        return fail(MC_ERR_INVALID, "batch %d outside [1, %d]", batch, s->Bcap);
    if (!prompts || !prompt_lens || !out_ids || out_cap <= 0 || !rng_states || !out_counts ||
        prompt_stride <= 0)
        return fail(MC_ERR_INVALID, "null or empty argument");
    if (!options_valid(o)) return fail(MC_ERR_INVALID, "generation options rejected (generate.c:526-551)");
    if (trace_logits && (trace_steps < 0 || trace_steps > s->cap))
        return fail(MC_ERR_INVALID, "trace_steps %d", trace_steps);
    MC_CUDA(cudaSetDevice(s->m->device));
    if (s->m->dtype == MC_WEIGHTS_BF16)
        return generate_t<__nv_bfloat16>(s, batch, prompts, prompt_stride, prompt_lens, out_ids,
                                         out_cap, o, rng_states, out_counts, final_pos, flags,
                                         trace_logits, trace_steps);
    return generate_t<float>(s, batch, prompts, prompt_stride, prompt_lens, out_ids, out_cap, o,
                             rng_states, out_counts, final_pos, flags, trace_logits, trace_steps);
}

}  // extern "C"

namespace {

template <typename WT>
mc_status model_forward_t(mc_session* s, int batch, int seq, const uint16_t* tokens, float* logits,
                          bool dev, const mc_forward_caches* caps = nullptr) {
    const mc_model* m = s->m;
    const uint16_t* dtok = tokens;
    if (s->kv_paged) {
        std::vector<int> need(batch, seq);
        const mc_status st = assign_pages(s, batch, need.data());
        if (st) return st;
    }
    if (!dev) {
        for (size_t i = 0; i < (size_t)batch * seq; i++)   // forward.c:179-186
            if (tokens[i] >= m->V) return fail(MC_ERR_INVALID, "model_forward: token id %d >= vocab", tokens[i]);
        MC_CUDA(cudaMemcpyAsync(s->prompts, tokens, (size_t)batch * seq * 2, cudaMemcpyHostToDevice, s->stream));
        dtok = s->prompts;
    }
    MC_CUDA(cudaMemsetAsync(s->status, 0, 256, s->stream));
    MC_CUDA(cudaEventRecord(s->ev0, s->stream));
    int launches = 0;
    const mc_status st = run_prefill<WT>(s, batch, dtok, seq, seq, launches, logits, dev, seq, caps);
    if (st) return st;
    MC_CUDA(cudaEventRecord(s->ev1, s->stream));
    int status = 0;
    MC_CUDA(cudaMemcpyAsync(&status, s->status, 4, cudaMemcpyDeviceToHost, s->stream));
    MC_CUDA(cudaStreamSynchronize(s->stream));
    MC_CUDA(cudaEventElapsedTime(&s->last_ms, s->ev0, s->ev1));
    s->last_launches = launches;
    s->last_T = 0;
    if (status == mc::ST_DEVICE) return fail(MC_ERR_INVALID, "model_forward: token id outside the vocabulary");
    if (status != 0) return fail(MC_ERR_DEVICE, "model_forward: kernel status %d", status);
    return MC_OK;
}

}  // namespace

extern "C" {

mc_status mc_model_forward(mc_session* s, int batch, int seq, const uint16_t* tokens, float* logits_out,
                           unsigned flags) {
    if (!s || !tokens || !logits_out) return fail(MC_ERR_INVALID, "null argument");
    if (batch <= 0 || batch > s->Bcap || seq <= 0 || seq > s->cap)
        return fail(MC_ERR_INVALID, "model_forward: batch %d, seq %d outside [1, %d] x [1, %d]", batch, seq,
                    s->Bcap, s->cap);
    if (!prefill_ok(s->m)) return fail(MC_ERR_UNSUPPORTED, "model_forward: no batched kernels for this shape");
    MC_CUDA(cudaSetDevice(s->m->device));
    const bool dev = flags & MC_DEVICE_POINTERS;
    if (s->m->dtype == MC_WEIGHTS_BF16)
        return model_forward_t<__nv_bfloat16>(s, batch, seq, tokens, logits_out, dev);
    return model_forward_t<float>(s, batch, seq, tokens, logits_out, dev);
}

mc_status mc_model_forward_caches(mc_session* s, int batch, int seq, const uint16_t* tokens,
                                  const mc_forward_caches* caps) {
    if (!s || !tokens || !caps) return fail(MC_ERR_INVALID, "null argument");
    if (batch <= 0 || batch > s->Bcap || seq <= 0 || seq > s->cap)
        return fail(MC_ERR_INVALID, "model_forward: batch %d, seq %d outside [1, %d] x [1, %d]", batch, seq,
                    s->Bcap, s->cap);
    if (!prefill_ok(s->m)) return fail(MC_ERR_UNSUPPORTED, "model_forward: no batched kernels for this shape");
    MC_CUDA(cudaSetDevice(s->m->device));
    if (s->m->dtype == MC_WEIGHTS_BF16)
        return model_forward_t<__nv_bfloat16>(s, batch, seq, tokens, caps->logits, false, caps);
    return model_forward_t<float>(s, batch, seq, tokens, caps->logits, false, caps);
}

mc_status mc_forward_logits(mc_session* s, int batch, const uint16_t* tokens, int n, float* out) {
    if (!s) return fail(MC_ERR_INVALID, "null session");
    if (batch <= 0 || batch > s->Bcap || n <= 0 || n > s->cap || !tokens || !out)
        return fail(MC_ERR_INVALID, "forward_logits: batch %d, n %d", batch, n);
    MC_CUDA(cudaSetDevice(s->m->device));
    if (s->m->dtype == MC_WEIGHTS_BF16) return forward_logits_t<__nv_bfloat16>(s, batch, tokens, n, out);
    return forward_logits_t<float>(s, batch, tokens, n, out);
}

mc_status mc_next_token_stats(mc_session* s, const uint16_t* tokens, int n, int top_n,
                              mc_token_stats* out) {
    if (!s || !tokens || !out) return fail(MC_ERR_INVALID, "null argument");
    if (n <= 0 || n > s->cap || top_n <= 0 || top_n > MC_STATS_MAX_TOP)
        return fail(MC_ERR_INVALID, "next_token_stats: n %d, top_n %d", n, top_n);
    MC_CUDA(cudaSetDevice(s->m->device));
    const mc_status st = s->m->dtype == MC_WEIGHTS_BF16
                             ? forward_logits_dev<__nv_bfloat16>(s, 1, tokens, n)
                             : forward_logits_dev<float>(s, 1, tokens, n);
    if (st) return st;
    if (!s->stats) MC_CUDA(cudaMalloc(&s->stats, sizeof(mc_token_stats)));
    MC_CUDA(cudaMemsetAsync(s->stats, 0, sizeof(mc_token_stats), s->stream));
    mc::next_token_stats_kernel<<<1, mc::kStatsThreads, 0, s->stream>>>(
        s->trace + (size_t)(n - 1) * s->m->V, s->m->V, top_n, s->stats);
    MC_CUDA(cudaGetLastError());
    MC_CUDA(cudaMemcpyAsync(out, s->stats, sizeof(*out), cudaMemcpyDeviceToHost, s->stream));
    MC_CUDA(cudaStreamSynchronize(s->stream));
    s->last_launches += 1;
    return MC_OK;
}

// Device buffers of mc_matmul, per device, grown on demand and kept.
namespace {
struct MatmulScratch {
    float* buf;
    size_t floats;
};
MatmulScratch g_mm[64];
}  // namespace

mc_status mc_matmul(float* out, const float* x, const float* w, int n, int d_in, int d_out) {
    if (!out || !x || !w || n <= 0 || d_in <= 0 || d_out <= 0)
        return fail(MC_ERR_INVALID, "matmul: null operand or empty shape");
    int dev = 0;
    MC_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(MC_ERR_UNSUPPORTED, "device index %d", dev);
    const size_t nx = (size_t)n * d_in, nw = (size_t)d_out * d_in, no = (size_t)n * d_out;
    MatmulScratch& sc = g_mm[dev];
    if (sc.floats < nx + nw + no) {
        cudaFree(sc.buf);
        sc.buf = nullptr;
        sc.floats = 0;
        MC_CUDA(cudaMalloc(&sc.buf, (nx + nw + no) * 4));
        sc.floats = nx + nw + no;
    }
    float* dx = sc.buf;
    float* dw = dx + nx;
    float* dout = dw + nw;
    MC_CUDA(cudaMemcpy(dx, x, nx * 4, cudaMemcpyHostToDevice));
    MC_CUDA(cudaMemcpy(dw, w, nw * 4, cudaMemcpyHostToDevice));
    const dim3 grid((d_out + mc::kMmTile - 1) / mc::kMmTile, (n + mc::kMmTile - 1) / mc::kMmTile);
    mc::matmul_f32_kernel<<<grid, 256>>>(dx, dw, dout, n, d_in, d_out);
    MC_CUDA(cudaGetLastError());
    MC_CUDA(cudaMemcpy(out, dout, no * 4, cudaMemcpyDeviceToHost));
    return MC_OK;
}

mc_status mc_last_kernel_ms(mc_session* s, float* ms) {
    if (!s || !ms) return fail(MC_ERR_INVALID, "null argument");
    *ms = s->last_ms;
    return MC_OK;
}

mc_status mc_last_prefill(mc_session* s, int* positions, float* ms) {
    if (!s || !positions || !ms) return fail(MC_ERR_INVALID, "null argument");
    *positions = s->last_prefill_pos;
    *ms = s->last_prefill_ms;
    return MC_OK;
}

mc_status mc_last_launch_count(mc_session* s, int* n) {
    if (!s || !n) return fail(MC_ERR_INVALID, "null argument");
    *n = s->last_launches;
    return MC_OK;
}

mc_status mc_last_step_times(mc_session* s, unsigned long long* ns, int cap, int* n) {
    if (!s || !ns || !n || cap < 0) return fail(MC_ERR_INVALID, "null argument");
    *n = 0;
    if (s->last_launches == 0) return MC_OK;
    const int count = std::min(cap, s->last_T + 1);
    MC_CUDA(cudaMemcpy(ns, s->stamps, (size_t)count * 8, cudaMemcpyDeviceToHost));
    *n = count;
    return MC_OK;
}

const char* mc_last_kernel_name(mc_session* s) {
    if (!s || s->last_launches == 0) return "";
    return s->last_path == 2 ? "mc::tc_gemm_kernel" : s->last_path == 1 ? "mc::cluster_loop_kernel" : "mc::token_loop_kernel";
}

mc_status mc_session_cluster_variant(mc_session* s, int* variant) {
    if (!s || !variant) return fail(MC_ERR_INVALID, "null argument");
    *variant = s->cl_ok ? s->cl_plan.v2 : -1;
    return MC_OK;
}

mc_status mc_session_stream(mc_session* s, void** stream) {
    if (!s || !stream) return fail(MC_ERR_INVALID, "null argument");
    *stream = (void*)s->stream;
    return MC_OK;
}

}  // extern "C"

// ===========================================================================
// mc_generate_static: the token loop with no device allocation at all.
//
// For callers that cannot call cudaMalloc: real-time hosts that must not take
// its cost (or the device-wide wait of a later cudaFree) mid-session, hosts
// whose device memory is carved up front by their own pool, and plugins that
// must not grow the process's device footprint after start-up.  Weights, prompts and outputs are the caller's device
// buffers; everything else the loop needs (KV cache, activations, split
// partials, counters, RoPE table, sequence table) lives in one file-scope
// __device__ array of MC_STATIC_SCRATCH_BYTES, which every GPU that loads
// this library holds until the process exits.
//
// Every call resolves the array's device address with cudaGetSymbolAddress
// (with the device current) and sets the kernel's shared-memory limit; the
// first call on a device also reads its properties and loads the kernel, so
// make that first call before any stream capture.  All calls share the one array and
// it keeps the last call's contents, so the barrier counter, status word and
// attention counters are cleared at the start of each call, and calls that
// overlap on the GPU (on different streams, or from several host threads)
// race.  Not thread-safe.
// ===========================================================================

static __device__ __align__(256) unsigned char g_static_scratch[MC_STATIC_SCRATCH_BYTES];

namespace {

struct StaticDevice {
    bool ready;
    int sms;
    size_t smem_optin;
};
StaticDevice g_static_dev[64];

// Host-side staging kept in static storage so that the call allocates no
// host memory either.
mc::SeqState g_static_seq[MC_STATIC_MAX_BATCH];
float2 g_static_rope[MC_STATIC_MAX_ROPE];
int g_static_pages[MC_STATIC_MAX_BATCH * (MC_MAX_SEQ / MC_MIN_PAGE_LEN)];
int g_static_status;

struct StaticPlan {
    size_t off[22];
    size_t total;
    size_t smem;
    int bc, xs_ld, max_split, pps;
};

// Carve the scratch array the same way mc_session_create sizes its buffers.
StaticPlan static_plan(const mc_model_desc* d, int batch, int cap, int grid, size_t smem_limit) {
    StaticPlan pl{};
    const size_t B = batch, L = d->n_layers, K = d->n_kv_heads, hd = d->head_dim, D = d->dim;
    const size_t F = d->ffn_dim, V = d->vocab_size, H = d->n_heads;
    pl.max_split = (cap + mc::kSplitLen - 1) / mc::kSplitLen;
    const size_t ms = pl.max_split;
    // KV pages of MC_MIN_PAGE_LEN positions, identity table
    pl.pps = (cap + MC_MIN_PAGE_LEN - 1) / MC_MIN_PAGE_LEN;
    const size_t kv_bytes = B * pl.pps * L * K * (size_t)MC_MIN_PAGE_LEN * hd * 4;
    const size_t sizes[22] = {
        kv_bytes, kv_bytes,                                   // kc, vc
        B * D * 4, B * D * 4, B * D * 4, B * F * 4,           // x, q, att, f
        B * V * 4,                                            // logits
        B * H * ms * hd * 4, B * H * ms * 4, B * H * ms * 4,  // part_o, part_m, part_l
        B * (size_t)grid * 4, B * (size_t)grid * 4,           // amax_v, amax_i
        B * K * 4, B * V * 4, B * ((V + 31) / 32) * 4,        // att_cnt, counts, banned
        256, 256,                                             // bar, status
        B * sizeof(mc::SeqState), (size_t)MC_MAX_STOP * 2,    // seq, stop ids
        (size_t)cap * (hd / 2 > 0 ? hd / 2 : 1) * sizeof(float2),  // rope
        B * (size_t)pl.pps * 4,                               // page table
        0};
    size_t off = 0;
    for (int i = 0; i < 22; i++) {
        pl.off[i] = off;
        off = align_up(off + sizes[i], 256);
    }
    pl.total = off;
    const int G = d->n_heads / d->n_kv_heads;
    pl.xs_ld = (int)align_up((size_t)std::max(d->dim, d->ffn_dim), 4);
    const size_t att_bytes = mc::att_phase_bytes(G, d->head_dim);
    const size_t samp_bytes = mc::sampler_smem_bytes(d->vocab_size);
    const size_t fixed = mc::loop_fixed_bytes(batch);
    const size_t wi_bytes = mc::kWarps * mc::kBCMax * 4;
    size_t phase = std::max(att_bytes, samp_bytes);
    const size_t row_bytes = (size_t)pl.xs_ld * 4;
    int bc = mc::kBCMax;
    while (bc > 1 && fixed + std::max(phase, bc * row_bytes + wi_bytes) > smem_limit) bc--;
    pl.bc = bc;
    phase = std::max(phase, bc * row_bytes + wi_bytes);
    pl.smem = align_up(fixed + phase, 16);
    return pl;
}

// Per-device set-up of the static path, with that device current.  The
// device properties are cached; the array's device address and the
// kernels' shared-memory limit are looked up on every call (both are cheap
// after the first), so nothing cached goes stale if the host resets the
// device between calls.
mc_status static_setup(int dev, unsigned char** scratch) {
    StaticDevice& sd = g_static_dev[dev];
    if (!sd.ready) {
        cudaDeviceProp prop;
        MC_CUDA(cudaGetDeviceProperties(&prop, dev));
        if (prop.major != 10)
            return fail(MC_ERR_UNSUPPORTED, "mc_generate_static: device %d is not sm_100", dev);
        sd.sms = prop.multiProcessorCount;
        sd.smem_optin = prop.sharedMemPerBlockOptin;
        sd.ready = true;
    }
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (e != cudaSuccess || !ptr)
        return fail(MC_ERR_CUDA, "mc_generate_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    const int optin = (int)sd.smem_optin;
    MC_CUDA(cudaFuncSetAttribute(mc::token_loop_kernel<float, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
    MC_CUDA(cudaFuncSetAttribute(mc::token_loop_kernel<float, false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
    *scratch = static_cast<unsigned char*>(ptr);
    return MC_OK;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace

extern "C" mc_status mc_generate_static(const mc_model_desc* w, int batch,
                                        const uint16_t* prompts, int prompt_stride,
                                        const int* prompt_lens, uint16_t* out_ids, int out_cap,
                                        const mc_sampling* o, uint64_t* rng_states,
                                        int* out_counts, int max_seq, void* stream) {
    mc_status st = validate_desc(w);
    if (st) return st;
    if (batch <= 0 || batch > MC_STATIC_MAX_BATCH)
        return fail(MC_ERR_INVALID, "mc_generate_static: batch %d outside [1, %d]", batch,
                    MC_STATIC_MAX_BATCH);
    if (max_seq <= 0 || max_seq > w->max_seq || max_seq > MC_STATIC_MAX_ROPE ||
        (size_t)max_seq * std::max(w->head_dim / 2, 1) > MC_STATIC_MAX_ROPE)
        return fail(MC_ERR_INVALID, "mc_generate_static: max_seq %d outside [1, %d]", max_seq,
                    std::min(w->max_seq, MC_STATIC_MAX_ROPE / std::max(w->head_dim / 2, 1)));
    if (!prompts || !prompt_lens || !out_ids || out_cap <= 0 || !rng_states || !out_counts ||
        prompt_stride <= 0)
        return fail(MC_ERR_INVALID, "mc_generate_static: null or empty argument");
    if (!options_valid(o))
        return fail(MC_ERR_INVALID, "mc_generate_static: options rejected (generate.c:526-551)");
    int dev = 0;
    MC_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(MC_ERR_UNSUPPORTED, "device index %d", dev);
    unsigned char* base = nullptr;
    st = static_setup(dev, &base);
    if (st) return st;
    const StaticDevice& sd = g_static_dev[dev];
    const StaticPlan pl = static_plan(w, batch, max_seq, sd.sms, sd.smem_optin);
    if (pl.total > (size_t)MC_STATIC_SCRATCH_BYTES)
        return fail(MC_ERR_INVALID,
                    "mc_generate_static: this model/batch/max_seq needs %zu bytes of scratch; the "
                    "static array holds %u (use mc_session_create + mc_generate instead)",
                    pl.total, (unsigned)MC_STATIC_SCRATCH_BYTES);
    if (pl.smem > sd.smem_optin)
        return fail(MC_ERR_UNSUPPORTED, "mc_generate_static: shared memory plan %zu B", pl.smem);
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    // Per-sequence bookkeeping exactly as generate.c:553-564.
    int T = 0;
    for (int b = 0; b < batch; b++) {
        const int P = prompt_lens[b];
        if (P <= 0 || P > out_cap || P > max_seq || P > prompt_stride)
            return fail(MC_ERR_INVALID, "mc_generate_static: prompt %d length %d", b, P);
        int nnew = o->max_new_tokens;
        nnew = std::min(nnew, out_cap - P);
        nnew = std::min(nnew, max_seq - P);
        mc::SeqState& q = g_static_seq[b];
        memset(&q, 0, sizeof(q));
        q.P = P;
        q.nnew = std::max(nnew, 0);
        q.done = nnew <= 0;
        q.result = P;
        if (nnew > 0) T = std::max(T, P + nnew - 1);
    }
    for (int i = 0; i < o->stop_sequence_len; i++)
        if (o->stop_sequence_ids[i] >= w->vocab_size)
            return fail(MC_ERR_INVALID, "mc_generate_static: stop id >= vocab");

    // RoPE table (rotary.h:19-24) with the host libm, as mc_model_create does.
    const int half = w->head_dim / 2;
    for (int pair = 0; pair < half; pair++) {
        const float exponent = (2.0f * (float)pair) / (float)w->head_dim;
        const float rbase = ::powf(10000.0f, -exponent);
        for (int pos = 0; pos < max_seq; pos++) {
            const float angle = (float)pos * rbase;
            g_static_rope[(size_t)pos * half + pair] = make_float2(::cosf(angle), ::sinf(angle));
        }
    }

    mc::LoopParams<float> p{};
    p.V = w->vocab_size; p.D = w->dim; p.L = w->n_layers; p.H = w->n_heads; p.K = w->n_kv_heads;
    p.hd = w->head_dim; p.kvd = w->kv_dim; p.Q = w->qkv_dim; p.F = w->ffn_dim;
    p.G = w->n_heads / w->n_kv_heads;
    p.tok_emb = w->tok_emb; p.w_qkv = w->attn_qkv; p.w_proj = w->attn_proj; p.w_up = w->ffn_up;
    p.w_gate = w->ffn_gate; p.w_down = w->ffn_down;
    p.rms1 = w->rms1_scale; p.rms2 = w->rms2_scale; p.rmsf = w->rms_final_scale;
    p.kc = reinterpret_cast<float*>(base + pl.off[0]);
    p.vc = reinterpret_cast<float*>(base + pl.off[1]);
    p.x = reinterpret_cast<float*>(base + pl.off[2]);
    p.q = reinterpret_cast<float*>(base + pl.off[3]);
    p.att = reinterpret_cast<float*>(base + pl.off[4]);
    p.f = reinterpret_cast<float*>(base + pl.off[5]);
    p.logits = reinterpret_cast<float*>(base + pl.off[6]);
    p.part_o = reinterpret_cast<float*>(base + pl.off[7]);
    p.part_m = reinterpret_cast<float*>(base + pl.off[8]);
    p.part_l = reinterpret_cast<float*>(base + pl.off[9]);
    p.amax_v = reinterpret_cast<float*>(base + pl.off[10]);
    p.amax_i = reinterpret_cast<int*>(base + pl.off[11]);
    p.att_cnt = reinterpret_cast<unsigned*>(base + pl.off[12]);
    p.counts = reinterpret_cast<unsigned*>(base + pl.off[13]);
    p.banned = reinterpret_cast<unsigned*>(base + pl.off[14]);
    p.bar = reinterpret_cast<unsigned*>(base + pl.off[15]);
    p.status = reinterpret_cast<int*>(base + pl.off[16]);
    mc::SeqState* dseq = reinterpret_cast<mc::SeqState*>(base + pl.off[17]);
    uint16_t* dstop = reinterpret_cast<uint16_t*>(base + pl.off[18]);
    float2* drope = reinterpret_cast<float2*>(base + pl.off[19]);
    int* dpages = reinterpret_cast<int*>(base + pl.off[20]);
    p.pg = mc::KvPages{dpages, pl.pps, 6};
    static_assert(MC_MIN_PAGE_LEN == 64, "the static path's pages are 2^6 positions");
    p.rope = drope; p.rope_len = max_seq;
    p.cap = max_seq; p.Bcap = batch; p.max_split = pl.max_split;
    p.seq = dseq; p.B = batch;
    p.prompts = prompts; p.prompt_stride = prompt_stride;
    p.out_ids = out_ids; p.out_cap = out_cap;
    p.s.temperature = o->temperature; p.s.top_p = o->top_p; p.s.rep = o->repetition_penalty;
    p.s.min_p = o->min_p; p.s.freq = o->frequency_penalty; p.s.pres = o->presence_penalty;
    p.s.top_k = std::min(std::min(std::max(o->top_k, 1), w->vocab_size), MC_MAX_TOPK);
    p.s.min_new = o->min_new_tokens; p.s.ngram = o->no_repeat_ngram_size;
    p.s.stop_ids = dstop; p.s.stop_len = o->stop_sequence_len;
    p.s.pen_active = o->repetition_penalty > 1.0f || o->frequency_penalty != 0.0f ||
                     o->presence_penalty != 0.0f;
    p.T = T;
    wait_hooks(p);
    p.bc = pl.bc; p.xs_ld = pl.xs_ld;

    // Clear what must start at zero; the array keeps the previous call's data.
    MC_CUDA(cudaMemsetAsync(p.bar, 0, 256, s));
    MC_CUDA(cudaMemsetAsync(p.status, 0, 256, s));
    MC_CUDA(cudaMemsetAsync(p.att_cnt, 0, (size_t)batch * w->n_kv_heads * 4, s));
    if (half > 0)
        MC_CUDA(cudaMemcpyAsync(drope, g_static_rope, (size_t)max_seq * half * sizeof(float2),
                                cudaMemcpyHostToDevice, s));
    if (o->stop_sequence_len > 0)
        MC_CUDA(cudaMemcpyAsync(dstop, o->stop_sequence_ids, o->stop_sequence_len * 2,
                                cudaMemcpyHostToDevice, s));
    for (int i = 0; i < batch * pl.pps; i++) g_static_pages[i] = i;
    MC_CUDA(cudaMemcpyAsync(dpages, g_static_pages, (size_t)batch * pl.pps * 4, cudaMemcpyHostToDevice, s));
    MC_CUDA(cudaMemcpyAsync(dseq, g_static_seq, batch * sizeof(mc::SeqState),
                            cudaMemcpyHostToDevice, s));
    for (int b = 0; b < batch; b++)
        MC_CUDA(cudaMemcpyAsync(&dseq[b].rng, rng_states + b, 8, cudaMemcpyDeviceToDevice, s));
    if (T > 0) {
        const bool vec = w->dim % 4 == 0 && w->ffn_dim % 4 == 0 && aligned16(w->tok_emb) &&
                         aligned16(w->attn_qkv) && aligned16(w->attn_proj) &&
                         aligned16(w->ffn_up) && aligned16(w->ffn_gate) && aligned16(w->ffn_down);
        const cudaError_t e = vec ? launch_loop<float, true>(p, sd.sms, pl.smem, s)
                                  : launch_loop<float, false>(p, sd.sms, pl.smem, s);
        if (e != cudaSuccess)
            return fail(MC_ERR_CUDA, "mc_generate_static launch: %s", cudaGetErrorString(e));
    }
    for (int b = 0; b < batch; b++) {
        MC_CUDA(cudaMemcpyAsync(rng_states + b, &dseq[b].rng, 8, cudaMemcpyDeviceToDevice, s));
        MC_CUDA(cudaMemcpyAsync(out_counts + b, &dseq[b].result, 4, cudaMemcpyDeviceToDevice, s));
        if (g_static_seq[b].nnew <= 0)  // generate.c:557-559
            MC_CUDA(cudaMemcpyAsync(out_ids + (size_t)b * out_cap, prompts + (size_t)b * prompt_stride,
                                    (size_t)g_static_seq[b].P * 2, cudaMemcpyDeviceToDevice, s));
    }
    MC_CUDA(cudaMemcpyAsync(&g_static_status, p.status, 4, cudaMemcpyDeviceToHost, s));
    MC_CUDA(cudaStreamSynchronize(s));
    if (g_static_status == mc::ST_TIMEOUT)
        return fail(MC_ERR_TIMEOUT, "mc_generate_static: a grid barrier passed its deadline");
    if (g_static_status != 0)
        return fail(MC_ERR_DEVICE, "mc_generate_static: kernel status %d", g_static_status);
    return MC_OK;
}

// ------------------------------------------------------------- checkpoints
namespace {

constexpr char kCkptMagicV4[8] = {'M', 'I', 'N', 'I', 'M', 'A', '0', '4'};
constexpr char kCkptMagicV5[8] = {'M', 'I', 'N', 'I', 'M', 'A', '0', '5'};
constexpr size_t kCkptChunkFloats = (size_t)8 << 20;   // 32 MiB per staging buffer

template <typename T>
void take_le(const unsigned char*& p, T& v) {
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
}

// Dimensions derived as model_init_config derives them (model.c:55-89).
mc_model_desc ckpt_desc(const mc_checkpoint_info& in) {
    mc_model_desc d{};
    d.vocab_size = in.vocab_size;
    d.dim = in.dim;
    d.n_layers = in.n_layers;
    d.n_heads = in.n_heads;
    d.ffn_dim = in.ffn_dim;
    d.max_seq = in.max_seq;
    if (in.n_heads > 0 && in.dim % in.n_heads == 0) {
        d.n_kv_heads = kv_head_count(in.n_heads);
        d.head_dim = in.dim / in.n_heads;
        d.kv_dim = d.n_kv_heads * d.head_dim;
        d.qkv_dim = in.dim + 2 * d.kv_dim;
    }
    return d;
}

// Floats per model array, MODEL_ARRAYS order (checkpoint.c:43-52).
void ckpt_counts(const mc_model_desc& d, size_t (&c)[9]) {
    const size_t V = d.vocab_size, D = d.dim, L = d.n_layers, Q = d.qkv_dim, F = d.ffn_dim;
    const size_t v[9] = {V * D, L * Q * D, L * D * D, L * F * D, L * F * D, L * D * F, L * D, L * D, D};
    for (int i = 0; i < 9; i++) c[i] = v[i];
}

// The header and length checks of checkpoint_load (checkpoint.c:319-400),
// in its order.  Leaves f positioned after the header.
mc_status ckpt_header(FILE* f, mc_checkpoint_info* out) {
    unsigned char h[116];
    if (std::fread(h, 1, 12, f) != 12) return fail(MC_ERR_INVALID, "checkpoint: short header");
    mc_checkpoint_info in{};
    const unsigned char* p = h + 8;
    take_le(p, in.version);
    const bool v4 = in.version == 4 && std::memcmp(h, kCkptMagicV4, 8) == 0;
    const bool v5 = in.version == 5 && std::memcmp(h, kCkptMagicV5, 8) == 0;
    if (!v4 && !v5) return fail(MC_ERR_INVALID, "checkpoint: bad magic or version");
    in.header_bytes = v5 ? 116 : 112;
    if (std::fread(h + 12, 1, in.header_bytes - 12, f) != in.header_bytes - 12)
        return fail(MC_ERR_INVALID, "checkpoint: short header");
    uint32_t dims[6];
    for (int i = 0; i < 6; i++) take_le(p, dims[i]);
    take_le(p, in.n_params);
    take_le(p, in.step);
    uint64_t rng = 0;
    take_le(p, rng);
    take_le(p, in.tokenizer_hash);
    take_le(p, in.lr);
    take_le(p, in.beta1);
    take_le(p, in.beta2);
    take_le(p, in.eps);
    take_le(p, in.weight_decay);
    take_le(p, in.schedule_base_lr);
    take_le(p, in.schedule_total_steps);
    take_le(p, in.schedule_warmup_steps);
    take_le(p, in.schedule_type);
    in.optimizer_type = 0;
    if (v5) take_le(p, in.optimizer_type);
    if (in.optimizer_type != 0 && in.optimizer_type != 1)
        return fail(MC_ERR_INVALID, "checkpoint: unknown optimizer type %d", in.optimizer_type);
    for (int i = 0; i < 6; i++)
        if (dims[i] > 0x7fffffffu) return fail(MC_ERR_INVALID, "checkpoint: dimension out of range");
    in.vocab_size = (int32_t)dims[0];
    in.dim = (int32_t)dims[1];
    in.n_layers = (int32_t)dims[2];
    in.n_heads = (int32_t)dims[3];
    in.ffn_dim = (int32_t)dims[4];
    in.max_seq = (int32_t)dims[5];
    in.rng_state = rng ? rng : 0x123456789abcdef0ULL;   // checkpoint.c:413
    const mc_model_desc d = ckpt_desc(in);
    mc_status st = validate_dims(&d);
    if (st) return st;
    size_t c[9];
    ckpt_counts(d, c);
    uint64_t params = 0;
    for (int i = 0; i < 9; i++) params += c[i];
    if (in.n_params != params)
        return fail(MC_ERR_INVALID, "checkpoint: %llu parameters stored, the dimensions give %llu",
                    (unsigned long long)in.n_params, (unsigned long long)params);
    const bool hyper_ok =
        in.step >= 0 && std::isfinite(in.lr) && in.lr >= 0.0f && std::isfinite(in.beta1) &&
        in.beta1 >= 0.0f && in.beta1 < 1.0f && std::isfinite(in.beta2) && in.beta2 >= 0.0f &&
        in.beta2 < 1.0f && std::isfinite(in.eps) && in.eps > 0.0f &&
        std::isfinite(in.weight_decay) && in.weight_decay >= 0.0f &&
        std::isfinite(in.schedule_base_lr) && in.schedule_base_lr > 0.0f &&
        in.schedule_total_steps >= 1 && in.step <= in.schedule_total_steps &&
        in.schedule_warmup_steps >= 0 && in.schedule_warmup_steps < in.schedule_total_steps &&
        (in.schedule_type == 0 || in.schedule_type == 1);
    if (!hyper_ok) return fail(MC_ERR_INVALID, "checkpoint: optimizer state out of range");
    // model arrays, then m (and v for AdamW) per array, then end of file
    const uint64_t floats = params * (in.optimizer_type == 0 ? 3u : 2u);
    in.file_bytes = in.header_bytes + floats * 4;
    const long here = std::ftell(f);
    if (here < 0 || std::fseek(f, 0, SEEK_END) != 0) return fail(MC_ERR_INVALID, "checkpoint: cannot seek");
    const long end = std::ftell(f);
    if (end < 0 || std::fseek(f, here, SEEK_SET) != 0) return fail(MC_ERR_INVALID, "checkpoint: cannot seek");
    if ((uint64_t)end < in.file_bytes) return fail(MC_ERR_INVALID, "checkpoint: truncated file");
    if ((uint64_t)end > in.file_bytes) return fail(MC_ERR_INVALID, "checkpoint: trailing bytes");
    *out = in;
    return MC_OK;
}

struct CkptStaging {
    float* pinned[2] = {nullptr, nullptr};
    float* dev[2] = {nullptr, nullptr};
    unsigned* bad = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t done[2] = {nullptr, nullptr};
    ~CkptStaging() {
        if (stream) cudaStreamSynchronize(stream);
        for (int i = 0; i < 2; i++) {
            if (pinned[i]) cudaFreeHost(pinned[i]);
            if (dev[i]) cudaFree(dev[i]);
            if (done[i]) cudaEventDestroy(done[i]);
        }
        if (bad) cudaFree(bad);
        if (stream) cudaStreamDestroy(stream);
    }
};

// Stream the arrays of an already validated file into m (fp32 or bf16).
mc_status ckpt_stream(FILE* f, const mc_checkpoint_info& in, mc_model* m) {
    CkptStaging st;
    MC_CUDA(cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking));
    for (int i = 0; i < 2; i++) {
        if (cudaHostAlloc(&st.pinned[i], kCkptChunkFloats * 4, cudaHostAllocDefault) != cudaSuccess ||
            cudaMalloc(&st.dev[i], kCkptChunkFloats * 4) != cudaSuccess) {
            cudaGetLastError();
            return fail(MC_ERR_NOMEM, "checkpoint: staging buffers");
        }
        MC_CUDA(cudaEventCreateWithFlags(&st.done[i], cudaEventDisableTiming));
    }
    MC_CUDA(cudaMalloc(&st.bad, 4));
    MC_CUDA(cudaMemsetAsync(st.bad, 0, 4, st.stream));
    const mc_model_desc d = ckpt_desc(in);
    size_t c[9];
    ckpt_counts(d, c);
    const size_t L = m->L, D = m->D;
    char* wb = static_cast<char*>(m->wblock);
    const bool bf16 = m->dtype == MC_WEIGHTS_BF16;
    // destinations: six matrices in wblock, three norm arrays in norms, then
    // the moments (checked only)
    struct Run {
        size_t n;
        float* f32;
        __nv_bfloat16* b16;
    };
    std::vector<Run> runs;
    for (int i = 0; i < 6; i++)
        runs.push_back({c[i], bf16 ? nullptr : reinterpret_cast<float*>(wb + m->off[i]),
                        bf16 ? reinterpret_cast<__nv_bfloat16*>(wb + m->off[i]) : nullptr});
    runs.push_back({c[6], m->norms, nullptr});
    runs.push_back({c[7], m->norms + L * D, nullptr});
    runs.push_back({c[8], m->norms + 2 * L * D, nullptr});
    runs.push_back({(size_t)in.n_params * (in.optimizer_type == 0 ? 2u : 1u), nullptr, nullptr});
    int k = 0;
    for (const Run& r : runs) {
        for (size_t o = 0; o < r.n; o += kCkptChunkFloats, k++) {
            const size_t n = std::min(kCkptChunkFloats, r.n - o);
            const int b = k & 1;
            MC_CUDA(cudaEventSynchronize(st.done[b]));     // its last copy has left the buffer
            if (std::fread(st.pinned[b], 4, n, f) != n) return fail(MC_ERR_INVALID, "checkpoint: read failed");
            MC_CUDA(cudaMemcpyAsync(st.dev[b], st.pinned[b], n * 4, cudaMemcpyHostToDevice, st.stream));
            const int grid = (int)std::min<size_t>((n + 255) / 256, 148 * 8);
            mc::ckpt_ingest_kernel<<<grid, 256, 0, st.stream>>>(st.dev[b], n, r.f32 ? r.f32 + o : nullptr,
                                                               r.b16 ? r.b16 + o : nullptr, st.bad);
            MC_CUDA(cudaGetLastError());
            MC_CUDA(cudaEventRecord(st.done[b], st.stream));
        }
    }
    unsigned bad = 0;
    MC_CUDA(cudaMemcpyAsync(&bad, st.bad, 4, cudaMemcpyDeviceToHost, st.stream));
    MC_CUDA(cudaStreamSynchronize(st.stream));
    if (bad) return fail(MC_ERR_INVALID, "checkpoint: non-finite values");
    return MC_OK;
}

}  // namespace

extern "C" {

mc_status mc_checkpoint_inspect(const char* path, mc_checkpoint_info* info) {
    if (!path || !info) return fail(MC_ERR_INVALID, "null argument");
    FILE* f = std::fopen(path, "rb");
    if (!f) return fail(MC_ERR_INVALID, "checkpoint: cannot open %s", path);
    mc_checkpoint_info in{};
    const mc_status st = ckpt_header(f, &in);
    std::fclose(f);
    if (st) return st;
    *info = in;
    return MC_OK;
}

mc_status mc_model_load_checkpoint(const char* path, int weights_dtype, uint64_t expected_tokenizer_hash,
                                   unsigned flags, mc_model** out, mc_checkpoint_info* info) {
    if (!path || !out) return fail(MC_ERR_INVALID, "null argument");
    *out = nullptr;
    if (weights_dtype != MC_WEIGHTS_F32 && weights_dtype != MC_WEIGHTS_BF16)
        return fail(MC_ERR_INVALID, "unknown weight dtype %d", weights_dtype);
    FILE* f = std::fopen(path, "rb");
    if (!f) return fail(MC_ERR_INVALID, "checkpoint: cannot open %s", path);
    mc_checkpoint_info in{};
    mc_status st = ckpt_header(f, &in);
    if (!st && !(flags & MC_CKPT_ANY_TOKENIZER) && in.tokenizer_hash != expected_tokenizer_hash)
        st = fail(MC_ERR_INVALID, "checkpoint: tokenizer fingerprint differs");
    mc_model* m = nullptr;
    if (!st) {
        const mc_model_desc d = ckpt_desc(in);
        st = model_alloc(&d, weights_dtype, &m);
    }
    if (!st) st = ckpt_stream(f, in, m);
    std::fclose(f);
    if (st) {
        if (m) mc_model_destroy(m);
        return st;
    }
    *out = m;
    if (info) *info = in;
    return MC_OK;
}

}  // extern "C"

// ------------------------------------------------------------ plain GEMM
extern "C" mc_status mc_gemm(int kind, const void* A, const void* B, float* C, int M, int N, int K,
                             unsigned flags, float* ms) {
    if (kind != MC_GEMM_TF32 && kind != MC_GEMM_BF16) return fail(MC_ERR_INVALID, "unknown GEMM kind %d", kind);
    const int es = kind == MC_GEMM_TF32 ? 4 : 2;
    if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0 || ((size_t)K * es) % 16 != 0)
        return fail(MC_ERR_INVALID, "mc_gemm: bad shape or null pointer (K * element size must be a multiple of 16)");
    const bool dev = flags & MC_DEVICE_POINTERS;
    const void* dA = A;
    const void* dB = B;
    float* dC = C;
    void* own[3] = {nullptr, nullptr, nullptr};
    int* dstatus = nullptr;
    mc_status st = MC_OK;
    auto cleanup = [&]() {
        for (void* p : own) cudaFree(p);
        cudaFree(dstatus);
    };
    if (!dev) {
        if (cudaMalloc(&own[0], (size_t)M * K * es) != cudaSuccess ||
            cudaMalloc(&own[1], (size_t)N * K * es) != cudaSuccess ||
            cudaMalloc(&own[2], (size_t)M * N * 4) != cudaSuccess) {
            cudaGetLastError();
            cleanup();
            return fail(MC_ERR_NOMEM, "mc_gemm: device buffers");
        }
        dA = own[0];
        dB = own[1];
        dC = static_cast<float*>(own[2]);
        if (cudaMemcpy(own[0], A, (size_t)M * K * es, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(own[1], B, (size_t)N * K * es, cudaMemcpyHostToDevice) != cudaSuccess) {
            cleanup();
            return fail(MC_ERR_CUDA, "mc_gemm: upload");
        }
    } else if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) {
        return fail(MC_ERR_INVALID, "mc_gemm: device operands must be 16-byte aligned");
    }
    CUtensorMap ma, mb;
    st = tc_map(&ma, dA, es, (uint64_t)K, (uint64_t)M, 0);
    if (!st) st = tc_map(&mb, dB, es, (uint64_t)K, (uint64_t)N, 1, 256);
    if (!st && cudaMalloc(&dstatus, 4) != cudaSuccess) {
        cudaGetLastError();
        st = fail(MC_ERR_NOMEM, "mc_gemm: status word");
    }
    if (st) {
        cleanup();
        return st;
    }
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaMemset(dstatus, 0, 4);
    mc::TcArgs g{};
    g.M = M; g.N = N; g.K = K; g.layer = 0; g.C = dC; g.ldc = N;
    g.status = dstatus;
    g.timeout_ns = 1000ull * 1000ull * 1000ull;
    cudaEventRecord(e0, 0);
    const cudaError_t le = kind == MC_GEMM_TF32 ? tc_launch<mc::TC_TF32, mc::TCE_STORE, 256>(ma, mb, mb, g, 0)
                                                : tc_launch<mc::TC_BF16, mc::TCE_STORE, 256>(ma, mb, mb, g, 0);
    cudaEventRecord(e1, 0);
    cudaError_t e = le != cudaSuccess ? le : cudaEventSynchronize(e1);
    int status = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&status, dstatus, 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && ms) cudaEventElapsedTime(ms, e0, e1);
    if (e == cudaSuccess && !dev) e = cudaMemcpy(C, dC, (size_t)M * N * 4, cudaMemcpyDeviceToHost);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cleanup();
    if (e != cudaSuccess) return fail(MC_ERR_CUDA, "mc_gemm: %s", cudaGetErrorString(e));
    if (status == mc::ST_TIMEOUT) return fail(MC_ERR_TIMEOUT, "mc_gemm: a pipeline wait passed its deadline");
    if (status != 0) return fail(MC_ERR_DEVICE, "mc_gemm: kernel status %d", status);
    return MC_OK;
}


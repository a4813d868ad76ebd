// attention.cu -- split-KV flash-decode attention for one query token.
//
// Replaces the reference's FlashAttentionDecodeBF16 + CombineFlashAttention
// (src/lib/backend/cuda/kernels/flash_attention.cuh:38-184), which runs one
// CTA per (query head, 16-token tile), re-reads every KV head once per query
// head of its GQA group and round-trips fp32 partials through HBM.  Here:
//   * grid = (splits, kv_heads, query-head blocks), cluster = (splits, 1, 1):
//     the splits of one (kv head, block) form a thread-block cluster; one CTA
//     handles up to four query heads of the GQA group, so K/V cross HBM once;
//   * the context's pages are divided evenly over the splits from the device
//     position at run time, so one launch shape (one CUDA graph) serves every
//     position;
//   * a producer warp streams 64-token K and V pages into a two-stage shared
//     ring with 1-D TMA bulk copies (one 16 KB copy per page in the paged
//     layout; 64 row copies in the reference's [capacity, kvh, 128] layout).
//     Pages older than the current position are fetched before
//     griddepcontrol.wait -- only the page receiving this token's K/V waits
//     for the QKV kernel;
//   * each half-warp owns 8 of a page's 64 tokens (16 lanes x 8 dims), with an
//     online softmax in fp32 (exp2 of log2e-scaled scores);
//   * half-warp states merge in shared memory in a fixed order; the splits then
//     merge across the cluster through distributed shared memory, each CTA
//     producing a slice of the outputs -- deterministic, no global partials.
#include <cooperative_groups.h>

#include <algorithm>
#include <cfloat>

#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace q3 {

namespace {

constexpr int kPage = 64;
constexpr int kHd = 128;
constexpr int kWarps = 4;
constexpr int kConsumers = kWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + producer warp
constexpr int kTileBytes = kPage * kHd * 2;  // 16 KB
constexpr int kStages = 2;
constexpr float kLog2e = 1.4426950408889634f;

template <int HG>
struct AttnSmem {
    uint8_t kv[kStages][2][kTileBytes];
    float m[8][HG];
    float l[8][HG];
    float acc[8][HG][kHd];
    float cm[HG];  // this CTA's merged state, read by the cluster
    float cl[HG];
    float cacc[HG][kHd];
    uint64_t full[kStages];
    uint64_t empty[kStages];
};

template <int HG>
__global__ void __launch_bounds__(kThreads, 2) attn_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    AttnSmem<HG>& S = *reinterpret_cast<AttnSmem<HG>*>(smem_raw);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.q_heads / a.kv_heads;
    const int nqb = G / HG;
    const int split = blockIdx.x, kvh = blockIdx.y, qb = blockIdx.z % nqb, qi = blockIdx.z / nqb;
    const bf16* qv = a.q + static_cast<size_t>(qi) * a.q_stride;
    bf16* out = a.out + static_cast<size_t>(qi) * a.out_stride;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], kWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    // The position is final here: every kernel triggers its dependents only
    // after its own griddepcontrol.wait, so when this grid runs, the kernel
    // before the QKV GEMV (which advanced the position) has completed.
    int pos = (a.pos_ptr ? *a.pos_ptr : a.pos_host) + qi;
    if (pos < 0) pos = 0;
    const int n_pages = pos / kPage + 1;
    const int pb = static_cast<int>(static_cast<long long>(split) * n_pages / a.splits);
    const int pe = static_cast<int>(static_cast<long long>(split + 1) * n_pages / a.splits);
    const int np = pe - pb;
    const int live_page = pos / kPage;  // receives this step's K/V from the QKV kernel

    if (warp == kWarps) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            bool waited = false;
            for (int i = 0; i < np; ++i) {
                const int s = i % kStages;
                if (i >= kStages && !mbar_wait(&S.empty[s], ((i / kStages) - 1) & 1, a.err, DEV_TMA_WAIT_TIMEOUT))
                    break;
                const int page = pb + i;
                if (page >= live_page && !waited) {
                    pdl_wait();
                    waited = true;
                }
                if (a.paged) {
                    const size_t base = (static_cast<size_t>(a.page_table[page]) * a.kv_heads + kvh) * kPage * kHd;
                    mbar_arrive_expect_tx(&S.full[s], 2 * kTileBytes);
                    bulk_g2s(S.kv[s][0], a.k + base, kTileBytes, &S.full[s], pol);
                    bulk_g2s(S.kv[s][1], a.v + base, kTileBytes, &S.full[s], pol);
                } else {
                    const int rows = min(kPage, pos + 1 - page * kPage);
                    mbar_arrive_expect_tx(&S.full[s], 2 * rows * kHd * 2);
                    for (int r = 0; r < rows; ++r) {
                        const size_t off = (static_cast<size_t>(page * kPage + r) * a.kv_heads + kvh) * kHd;
                        bulk_g2s(S.kv[s][0] + r * kHd * 2, a.k + off, kHd * 2, &S.full[s], pol);
                        bulk_g2s(S.kv[s][1] + r * kHd * 2, a.v + off, kHd * 2, &S.full[s], pol);
                    }
                }
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        pdl_wait();  // q comes from the QKV kernel
        pdl_trigger();
        const int hw = tid >> 4;  // half-warp 0..7
        const int hl = tid & 15;  // lane within half-warp: dims [8 hl, 8 hl + 8)
        const int qh0 = kvh * G + qb * HG;
        const float qscale = (1.0f / sqrtf(static_cast<float>(kHd))) * kLog2e;

        float q[HG][8];
#pragma unroll
        for (int g = 0; g < HG; ++g) {
            const uint4 v = reinterpret_cast<const uint4*>(qv + static_cast<size_t>(qh0 + g) * kHd)[hl];
            const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                q[g][2 * j] = bf_lo(w[j]);
                q[g][2 * j + 1] = bf_hi(w[j]);
            }
        }
        float m[HG], l[HG], acc[HG][8];
#pragma unroll
        for (int g = 0; g < HG; ++g) {
            m[g] = -INFINITY;
            l[g] = 0.f;
#pragma unroll
            for (int d = 0; d < 8; ++d) acc[g][d] = 0.f;
        }

        bool failed = false;
        for (int i = 0; i < np; ++i) {
            const int s = i % kStages;
            const bool ok = !failed && mbar_wait(&S.full[s], (i / kStages) & 1, a.err, DEV_TMA_WAIT_TIMEOUT);
            failed = failed || !ok;
            if (ok) {
                const int page = pb + i;
                const int valid = min(kPage, pos + 1 - page * kPage);
                const uint4* kt = reinterpret_cast<const uint4*>(S.kv[s][0]);
                const uint4* vt = reinterpret_cast<const uint4*>(S.kv[s][1]);
                float sc[8][HG];
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    const int j = hw + 8 * t;
                    const uint4 kv = kt[j * 16 + hl];
                    const uint32_t* w = reinterpret_cast<const uint32_t*>(&kv);
#pragma unroll
                    for (int g = 0; g < HG; ++g) {
                        float d = 0.f;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            d = fmaf(q[g][2 * e], bf_lo(w[e]), d);
                            d = fmaf(q[g][2 * e + 1], bf_hi(w[e]), d);
                        }
                        d += __shfl_xor_sync(0xffffffffu, d, 8);
                        d += __shfl_xor_sync(0xffffffffu, d, 4);
                        d += __shfl_xor_sync(0xffffffffu, d, 2);
                        d += __shfl_xor_sync(0xffffffffu, d, 1);
                        sc[t][g] = (j < valid) ? d * qscale : -INFINITY;
                    }
                }
#pragma unroll
                for (int g = 0; g < HG; ++g) {
                    float mx = sc[0][g];
#pragma unroll
                    for (int t = 1; t < 8; ++t) mx = fmaxf(mx, sc[t][g]);
                    const float mn = fmaxf(m[g], mx);
                    if (mn == -INFINITY) continue;
                    const float corr = exp2f(m[g] - mn);
                    m[g] = mn;
                    l[g] *= corr;
#pragma unroll
                    for (int d = 0; d < 8; ++d) acc[g][d] *= corr;
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        const float pr = exp2f(sc[t][g] - mn);
                        sc[t][g] = pr;
                        l[g] += pr;
                    }
                }
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    const int j = hw + 8 * t;
                    if (j >= valid) continue;  // rows past the position hold stale data
                    const uint4 vv = vt[j * 16 + hl];
                    const uint32_t* w = reinterpret_cast<const uint32_t*>(&vv);
                    float vf[8];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        vf[2 * e] = bf_lo(w[e]);
                        vf[2 * e + 1] = bf_hi(w[e]);
                    }
#pragma unroll
                    for (int g = 0; g < HG; ++g) {
                        const float pr = (m[g] == -INFINITY) ? 0.f : sc[t][g];
#pragma unroll
                        for (int d = 0; d < 8; ++d) acc[g][d] = fmaf(pr, vf[d], acc[g][d]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[s]);
        }

        // ---- merge the 8 half-warp states (fixed order) into this CTA's state
#pragma unroll
        for (int g = 0; g < HG; ++g) {
            if (hl == 0) {
                S.m[hw][g] = m[g];
                S.l[hw][g] = l[g];
            }
#pragma unroll
            for (int d = 0; d < 8; ++d) S.acc[hw][g][8 * hl + d] = acc[g][d];
        }
        named_bar(1, kConsumers);
        for (int o = tid; o < HG * kHd; o += kConsumers) {
            const int g = o / kHd, d = o % kHd;
            float M = -INFINITY;
            for (int h = 0; h < 8; ++h) M = fmaxf(M, S.m[h][g]);
            float Lsum = 0.f, A = 0.f;
            if (M != -INFINITY) {
                for (int h = 0; h < 8; ++h) {
                    const float f = exp2f(S.m[h][g] - M);
                    Lsum += S.l[h][g] * f;
                    A += S.acc[h][g][d] * f;
                }
            }
            if (a.splits == 1) {
                out[static_cast<size_t>(qh0 + g) * kHd + d] = f2bf(A / Lsum);
            } else {
                S.cacc[g][d] = A;
                if (d == 0) {
                    S.cm[g] = M;
                    S.cl[g] = Lsum;
                }
            }
        }
    }
    if (a.splits == 1) return;

    // ---- merge the splits across the cluster through distributed shared memory
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (warp < kWarps) {
        const int n_out = HG * kHd;
        const int slice = n_out / a.splits;                   // outputs this CTA finishes
        const int tpo = slice >= kConsumers ? 1 : kConsumers / slice;  // threads per output
        const int per_pass = kConsumers / tpo;
        const int sub = tid % tpo;
        for (int base = 0; base < slice; base += per_pass) {
            const int o = split * slice + base + tid / tpo;
            const int g = o / kHd, d = o % kHd;
            float M = -INFINITY;
            for (int sp = 0; sp < a.splits; ++sp) {
                const AttnSmem<HG>* R = cluster.map_shared_rank(&S, sp);
                M = fmaxf(M, R->cm[g]);
            }
            float Lsum = 0.f, A = 0.f;
            for (int sp = sub; sp < a.splits; sp += tpo) {
                const AttnSmem<HG>* R = cluster.map_shared_rank(&S, sp);
                const float ms = R->cm[g];
                if (ms == -INFINITY) continue;
                const float f = exp2f(ms - M);
                Lsum += R->cl[g] * f;
                A += R->cacc[g][d] * f;
            }
            // tpo consecutive lanes hold parts of one output: reduce in a fixed tree
            for (int off = tpo >> 1; off > 0; off >>= 1) {
                Lsum += __shfl_xor_sync(0xffffffffu, Lsum, off);
                A += __shfl_xor_sync(0xffffffffu, A, off);
            }
            if (sub == 0) {
                const int qh = kvh * G + qb * HG + g;
                out[static_cast<size_t>(qh) * kHd + d] = f2bf(A / Lsum);
            }
        }
    }
    cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
}

int heads_per_cta(int G) { return G >= 4 ? 4 : G; }

template <int HG>
cudaError_t launch_hg(const AttnArgs& a, cudaStream_t s, bool pdl, int nqb) {
    auto* fn = attn_kernel<HG>;
    const size_t smem = sizeof(AttnSmem<HG>);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.splits, a.kv_heads, nqb * (a.n_queries > 1 ? a.n_queries : 1));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int n = 0;
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = a.splits;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
    if (pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, fn, a);
}

template <int HG>
cudaError_t configure_hg() {
    cudaError_t e = cudaFuncSetAttribute(attn_kernel<HG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(sizeof(AttnSmem<HG>)));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_kernel<HG>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    return e;
}

int g_max_cluster = 0;  // largest split cluster that can be resident (16 or 8)

}  // namespace

cudaError_t configure_attention_kernels() {
    cudaError_t e = configure_hg<1>();
    if (e == cudaSuccess) e = configure_hg<2>();
    if (e == cudaSuccess) e = configure_hg<4>();
    if (e != cudaSuccess) return e;
    // Can a 16-CTA cluster of the largest variant be resident at all?
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(16, 1, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = sizeof(AttnSmem<4>);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 16;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, attn_kernel<4>, &cfg) == cudaSuccess && clusters > 0)
        g_max_cluster = 16;
    else
        g_max_cluster = 8;
    cudaGetLastError();
    return cudaSuccess;
}

// Splits per (kv head, block): a power of two forming one cluster, at most 16
// (8 where a 16-CTA cluster cannot be resident), and no more than the pages.
int attn_splits(int kv_heads, int max_pos, int page_size, int sms) {
    (void)page_size;
    (void)kv_heads;
    (void)sms;
    const int max_pages = max_pos / kPage + 1;
    const int cap = g_max_cluster > 0 ? g_max_cluster : 8;
    int s = 1;
    while (s * 2 <= cap && s * 2 <= max_pages) s *= 2;
    return s;
}

size_t attn_workspace_bytes(int q_heads, int kv_heads, int splits) {
    // Splits merge through distributed shared memory: no global scratch.
    (void)q_heads;
    (void)kv_heads;
    (void)splits;
    return 256;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl) {
    const int G = a.q_heads / a.kv_heads;
    if (a.q_heads % a.kv_heads != 0 || !(G == 1 || G == 2 || G == 4 || G == 8)) return cudaErrorInvalidValue;
    if (a.splits < 1 || a.splits > 16 || (a.splits & (a.splits - 1)) != 0) return cudaErrorInvalidValue;
    if (a.n_queries > 1 && static_cast<long long>(a.n_queries) * (G / heads_per_cta(G)) > 65535)
        return cudaErrorInvalidValue;
    const int HG = heads_per_cta(G);
    const int nqb = G / HG;
    switch (HG) {
        case 1: return launch_hg<1>(a, s, pdl, nqb);
        case 2: return launch_hg<2>(a, s, pdl, nqb);
        default: return launch_hg<4>(a, s, pdl, nqb);
    }
}

}  // namespace q3

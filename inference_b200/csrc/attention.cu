// attention.cu -- split-KV flash-decode attention for one query token.
//
// Replaces the reference's FlashAttentionDecodeBF16 + CombineFlashAttention
// (src/lib/backend/cuda/kernels/flash_attention.cuh:38-184), which runs one
// CTA per (query head, 16-token tile) and so re-reads every KV head once per
// query head of its GQA group.  Here one CTA handles a (kv head, page range)
// pair for up to four query heads of the group, so K/V cross HBM once:
//   * grid = (splits, kv_heads, query-head blocks); the context's pages are
//     divided evenly over the splits at run time from the device position, so
//     one launch shape (and one CUDA graph) serves every position;
//   * a producer warp streams 64-token K and V pages into a two-stage shared
//     memory ring with 1-D TMA bulk copies (one 16 KB copy per page in the
//     paged layout; 64 row copies in the reference's [capacity, kvh, 128]
//     layout);
//   * each half-warp owns 8 of a page's 64 tokens, 16 lanes x 8 dims per
//     token, an online softmax in fp32 (exp2 of log2e-scaled scores);
//   * half-warp states merge in shared memory in a fixed order; splits merge
//     in the last CTA of each (kv head, block) -- deterministic.
#include <algorithm>
#include <cfloat>

#include "kernels.cuh"

namespace q3 {

namespace {

constexpr int kPage = 64;
constexpr int kHd = 128;
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32 + 32;  // + producer warp
constexpr int kTileBytes = kPage * kHd * 2;  // 16 KB
constexpr int kStages = 2;
constexpr float kLog2e = 1.4426950408889634f;

template <int HG>
struct AttnSmem {
    uint8_t kv[kStages][2][kTileBytes];
    float m[8][HG];
    float l[8][HG];
    float acc[8][HG][kHd];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint32_t last;
};

// HG = query heads handled per CTA (<= 4); G = query heads per kv head.
template <int HG>
__global__ void __launch_bounds__(kThreads, 2) attn_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    AttnSmem<HG>& S = *reinterpret_cast<AttnSmem<HG>*>(smem_raw);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, kvh = blockIdx.y, qb = blockIdx.z;
    const int G = a.q_heads / a.kv_heads;
    const int nqb = gridDim.z;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], kWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();
    pdl_trigger();
    // K/V pages and the position come from earlier kernels.
    pdl_wait();

    int pos = a.pos_ptr ? *a.pos_ptr : a.pos_host;
    if (pos < 0) pos = 0;
    const int n_pages = pos / kPage + 1;
    const int pb = static_cast<int>(static_cast<long long>(split) * n_pages / a.splits);
    const int pe = static_cast<int>(static_cast<long long>(split + 1) * n_pages / a.splits);
    const int np = pe - pb;

    // ------------------------------------------------------------ producer
    if (warp == kWarps) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            for (int i = 0; i < np; ++i) {
                const int s = i % kStages;
                if (i >= kStages && !mbar_wait(&S.empty[s], ((i / kStages) - 1) & 1, a.err, DEV_TMA_WAIT_TIMEOUT))
                    break;
                const int page = pb + i;
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
        return;
    }

    // ------------------------------------------------------------ consumers
    const int hw = tid >> 4;        // half-warp 0..7
    const int hl = tid & 15;        // lane within half-warp: dims [8 hl, 8 hl + 8)
    const int qh0 = kvh * G + qb * HG;
    const float qscale = (1.0f / sqrtf(static_cast<float>(kHd))) * kLog2e;

    float q[HG][8];
#pragma unroll
    for (int g = 0; g < HG; ++g) {
        const uint4 v = reinterpret_cast<const uint4*>(a.q + static_cast<size_t>(qh0 + g) * kHd)[hl];
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
#pragma unroll
                for (int g = 0; g < HG; ++g) {
                    const uint32_t* w = reinterpret_cast<const uint32_t*>(&kv);
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

    // ---- merge the 8 half-warp states (fixed order)
#pragma unroll
    for (int g = 0; g < HG; ++g) {
        if (hl == 0) {
            S.m[hw][g] = m[g];
            S.l[hw][g] = l[g];
        }
#pragma unroll
        for (int d = 0; d < 8; ++d) S.acc[hw][g][8 * hl + d] = acc[g][d];
    }
    named_bar(1, kWarps * 32);

    const int n_out = HG * kHd;
    float* part_ml = a.part_ml + ((static_cast<size_t>(kvh) * nqb + qb) * a.splits + split) * HG * 2;
    float* part_acc = a.part_acc + ((static_cast<size_t>(kvh) * nqb + qb) * a.splits + split) * HG * kHd;
    for (int o = tid; o < n_out; o += kWarps * 32) {
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
            a.out[static_cast<size_t>(qh0 + g) * kHd + d] = f2bf(A / Lsum);
        } else {
            part_acc[g * kHd + d] = A;
            if (d == 0) {
                part_ml[2 * g] = M;
                part_ml[2 * g + 1] = Lsum;
            }
        }
    }
    if (a.splits == 1) return;

    // ---- last CTA of this (kv head, block) merges the splits in order
    __threadfence();
    named_bar(1, kWarps * 32);
    if (tid == 0) {
        const uint32_t old = atomicAdd(&a.counters[kvh * nqb + qb], 1u);
        S.last = (old == static_cast<uint32_t>(a.splits - 1)) ? 1u : 0u;
    }
    named_bar(1, kWarps * 32);
    if (!S.last) return;
    __threadfence();
    const float* ml0 = a.part_ml + (static_cast<size_t>(kvh) * nqb + qb) * a.splits * HG * 2;
    const float* acc0 = a.part_acc + (static_cast<size_t>(kvh) * nqb + qb) * a.splits * HG * kHd;
    for (int o = tid; o < n_out; o += kWarps * 32) {
        const int g = o / kHd, d = o % kHd;
        float M = -INFINITY;
        for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, __ldcg(ml0 + (sp * HG + g) * 2));
        float Lsum = 0.f, A = 0.f;
        for (int sp = 0; sp < a.splits; ++sp) {
            const float ms = __ldcg(ml0 + (sp * HG + g) * 2);
            if (ms == -INFINITY) continue;
            const float f = exp2f(ms - M);
            Lsum += __ldcg(ml0 + (sp * HG + g) * 2 + 1) * f;
            A += __ldcg(acc0 + (sp * HG + g) * kHd + d) * f;
        }
        a.out[static_cast<size_t>(qh0 + g) * kHd + d] = f2bf(A / Lsum);
    }
    if (tid == 0) a.counters[kvh * nqb + qb] = 0u;
}

int heads_per_cta(int G) { return G >= 4 ? 4 : G; }

template <int HG>
cudaError_t launch_hg(const AttnArgs& a, cudaStream_t s, bool pdl, int nqb) {
    auto* fn = attn_kernel<HG>;
    const size_t smem = sizeof(AttnSmem<HG>);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.splits, a.kv_heads, nqb);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, a);
}

}  // namespace

cudaError_t configure_attention_kernels() {
    cudaError_t e = cudaFuncSetAttribute(attn_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(sizeof(AttnSmem<1>)));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(sizeof(AttnSmem<2>)));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(sizeof(AttnSmem<4>)));
    return e;
}

int attn_splits(int kv_heads, int max_pos, int page_size, int sms) {
    (void)page_size;
    const int max_pages = max_pos / kPage + 1;
    const int want = (2 * sms + kv_heads - 1) / kv_heads;
    return std::max(1, std::min(want, max_pages));
}

size_t attn_workspace_bytes(int q_heads, int kv_heads, int splits) {
    const int G = q_heads / kv_heads;
    const int HG = heads_per_cta(G);
    const int nqb = G / HG;
    const size_t slots = static_cast<size_t>(kv_heads) * nqb * splits * HG;
    // part_ml | part_acc | counters
    return slots * 2 * sizeof(float) + slots * kHd * sizeof(float) + static_cast<size_t>(kv_heads) * nqb * 4 + 256;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl) {
    const int G = a.q_heads / a.kv_heads;
    if (a.q_heads % a.kv_heads != 0 || !(G == 1 || G == 2 || G == 4 || G == 8)) return cudaErrorInvalidValue;
    const int HG = heads_per_cta(G);
    const int nqb = G / HG;
    switch (HG) {
        case 1: return launch_hg<1>(a, s, pdl, nqb);
        case 2: return launch_hg<2>(a, s, pdl, nqb);
        default: return launch_hg<4>(a, s, pdl, nqb);
    }
}

}  // namespace q3

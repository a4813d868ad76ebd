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
//   * each consumer warp owns 16 of a page's 64 tokens and does its math on the
//     tensor cores (mma.sync: S = Q K^T, online softmax in fp32 on the
//     fragments, O += P V with P in BF16 hi + lo parts);
//   * warp states merge in shared memory in a fixed order; each split then
//     pushes its state of every output slice into the shared memory of the
//     cluster CTA that owns the slice (distributed shared memory stores), and
//     after one cluster barrier every CTA merges its slice locally in a fixed
//     split order -- deterministic, no global partials.

#include <algorithm>
#include <cfloat>

#include "kernels.cuh"

namespace q3 {

namespace {

constexpr int kPage = 64;
constexpr int kHd = 128;
constexpr int kWarps = 4;
constexpr int kConsumers = kWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + producer warp
constexpr int kTileBytes = kPage * kHd * 2;  // 16 KB
constexpr float kLog2e = 1.4426950408889634f;

// K/V pages in flight per CTA (ring stages).  Deeper rings (3 at two CTAs per
// SM, 4 at one) were measured on B200 and gained nothing at Qwen3-8B context
// 2300 or Qwen3-0.6B context 8192: the split count, not the ring, bounds the
// pages a CTA streams.
constexpr int kStages = 2;

template <int HG>
struct AttnSmem {
    uint8_t kv[kStages][2][kTileBytes];
    float m[kWarps][HG];  // per consumer warp: running max, sum, accumulators
    float l[kWarps][HG];
    float acc[kWarps][HG][kHd];
    // split merge: CTA `o` of the cluster owns outputs [o * slice, (o + 1) * slice) of the
    // HG x 128 (slice = HG * 128 / splits); every split pushes into the owner's shared
    // memory its running max and sum per head, and its accumulators of those outputs,
    // at [split][...] -- splits x slice = HG x 128 accumulators in all
    float rx_m[16][HG];
    float rx_l[16][HG];
    float rx_acc[HG * kHd];
    bf16 qn[HG][kHd];  // normalised, rotated q heads (fused q/k norm)
    bf16 kn[kHd];      // normalised, rotated key row of the position
    uint64_t full[kStages];
    uint64_t empty[kStages];
};

__device__ __forceinline__ void ldmatrix_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldmatrix_x4_trans(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
// One 128-wide head: RMSNorm (weights nw) then RoPE at `pos`, rounded once
// (qk_norm_rope.cuh:14-90); a warp, lane l holding dims l, l + 32, l + 64,
// l + 96.  The weights and the RoPE row do not depend on earlier kernels and
// are loaded (load) before griddepcontrol.wait; apply runs on the head after.
struct NormRope {
    float w[4], c[2], s[2];
    __device__ __forceinline__ void load(const bf16* nw, const float* cs, const float* sn, int pos, int lane) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int i = lane + 32 * j;
            w[j] = bf2f(nw[i]);
            w[j + 2] = bf2f(nw[i + 64]);
            c[j] = cs[static_cast<size_t>(pos) * 64 + i];
            s[j] = sn[static_cast<size_t>(pos) * 64 + i];
        }
    }
    __device__ __forceinline__ void apply(const bf16* src, float eps, bf16* dst, int lane) const {
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = bf2f(src[lane + 32 * j]);
        const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
        const float scale = 1.0f / sqrtf(ss / 128.0f + eps);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int i = lane + 32 * j;
            const float x = v[j] * w[j] * scale;
            const float y = v[j + 2] * w[j + 2] * scale;
            dst[i] = f2bf(x * c[j] - y * s[j]);
            dst[i + 64] = f2bf(y * c[j] + x * s[j]);
        }
    }
};

// D (16 x 8, fp32) += A (16 x 16, BF16, row) B (16 x 8, BF16, col)
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void fence_proxy_async_cta() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int HG>
__global__ void __launch_bounds__(kThreads, 2) attn_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    AttnSmem<HG>& S = *reinterpret_cast<AttnSmem<HG>*>(smem_raw);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool tracing = a.trace.buf != nullptr;
    // trace marks (thread 0, a consumer): start, dependency released, q/k norm done,
    // page loop done
    unsigned long long tr_t0 = 0, tr_c0 = 0, tr_c1 = 0, tr_cq = 0, tr_cp = 0, tr_cs = 0;
    if (tracing && tid == 0) {
        tr_t0 = globaltimer_ns();
        tr_c0 = clock64();
    }
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
    // Every CTA of the cluster must be running before any pushes into its shared
    // memory: arrive now, wait just before the first push (long after all started).
    if (a.splits > 1) cluster_arrive_relaxed();

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
        // Tensor cores (mma.sync m16n8k16, BF16 -> FP32): warp w owns tokens
        // 16w .. 16w + 15 of each 64-token page.  S = Q K^T with Q as the A
        // operand (rows = the CTA's HG query heads, padded to 16 with zeros),
        // online softmax on the accumulator fragments, then O += P V with P
        // reused as the A operand, split into BF16 hi + lo parts so the
        // probabilities keep ~16 bits.  Each warp first XOR-swizzles its own
        // 16 rows of the K and V tiles in place (16-byte chunk c of row r to
        // c ^ (r & 7)), so every ldmatrix phase hits 8 distinct bank groups.
        const bool fused = a.k_raw != nullptr;
        const bool has_live = fused && live_page >= pb && live_page < pe;
        NormRope nq, nk;
        if (fused) {
            nq.load(a.q_norm, a.rope_cos, a.rope_sin, pos, lane);
            if (warp == kWarps - 1 && has_live) nk.load(a.k_norm, a.rope_cos, a.rope_sin, pos, lane);
        }
        pdl_wait();  // q comes from the QKV kernel
        pdl_trigger();
        if (tracing && tid == 0) tr_c1 = clock64();
        const int g = lane >> 2, t4 = lane & 3;  // fragment row (query head) and column pair
        const int qh0 = kvh * G + qb * HG;
        const float qscale = (1.0f / sqrtf(static_cast<float>(kHd))) * kLog2e;
        if (fused) {
            // q/k norm + RoPE of this step: warp w < HG takes q head qh0 + w, the last
            // warp (after its q head) the key row when this split holds the live page
            if (warp < HG) nq.apply(qv + static_cast<size_t>(qh0 + warp) * kHd, a.eps, S.qn[warp], lane);
            if (warp == kWarps - 1 && has_live) {
                nk.apply(a.k_raw + static_cast<size_t>(kvh) * kHd, a.eps, S.kn, lane);
                if (qb == 0) {
                    __syncwarp();
                    bf16* slot = const_cast<bf16*>(a.k) +
                                 ((static_cast<size_t>(a.page_table[live_page]) * a.kv_heads + kvh) * kPage +
                                  pos % kPage) * kHd;
                    if (lane < 16) reinterpret_cast<uint4*>(slot)[lane] = reinterpret_cast<const uint4*>(S.kn)[lane];
                }
            }
            named_bar(1, kConsumers);
        }

        if (tracing && tid == 0) tr_cq = clock64();
        uint32_t qa[8][2];  // A fragments of q: rows g (dims 16kk + 2t4, +1) and (+8); rows 8-15 are zero
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            qa[kk][0] = qa[kk][1] = 0u;
            if (g < HG) {
                const uint32_t* qr = fused ? reinterpret_cast<const uint32_t*>(S.qn[g])
                                           : reinterpret_cast<const uint32_t*>(qv + static_cast<size_t>(qh0 + g) * kHd);
                qa[kk][0] = qr[kk * 8 + t4];
                qa[kk][1] = qr[kk * 8 + 4 + t4];
            }
        }
        float o[16][4];
#pragma unroll
        for (int d = 0; d < 16; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
        float m_run = -INFINITY, l_run = 0.f;  // row g: running max (log2 units), this lane's partial sum

        bool failed = false;
        for (int i = 0; i < np; ++i) {
            const int s = i % kStages;
            const bool ok = !failed && mbar_wait(&S.full[s], (i / kStages) & 1, a.err, DEV_TMA_WAIT_TIMEOUT);
            failed = failed || !ok;
            if (ok) {
                const int page = pb + i;
                const int valid = min(kPage, pos + 1 - page * kPage);
                uint8_t* kt = S.kv[s][0];
                uint8_t* vt = S.kv[s][1];
                if (has_live && page == live_page && warp == (pos % kPage) / 16) {
                    // this step's key row: the cache slot still holds the raw row (or older data)
                    if (lane < 16)
                        reinterpret_cast<uint4*>(kt + (pos % kPage) * 256)[lane] =
                            reinterpret_cast<const uint4*>(S.kn)[lane];
                    __syncwarp();
                }
                // ---- swizzle this warp's rows in place; rows past the position become zeros in V
#pragma unroll
                for (int tile = 0; tile < 2; ++tile) {
                    uint8_t* base = tile ? vt : kt;
                    const int c = lane & 15;
                    uint4 rr[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int r = warp * 16 + (lane >> 4) + 2 * j;
                        rr[j] = *reinterpret_cast<const uint4*>(base + r * 256 + c * 16);
                    }
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int r = warp * 16 + (lane >> 4) + 2 * j;
                        *reinterpret_cast<uint4*>(base + r * 256 + (c ^ (r & 7)) * 16) =
                            (tile == 0 || r < valid) ? rr[j] : make_uint4(0u, 0u, 0u, 0u);
                    }
                    __syncwarp();
                }
                // ---- S = Q K^T for this warp's two 8-token n-tiles
                float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                {
                    const int q = lane >> 3, r8 = lane & 7;
                    const int row = warp * 16 + (q >> 1) * 8 + r8;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const int chunk = kk * 2 + (q & 1);
                        uint32_t b0, b1, b2, b3;
                        ldmatrix_x4(kt + row * 256 + ((chunk ^ (row & 7)) * 16), b0, b1, b2, b3);
                        mma_bf16_16816(sc[0], qa[kk][0], 0u, qa[kk][1], 0u, b0, b1);
                        mma_bf16_16816(sc[1], qa[kk][0], 0u, qa[kk][1], 0u, b2, b3);
                    }
                }
                // ---- online softmax on row g (tokens 16w + 8jn + 2t4 + e)
                float mx = -INFINITY;
#pragma unroll
                for (int jn = 0; jn < 2; ++jn)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int tok = warp * 16 + jn * 8 + 2 * t4 + e;
                        sc[jn][e] = tok < valid ? sc[jn][e] * qscale : -INFINITY;
                        mx = fmaxf(mx, sc[jn][e]);
                    }
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float m_new = fmaxf(m_run, mx);
                float p[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
                if (m_new != -INFINITY) {
                    const float corr = exp2f(m_run - m_new);
                    m_run = m_new;
                    l_run *= corr;
#pragma unroll
                    for (int d = 0; d < 16; ++d) {
                        o[d][0] *= corr;
                        o[d][1] *= corr;
                    }
#pragma unroll
                    for (int jn = 0; jn < 2; ++jn)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            p[jn][e] = exp2f(sc[jn][e] - m_new);
                            l_run += p[jn][e];
                        }
                }
                // ---- O += P V: P rows g, k = the warp's 16 tokens (hi + lo BF16 parts)
                uint32_t ph[2], pl[2];
#pragma unroll
                for (int jn = 0; jn < 2; ++jn) {
                    const bf16 h0 = f2bf(p[jn][0]), h1 = f2bf(p[jn][1]);
                    const bf16 l0 = f2bf(p[jn][0] - bf2f(h0)), l1 = f2bf(p[jn][1] - bf2f(h1));
                    ph[jn] = static_cast<uint32_t>(__bfloat16_as_ushort(h0)) |
                             (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
                    pl[jn] = static_cast<uint32_t>(__bfloat16_as_ushort(l0)) |
                             (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16);
                }
                {
                    const int q = lane >> 3, r8 = lane & 7;
                    const int row = warp * 16 + (q & 1) * 8 + r8;
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int chunk = 2 * e + (q >> 1);
                        uint32_t b0, b1, b2, b3;
                        ldmatrix_x4_trans(vt + row * 256 + ((chunk ^ (row & 7)) * 16), b0, b1, b2, b3);
                        mma_bf16_16816(o[2 * e], ph[0], 0u, ph[1], 0u, b0, b1);
                        mma_bf16_16816(o[2 * e], pl[0], 0u, pl[1], 0u, b0, b1);
                        mma_bf16_16816(o[2 * e + 1], ph[0], 0u, ph[1], 0u, b2, b3);
                        mma_bf16_16816(o[2 * e + 1], pl[0], 0u, pl[1], 0u, b2, b3);
                    }
                }
            }
            // the slot is refilled by the async proxy after this warp's generic-proxy
            // writes to it (the swizzle, the patched rows): order them first
            if (i + kStages < np) fence_proxy_async_cta();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[s]);
        }
        l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
        l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
        if (tracing && tid == 0) tr_cp = clock64();

        // ---- merge the 4 warp states (fixed order) into this CTA's state
        if (g < HG) {
            if (t4 == 0) {
                S.m[warp][g] = m_run;
                S.l[warp][g] = l_run;
            }
#pragma unroll
            for (int d = 0; d < 16; ++d) {
                S.acc[warp][g][8 * d + 2 * t4] = o[d][0];
                S.acc[warp][g][8 * d + 2 * t4 + 1] = o[d][1];
            }
        }
        named_bar(1, kConsumers);
        if (a.splits > 1) cluster_wait();  // phase 0: every CTA of the cluster has started
        const int slice = HG * kHd / a.splits;  // outputs each CTA of the cluster finishes
        for (int oi = tid; oi < HG * kHd; oi += kConsumers) {
            const int gg = oi / kHd, d = oi % kHd;
            float M = -INFINITY;
            for (int h = 0; h < kWarps; ++h) M = fmaxf(M, S.m[h][gg]);
            float Lsum = 0.f, A = 0.f;
            if (M != -INFINITY) {
                for (int h = 0; h < kWarps; ++h) {
                    const float f = exp2f(S.m[h][gg] - M);
                    Lsum += S.l[h][gg] * f;
                    A += S.acc[h][gg][d] * f;
                }
            }
            if (a.splits == 1) {
                out[static_cast<size_t>(qh0 + gg) * kHd + d] = f2bf(A / Lsum);
            } else {
                // push this split's state of output oi into its owner's shared memory
                const int owner = oi / slice, j = oi % slice;
                AttnSmem<HG>* R = static_cast<AttnSmem<HG>*>(map_cluster_rank(&S, owner));
                R->rx_acc[split * slice + j] = A;
                if (j == 0 || d == 0) {  // the first output of each (owner, head) pair carries m, l
                    R->rx_m[split][gg] = M;
                    R->rx_l[split][gg] = Lsum;
                }
            }
        }
    }
    if (a.splits == 1) return;

    // ---- phase 1: every split's pushes are in (release / acquire), then each CTA
    // finishes its own outputs from its shared memory; no CTA reads a peer's memory,
    // so none has to outlive the barrier for the others
    __syncwarp();  // the cluster barrier instructions below are warp-aligned
    if (warp == kWarps) cluster_wait();  // the producer warp's phase-0 wait
    cluster_arrive_release();
    cluster_wait();
    if (tracing && tid == 0) tr_cs = clock64();
    if (warp < kWarps) {
        const int slice = HG * kHd / a.splits;
        for (int j = tid; j < slice; j += kConsumers) {
            const int o = split * slice + j;
            const int g = o / kHd, d = o % kHd;
            float M = -INFINITY;
            for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, S.rx_m[sp][g]);
            float Lsum = 0.f, A = 0.f;
            for (int sp = 0; sp < a.splits; ++sp) {  // fixed split order
                const float ms = S.rx_m[sp][g];
                if (ms == -INFINITY) continue;
                const float f = exp2f(ms - M);
                Lsum += S.rx_l[sp][g] * f;
                A += S.rx_acc[sp * slice + j] * f;
            }
            const int qh = kvh * G + qb * HG + g;
            out[static_cast<size_t>(qh) * kHd + d] = f2bf(A / Lsum);
        }
    }
    const int cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    if (tracing && tid == 0 && cta < a.trace.ctas) {
        unsigned long long* t = a.trace.buf + (static_cast<size_t>(cta) * a.trace.phases + a.trace.phase) * kTraceWords;
        const unsigned long long c4 = clock64();
        t[0] = tr_t0;
        t[1] = globaltimer_ns();
        t[2] = tr_c0;
        t[3] = c4;
        t[4] = tr_c1 - tr_c0;
        t[5] = tr_cq - tr_c1;  // q/k RMSNorm + RoPE (the "prologue")
        t[6] = tr_cp - tr_cq;  // page loop
        t[7] = c4 - tr_cp;     // warp merge, cluster merge (the "epilogue")
        t[9] = tr_cs ? c4 - tr_cs : 0;  // of which: after the cluster barrier (the owner's merge)
        t[8] = sm_id();
    }
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
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_kernel<HG>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    return e;
}

// Clusters of `splits` CTAs of attn_kernel<HG> that can be resident at once.
template <int HG>
int max_clusters(int splits) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(splits, 1, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = sizeof(AttnSmem<HG>);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, attn_kernel<HG>, &cfg) != cudaSuccess) clusters = 0;
    cudaGetLastError();
    return clusters;
}

int g_max_cluster = 0;  // largest split cluster that can be resident (16 or 8)

}  // namespace

cudaError_t configure_attention_kernels() {
    cudaError_t e = configure_hg<1>();
    if (e == cudaSuccess) e = configure_hg<2>();
    if (e == cudaSuccess) e = configure_hg<4>();
    if (e != cudaSuccess) return e;
    // Can a 16-CTA cluster of the largest variant be resident at all?
    g_max_cluster = max_clusters<4>(16) > 0 ? 16 : 8;
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

// attention.cu -- split-KV flash-decode attention for one query token.
//
// Replaces the reference's FlashAttentionDecodeBF16 + CombineFlashAttention
// (src/lib/backend/cuda/kernels/flash_attention.cuh:38-184), which runs one
// CTA per (query head, 16-token tile), re-reads every KV head once per query
// head of its GQA group and round-trips fp32 partials through HBM.  Here:
//   * grid = (splits, kv_heads, query-head blocks), cluster = (splits, 1, 1):
//     the splits of one (kv head, block) form a thread-block cluster; one CTA
//     handles up to eight query heads of the GQA group, so K/V cross HBM once;
//   * the context's pages are divided evenly over the splits from the device
//     position at run time, so one launch shape (one CUDA graph) serves every
//     position;
//   * a producer warp streams 64-token K and V pages into a four-stage shared
//     ring with 3-D TMA tensor copies (128-byte swizzle: two 64-column boxes
//     per 64-row tile, from the paged pool or the reference's [capacity, kvh,
//     128] layout alike), so ldmatrix reads conflict-free rows with no pass
//     over the tile first; pages older than the current position are fetched
//     before griddepcontrol.wait -- only the page receiving this token's K/V
//     waits for the QKV kernel;
//   * each consumer warp owns 16 of a page's 64 tokens and does its math on the
//     tensor cores with the tokens as the 16-row M dimension and the CTA's
//     query heads (up to 8) as N: S^T = K Q^T, online softmax in fp32 on the
//     fragments, O^T += V^T P^T with P in BF16 hi + lo parts, transposed from
//     the accumulator layout into the B operand by movmatrix;
//   * warp states merge in shared memory in a fixed order; each split then
//     pushes its state of every output slice into the shared memory of the
//     cluster CTA that owns the slice (distributed shared memory stores), and
//     after one cluster barrier every CTA merges its slice locally in a fixed
//     split order -- deterministic, no global partials.

#include <algorithm>
#include <cfloat>
#include <cstddef>

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

// K/V pages in flight per CTA (ring stages).  Four 32 KB stages also make the
// CTA too large for two to share an SM: the 16-CTA clusters would otherwise be
// packed two CTAs per SM onto half the SMs (measured on B200: 128 CTAs on 64
// SMs), leaving the other half idle while attention runs.
constexpr int kStages = 4;

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
    float fw[kWarps][HG];  // per head: each warp's weight in the CTA's merge, the max, the sum
    float cm[HG];
    float cl[HG];
    float rf[16][HG];      // per head: each split's weight in the owner's merge, the sum
    float rl[HG];
    alignas(16) bf16 qn[HG][kHd];  // normalised, rotated q heads (fused q/k norm)
    alignas(16) bf16 kn[kHd];      // normalised, rotated key row of the position (read as uint4)
    uint64_t full[kStages];
    uint64_t empty[kStages];
};

// The K/V ring and the key row are read and written as 16-byte vectors.
template <int HG>
constexpr bool smem_aligned() {
    return offsetof(AttnSmem<HG>, kv) % 16 == 0 && offsetof(AttnSmem<HG>, qn) % 16 == 0 &&
           offsetof(AttnSmem<HG>, kn) % 16 == 0 && offsetof(AttnSmem<HG>, full) % 8 == 0;
}
static_assert(smem_aligned<1>() && smem_aligned<2>() && smem_aligned<4>() && smem_aligned<8>(),
              "attention shared-memory layout");

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
// 8 x 8 BF16 matrix held in the fragment layout (lane 4r + c: row r, columns
// 2c, 2c + 1) -> its transpose in the same layout.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_bf2(bf16 lo, bf16 hi) {
    return static_cast<uint32_t>(__bfloat16_as_ushort(lo)) | (static_cast<uint32_t>(__bfloat16_as_ushort(hi)) << 16);
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

// Byte offset of 16-byte column chunk `chunk` (0..15) of row `row` in a 64 x 128
// BF16 tile as two 64-column boxes loaded with the 128-byte swizzle: box
// chunk >> 3 at 8 KB steps, rows of 128 bytes, chunk c of row r at c ^ (r & 7).
__device__ __forceinline__ int tile_off(int row, int chunk) {
    return (chunk >> 3) * 8192 + row * 128 + (((chunk & 7) ^ (row & 7)) << 4);
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

template <int HG>
__global__ void __launch_bounds__(kThreads, 1) attn_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // the swizzled TMA boxes want 1024-byte aligned destinations
    uint8_t* smem_base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    AttnSmem<HG>& S = *reinterpret_cast<AttnSmem<HG>*>(smem_base);

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
    int pos = a.row_pos ? a.row_pos[qi] : (a.pos_ptr ? *a.pos_ptr : a.pos_host) + qi;
    if (pos < 0) pos = 0;
    const int32_t* page_table = a.row_pos ? a.page_table + static_cast<size_t>(qi) * a.pt_stride : a.page_table;
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
                // paged: (column, row, physical page x kv heads + head); flat: (column, head, position)
                const int y = a.paged ? 0 : kvh;
                const int z = a.paged ? page_table[page] * a.kv_heads + kvh : page * kPage;
                mbar_arrive_expect_tx(&S.full[s], 2 * kTileBytes);
                tma_load_3d(S.kv[s][0], &a.tk, 0, y, z, &S.full[s], pol);
                tma_load_3d(S.kv[s][0] + kTileBytes / 2, &a.tk, 64, y, z, &S.full[s], pol);
                tma_load_3d(S.kv[s][1], &a.tv, 0, y, z, &S.full[s], pol);
                tma_load_3d(S.kv[s][1] + kTileBytes / 2, &a.tv, 64, y, z, &S.full[s], pol);
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        // Tensor cores (mma.sync m16n8k16, BF16 -> FP32): warp w owns tokens
        // 16w .. 16w + 15 of each 64-token page, the M dimension.  S^T = K Q^T
        // with the warp's key rows as the A operand (ldmatrix) and the CTA's HG
        // query heads as N (columns past HG are zero), online softmax on the
        // accumulator fragments, then O^T += V^T P^T with V^T from
        // ldmatrix.trans and P, split into BF16 hi + lo parts so the
        // probabilities keep ~16 bits, moved into the B operand by movmatrix.
        // The tiles arrive 128-byte swizzled by the TMA (16-byte chunk c of row
        // r at c ^ (r & 7), tile_off), so every ldmatrix phase hits 8 distinct
        // bank groups.
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
            for (int h = warp; h < HG; h += kWarps) nq.apply(qv + static_cast<size_t>(qh0 + h) * kHd, a.eps, S.qn[h], lane);
            if (warp == kWarps - 1 && has_live) {
                nk.apply(a.k_raw + static_cast<size_t>(kvh) * kHd, a.eps, S.kn, lane);
                if (qb == 0) {
                    __syncwarp();
                    bf16* slot = const_cast<bf16*>(a.k) +
                                 ((static_cast<size_t>(page_table[live_page]) * a.kv_heads + kvh) * kPage +
                                  pos % kPage) * kHd;
                    if (lane < 16) reinterpret_cast<uint4*>(slot)[lane] = reinterpret_cast<const uint4*>(S.kn)[lane];
                }
            }
            named_bar(1, kConsumers);
        }

        if (tracing && tid == 0) tr_cq = clock64();
        // B fragments of Q^T (k = dims 16kk + 2t4, +1 and + 8, n = query head g; heads >= HG are zero)
        uint32_t qb[8][2];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            qb[kk][0] = qb[kk][1] = 0u;
            if (g < HG) {
                const uint32_t* qr = fused ? reinterpret_cast<const uint32_t*>(S.qn[g])
                                           : reinterpret_cast<const uint32_t*>(qv + static_cast<size_t>(qh0 + g) * kHd);
                qb[kk][0] = qr[kk * 8 + t4];
                qb[kk][1] = qr[kk * 8 + 4 + t4];
            }
        }
        // O^T accumulators: d-tile dt, rows (dims) 16dt + g and + 8, columns (heads) 2t4 and 2t4 + 1
        float o[8][4];
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
        // heads 2t4 and 2t4 + 1: running max (log2 units) and this lane's partial sum (tokens g, g + 8)
        float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

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
                    const int r = pos % kPage;
                    if (lane < 16)
                        *reinterpret_cast<uint4*>(kt + tile_off(r, lane)) = reinterpret_cast<const uint4*>(S.kn)[lane];
                    __syncwarp();
                }
                if (valid < kPage) {
                    // rows past the position become zeros in V (their P is 0; the slots may hold
                    // anything, NaN included); each row is two 128-byte box rows
                    for (int r = max(valid, warp * 16); r < warp * 16 + 16; ++r)
                        reinterpret_cast<uint2*>(vt + (lane >> 4) * 8192 + r * 128)[lane & 15] = make_uint2(0u, 0u);
                    __syncwarp();
                }
                // ---- S^T = K Q^T: A = this warp's 16 key rows, two accumulators (even / odd k-steps)
                float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
                {
                    const int q = lane >> 3, r8 = lane & 7;
                    const int row = warp * 16 + (q & 1) * 8 + r8;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const int chunk = kk * 2 + (q >> 1);
                        uint32_t a0, a1, a2, a3;
                        ldmatrix_x4(kt + tile_off(row, chunk), a0, a1, a2, a3);
                        if (kk & 1)
                            mma_bf16_16816(sb, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
                        else
                            mma_bf16_16816(sa, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
                    }
                }
                // ---- online softmax per head column: tokens g (elements 0, 1) and g + 8 (2, 3)
                const int tok = warp * 16 + g;
                float sc[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    sc[e] = (tok + (e >> 1) * 8) < valid ? (sa[e] + sb[e]) * qscale : -INFINITY;
                float mx0 = fmaxf(sc[0], sc[2]), mx1 = fmaxf(sc[1], sc[3]);
#pragma unroll
                for (int off = 4; off < 32; off <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
                }
                float p[4] = {0.f, 0.f, 0.f, 0.f};
                float corr0 = 1.f, corr1 = 1.f;
                const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
                if (mn0 != -INFINITY) {
                    corr0 = exp2f(m_run[0] - mn0);
                    m_run[0] = mn0;
                    p[0] = exp2f(sc[0] - mn0);
                    p[2] = exp2f(sc[2] - mn0);
                }
                if (mn1 != -INFINITY) {
                    corr1 = exp2f(m_run[1] - mn1);
                    m_run[1] = mn1;
                    p[1] = exp2f(sc[1] - mn1);
                    p[3] = exp2f(sc[3] - mn1);
                }
                l_run[0] = l_run[0] * corr0 + p[0] + p[2];
                l_run[1] = l_run[1] * corr1 + p[1] + p[3];
#pragma unroll
                for (int dt = 0; dt < 8; ++dt) {
                    o[dt][0] *= corr0;
                    o[dt][1] *= corr1;
                    o[dt][2] *= corr0;
                    o[dt][3] *= corr1;
                }
                // ---- P^T as the B operand (k = tokens, n = heads): BF16 hi + lo parts, each
                // 8 x 8 block (tokens g / g + 8 by heads) transposed by movmatrix
                bf16 hb[4], lb[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    hb[e] = f2bf(p[e]);
                    lb[e] = f2bf(p[e] - bf2f(hb[e]));
                }
                const uint32_t bh0 = movmatrix_trans(pack_bf2(hb[0], hb[1]));
                const uint32_t bh1 = movmatrix_trans(pack_bf2(hb[2], hb[3]));
                const uint32_t bl0 = movmatrix_trans(pack_bf2(lb[0], lb[1]));
                const uint32_t bl1 = movmatrix_trans(pack_bf2(lb[2], lb[3]));
                // ---- O^T += V^T P^T: A = V^T tiles (dims 16dt.., tokens of this warp) by ldmatrix.trans
                {
                    const int q = lane >> 3, r8 = lane & 7;
                    const int row = warp * 16 + (q >> 1) * 8 + r8;
#pragma unroll
                    for (int dt = 0; dt < 8; ++dt) {
                        const int chunk = 2 * dt + (q & 1);
                        uint32_t a0, a1, a2, a3;
                        ldmatrix_x4_trans(vt + tile_off(row, chunk), a0, a1, a2, a3);
                        mma_bf16_16816(o[dt], a0, a1, a2, a3, bh0, bh1);
                        mma_bf16_16816(o[dt], a0, a1, a2, a3, bl0, bl1);
                    }
                }
            }
            // the slot is refilled by the async proxy after this warp's generic-proxy
            // writes to it (the patched key row, the zeroed V rows): order them first
            if (i + kStages < np) fence_proxy_async_cta();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[s]);
        }
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], off);
            l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], off);
        }
        if (tracing && tid == 0) tr_cp = clock64();

        // ---- merge the 4 warp states (fixed order) into this CTA's state
        {
            const int h0 = 2 * t4, h1 = 2 * t4 + 1;
            if (g == 0) {
                if (h0 < HG) {
                    S.m[warp][h0] = m_run[0];
                    S.l[warp][h0] = l_run[0];
                }
                if (h1 < HG) {
                    S.m[warp][h1] = m_run[1];
                    S.l[warp][h1] = l_run[1];
                }
            }
#pragma unroll
            for (int dt = 0; dt < 8; ++dt) {
                if (h0 < HG) {
                    S.acc[warp][h0][16 * dt + g] = o[dt][0];
                    S.acc[warp][h0][16 * dt + g + 8] = o[dt][2];
                }
                if (h1 < HG) {
                    S.acc[warp][h1][16 * dt + g] = o[dt][1];
                    S.acc[warp][h1][16 * dt + g + 8] = o[dt][3];
                }
            }
        }
        named_bar(1, kConsumers);
        if (tid < HG) {  // per head: the CTA's max, each warp's weight, the weighted sum
            float M = -INFINITY;
            for (int h = 0; h < kWarps; ++h) M = fmaxf(M, S.m[h][tid]);
            float Lsum = 0.f;
            for (int h = 0; h < kWarps; ++h) {
                const float f = M == -INFINITY ? 0.f : exp2f(S.m[h][tid] - M);
                S.fw[h][tid] = f;
                Lsum += S.l[h][tid] * f;
            }
            S.cm[tid] = M;
            S.cl[tid] = Lsum;
        }
        named_bar(1, kConsumers);
        if (a.splits > 1) cluster_wait();  // phase 0: every CTA of the cluster has started
        const int slice = HG * kHd / a.splits;  // outputs each CTA of the cluster finishes
        for (int oi = tid; oi < HG * kHd; oi += kConsumers) {
            const int gg = oi / kHd, d = oi % kHd;
            const float M = S.cm[gg], Lsum = S.cl[gg];
            float A = 0.f;
#pragma unroll
            for (int h = 0; h < kWarps; ++h) A += S.acc[h][gg][d] * S.fw[h][gg];
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
        // per head (a warp each, lane = split): the max over splits, each split's weight
        // and the weighted sum (fixed shuffle tree)
        for (int h = warp; h < HG; h += kWarps) {
            const float ms = lane < a.splits ? S.rx_m[lane][h] : -INFINITY;
            float M = ms;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
            const float f = ms == -INFINITY ? 0.f : exp2f(ms - M);
            float L = lane < a.splits ? S.rx_l[lane][h] * f : 0.f;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
            if (lane < 16) S.rf[lane][h] = f;
            if (lane == 0) S.rl[h] = L;
        }
        named_bar(1, kConsumers);
        const int slice = HG * kHd / a.splits;
        for (int j = tid; j < slice; j += kConsumers) {
            const int o = split * slice + j;
            const int g = o / kHd, d = o % kHd;
            float A = 0.f;
#pragma unroll
            for (int sp = 0; sp < 16; ++sp)  // fixed split order
                if (sp < a.splits) A += S.rx_acc[sp * slice + j] * S.rf[sp][g];
            const int qh = kvh * G + qb * HG + g;
            out[static_cast<size_t>(qh) * kHd + d] = f2bf(A / S.rl[g]);
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


template <int HG>
cudaError_t launch_hg(const AttnArgs& a, cudaStream_t s, bool pdl, int nqb) {
    auto* fn = attn_kernel<HG>;
    const size_t smem = sizeof(AttnSmem<HG>) + 1024;  // + alignment of the TMA boxes
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
                                         static_cast<int>(sizeof(AttnSmem<HG>) + 1024));
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
    cfg.dynamicSmemBytes = sizeof(AttnSmem<HG>) + 1024;
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
int g_clusters16 = 0;   // 16-CTA clusters of the largest variant resident at once

}  // namespace

int attn_heads_per_cta(int G) { return G >= 8 ? 8 : G; }

int attn_sms_used(int q_heads, int kv_heads, int splits) {
    const int G = q_heads / kv_heads;
    return splits * kv_heads * (G / attn_heads_per_cta(G));  // one CTA per SM
}

cudaError_t configure_attention_kernels() {
    cudaError_t e = configure_hg<1>();
    if (e == cudaSuccess) e = configure_hg<2>();
    if (e == cudaSuccess) e = configure_hg<4>();
    if (e == cudaSuccess) e = configure_hg<8>();
    if (e != cudaSuccess) return e;
    // How many 16-CTA clusters of the largest variant can be resident at once (one CTA
    // per SM: a cluster needs 16 SMs of one GPC)?
    g_clusters16 = max_clusters<8>(16);
    g_max_cluster = g_clusters16 > 0 ? 16 : 8;
    return cudaSuccess;
}

// Splits per (kv head, block): a power of two forming one cluster, no more than
// the pages; 16 when the decode launch's kv_heads clusters of 16 are all resident
// at once, else 8.
int attn_splits(int kv_heads, int max_pos, int page_size, int sms) {
    (void)page_size;
    (void)sms;
    const int max_pages = max_pos / kPage + 1;
    const int cap = (g_max_cluster == 16 && g_clusters16 >= kv_heads) ? 16 : 8;
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

// 3-D tensor map of a K or V cache for the page loads: paged [pages][kvh][64][128]
// as (column, row, page x kvh + head), box 64 x 64 x 1; flat [positions][kvh][128]
// as (column, head, position), box 64 x 1 x 64.  128-byte swizzle, zero fill past
// the extent.
bool make_cache_map(CUtensorMap* map, const bf16* base, int paged, int kv_heads, long long extent) {
    auto fn = tensor_map_encoder();
    if (!fn || !base || (reinterpret_cast<uintptr_t>(base) & 15) || extent <= 0) return false;
    cuuint64_t dims[3];
    cuuint64_t strides[2];
    cuuint32_t box[3];
    if (paged) {
        dims[0] = kHd, dims[1] = kPage, dims[2] = static_cast<cuuint64_t>(extent) * kv_heads;
        strides[0] = kHd * 2, strides[1] = static_cast<cuuint64_t>(kPage) * kHd * 2;
        box[0] = 64, box[1] = kPage, box[2] = 1;
    } else {
        dims[0] = kHd, dims[1] = static_cast<cuuint64_t>(kv_heads), dims[2] = static_cast<cuuint64_t>(extent);
        strides[0] = kHd * 2, strides[1] = static_cast<cuuint64_t>(kv_heads) * kHd * 2;
        box[0] = 64, box[1] = 1, box[2] = kPage;
    }
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<bf16*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_attention(const AttnArgs& args, cudaStream_t s, bool pdl) {
    AttnArgs a = args;
    if (!a.paged && (a.pos_ptr || a.row_pos) && a.pool <= 0) return cudaErrorInvalidValue;  // the extent must be known
    if (a.row_pos && !a.paged) return cudaErrorInvalidValue;
    // paged pool of unknown size: the page table is trusted, as it is for the addresses
    const long long extent = a.pool > 0 ? a.pool
                             : a.paged ? (1ll << 20)
                                       : static_cast<long long>(a.pos_host) + (a.n_queries > 1 ? a.n_queries : 1);
    if (!make_cache_map(&a.tk, a.k, a.paged, a.kv_heads, extent) ||
        !make_cache_map(&a.tv, a.v, a.paged, a.kv_heads, extent))
        return cudaErrorInvalidValue;
    const int G = a.q_heads / a.kv_heads;
    if (a.q_heads % a.kv_heads != 0 || !(G == 1 || G == 2 || G == 4 || G == 8)) return cudaErrorInvalidValue;
    if (a.splits < 1 || a.splits > 16 || (a.splits & (a.splits - 1)) != 0) return cudaErrorInvalidValue;
    if (a.n_queries > 1 && static_cast<long long>(a.n_queries) * (G / attn_heads_per_cta(G)) > 65535)
        return cudaErrorInvalidValue;
    const int HG = attn_heads_per_cta(G);
    const int nqb = G / HG;
    switch (HG) {
        case 1: return launch_hg<1>(a, s, pdl, nqb);
        case 2: return launch_hg<2>(a, s, pdl, nqb);
        case 4: return launch_hg<4>(a, s, pdl, nqb);
        default: return launch_hg<8>(a, s, pdl, nqb);
    }
}

}  // namespace q3

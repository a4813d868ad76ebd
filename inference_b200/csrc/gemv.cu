// gemv.cu -- batch-1 BF16 GEMV for B200, the weight-streaming kernel of the
// decode step.  Replaces the reference's cuBLAS call
// (src/lib/backend/cuda/kernels/matmul.cuh:8-18) and fuses the small ops
// around each matmul of Model::forward (src/lib/model/qwen3/qwen3.hpp:131-166).
//
// Design (one CTA per SM, 8 consumer warps + 1 producer warp):
//   * The CTA owns a contiguous band of weight rows.  The producer lane streams
//     it as tiles of rb rows x kc columns with 1-D TMA bulk copies
//     (cp.async.bulk, one per row segment, L2 evict-first) into a ring of
//     shared-memory stages guarded by full/empty mbarriers.
//   * Weights do not depend on the previous kernel, so the producer starts
//     before griddepcontrol.wait: with programmatic dependent launch the next
//     GEMV's weight prefetch overlaps the tail of the current kernel.
//   * Consumers build x in shared memory (the prologue: copy, RMSNorm,
//     embedding lookup, residual add), then each warp dots its row segment
//     with 16-byte vectors, fp32 FMA, warp-shuffle reduction, and a fixed-order
//     cross-warp sum, so results are deterministic.
//   * Epilogues apply the reference's BF16 rounding points exactly: matmul
//     output rounded to BF16, then the following op on the rounded value.
//   * FP8 E4M3 weights (F8) take the tensor cores instead: an item is a tile
//     of 16 rows x 256 columns, stored contiguously and bank-swizzled by the
//     packed layout (F8Pack) so one bulk copy brings it, each weight pair converts exactly to
//     f16x2 (cvt.rn.f16x2.e4m3x2) as the A operand of mma.sync m16n8k16, and
//     x enters as the B operand in f16, scaled by a power of two 2^-s chosen
//     per CTA so that max|x| 2^-s lies in [2^14, 2^15) (exact for every
//     |x| >= max|x| 2^-29; the few smaller ones round as f16 subnormals).
//     Row sums are multiplied back by 2^s and by the row's scale in the
//     epilogue.
//   * NVFP4 weights (F4) take the same path with 16-row x 512-column items:
//     each lane's 16 columns of a 64-column block are one NVFP4 block, so
//     its E2M1 nibbles turn into f16 by a byte-permute lookup (integer pipe,
//     not the conversion unit) and one f16x2 multiply by the block's E4M3
//     scale gives the exact weights (at most six significant bits).
#include <algorithm>
#include <cmath>

#include "kernels.cuh"

namespace q3 {

namespace {

#ifndef Q3_GEMV_WARPS
#define Q3_GEMV_WARPS 16
#endif
#ifndef Q3_GEMV_CHUNK
#define Q3_GEMV_CHUNK 2048
#endif
#ifndef Q3_GEMV_SMEM_KB
#define Q3_GEMV_SMEM_KB 210
#endif
#ifndef Q3_GEMV_MAX_STAGES
#define Q3_GEMV_MAX_STAGES 3
#endif
#ifndef Q3_GEMV_MIN_BLOCKS
#define Q3_GEMV_MIN_BLOCKS 1
#endif
constexpr int kWarps = Q3_GEMV_WARPS;
constexpr int kThreads = kWarps * 32;
constexpr int kChunk = Q3_GEMV_CHUNK;   // BF16 columns per item (4 KB); FP8 items take twice the columns
constexpr int kMaxItems = 4096;         // (row, chunk) partial sums per CTA
// One CTA per SM with a ~192 KB ring: loaded HBM latency needs well over
// 100 KB in flight per SM to sustain its share of the bandwidth (measured:
// 8 warps x 3 x 4 KB reached 71% of peak on a 201 MB GEMV, 16 x 3 x 4 KB 85%).
constexpr size_t kSmemBudget = Q3_GEMV_SMEM_KB * 1024;
constexpr int kMaxDynSmem = 227 * 1024;   // the opt-in maximum per block
constexpr size_t kSmemBudgetF8 = 226 * 1024;

constexpr int kF8Rows = kF8TileRows;          // rows per FP8 tile (the mma M dimension)
constexpr int kF8Cols = kF8TileCols;          // columns per FP8 item
constexpr int kF8Slot = kF8Rows * kF8Cols;    // bytes per FP8 ring slot (one packed item)
constexpr int kF4Slot = kF8Rows * kF4RowBytes;  // bytes per NVFP4 ring slot (nibbles + block scales)

struct SmemLayout {
    size_t stage_off, x_off, part_off, bar_off, misc_off, total;
};

// plan.wb: 2 = BF16, 1 = E4M3, 0 = NVFP4 (WF = 2 - wb in the kernel)
__host__ __device__ inline size_t slot_bytes_of(int wb, int kc) {
    return wb == 2 ? static_cast<size_t>(kc) * 2 : wb == 1 ? static_cast<size_t>(kF8Slot)
                                                          : static_cast<size_t>(kF4Slot);
}
__host__ __device__ inline size_t slot_bytes(const GemvPlan& p) { return slot_bytes_of(p.wb, p.kc); }

// `wb` a compile-time constant in the kernel (its weight format)
__host__ __device__ inline SmemLayout smem_layout_wb(const GemvPlan& p, int wb, int K, int max_rows) {
    SmemLayout L;
    L.stage_off = 0;
    L.x_off = static_cast<size_t>(kWarps) * p.stages * slot_bytes_of(wb, p.kc);
    L.part_off = L.x_off + (static_cast<size_t>(K) * 2 + 15) / 16 * 16;
    L.bar_off = L.part_off + (static_cast<size_t>(max_rows) * p.nch * 4 + 15) / 16 * 16;
    L.misc_off = L.bar_off + static_cast<size_t>(kWarps) * p.stages * 8;
    L.total = L.misc_off + 128;
    return L;
}
__host__ __device__ inline SmemLayout smem_layout(const GemvPlan& p, int K, int max_rows) {
    return smem_layout_wb(p, p.wb, K, max_rows);
}

__device__ __forceinline__ size_t kv_slot(const GemvArgs& a, int pos, int head) {
    const int page = a.page_table[pos / a.page_size];
    return ((static_cast<size_t>(page) * a.kv_heads_local + head) * a.page_size + (pos % a.page_size)) * 128;
}

// Sum over the CTA's threads, fixed order.
__device__ __forceinline__ float cta_sum(float v, float* scratch) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    v = warp_sum(v);
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) t += scratch[w];
    __syncthreads();
    return t;
}

// Maximum over the CTA's threads.
__device__ __forceinline__ float cta_max(float v, float* scratch) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) t = fmaxf(t, scratch[w]);
    __syncthreads();
    return t;
}

// Four E4M3 weights w (byte i = column i) as two f16x2 registers, exact values,
// by the conversion unit: lo = bytes 0-1, hi = bytes 2-3.
__device__ __forceinline__ void e4m3x4_f16x2_cvt(uint32_t w, uint32_t& lo, uint32_t& hi) {
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.rn.f16x2.e4m3x2 %0, l;\n\tcvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
        : "=r"(lo), "=r"(hi)
        : "r"(w));
}

// D (16 x 8, fp32) += A (16 x 16, f16, row) B (16 x 8, f16, col); A rows g / g + 8 of
// lane (g, t) come as 4-byte E4M3 words: bytes 0-1 = k 2t, 2t+1, bytes 2-3 = k 2t+8,
// 2t+9 (exact f16 values).
__device__ __forceinline__ void mma_e4m3_f16(float (&d)[4], uint32_t wg, uint32_t wg8, uint32_t b0, uint32_t b1) {
    uint32_t a0, a1, a2, a3;
    e4m3x4_f16x2_cvt(wg, a0, a2);
    e4m3x4_f16x2_cvt(wg8, a1, a3);
    // not volatile: a pure function of its operands, free to be scheduled among the conversions
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two E2M1 weights (one byte: column 2 i in the low nibble) as an f16x2, by a
// byte-permute lookup of the f16 high byte (the low byte of every E2M1 value in
// f16 is zero): magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6 -> 0x00, 0x38, 0x3C,
// 0x3E, 0x40, 0x42, 0x44, 0x46, entry 0 also filling the low bytes; the signs
// go to bits 15 and 31.
__device__ __forceinline__ uint32_t e2m1x2_f16x2(uint32_t byte) {
    const uint32_t sel = ((byte & 0x7u) << 4) | ((byte & 0x70u) << 8);
    uint32_t v;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(v) : "r"(0x3E3C3800u), "r"(0x46444240u), "r"(sel));
    return v | ((byte & 0x8u) << 12) | ((byte & 0x80u) << 24);
}

__device__ __forceinline__ uint32_t mul_f16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// An E4M3 scale byte as (s, s) in f16 (exact).
__device__ __forceinline__ uint32_t e4m3_f16x2_splat(uint32_t q) {
    uint32_t d;
    asm("{\n\t.reg .b16 p;\n\tcvt.u16.u32 p, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, p;\n\t}" : "=r"(d) : "r"(q | (q << 8)));
    return d;
}

// The mma of four consecutive columns of NVFP4 rows g and g + 8: h / h8 hold the
// two bytes (four nibbles) of each row, sa / sb the rows' block scales as f16x2.
__device__ __forceinline__ void mma_nvfp4(float (&d)[4], uint32_t h, uint32_t h8, uint32_t sa, uint32_t sb,
                                          uint32_t b0, uint32_t b1) {
    const uint32_t a0 = mul_f16x2(e2m1x2_f16x2(h & 0xFFu), sa), a2 = mul_f16x2(e2m1x2_f16x2((h >> 8) & 0xFFu), sa);
    const uint32_t a1 = mul_f16x2(e2m1x2_f16x2(h8 & 0xFFu), sb), a3 = mul_f16x2(e2m1x2_f16x2((h8 >> 8) & 0xFFu), sb);
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- tensor-parallel exchange through peer memory
constexpr uint32_t kPeerPolls = 1u << 20;

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long peer_seq(const PeerLinks& x) {
    return *reinterpret_cast<volatile unsigned long long*>(x.seq);
}
// Tag of partial exchange xtag in the current step (unique for 2^24 steps).
__device__ __forceinline__ uint32_t pair_tag(const PeerLinks& x, int xtag) {
    return static_cast<uint32_t>(peer_seq(x)) * 256u + static_cast<uint32_t>(xtag);
}
__device__ __forceinline__ void ld_pairs(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Consumer side: every CTA waits (bounded) until all ranks filled the slot of
// exchange s, the one the kernel before produced.
__device__ __forceinline__ void peer_wait(const PeerLinks& x, unsigned long long s, uint32_t* err) {
    const uint32_t* fl = x.flags[x.rank] + (s & 1) * x.world;
    if (threadIdx.x < static_cast<unsigned>(x.world)) {
        uint32_t polls = 0;
        while (ld_acquire_sys(fl + threadIdx.x) != static_cast<uint32_t>(s)) {
            // after any recorded failure stop waiting at once (the engine reports it)
            if ((++polls & 1023) == 0 && *reinterpret_cast<volatile uint32_t*>(err)) break;
            if (polls > kPeerPolls) {
                record_error(err, DEV_PEER_WAIT_TIMEOUT);
                break;
            }
        }
    }
    __syncthreads();
}

// WF (weight format): 0 BF16; 1 E4M3 bytes (a.W8) with a scale per row (a.wscale),
// ring slots of 4 KB holding twice the columns; 2 NVFP4 (a.W8 in the NVFP4 pack,
// row scales in a.wscale), slots of 16 rows x 512 columns with their block scales.
template <int PRO, int EPI, int WF>
__global__ void __launch_bounds__(kThreads, Q3_GEMV_MIN_BLOCKS) gemv_kernel(const __grid_constant__ GemvArgs a) {
    constexpr bool F8 = WF != 0;  // packed 16-row tiles on the tensor cores (E4M3 or NVFP4)
    constexpr bool F4 = WF == 2;
    constexpr int WB = F8 ? 1 : 2;  // bytes per weight (BF16 items)
    constexpr int kUnit = F4 ? kF4RowBytes : kF8Cols;  // bytes of one row of a packed item
    constexpr int kSlot = kF8Rows * kUnit;
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvPlan& p = a.plan;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int pro = PRO, epi = EPI;
    const bool tracing = a.trace.buf != nullptr;
    unsigned long long tr_t0 = 0, tr_c0 = 0, tr_c1 = 0, tr_c2 = 0, tr_c3 = 0, tr_cx = 0;
    if (tracing && tid == 0) {
        tr_t0 = globaltimer_ns();
        tr_c0 = clock64();
    }

    // ---- this CTA's rows and this warp's contiguous run of (row, chunk) items
    const int units = a.N / p.row_gran;
    int u0, u1;
    gemv_band(p, units, blockIdx.x, u0, u1);
    const int r0 = u0 * p.row_gran, r1 = u1 * p.row_gran;
    const int nrows = r1 - r0;
    const int max_rows = p.max_units * p.row_gran;
    constexpr int kWb = 2 - WF;  // the plan's wb of this weight format
    const SmemLayout L = smem_layout_wb(p, kWb, a.K, max_rows);
    bf16* xs = reinterpret_cast<bf16*>(smem + L.x_off);
    float* part = reinterpret_cast<float*>(smem + L.part_off);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off) + warp * p.stages;
    float* misc = reinterpret_cast<float*>(smem + L.misc_off);
    unsigned long long* cta_key = reinterpret_cast<unsigned long long*>(misc + 16);
    uint8_t* ring = smem + L.stage_off + static_cast<size_t>(warp) * p.stages * slot_bytes_of(kWb, p.kc);

    // items: (row, chunk) pairs; FP8: (16-row tile, 256-column chunk) pairs
    const int n_items = (F8 ? (nrows + kF8Rows - 1) / kF8Rows : nrows) * p.nch;
    const int i0 = static_cast<int>(static_cast<long long>(warp) * n_items / kWarps);
    const int i1 = static_cast<int>(static_cast<long long>(warp + 1) * n_items / kWarps);
    const int cnt = i1 - i0;

    if (lane == 0) {
        for (int s = 0; s < p.stages; ++s) mbar_init(&bars[s], 1);
        fence_barrier_init();
    }
    __syncwarp();

    uint64_t pol = 0;
    // BF16: lane 0 copies one row segment.  FP8 (whole warp): lane r < 16 copies row r of the tile.
    auto issue = [&](int item, int slot) {
        const int c = item % p.nch;
        const int cols = (c == p.nch - 1) ? a.K - c * p.kc : p.kc;
        if constexpr (F8) {
            (void)cols;
            const int tile = item / p.nch;
            const int rows = min(kF8Rows, nrows - tile * kF8Rows);
            if (lane == 0) {
                const uint32_t bytes = static_cast<uint32_t>(rows * kUnit);
                mbar_arrive_expect_tx(&bars[slot], bytes);
                bulk_g2s(ring + static_cast<size_t>(slot) * kSlot,
                         a.W8 + (static_cast<size_t>(r0) * p.nch + static_cast<size_t>(tile) * kF8Rows * p.nch +
                                 static_cast<size_t>(c) * rows) * kUnit,
                         bytes, &bars[slot], pol);
            }
        } else {
            const int row = r0 + item / p.nch;
            const uint32_t bytes = static_cast<uint32_t>(cols) * WB;
            mbar_arrive_expect_tx(&bars[slot], bytes);
            bulk_g2s(ring + static_cast<size_t>(slot) * p.kc * WB,
                     reinterpret_cast<const uint8_t*>(a.W) + (static_cast<size_t>(row) * a.K + c * p.kc) * WB, bytes,
                     &bars[slot], pol);
        }
    };
    // Weights never depend on earlier kernels: start streaming before the wait.
    if (F8 || lane == 0) {
        pol = policy_evict_first();
        for (int j = 0; j < p.stages && j < cnt; ++j) issue(i0 + j, j);
    }
    for (int i = tid; i < nrows * p.nch; i += kThreads) part[i] = 0.f;
    if (tid == 0) *cta_key = 0ull;
    // RMSNorm weights never depend on earlier kernels: this thread's first two
    // 16-byte vectors of them load before the wait (the rest in the norm pass)
    const int kv8 = a.K / 8;
    uint4 wpre[2];
    if (pro != PRO_PLAIN) {
#pragma unroll
        for (int k = 0; k < 2; ++k)
            if (tid + k * kThreads < kv8) wpre[k] = reinterpret_cast<const uint4*>(a.norm_w)[tid + k * kThreads];
    }

    pdl_wait();
    pdl_trigger();
    if (tracing && tid == 0) tr_c1 = clock64();
    // the residual rows this thread updates in the epilogue (first pass), read now
    bf16 hs_pre = __float2bfloat16(0.f);
    if ((epi == EPI_RESID || epi == EPI_RESID_F32) && tid < nrows) hs_pre = a.hs[r0 + tid];
    // The position: the embedding prologue needs it at once; the QKV epilogue only at the
    // end, so there its load is issued now and checked after the prologue (a branch on it
    // here would hold the whole prologue for the load's round trip)
    int pos = 0;
    if (epi == EPI_QKV || pro == PRO_EMBED_NORM) pos = *a.pos_ptr;
    auto check_pos = [&]() {
        if (pos < 0 || pos >= a.capacity) {
            if (tid == 0) record_error(a.err, DEV_BAD_POSITION);
            pos = 0;
        }
    };
    if (pro == PRO_EMBED_NORM) check_pos();

    // ---- prologue: x in shared memory
    if (pro == PRO_PLAIN) {
        const uint4* src = reinterpret_cast<const uint4*>(a.x);
        uint4* dst = reinterpret_cast<uint4*>(xs);
        for (int i = tid; i < kv8; i += kThreads) dst[i] = src[i];
    } else {
        const bf16* src = a.hs;
        if (pro == PRO_EMBED_NORM) {
            const int nf = *a.n_forced;
            uint64_t best = 0;
            if (a.peer.world) {
                // the previous step's lm_head exchanged every rank's key (none before the first step)
                const unsigned long long s = peer_seq(a.peer);
                if (s) {
                    peer_wait(a.peer, s, a.err);
                    const unsigned long long* k = a.peer.keys[a.peer.rank] + (s & 1) * a.peer.world;
                    for (int r = 0; r < a.peer.world; ++r) best = max(best, static_cast<uint64_t>(__ldcg(k + r)));
                }
            } else {
                for (int r = 0; r < a.n_keys; ++r) best = max(best, static_cast<uint64_t>(a.keys[r]));
            }
            const uint32_t greedy = argmax_key_index(best);
            int token = (pos < nf) ? a.tokens[pos] : static_cast<int>(greedy);
            if (token < 0 || token >= a.vocab) {
                if (tid == 0) record_error(a.err, DEV_BAD_TOKEN);
                token = 0;
            }
            if (blockIdx.x == 0 && tid == 0) {
                if (pos >= 1) a.argmax_hist[pos - 1] = static_cast<int32_t>(greedy);
                if (pos >= nf) a.tokens[pos] = token;
            }
            src = a.embed + static_cast<size_t>(token) * a.K;
        }
        // tensor parallel through peer memory: the (value, tag) pairs every rank stored here
        const unsigned long long* parts = nullptr;
        uint32_t tag = 0;
        if (pro == PRO_RESID_NORM) {
            if (a.peer.world) {
                tag = pair_tag(a.peer, a.xtag);
                parts = a.peer.recv[a.peer.rank] + ((a.xtag - 1) & 1) * static_cast<size_t>(a.peer.world) * a.peer.H;
            }
        }
        float ss = 0.f;
        for (int i = tid; i < kv8; i += kThreads) {
            uint4 h = reinterpret_cast<const uint4*>(src)[i];
            if (pro == PRO_NORM_F32) {
                const float4 v0 = reinterpret_cast<const float4*>(a.vsum)[2 * i];
                const float4 v1 = reinterpret_cast<const float4*>(a.vsum)[2 * i + 1];
                ss += v0.x * v0.x + v0.y * v0.y + v0.z * v0.z + v0.w * v0.w;
                ss += v1.x * v1.x + v1.y * v1.y + v1.z * v1.z + v1.w * v1.w;
            } else if (pro == PRO_RESID_NORM) {
                float4 v0, v1;
                if (parts) {
                    // sum of the ranks' partials in rank order (the same bits on every rank),
                    // each pair read until it carries this exchange's tag (bounded)
                    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                    for (int r = 0; r < a.peer.world; ++r) {
                        const unsigned long long* pr = parts + static_cast<size_t>(r) * a.peer.H + 8 * i;
                        unsigned long long q[8];
                        for (uint32_t polls = 0;; ++polls) {
#pragma unroll
                            for (int e = 0; e < 4; ++e) ld_pairs(pr + 2 * e, q[2 * e], q[2 * e + 1]);
                            bool all = true;
#pragma unroll
                            for (int e = 0; e < 8; ++e) all = all && static_cast<uint32_t>(q[e] >> 32) == tag;
                            if (all) break;
                            if ((polls & 1023) == 1023 && *reinterpret_cast<volatile uint32_t*>(a.err)) break;
                            if (polls > kPeerPolls) {
                                record_error(a.err, DEV_PEER_WAIT_TIMEOUT);
                                break;
                            }
                        }
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[e] += __uint_as_float(static_cast<uint32_t>(q[e]));
                    }
                    v0 = make_float4(acc[0], acc[1], acc[2], acc[3]);
                    v1 = make_float4(acc[4], acc[5], acc[6], acc[7]);
                } else {
                    v0 = reinterpret_cast<const float4*>(a.vsum)[2 * i];
                    v1 = reinterpret_cast<const float4*>(a.vsum)[2 * i + 1];
                }
                // timeline: when thread 0 holds every rank's partials of its first rows
                if (tracing && parts && tid == 0 && tr_cx == 0) tr_cx = clock64();
                const float rs[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
                uint32_t* hw = reinterpret_cast<uint32_t*>(&h);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float a0 = bf_lo(hw[j]) + round_bf(rs[2 * j]);
                    const float a1 = bf_hi(hw[j]) + round_bf(rs[2 * j + 1]);
                    const bf16 b0 = f2bf(a0), b1 = f2bf(a1);
                    const float s0 = a.ss_unrounded ? a0 : bf2f(b0);
                    const float s1 = a.ss_unrounded ? a1 : bf2f(b1);
                    ss += s0 * s0 + s1 * s1;
                    hw[j] = static_cast<uint32_t>(__bfloat16_as_ushort(b0)) |
                            (static_cast<uint32_t>(__bfloat16_as_ushort(b1)) << 16);
                }
            } else {
                const uint32_t* hw = reinterpret_cast<const uint32_t*>(&h);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float lo = bf_lo(hw[j]), hi = bf_hi(hw[j]);
                    ss += lo * lo + hi * hi;
                }
            }
            reinterpret_cast<uint4*>(xs)[i] = h;
            if (pro == PRO_EMBED_NORM || pro == PRO_RESID_NORM) {
                if (blockIdx.x == 0) reinterpret_cast<uint4*>(a.hs_out)[i] = h;
            }
        }
        ss = cta_sum(ss, misc);
        const float scale = 1.0f / sqrtf(ss / static_cast<float>(a.K) + a.eps);
        for (int i = tid, k = 0; i < kv8; i += kThreads, ++k) {
            uint4 h = reinterpret_cast<uint4*>(xs)[i];
            const uint4 w = k == 0 ? wpre[0] : k == 1 ? wpre[1] : reinterpret_cast<const uint4*>(a.norm_w)[i];
            uint32_t* hw = reinterpret_cast<uint32_t*>(&h);
            const uint32_t* ww = reinterpret_cast<const uint32_t*>(&w);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const bf16 b0 = f2bf(bf_lo(hw[j]) * scale * bf_lo(ww[j]));
                const bf16 b1 = f2bf(bf_hi(hw[j]) * scale * bf_hi(ww[j]));
                hw[j] = static_cast<uint32_t>(__bfloat16_as_ushort(b0)) |
                        (static_cast<uint32_t>(__bfloat16_as_ushort(b1)) << 16);
            }
            reinterpret_cast<uint4*>(xs)[i] = h;
        }
    }
    __syncthreads();
    int xshift = 0;  // FP8: x in shared memory holds f16(x 2^-xshift)
    if constexpr (F8) {
        float mx = 0.f;
        for (int i = tid; i < kv8; i += kThreads) {
            const uint4 h = reinterpret_cast<const uint4*>(xs)[i];
            const uint32_t* hw = reinterpret_cast<const uint32_t*>(&h);
#pragma unroll
            for (int j = 0; j < 4; ++j) mx = fmaxf(mx, fmaxf(fabsf(bf_lo(hw[j])), fabsf(bf_hi(hw[j]))));
        }
        mx = cta_max(mx, misc);
        if (mx > 0.f) {
            int k;
            frexpf(mx, &k);  // mx < 2^k
            xshift = k - 15;
        }
        for (int i = tid; i < kv8; i += kThreads) {
            uint4 h = reinterpret_cast<const uint4*>(xs)[i];
            uint32_t* hw = reinterpret_cast<uint32_t*>(&h);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const __half lo = __float2half_rn(ldexpf(bf_lo(hw[j]), -xshift));
                const __half hi = __float2half_rn(ldexpf(bf_hi(hw[j]), -xshift));
                hw[j] = static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
            }
            reinterpret_cast<uint4*>(xs)[i] = h;
        }
        __syncthreads();
    }
    if (tracing && tid == 0) tr_c2 = clock64();
    // EPI_QKV: the V page slot of this position, looked up now for the epilogue
    size_t v_slot = 0;
    if (epi == EPI_QKV) {
        if (pro != PRO_EMBED_NORM) check_pos();
        v_slot = kv_slot(a, pos, 0);
    }

    // ---- main loop: each warp streams its own items; no CTA-wide barrier
    float acc0 = 0.f, acc1 = 0.f;
    bool failed = false;
    if constexpr (F8) {
        const int g = lane >> 2, t = lane & 3;
        float d[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};  // two independent mma chains
        for (int j = 0; j < cnt; ++j) {
            const int slot = j % p.stages;
            bool ok = !failed && mbar_wait(&bars[slot], (j / p.stages) & 1, a.err, DEV_TMA_WAIT_TIMEOUT);
            ok = __all_sync(0xffffffffu, ok);  // the mma and the refill need the whole warp
            failed = failed || !ok;
            const int item = i0 + j;
            const int tile = item / p.nch, c = item % p.nch;
            if (ok && F4) {
                const int cols = (c == p.nch - 1) ? a.K - c * p.kc : p.kc;
                const uint8_t* ws = ring + static_cast<size_t>(slot) * kSlot;
                const uint8_t* sc = ws + min(kF8Rows, nrows - tile * kF8Rows) * 256;  // the item's block scales
                const uint4* xq = reinterpret_cast<const uint4*>(xs) + c * (p.kc / 8);
#pragma unroll 2
                for (int blk = 0; blk < cols / 64; ++blk) {
                    // lane (g, t): block 4 blk + t of rows g and g + 8 (8 bytes each, 32-byte units
                    // swizzled by the row), its scales, and the matching 16 x values
                    const int unit = ((blk ^ g) << 5) + (t << 3);
                    const uint2 wa = *reinterpret_cast<const uint2*>(ws + g * 256 + unit);
                    const uint2 wb = *reinterpret_cast<const uint2*>(ws + (g + 8) * 256 + unit);
                    const uint32_t sa = e4m3_f16x2_splat(sc[g * 32 + 4 * blk + t]);
                    const uint32_t sb = e4m3_f16x2_splat(sc[(g + 8) * 32 + 4 * blk + t]);
                    const uint4 x0 = xq[blk * 8 + 2 * t], x1 = xq[blk * 8 + 2 * t + 1];
                    mma_nvfp4(d, wa.x, wb.x, sa, sb, x0.x, x0.y);
                    mma_nvfp4(e, wa.x >> 16, wb.x >> 16, sa, sb, x0.z, x0.w);
                    mma_nvfp4(d, wa.y, wb.y, sa, sb, x1.x, x1.y);
                    mma_nvfp4(e, wa.y >> 16, wb.y >> 16, sa, sb, x1.z, x1.w);
                }
            } else if (ok) {
                const int cols = (c == p.nch - 1) ? a.K - c * p.kc : p.kc;
                const uint8_t* ws = ring + static_cast<size_t>(slot) * kSlot;
                const uint4* xq = reinterpret_cast<const uint4*>(xs) + c * (kF8Cols / 8);
#pragma unroll 4
                for (int blk = 0; blk < cols / 64; ++blk) {
                    // lane (g, t): bytes 16t .. 16t + 15 of the block in rows g and g + 8 (16-byte group
                    // 4 blk + t, stored at group (4 blk + t) ^ g), and the matching x halves; 4-byte
                    // step s feeds one mma
                    const int grp = ((4 * blk + t) ^ g) * 16;
                    const uint4 wa = *reinterpret_cast<const uint4*>(ws + g * kF8Cols + grp);
                    const uint4 wb = *reinterpret_cast<const uint4*>(ws + (g + 8) * kF8Cols + grp);
                    const uint4 x0 = xq[blk * 8 + 2 * t], x1 = xq[blk * 8 + 2 * t + 1];
                    mma_e4m3_f16(d, wa.x, wb.x, x0.x, x0.y);
                    mma_e4m3_f16(e, wa.y, wb.y, x0.z, x0.w);
                    mma_e4m3_f16(d, wa.z, wb.z, x1.x, x1.y);
                    mma_e4m3_f16(e, wa.w, wb.w, x1.z, x1.w);
                }
            }
            // flush at the end of this warp's part of a tile: column 0 of D (lanes t == 0)
            if (c == p.nch - 1 || j == cnt - 1) {
                const int rl = tile * kF8Rows + g;
                if (t == 0) {
                    if (rl < nrows) part[rl * p.nch + c] = d[0] + e[0];
                    if (rl + 8 < nrows) part[(rl + 8) * p.nch + c] = d[2] + e[2];
                }
                d[0] = d[1] = d[2] = d[3] = 0.f;
                e[0] = e[1] = e[2] = e[3] = 0.f;
            }
            __syncwarp();
            if (!failed && j + p.stages < cnt) {
                fence_proxy_async();  // generic-proxy reads of this slot precede the async refill
                issue(i0 + j + p.stages, slot);
            }
        }
    }
    for (int j = 0; j < (F8 ? 0 : cnt); ++j) {  // BF16 (FP8 took the loop above)
        const int slot = j % p.stages;
        const bool ok = !failed && mbar_wait(&bars[slot], (j / p.stages) & 1, a.err, DEV_TMA_WAIT_TIMEOUT);
        failed = failed || !ok;
        const int item = i0 + j;
        const int rl = item / p.nch, c = item % p.nch;
        if (ok) {
            const int cols = (c == p.nch - 1) ? a.K - c * p.kc : p.kc;
            const int nv = cols * WB / 16;  // 16-byte weight vectors
            const uint4* wv = reinterpret_cast<const uint4*>(ring + static_cast<size_t>(slot) * p.kc * WB);
            const uint4* xv = reinterpret_cast<const uint4*>(xs + static_cast<size_t>(c) * p.kc);
            int v = lane;
            for (; v + 32 < nv; v += 64) {
                acc0 = dot8(wv[v], xv[v], acc0);
                acc1 = dot8(wv[v + 32], xv[v + 32], acc1);
            }
            if (v < nv) acc0 = dot8(wv[v], xv[v], acc0);
        }
        // flush at the end of this warp's part of a row
        if (c == p.nch - 1 || j == cnt - 1) {
            const float sum = warp_sum(acc0 + acc1);
            acc0 = acc1 = 0.f;
            if (lane == 0) part[rl * p.nch + c] = sum;
        }
        __syncwarp();
        if (lane == 0 && !failed && j + p.stages < cnt) {
            fence_proxy_async();  // generic-proxy reads of this slot precede the async refill
            issue(i0 + j + p.stages, slot);
        }
    }
    __syncthreads();
    if (tracing && tid == 0) tr_c3 = clock64();

    // ---- epilogue: row sums in fixed chunk order (FP8: times the row's power-of-two scale)
    auto row_sum = [&](int rl) {
        float r = 0.f;
        for (int c = 0; c < p.nch; ++c) r += part[rl * p.nch + c];
        if constexpr (F8) r = ldexpf(r, xshift) * a.wscale[r0 + rl];  // x carried 2^-xshift
        return r;
    };
    uint64_t best_key = 0;
    if (epi == EPI_SWIGLU) {
        for (int m = tid; m < nrows / 2; m += kThreads) {
            // qwen3.hpp:154-156 -> silu.cuh:18-20 on the BF16-rounded matmul outputs
            const float gv = round_bf(row_sum(2 * m)), uv = round_bf(row_sum(2 * m + 1));
            const float silu = gv / (1.0f + expf(-gv));
            a.y[(r0 >> 1) + m] = f2bf(silu * uv);
        }
    } else {
        // tensor parallel through peer memory: this kernel produces partial exchange xtag
        uint32_t tag = 0;
        if (epi == EPI_PARTIAL) {
            if (a.peer.world) tag = pair_tag(a.peer, a.xtag);
        }
        for (int rl = tid; rl < nrows; rl += kThreads) {
            const float r = row_sum(rl);
            const int gr = r0 + rl;
            if (epi == EPI_STORE) {
                a.y[gr] = f2bf(r);
            } else if (epi == EPI_PARTIAL) {
                if (a.peer.world) {
                    // this rank's partial row into every rank's slot: one 8-byte (value, tag)
                    // store per rank (NVLink to peers); no fence or flag needed
                    const size_t off =
                        (((a.xtag - 1) & 1) * static_cast<size_t>(a.peer.world) + a.peer.rank) * a.peer.H + gr;
                    const unsigned long long pair =
                        (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(r);
                    for (int j = 0; j < a.peer.world; ++j) a.peer.recv[j][off] = pair;
                } else {
                    a.yf[gr] = r;
                }
            } else if (epi == EPI_RESID) {
                // qwen3.hpp:158-159: hidden = bf16(down); hs = bf16(hs + hidden)
                const bf16 h = rl < kThreads ? hs_pre : a.hs[gr];
                a.hs[gr] = f2bf(bf2f(h) + round_bf(r));
            } else if (epi == EPI_RESID_F32) {
                // qwen3.hpp:151-152 -> rmsnorm.cuh:58-60
                const float v = bf2f(rl < kThreads ? hs_pre : a.hs[gr]) + round_bf(r);
                a.hs[gr] = f2bf(v);
                a.vsum_out[gr] = v;
            } else if (epi == EPI_QKV) {
                // q and k rows raw (the attention kernel normalises and rotates them), v to its slot
                const bf16 b = f2bf(r);
                if (gr < a.q_rows + a.kv_rows) {
                    a.q_out[gr] = b;
                } else {
                    const int k = gr - a.q_rows - a.kv_rows;
                    // head h of the page sits h * page_size rows after head 0
                    a.v_pages[v_slot + static_cast<size_t>(k >> 7) * a.page_size * 128 + (k & 127)] = b;
                }
            } else if (epi == EPI_ARGMAX) {
                const bf16 b = f2bf(r);
                a.y[gr] = b;
                best_key = max(best_key, argmax_key(bf2f(b), static_cast<uint32_t>(gr) + a.vocab_offset));
            }
        }
    }

    // ---- post-loop finishers
    if (epi == EPI_ARGMAX) {
        if (best_key) atomicMax(cta_key, static_cast<unsigned long long>(best_key));
        __syncthreads();
        if (tid == 0) {
            atomicMax(reinterpret_cast<unsigned long long*>(a.key_slot), *cta_key);
            __threadfence();
            const uint32_t old = atomicAdd(a.done_counter, 1u);
            if (old == gridDim.x - 1) {
                __threadfence();
                const unsigned long long k = atomicExch(reinterpret_cast<unsigned long long*>(a.key_slot), 0ull);
                if (a.peer.world) {
                    // this rank's best key to every rank, then the exchange flag
                    const unsigned long long s1 = peer_seq(a.peer) + 1;
                    const size_t off = (s1 & 1) * static_cast<size_t>(a.peer.world) + a.peer.rank;
                    for (int j = 0; j < a.peer.world; ++j) a.peer.keys[j][off] = k;
                    __threadfence_system();
                    for (int j = 0; j < a.peer.world; ++j)
                        st_release_sys(a.peer.flags[j] + (s1 & 1) * a.peer.world + a.peer.rank, static_cast<uint32_t>(s1));
                    *a.peer.seq = s1;
                } else {
                    *a.key_out = k;
                }
                *a.done_counter = 0u;
                atomicAdd(a.pos_inc, 1);
            }
        }
    }
    if (tracing) {
        __syncthreads();
        if (tid == 0 && static_cast<int>(blockIdx.x) < a.trace.ctas) {
            unsigned long long* t =
                a.trace.buf + (static_cast<size_t>(blockIdx.x) * a.trace.phases + a.trace.phase) * kTraceWords;
            const unsigned long long c4 = clock64();
            t[0] = tr_t0;
            t[1] = globaltimer_ns();
            t[2] = tr_c0;
            t[3] = c4;
            t[4] = tr_c1 - tr_c0;
            t[5] = tr_c2 - tr_c1;
            t[6] = tr_c3 - tr_c2;
            t[7] = c4 - tr_c3;
            t[8] = sm_id();
            t[9] = tr_cx ? tr_cx - tr_c1 : 0;  // exchange-consuming prologue: thread 0's rows complete
        }
    }
}

// The keys of the last exchange (lm_head of the last step) into out[world],
// for the host-side readers of the greedy token.
__global__ void peer_keys_kernel(const PeerLinks x, unsigned long long* out, uint32_t* err) {
    const unsigned long long s = peer_seq(x);
    if (s == 0) return;
    peer_wait(x, s, err);
    if (threadIdx.x < static_cast<unsigned>(x.world))
        out[threadIdx.x] = __ldcg(x.keys[x.rank] + (s & 1) * x.world + threadIdx.x);
}

template <int PRO, int EPI>
cudaError_t launch_t(const GemvArgs& a, cudaStream_t s, bool pdl) {
    auto* fn = !a.W8 ? gemv_kernel<PRO, EPI, 0> : a.plan.wb == 0 ? gemv_kernel<PRO, EPI, 2> : gemv_kernel<PRO, EPI, 1>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.plan.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = a.plan.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, a);
}

}  // namespace

cudaError_t launch_peer_keys(const PeerLinks& x, unsigned long long* out, uint32_t* err, cudaStream_t s) {
    peer_keys_kernel<<<1, 32, 0, s>>>(x, out, err);
    return cudaGetLastError();
}

template <int PRO, int EPI>
cudaError_t configure_pair() {
    for (const void* f : {reinterpret_cast<const void*>(gemv_kernel<PRO, EPI, 0>),
                          reinterpret_cast<const void*>(gemv_kernel<PRO, EPI, 1>),
                          reinterpret_cast<const void*>(gemv_kernel<PRO, EPI, 2>)}) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
        // the whole carve-out as shared memory, so a CTA of the next (PDL-launched) kernel fits beside
        // this one where the two footprints allow
        if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t configure_gemv_kernels() {
    cudaError_t e = cudaSuccess;
#define Q3_CFG(P, E) \
    if (e == cudaSuccess) e = configure_pair<P, E>();
    Q3_CFG(PRO_PLAIN, EPI_STORE)
    Q3_CFG(PRO_PLAIN, EPI_RESID)
    Q3_CFG(PRO_PLAIN, EPI_RESID_F32)
    Q3_CFG(PRO_PLAIN, EPI_PARTIAL)
    Q3_CFG(PRO_NORM, EPI_STORE)
    Q3_CFG(PRO_NORM, EPI_QKV)
    Q3_CFG(PRO_EMBED_NORM, EPI_QKV)
    Q3_CFG(PRO_RESID_NORM, EPI_QKV)
    Q3_CFG(PRO_NORM_F32, EPI_SWIGLU)
    Q3_CFG(PRO_RESID_NORM, EPI_SWIGLU)
    Q3_CFG(PRO_NORM, EPI_ARGMAX)
    Q3_CFG(PRO_RESID_NORM, EPI_ARGMAX)
#undef Q3_CFG
    return e;
}

F8Pack f8_pack_for(int N, int K, int epi, int sms) {
    const GemvPlan p = plan_gemv(N, K, epi, sms, 1);
    return F8Pack{N, K, (K + kF8TileCols - 1) / kF8TileCols, p.grid, p.row_gran, 0};
}

F8Pack f4_pack_for(int N, int K, int epi, int sms) {
    const GemvPlan p = plan_gemv(N, K, epi, sms, 0);
    return F8Pack{N, K, (K + kF4TileCols - 1) / kF4TileCols, p.grid, p.row_gran, 1};
}

GemvPlan plan_gemv(int N, int K, int epi, int sms, int wb) {
    GemvPlan p{};
    p.row_gran = (epi == EPI_SWIGLU) ? 2 : 1;
    p.wb = wb;
    // BF16: 4 KB row segments; FP8: 16-row tiles of 256 columns; NVFP4: of 512
    const int chunk = wb == 2 ? kChunk : wb == 1 ? kF8Cols : kF4TileCols;
    p.kc = K < chunk ? K : chunk;
    p.nch = (K + p.kc - 1) / p.kc;
    const int units = N / p.row_gran;
    // one CTA per SM, more only if the per-CTA partial sums would not fit
    const long long items = static_cast<long long>(N) * p.nch;
    int grid = std::min(sms, units);
    const long long min_grid = (items + kMaxItems - 1) / kMaxItems;
    if (grid < min_grid) grid = static_cast<int>(std::min<long long>(min_grid, units));
    p.grid = std::max(1, grid);
    p.max_units = (units + p.grid - 1) / p.grid;
    const int max_rows = p.max_units * p.row_gran;
    const size_t budget = wb == 2 ? kSmemBudget : kSmemBudgetF8;
    for (p.stages = Q3_GEMV_MAX_STAGES; p.stages > 2; --p.stages)
        if (smem_layout(p, K, max_rows).total <= budget) break;
    p.smem = smem_layout(p, K, max_rows).total;
    return p;
}

GemvPlan plan_gemv_early(int N, int K, int epi, int sms, int early_ctas) {
    GemvPlan p = plan_gemv(N, K, epi, sms, 2);
    const int units = N / p.row_gran, E = early_ctas;
    if (E <= 0 || E >= p.grid) return p;
    // the ring an early CTA fills before the dependency release, in units of rows
    const double ring_units = static_cast<double>(kWarps) * p.stages * slot_bytes(p) /
                              (static_cast<double>(K) * 2 * p.row_gran);
    // equal bytes left after the release: b_E - ring = b_L, E b_E + (grid - E) b_L = units
    const double b_late = std::max(0.0, (units - E * ring_units) / p.grid);
    long long early_units = std::llround(E * (b_late + ring_units));
    early_units = std::min<long long>(std::max<long long>(early_units, (static_cast<long long>(units) * E) / p.grid),
                                      units);
    const int max_early = static_cast<int>((early_units + E - 1) / E);
    // the per-CTA partial sums must still fit
    if (static_cast<long long>(max_early) * p.row_gran * p.nch > kMaxItems) return p;
    p.early = E;
    p.early_units = static_cast<int>(early_units);
    p.max_units = std::max(max_early, (units - p.early_units + (p.grid - E) - 1) / (p.grid - E));
    const int max_rows = p.max_units * p.row_gran;
    for (p.stages = Q3_GEMV_MAX_STAGES; p.stages > 2; --p.stages)
        if (smem_layout(p, K, max_rows).total <= kSmemBudget) break;
    p.smem = smem_layout(p, K, max_rows).total;
    return p;
}

cudaError_t launch_gemv(int pro, int epi, const GemvArgs& a, cudaStream_t s, bool pdl) {
    // the plan's item width must match the weight format; packed rows are whole 64-column blocks
    if ((a.W8 ? a.plan.wb == 2 : a.plan.wb != 2) || (a.W8 && (a.K % 64 != 0 || !a.wscale)))
        return cudaErrorInvalidValue;
#define Q3_CASE(P, E) \
    if (pro == P && epi == E) return launch_t<P, E>(a, s, pdl);
    Q3_CASE(PRO_PLAIN, EPI_STORE)
    Q3_CASE(PRO_PLAIN, EPI_RESID)
    Q3_CASE(PRO_PLAIN, EPI_RESID_F32)
    Q3_CASE(PRO_PLAIN, EPI_PARTIAL)
    Q3_CASE(PRO_NORM, EPI_STORE)
    Q3_CASE(PRO_NORM, EPI_QKV)
    Q3_CASE(PRO_EMBED_NORM, EPI_QKV)
    Q3_CASE(PRO_RESID_NORM, EPI_QKV)
    Q3_CASE(PRO_NORM_F32, EPI_SWIGLU)
    Q3_CASE(PRO_RESID_NORM, EPI_SWIGLU)
    Q3_CASE(PRO_NORM, EPI_ARGMAX)
    Q3_CASE(PRO_RESID_NORM, EPI_ARGMAX)
#undef Q3_CASE
    return cudaErrorInvalidValue;
}

}  // namespace q3

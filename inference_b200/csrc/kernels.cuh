// kernels.cuh -- argument blocks and host launchers of the sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace q3 {

// ---------------------------------------------------------------- launch timeline
// Graph-path tracing (q3_engine_trace): launch `phase` of a step writes, per
// CTA (linear block index below `ctas`), Q3_TRACE_WORDS words at
// buf[(cta * phases + phase) * Q3_TRACE_WORDS]: [0] / [1] %globaltimer at CTA
// start / end, [2] / [3] clock64 there, SM cycles of [4] start -> dependency
// wait returned, [5] prologue, [6] main loop, [7] epilogue, [8] SM id, [9] (a
// prologue over the ranks' partials) cycles from [4]'s end until thread 0 held
// every rank's partials of its first rows.
struct LaunchTrace {
    unsigned long long* buf;  // null: off
    int phase, phases, ctas;
};
constexpr int kTraceWords = Q3_TRACE_WORDS;

// ---------------------------------------------------------------- GEMV
// y = W x for one token, W row-major [N, K] BF16, fp32 accumulation.
// The prologue builds x in shared memory; the epilogue consumes each row sum.
enum GemvPro : int {
    PRO_PLAIN = 0,       // x = src (BF16 vector of K)
    PRO_NORM = 1,        // x = rmsnorm(hs) over rounded hs
    PRO_NORM_F32 = 2,    // x = rmsnorm with sum of squares over fp32 vsum, values bf16(vsum)
    PRO_EMBED_NORM = 3,  // token -> hs = embed[token]; x = rmsnorm(hs)
    PRO_RESID_NORM = 4,  // hs' = bf16(hs + bf16(reduced)); x = rmsnorm(hs') (tensor parallel)
};
enum GemvEpi : int {
    EPI_STORE = 0,      // y[r] = bf16(acc)
    EPI_RESID = 1,      // hs[r] = bf16(hs[r] + bf16(acc))
    EPI_RESID_F32 = 2,  // v = hs[r] + bf16(acc); hs[r] = bf16(v); vsum[r] = v
    EPI_SWIGLU = 3,     // rows (2j, 2j+1) = (gate_j, up_j): y[j] = bf16(silu(bf16 g) * bf16 u)
    EPI_QKV = 4,        // q and k rows (raw) to q_out, v rows to the paged KV slot
    EPI_ARGMAX = 5,     // logits[r] = bf16(acc); running (max, first index) across the grid
    EPI_PARTIAL = 6,    // yf[r] = acc (fp32 partial for a tensor-parallel reduction)
};

struct GemvPlan {
    int kc;        // columns per (row, chunk) work item: min(K, 2048), a multiple of 8
    int nch;       // chunks per row, ceil(K / kc); the last may be shorter
    int stages;    // per-warp shared-memory ring depth
    int grid;      // CTAs
    int row_gran;  // rows assigned to CTAs in units of this many (2 for SWIGLU)
    int wb;        // bytes per weight: 2 = BF16, 1 = FP8 E4M3
    size_t smem;   // dynamic shared memory bytes
    // Row bands: by default units (row_gran rows each) are spread evenly over the grid.
    // early > 0: CTAs [0, early) share early_units units and the rest the remainder --
    // for a GEMV launched beside a kernel that occupies some SMs, whose first CTAs start
    // (and fill their rings) early while the others wait for SMs to free up.
    int early, early_units;
    int max_units;  // the largest band
};
// Units [u0, u1) of CTA b's band.
__host__ __device__ inline void gemv_band(const GemvPlan& p, int units, int b, int& u0, int& u1) {
    if (p.early > 0 && p.early < p.grid) {
        const int late = p.grid - p.early;
        if (b < p.early) {
            u0 = static_cast<int>(static_cast<long long>(b) * p.early_units / p.early);
            u1 = static_cast<int>(static_cast<long long>(b + 1) * p.early_units / p.early);
        } else {
            const int r = b - p.early, rest = units - p.early_units;
            u0 = p.early_units + static_cast<int>(static_cast<long long>(r) * rest / late);
            u1 = p.early_units + static_cast<int>(static_cast<long long>(r + 1) * rest / late);
        }
    } else {
        u0 = static_cast<int>(static_cast<long long>(b) * units / p.grid);
        u1 = static_cast<int>(static_cast<long long>(b + 1) * units / p.grid);
    }
}

// Tensor-parallel exchange through peer memory (CUDA IPC mappings over
// NVLink).  Rank j's buffer holds, per slot (exchange parity), every rank's
// fp32 partial vector as [world][H] 8-byte (value, tag) pairs -- a pair is
// one store, so a reader that sees the expected tag sees the value -- plus a
// flag and an argmax key per rank for the lm_head exchange.  world == 0
// selects the NCCL path.
constexpr int kMaxRanks = 8;
struct PeerLinks {
    unsigned long long* recv[kMaxRanks];  // rank j's [2][world][H] (value, tag) pairs, mapped into this process
    uint32_t* flags[kMaxRanks];           // rank j's [2][world]: exchange number that filled the slot
    unsigned long long* keys[kMaxRanks];  // rank j's [2][world] argmax keys
    unsigned long long* seq;              // lm_head exchanges (= steps) this rank has run (never reset)
    uint32_t* counter;                    // CTA arrivals of the producing kernel
    int rank, world, H;
};

struct GemvArgs {
    const bf16* W;
    // FP8 weights (used when W8 is set): E4M3 bytes, row-major [N, K], and a
    // power-of-two scale per row; row r of the matrix is W8[r, :] * wscale[r]
    const uint8_t* W8;
    const float* wscale;
    int N, K;
    GemvPlan plan;
    // ---- prologue
    const bf16* x;             // PRO_PLAIN source
    bf16* hs;                  // residual stream read by PRO_NORM*/PRO_RESID_NORM, updated by EPI_RESID*
    bf16* hs_out;              // PRO_EMBED_NORM / PRO_RESID_NORM: residual written by CTA 0
    const bf16* norm_w;        // RMSNorm weight [K]
    float eps;
    const float* vsum;         // PRO_NORM_F32 fp32 sums; PRO_RESID_NORM: fp32 reduced partials
    int ss_unrounded;          // PRO_RESID_NORM: sum of squares over unrounded (rmsnorm_add) values
    const bf16* embed;         // PRO_EMBED_NORM table [vocab, K]
    int vocab;                 // full vocabulary
    int32_t* tokens;           // tokens by position (forced prefix + greedy)
    int32_t* argmax_hist;      // greedy argmax by position
    const int32_t* n_forced;   // forced prefix length
    const uint64_t* keys;      // per-rank argmax keys of the previous step
    int n_keys;
    const int32_t* pos_ptr;    // current position
    int capacity;
    // ---- epilogue
    bf16* y;
    float* yf;
    float* vsum_out;
    // EPI_QKV: q rows then k rows to q_out, v rows to the v page slot of pos
    int q_rows, kv_rows, head_dim, kv_heads_local, page_size;
    bf16* q_out;
    bf16* v_pages;
    const int32_t* page_table;
    // EPI_ARGMAX
    uint64_t* key_slot;
    uint32_t* done_counter;
    uint64_t* key_out;
    int32_t* pos_inc;          // incremented once by the last CTA
    uint32_t vocab_offset;
    // ---- tensor-parallel exchange (EPI_PARTIAL / EPI_ARGMAX produce, PRO_RESID_NORM /
    // PRO_EMBED_NORM consume); peer.world == 0: NCCL path through yf / vsum / keys.
    // xtag: the partial exchange produced (EPI_PARTIAL) or consumed (PRO_RESID_NORM),
    // 1 .. 2 L within a step (o_proj of layer l: 2 l + 1, down_proj: 2 l + 2)
    PeerLinks peer;
    int xtag;
    uint32_t tune;             // Q3_TUNE_PEER_* bits (q3_engine_set_tuning)
    // ---- errors
    uint32_t* err;
    LaunchTrace trace;
};

GemvPlan plan_gemv(int N, int K, int epi, int num_sms, int wb = 2);
// plan_gemv for a BF16 GEMV whose first `early_ctas` CTAs start beside the kernel
// before it: their bands grow by what their shared-memory rings prefetch there, so
// that every CTA has the same bytes left to stream once the dependency is released.
GemvPlan plan_gemv_early(int N, int K, int epi, int num_sms, int early_ctas);
cudaError_t launch_gemv(int pro, int epi, const GemvArgs& a, cudaStream_t s, bool pdl);

// ---------------------------------------------------------------- attention
struct AttnArgs {
    const bf16* q;            // [q_heads, 128]
    const bf16* k;            // paged: [pages, kvh, page, 128]; flat: [capacity, kvh, 128]
    const bf16* v;
    const int32_t* page_table;
    bf16* out;                // [q_heads, 128]
    int q_heads, kv_heads, page_size;
    int paged;                // 1 = paged layout, 0 = reference layout
    const int32_t* pos_ptr;   // device position (or null -> pos_host)
    int pos_host;
    int splits;               // grid.x = cluster size: a power of two <= 16
    uint32_t* err;
    // batch of consecutive query positions (prefill): query i sits at position
    // pos + i, reads q + i * q_stride and writes out + i * out_stride.  0 or 1 =
    // the single decode query.
    int n_queries, q_stride, out_stride;
    // Decode step with q/k RMSNorm + RoPE fused in (qk_norm_rope.cuh:14-90), k_raw
    // set: q holds the raw q heads, k_raw [kv_heads, 128] this position's raw key
    // rows; every CTA normalises and rotates its q heads, the CTAs whose split
    // holds the position's page put the normalised key row into their K tile,
    // and those of the first query-head block store it to its cache slot.
    const bf16* k_raw;
    const bf16* q_norm;
    const bf16* k_norm;
    const float* rope_cos;
    const float* rope_sin;
    float eps;
    LaunchTrace trace;
    // batched decode (paged, n_queries rows): query i sits at position row_pos[i] and
    // uses the page table page_table + i * pt_stride
    const int32_t* row_pos;
    int pt_stride;
    // Extent of the cache the tensor maps cover: paged, physical pages in the pool
    // (0 = not known: the page table is trusted); flat, positions (0 = pos + queries).
    int pool;
    // Filled by launch_attention: 3-D tensor maps of K and V (128-byte swizzle, boxes
    // of 64 rows x 64 columns) for the page loads.
    CUtensorMap tk, tv;
};
int attn_splits(int kv_heads, int max_pos, int page_size, int num_sms);
// Query heads one attention CTA handles (of a GQA group of G), and the SMs a decode
// launch occupies (one CTA per SM).
int attn_heads_per_cta(int G);
int attn_sms_used(int q_heads, int kv_heads, int splits);
size_t attn_workspace_bytes(int q_heads, int kv_heads, int splits);
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl);

// cuTensorMapEncodeTiled, resolved once through the runtime (null if unavailable).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// ---------------------------------------------------------------- prefill GEMM (tcgen05)
enum GemmEpi : int { GEMM_STORE = 0, GEMM_SWIGLU = 1, GEMM_RESID = 2, GEMM_F32 = 3 };
struct GemmArgs {
    const bf16* x;  // [M, K] row-major (tokens)
    const bf16* w;  // [N, K] row-major (weights as stored)
    bf16* y;        // STORE: [M, ldy] <- XW^T; SWIGLU: [M, ldy] <- swiglu of column pairs; RESID: [M, ldy] += XW^T
    float* vsum;    // RESID only (optional): [M, ldy] fp32 sums before rounding
    float* yf;      // F32 only: [M, ldy] <- XW^T unrounded (a tensor-parallel partial)
    int M, N, K, ldy;
    int epi;        // GemmEpi
    int bn;         // output tile width 128 / 256, 0 = choose
    uint32_t* err;
    // Split-K for one 128-row tile with few output tiles (batched decode): ws holds
    // ws_floats fp32 for the splits' partial tiles; null = no split.  Set by the
    // caller; launch_gemm picks the split count.
    float* ws;
    size_t ws_floats;
    int sms;
    // internal (launch_gemm): k-tiles per split, fp32 elements between splits' partials
    int kt_per;
    size_t yf_split;
};
cudaError_t launch_peer_keys(const PeerLinks& x, unsigned long long* out, uint32_t* err, cudaStream_t s);
int gemm_tile_n(int M, int N, int sms);
cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t s);
cudaError_t configure_gemm_kernels();  // every variant's shared-memory opt-in (before graph capture)

// ---------------------------------------------------------------- prefill rows
struct PrefillQkvArgs {
    bf16* qkv;                  // [n, ld]: q heads, k heads, v heads of each token
    int ld, q_heads, kv_heads, p0;
    const bf16 *q_norm, *k_norm;
    const float *rope_cos, *rope_sin;
    bf16 *k_pages, *v_pages;
    const int32_t* page_table;
    float eps;
    // batched decode: row r sits at position row_pos[r] (not p0 + r) and uses the page
    // table page_table + r * pt_stride
    const int32_t* row_pos;
    int pt_stride;
};
// Row r takes token row_tokens[r] when row_tokens is set, else tokens[p0 + r].
cudaError_t launch_embed_rows(const bf16* table, const int32_t* tokens, int p0, int n, int vocab, int H, bf16* x,
                              uint32_t* err, cudaStream_t s, const int32_t* row_tokens = nullptr);
// out[r] = first index of the largest BF16 value of logits[r * ld .. r * ld + n) (the
// greedy sampler, backend.cu:107-112, per row).
cudaError_t launch_argmax_rows(const bf16* logits, int rows, int n, int ld, int32_t* out, cudaStream_t s);
cudaError_t launch_rmsnorm_rows(const bf16* x, const float* vsum, const bf16* w, bf16* xn, int n, int H, float eps,
                                cudaStream_t s);
cudaError_t launch_qkv_rows(const PrefillQkvArgs& a, int n, cudaStream_t s);

// Tensor-parallel prefill exchange.  Every rank's GEMM (GEMM_F32) writes its
// fp32 partial rows into slot (seq & 1) of its own buffer (part[rank], slots
// slot_floats apart), raises flags[j][slot * kMaxRanks + rank] = seq in every
// rank's buffer (launch_tp_signal), and every rank adds the sum over all ranks'
// slots, in rank order, to its residual rows (launch_tp_resid_rows; part[j] of
// a peer is its CUDA IPC mapping).  flags[rank] == null: no flags to wait for
// (world 1: a buffer NCCL has already allreduced).  A rank overwrites a slot
// two exchanges later, after every rank raised its flag for the exchange in
// between, which it does only after reading the slot.
struct TpExchange {
    const float* part[kMaxRanks];
    uint32_t* flags[kMaxRanks];
    size_t slot_floats;
    int rank, world;
};
cudaError_t launch_tp_signal(const TpExchange& x, uint32_t seq, cudaStream_t s);
cudaError_t launch_tp_resid_rows(const TpExchange& x, uint32_t seq, int n, int H, bf16* xr, float* vsum, uint32_t* err,
                                 int num_sms, cudaStream_t s);

// ---------------------------------------------------------------- small ops
cudaError_t launch_embedding(const bf16* table, int hidden, uint32_t token, bf16* out, cudaStream_t s);
cudaError_t launch_rmsnorm(const bf16* x, const bf16* w, bf16* out, int n, float eps, cudaStream_t s);
cudaError_t launch_rmsnorm_add(bf16* res, const bf16* upd, const bf16* w, bf16* out, int n, float eps,
                               cudaStream_t s);
cudaError_t launch_qk_norm_rope(bf16* q, bf16* k, const bf16* qn, const bf16* kn, const float* cos_t,
                                const float* sin_t, int q_heads, int kv_heads, int pos, float eps, cudaStream_t s);
cudaError_t launch_rope(bf16* v, const float* cos_t, const float* sin_t, int heads, int head_dim, int pos,
                        cudaStream_t s);
cudaError_t launch_add(const bf16* a, const bf16* b, bf16* out, size_t n, cudaStream_t s);
cudaError_t launch_silu_mul(const bf16* g, const bf16* u, bf16* out, size_t n, cudaStream_t s);
cudaError_t launch_argmax(const bf16* logits, size_t n, uint32_t* index, uint64_t* scratch, cudaStream_t s);
cudaError_t launch_fill_normal(bf16* dst, uint64_t seed, uint64_t tensor_id, size_t rows, size_t cols, size_t row0,
                               size_t col0, size_t full_cols, size_t dst_row_stride, cudaStream_t s);
cudaError_t launch_fill_const(bf16* dst, size_t n, float value, cudaStream_t s);
cudaError_t launch_resolve_tokens(const uint64_t* keys, int n_keys, int32_t* tokens, int32_t* argmax_hist,
                                  const int32_t* pos_ptr, const int32_t* n_forced, int vocab, uint32_t* err,
                                  cudaStream_t s);

uint64_t seed_key(uint64_t seed);
// Shared-memory opt-in of every kernel instantiation on the current device;
// called once per device before any launch (and before graph capture).
cudaError_t configure_kernels();
cudaError_t configure_gemv_kernels();

// ---------------------------------------------------------------- FP8 weights
// The FP8 GEMV's weight layout ("packed"): the [N, K] E4M3 matrix cut into the
// row bands of its CTAs (the GEMV plan: `grid` bands of whole row_gran units),
// each band into 16-row tiles (the last one shorter) and each tile into
// 256-column chunks; item (tile, chunk) of a band is rows_t x 256 contiguous
// bytes (rows_t = the tile's rows; columns past K are zero), so one bulk copy
// fetches it, and inside an item row r keeps its 16-byte column group j at
// group j ^ (r & 7), so the tensor-core fragment loads hit distinct banks.
struct F8Pack {
    int N, K, nch, grid, row_gran;  // N == 0: plain row-major with pitch K
    int fmt;                        // 0: E4M3 (256-column chunks); 1: NVFP4 (512-column chunks)
};
constexpr int kF8TileRows = 16;
constexpr int kF8TileCols = 256;
// The band of GEMV rows holding `row` (the plan's uniform split into whole
// row_gran units), and the row's tile t, row rr in the tile and the tile's rows.
__host__ __device__ inline void pack_tile(const F8Pack& L, int row, int& r0, int& t, int& rr, int& rows_t) {
    const int U = L.N / L.row_gran, u = row / L.row_gran;
    int b = static_cast<int>(static_cast<long long>(u) * L.grid / U);
    while (b + 1 < L.grid && static_cast<int>(static_cast<long long>(b + 1) * U / L.grid) <= u) ++b;
    const int u0 = static_cast<int>(static_cast<long long>(b) * U / L.grid);
    const int u1 = static_cast<int>(static_cast<long long>(b + 1) * U / L.grid);
    r0 = u0 * L.row_gran;
    const int nrows = (u1 - u0) * L.row_gran;
    const int rl = row - r0;
    t = rl / kF8TileRows;
    rr = rl % kF8TileRows;
    rows_t = nrows - t * kF8TileRows < kF8TileRows ? nrows - t * kF8TileRows : kF8TileRows;
}
__host__ __device__ inline size_t f8_offset(const F8Pack& L, int row, int col) {
    if (L.N == 0) return static_cast<size_t>(row) * L.K + col;
    int r0, t, rr, rows_t;
    pack_tile(L, row, r0, t, rr, rows_t);
    const int c = col / kF8TileCols, g = (col % kF8TileCols) / 16;
    return (static_cast<size_t>(r0) * L.nch + static_cast<size_t>(t) * kF8TileRows * L.nch +
            static_cast<size_t>(c) * rows_t + rr) * kF8TileCols + ((g ^ (rr & 7)) << 4) + (col & 15);
}
// NVFP4 (fmt 1): E2M1 weights in 512-column chunks, one E4M3 scale per 16 columns.
// Item (tile, chunk) = rows_t x 256 bytes of nibbles, then rows_t x 32 block
// scales.  In row rr of an item: columns 64 u .. 64 u + 63 (unit u) sit in the
// 32 bytes at (u ^ (rr & 7)) * 32, the unit's 16-column block j at byte 8 j of
// them, column 2 i of the block in the low nibble of byte i; block b of the
// chunk has its scale at byte rows_t * 256 + rr * 32 + b.
constexpr int kF4TileCols = 512;
constexpr int kF4RowBytes = 256 + 32;
__host__ __device__ inline size_t f4_item_base(const F8Pack& L, int row, int col, int& rr, int& rows_t) {
    int r0, t;
    pack_tile(L, row, r0, t, rr, rows_t);
    const int c = col / kF4TileCols;
    return (static_cast<size_t>(r0) * L.nch + static_cast<size_t>(t) * kF8TileRows * L.nch +
            static_cast<size_t>(c) * rows_t) * kF4RowBytes;
}
// The byte holding column col (a multiple of 2: the low nibble; col + 1 the high one).
__host__ __device__ inline size_t f4_nibble_offset(const F8Pack& L, int row, int col) {
    int rr, rows_t;
    const size_t base = f4_item_base(L, row, col, rr, rows_t);
    const int cc = col % kF4TileCols, u = cc / 64;
    return base + static_cast<size_t>(rr) * 256 + ((u ^ (rr & 7)) << 5) + ((cc % 64) / 16) * 8 + (cc % 16) / 2;
}
// The scale byte of column col's 16-column block.
__host__ __device__ inline size_t f4_scale_offset(const F8Pack& L, int row, int col) {
    int rr, rows_t;
    const size_t base = f4_item_base(L, row, col, rr, rows_t);
    return base + static_cast<size_t>(rows_t) * 256 + static_cast<size_t>(rr) * 32 + (col % kF4TileCols) / 16;
}
inline size_t f4_packed_bytes(int N, int K) {
    return static_cast<size_t>(N) * ((K + kF4TileCols - 1) / kF4TileCols) * kF4RowBytes;
}
F8Pack f4_pack_for(int N, int K, int epi, int num_sms);
inline size_t f8_packed_bytes(int N, int K) {
    return static_cast<size_t>(N) * ((K + kF8TileCols - 1) / kF8TileCols) * kF8TileCols;
}
// The packed layout the GEMV with this epilogue uses for an [N, K] matrix.
F8Pack f8_pack_for(int N, int K, int epi, int num_sms);

// Where quantized rows go: source row r to matrix row row0 + r * row_step of
// `base` (laid out by `pack`), its scale to scale[row0 + r * row_step].
struct F8Dst {
    uint8_t* base;
    float* scale;
    F8Pack pack;
    int row0, row_step;
};
// Row-wise E4M3 quantization with power-of-two scales: for each of `rows`
// rows of src (BF16, row pitch ld_src elements, full_cols columns) the scale
// is 2^e, e the smallest integer with max|row| <= 448 * 2^e; columns
// [c0, c0 + cols) are written as E4M3(x / 2^e) (round to nearest even,
// saturating) to columns 0 .. cols - 1 of the destination rows.
cudaError_t launch_quantize_e4m3(const bf16* src, size_t ld_src, int rows, int full_cols, int c0, int cols,
                                 const F8Dst& dst, cudaStream_t s);
// Row-major E4M3 [N, K] (pitch K) -> the packed layout `pack` (zero padding included).
cudaError_t launch_pack_e4m3(const uint8_t* q, const F8Pack& pack, uint8_t* packed, cudaStream_t s);
// The packed matrix's exact BF16 values times the row scales, row-major [N, K] (K % 16 == 0).
cudaError_t launch_dequant_e4m3(const uint8_t* packed, const float* scale, const F8Pack& pack, bf16* out,
                                cudaStream_t s);
// NVFP4 with power-of-two row scales: for each of `rows` rows of src the row scale
// is 2^e, e the smallest integer with max|row| / 6 <= 448 * 2^e; each block b of
// 16 columns of [c0, c0 + cols) gets the E4M3 scale s = E4M3(amax_b / 6 * 2^-e)
// and its weights E2M1(w * 2^-e / s) (nearest, ties to even, saturating at 6;
// 0 when s is 0), written to columns 0 .. cols - 1 of the destination rows of
// an NVFP4 pack (c0 and cols multiples of 16).
cudaError_t launch_quantize_nvfp4(const bf16* src, size_t ld_src, int rows, int full_cols, int c0, int cols,
                                  const F8Dst& dst, cudaStream_t s);
// The NVFP4-packed matrix's exact BF16 values (E2M1 x block scale x row scale), row-major [N, K].
cudaError_t launch_dequant_nvfp4(const uint8_t* packed, const float* scale, const F8Pack& pack, bf16* out,
                                 cudaStream_t s);
cudaError_t configure_attention_kernels();
int num_sms(int device);

}  // namespace q3

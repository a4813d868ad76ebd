// engine_state.hpp -- the decode engine's state (struct q3_engine), shared by
// engine.cu (the single-sequence engine) and batch.cu (batched decode on the
// same weights).
#pragma once

#include <vector>

#include "host_util.hpp"
#include "kernels.cuh"
#include "nccl_dyn.hpp"

namespace q3 {

constexpr int kPageSize = 64;

struct LayerW {
    bf16 *w_qkv, *w_o, *w_gu, *w_down;  // BF16 engines
    // FP8 engines: E4M3 matrices of the same shapes and one scale per row
    uint8_t *f_qkv, *f_o, *f_gu, *f_down;
    float *s_qkv, *s_o, *s_gu, *s_down;
    bf16 *in_norm, *post_norm, *q_norm, *k_norm;
    bf16 *k_pages, *v_pages;
};

}  // namespace q3

struct q3_engine {
    q3_model_config cfg{};
    int device = 0, rank = 0, world = 1, sms = 148;
    cudaStream_t stream = nullptr;
    // local (per-rank) dimensions
    int H = 0, qh = 0, kvh = 0, qd = 0, kd = 0, il = 0, vl = 0;
    uint32_t voff = 0;
    // weights
    q3::bf16 *embed = nullptr, *lm_head = nullptr, *final_norm = nullptr;
    bool fp8 = false;  // packed GEMV matrices (Q3_WEIGHTS_FP8_E4M3 or Q3_WEIGHTS_NVFP4) + row scales
    bool fp4 = false;  // ... and they are NVFP4
    uint8_t* f_lm = nullptr;
    float* s_lm = nullptr;
    std::vector<q3::LayerW> layers;
    int n_pages = 0;
    int32_t* page_table = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    // activations
    q3::bf16 *hs[2] = {nullptr, nullptr}, *q = nullptr, *attn = nullptr, *g = nullptr, *logits = nullptr;
    float *vsum = nullptr, *partial = nullptr;
    // control state
    int32_t *pos = nullptr, *n_forced = nullptr, *tokens = nullptr, *argmax_hist = nullptr;
    uint64_t *key_slot = nullptr, *key_send = nullptr, *keys = nullptr;
    uint32_t *done_counter = nullptr, *err = nullptr;
    int attn_splits = 1;
    int o_early = 0;  // o_proj GEMV CTAs that start beside attention (plan_gemv_early)
    // opt-in variants of the graph path (Q3_TUNE_*)
    uint32_t tune = 0;
    // CUDA-graph path timeline: per launch of a step and CTA (q3_engine_trace)
    bool gtrace = false;
    unsigned long long* d_gtrace = nullptr;
    int gtrace_ctas = 0;
    // batched prefill: token-row buffers of prefill_rows rows (allocated on first use)
    int prefill_rows = 0;
    q3::bf16 *px = nullptr, *pxn = nullptr, *pqkv = nullptr, *pattn = nullptr, *pg = nullptr;
    q3::bf16* pw = nullptr;  // FP8 engines (Q3_TUNE_FP8_PREFILL): one layer matrix expanded to BF16
    float* pvsum = nullptr;
    // split-K partial tiles of the row GEMMs with one 128-row tile (batched decode, short prompts)
    float* split_ws = nullptr;
    size_t split_ws_floats = 0;
    // tensor-parallel exchange through peer memory: this rank's buffer (shared
    // with the peers by CUDA IPC), the peers' mappings, local counters
    void* xbuf = nullptr;
    size_t xbuf_bytes = 0;
    void* xpeer[q3::kMaxRanks] = {};
    q3::PeerLinks links{};
    bool peer_mode = false;
    // tensor-parallel batched prefill (Q3_TUNE_TP_PREFILL): the partial-row slots
    // and flags appended to xbuf, and the exchanges run so far (all ranks agree)
    q3::TpExchange tpx{};
    uint32_t tp_seq = 0;
    // graph / comms
    cudaGraphExec_t graph = nullptr;
    ncclComm_t comm = nullptr;
    // NCCL exchange bounds (q3_engine_set_comm_timeout): a host wait on this rank's stream
    // gives up comm_timeout_s (plus a per-step allowance for the queued steps) after it
    // starts, aborts the communicator and reports Q3_ERR_NCCL; comm_dead after that
    double comm_timeout_s = 60.0;
    size_t queued_steps = 0;
    bool comm_dead = false;
    size_t host_pos = 0, host_forced = 0, host_max_pos = 0;
    size_t weight_bytes = 0;
    std::vector<void*> allocs;
};

namespace q3 {

// Rows through the model with the batched kernels (row RMSNorm, tcgen05 GEMMs,
// per-row q/k norm + RoPE + cache writes, split-KV attention over each row's own
// prefix): the batched prefill of one sequence, or one batched decode step of
// several sequences.
struct RowsSpec {
    int n = 0;
    // row r: token tokens[p0 + r] at position p0 + r (one sequence's prompt) ...
    const int32_t* tokens = nullptr;
    int p0 = 0;
    // ... or token row_tokens[r] at position row_pos[r] with its page table
    // page_table + r * pt_stride (device arrays)
    const int32_t* row_tokens = nullptr;
    const int32_t* row_pos = nullptr;
    const int32_t* page_table = nullptr;
    int pt_stride = 0;
    // per layer K and V page pools of pool_pages pages (null: the engine's own)
    bf16* const* k_pools = nullptr;
    bf16* const* v_pools = nullptr;
    int pool_pages = 0;
    int max_pos = 0;      // the largest position of any row (sizes the attention splits)
    int attn_splits = 0;  // 0: from max_pos, at least 8 pages per split (many rows of one prompt)
    // set: the whole last layer, the final RMSNorm and lm_head into logits [n][vocab]
    bf16* logits = nullptr;
};
int forward_rows(q3_engine* e, const RowsSpec& r);
// The batched-row buffers (px, pxn, ...) for kPrefillRows rows, allocated on first use.
int ensure_rows(q3_engine* e);
constexpr int kPrefillRows = 512;  // rows per batched forward

}  // namespace q3

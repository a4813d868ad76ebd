// engine.cu -- the decode engine: Qwen3 Model + paged KVCache + greedy loop on
// one GPU (one tensor-parallel rank), behind the q3_engine_* C ABI.
//
// Reference semantics followed: Model::build / forward / prefill
// (src/lib/model/qwen3/qwen3.hpp:105-173), KVCache (src/lib/kv_cache/
// kv_cache.hpp:6-29), make_rope_cache (src/lib/backend/util/rope_cache.hpp:
// 23-45) and the Generator loop (src/lib/inference/generator.cpp:37-63).
//
// B200 design:
//   * one decode step = 5 kernels per layer + 1 (QKV, attention, O, gate/up,
//     down; lm_head+argmax), all PDL-launched, captured once into a CUDA graph
//     and replayed per token; the token id, position and argmax live in device
//     memory so consecutive steps run back to back with no host round trip;
//   * weights are pre-packed once: q/k/v rows concatenated, gate/up rows
//     interleaved (gate_j, up_j), each rank holding its tensor-parallel shard;
//   * KV cache: per layer [pages, kv_heads, 64, 128] BF16 pages and a page
//     table; a (page, head) block is one contiguous 16 KB TMA copy;
//   * tensor parallel ranks run the row-parallel GEMVs (o_proj, down_proj)
//     into fp32 partials, allreduce them with NCCL, and fold the residual add
//     into the next GEMV's prologue; lm_head is vocab-sharded and the per-rank
//     (value, index) keys are all-gathered and resolved in the next step.

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "engine_state.hpp"

namespace q3 {
bool engine_tied(const q3_engine* e) { return e->cfg.tied != 0; }
size_t engine_layers(const q3_engine* e) { return e->layers.size(); }
size_t engine_capacity(const q3_engine* e) { return e->cfg.capacity; }
}  // namespace q3

namespace q3 {
namespace {

// Tensor-parallel exchange buffer, one per rank, shared by CUDA IPC:
// decode pairs [2][world][H] u64 | flags [2][world] u32 | keys [2][world] u64 |
// (256-aligned) prefill flags [2][kMaxRanks] u32 | (at +256) prefill partial
// rows [2][rows][H] fp32.
struct XbufLayout {
    size_t flags_off, keys_off, pf_flags_off, pf_part_off, total;
};
XbufLayout xbuf_layout(size_t world, size_t H, size_t rows) {
    XbufLayout L{};
    L.flags_off = 2 * world * H * 8;
    L.keys_off = (L.flags_off + 2 * world * 4 + 15) / 16 * 16;
    L.pf_flags_off = (L.keys_off + 2 * world * 8 + 255) / 256 * 256;
    L.pf_part_off = L.pf_flags_off + 256;
    L.total = L.pf_part_off + 2 * rows * H * 4;
    return L;
}

int dalloc(q3_engine* e, void** p, size_t bytes) {
    if (bytes == 0) bytes = 16;
    cudaError_t st = cudaMalloc(p, bytes);
    if (st != cudaSuccess) {
        set_error(std::string("cudaMalloc(") + std::to_string(bytes) + "): " + cudaGetErrorString(st));
        return st == cudaErrorMemoryAllocation ? Q3_ERR_OOM : Q3_ERR_CUDA;
    }
    e->allocs.push_back(*p);
    return Q3_OK;
}

template <class T>
int dalloc_t(q3_engine* e, T** p, size_t count) {
    return dalloc(e, reinterpret_cast<void**>(p), count * sizeof(T));
}

// Bytes of an [N, K] GEMV matrix in the engine's packed weight format.
size_t packed_bytes(const q3_engine* e, int N, int K) {
    return e->fp4 ? f4_packed_bytes(N, K) : f8_packed_bytes(N, K);
}

// Device bytes, zeroed.
int dalloc_zero(q3_engine* e, uint8_t** p, size_t bytes) {
    int rc = dalloc(e, reinterpret_cast<void**>(p), bytes);
    if (rc == Q3_OK && cudaMemset(*p, 0, bytes) != cudaSuccess) return fail(Q3_ERR_CUDA, "cudaMemset failed");
    return rc;
}

#define Q3_TRY(x)                  \
    do {                           \
        int rc_ = (x);             \
        if (rc_ != Q3_OK) return rc_; \
    } while (0)

// ------------------------------------------------------------ NCCL, bounded
// The communicator is non-blocking (ncclConfig_t.blocking = 0): every call
// returns at once, and ncclCommGetAsyncError reports when it has settled.  A
// peer that never arrives would otherwise hold this rank forever, so every
// host-side wait is bounded and ends by aborting the communicator.
void abort_comm(q3_engine* e) {
    if (e->comm) nccl().CommAbort(e->comm);  // also stops this rank's NCCL kernels still waiting on peers
    e->comm = nullptr;
    e->comm_dead = true;
}

double seconds_since(const std::chrono::steady_clock::time_point& t0) {
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

// Waits (bounded) until the communicator's last non-blocking call has settled.
int nccl_settle(q3_engine* e, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t r = nccl().CommGetAsyncError(e->comm, &st);
        if (r != ncclSuccess) st = r;
        if (st == ncclSuccess) return Q3_OK;
        if (st != ncclInProgress) {
            const std::string msg = std::string(what) + ": " + nccl().GetErrorString(st);
            abort_comm(e);
            return fail(Q3_ERR_NCCL, msg);
        }
        if (seconds_since(t0) > e->comm_timeout_s) {
            abort_comm(e);
            return fail(Q3_ERR_NCCL, std::string(what) + ": timed out; communicator aborted");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

// A NCCL call's immediate result: in progress means settle before going on.
int nccl_check(q3_engine* e, ncclResult_t nr, const char* what) {
    if (nr == ncclInProgress) return nccl_settle(e, what);
    if (nr != ncclSuccess) {
        const std::string msg = std::string(what) + ": " + nccl().GetErrorString(nr);
        abort_comm(e);
        return fail(Q3_ERR_NCCL, msg);
    }
    return Q3_OK;
}

// Host wait for the engine's stream.  NCCL engines poll it with a deadline of
// comm_timeout_s plus 0.25 s per step queued since the last wait: a rank whose
// peer has gone aborts the communicator (its NCCL kernels then return) and
// reports Q3_ERR_NCCL instead of waiting without end.
int stream_wait(q3_engine* e) {
    if (e->comm_dead) return fail(Q3_ERR_NCCL, "NCCL communicator aborted after a failed exchange");
    if (!e->comm) {
        Q3_CUDA(cudaStreamSynchronize(e->stream));
        e->queued_steps = 0;
        return Q3_OK;
    }
    const double limit = e->comm_timeout_s + 0.25 * static_cast<double>(e->queued_steps);
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(e->stream);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) return fail(Q3_ERR_CUDA, std::string("stream: ") + cudaGetErrorString(q));
        ncclResult_t st = ncclSuccess;
        if (nccl().CommGetAsyncError(e->comm, &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress) {
            const std::string msg = std::string("NCCL exchange failed: ") + nccl().GetErrorString(st);
            abort_comm(e);
            return fail(Q3_ERR_NCCL, msg);
        }
        if (seconds_since(t0) > limit) {
            // No wait for the stream after the abort: a collective captured in the step
            // graph may keep its kernel waiting on the departed peer, and the host must
            // get control back.  The engine refuses further work; the process should
            // tear down its CUDA context (exit) to reclaim that kernel.
            abort_comm(e);
            return fail(Q3_ERR_NCCL, "NCCL exchange: a peer did not arrive within " + std::to_string(limit) +
                                         " s; communicator aborted");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    e->queued_steps = 0;
    return Q3_OK;
}

// ------------------------------------------------------------ one decode step
struct Recorder {
    q3_engine* e;
    bool pdl;
    // optional per-kernel timing (eager profiling)
    int klass = -1;  // 0 GEMV, 1 attention, 2 all
    std::vector<cudaEvent_t>* ev = nullptr;
    double* bytes = nullptr;
    size_t launches = 0;
    int phase = 0;  // launches recorded so far in this step (the timeline's phase index)

    LaunchTrace trace() {
        LaunchTrace t{};
        if (e->gtrace) t = LaunchTrace{e->d_gtrace, phase, static_cast<int>(e->layers.size()) * 5 + 1, e->gtrace_ctas};
        ++phase;
        return t;
    }

    void mark(bool begin, int kind) {
        if (!ev || !(klass == 2 || klass == kind)) return;
        cudaEvent_t x;
        cudaEventCreate(&x);
        cudaEventRecord(x, e->stream);
        ev->push_back(x);
        if (!begin) ++launches;
    }
};

GemvArgs base_args(q3_engine* e) {
    GemvArgs a{};
    if (e->peer_mode) a.peer = e->links;
    a.tune = e->tune;
    a.eps = e->cfg.eps;
    a.err = e->err;
    a.capacity = static_cast<int>(e->cfg.capacity);
    a.pos_ptr = e->pos;
    return a;
}

// One GEMV matrix in either storage format.
struct WMat {
    const bf16* w;
    const uint8_t* q;  // FP8 E4M3 (q and s set) or null
    const float* s;
};

// early_ctas > 0 (BF16 weights): the GEMV runs after a kernel that leaves that many
// SMs free, so its first CTAs start beside it (plan_gemv_early)
int gemv(Recorder& r, int pro, int epi, GemvArgs a, WMat W, int N, int K, int early_ctas = 0) {
    a.W = W.w;
    a.W8 = W.q;
    a.wscale = W.s;
    a.N = N;
    a.K = K;
    a.plan = (early_ctas > 0 && !W.q) ? plan_gemv_early(N, K, epi, r.e->sms, early_ctas)
                                      : plan_gemv(N, K, epi, r.e->sms, W.q ? (r.e->fp4 ? 0 : 1) : 2);
    a.trace = r.trace();
    r.mark(true, 0);
    cudaError_t st = launch_gemv(pro, epi, a, r.e->stream, r.pdl);
    r.mark(false, 0);
    if (r.bytes && (r.klass == 0 || r.klass == 2))
        *r.bytes += W.q ? static_cast<double>(N) * K * (r.e->fp4 ? 0.5625 : 1.0) + N * 4.0 + K * 2.0 + N * 2.0
                        : static_cast<double>(N) * K * 2 + K * 2.0 + N * 2.0;
    if (st != cudaSuccess) return fail(Q3_ERR_CUDA, std::string("gemv launch: ") + cudaGetErrorString(st));
    return Q3_OK;
}

int attention(Recorder& r, const LayerW& L, size_t pos_now) {
    q3_engine* e = r.e;
    AttnArgs a{};
    a.q = e->q;
    a.k = L.k_pages;
    a.v = L.v_pages;
    a.page_table = e->page_table;
    a.out = e->attn;
    a.q_heads = e->qh;
    a.kv_heads = e->kvh;
    a.page_size = kPageSize;
    a.paged = 1;
    a.pool = e->n_pages;
    a.pos_ptr = e->pos;
    a.splits = e->attn_splits;
    a.err = e->err;
    // q/k RMSNorm + RoPE of this step (the QKV GEMV leaves the raw k rows after q)
    a.k_raw = e->q + e->qd;
    a.q_norm = L.q_norm;
    a.k_norm = L.k_norm;
    a.rope_cos = e->rope_cos;
    a.rope_sin = e->rope_sin;
    a.eps = e->cfg.eps;
    a.trace = r.trace();
    r.mark(true, 1);
    cudaError_t st = launch_attention(a, e->stream, r.pdl);
    r.mark(false, 1);
    if (r.bytes && (r.klass == 1 || r.klass == 2))
        *r.bytes += 2.0 * (pos_now + 1) * e->kvh * 128 * 2 + 2.0 * e->qd * 2;
    if (st != cudaSuccess) return fail(Q3_ERR_CUDA, std::string("attention launch: ") + cudaGetErrorString(st));
    return Q3_OK;
}

int allreduce(q3_engine* e, float* buf, size_t n) {
    if (e->peer_mode) return Q3_OK;  // the producing GEMV exchanged its partials through peer memory
    if (!e->comm) return fail(Q3_ERR_NCCL, "NCCL communicator aborted");
    return nccl_check(e, nccl().AllReduce(buf, buf, n, ncclFloat32, ncclSum, e->comm, e->stream), "ncclAllReduce");
}

int record_step(Recorder& r, size_t pos_now) {
    q3_engine* e = r.e;
    const q3_model_config& c = e->cfg;
    const bool tp = e->world > 1;
    int cur = 0;  // residual buffer holding hs (tensor-parallel ping-pong)
    for (size_t l = 0; l < e->layers.size(); ++l) {
        const LayerW& L = e->layers[l];
        const WMat w_qkv{L.w_qkv, L.f_qkv, L.s_qkv}, w_o{L.w_o, L.f_o, L.s_o};
        const WMat w_gu{L.w_gu, L.f_gu, L.s_gu}, w_down{L.w_down, L.f_down, L.s_down};
        // ---- QKV (+ embedding / residual / RMSNorm prologue, qk-norm + RoPE + KV write epilogue)
        GemvArgs a = base_args(e);
        a.norm_w = L.in_norm;
        a.q_rows = e->qd;
        a.kv_rows = e->kd;
        a.head_dim = 128;
        a.kv_heads_local = e->kvh;
        a.page_size = kPageSize;
        a.q_out = e->q;  // q rows, then the raw key rows (normalised by the attention kernel)
        a.v_pages = L.v_pages;
        a.page_table = e->page_table;
        int pro;
        if (l == 0) {
            pro = PRO_EMBED_NORM;
            a.embed = e->embed;
            a.vocab = static_cast<int>(c.vocab);
            a.tokens = e->tokens;
            a.argmax_hist = e->argmax_hist;
            a.n_forced = e->n_forced;
            a.keys = e->keys;
            a.n_keys = e->world;
            a.hs_out = e->hs[0];
            cur = 0;
        } else if (tp) {
            pro = PRO_RESID_NORM;
            a.xtag = 2 * static_cast<int>(l);  // the previous layer's down_proj exchange
            a.hs = e->hs[cur];
            a.hs_out = e->hs[cur ^ 1];
            a.vsum = e->partial;
            a.ss_unrounded = 0;  // qwen3.hpp:159 add, then :137 rmsnorm of the rounded residual
            cur ^= 1;
        } else {
            pro = PRO_NORM;
            a.hs = e->hs[0];
        }
        Q3_TRY(gemv(r, pro, EPI_QKV, a, w_qkv, e->qd + 2 * e->kd, e->H));
        // ---- attention
        Q3_TRY(attention(r, L, pos_now));
        // ---- o_proj (+ residual add); its first CTAs start on the SMs attention leaves free
        GemvArgs o = base_args(e);
        o.x = e->attn;
        if (tp) {
            o.yf = e->partial;
            o.xtag = 2 * static_cast<int>(l) + 1;
            Q3_TRY(gemv(r, PRO_PLAIN, EPI_PARTIAL, o, w_o, e->H, e->qd, e->o_early));
            Q3_TRY(allreduce(e, e->partial, e->H));
        } else {
            o.hs = e->hs[0];
            o.vsum_out = e->vsum;
            Q3_TRY(gemv(r, PRO_PLAIN, EPI_RESID_F32, o, w_o, e->H, e->qd, e->o_early));
        }
        // ---- gate/up (+ RMSNorm prologue, SwiGLU epilogue)
        GemvArgs gu = base_args(e);
        gu.norm_w = L.post_norm;
        gu.y = e->g;
        if (tp) {
            gu.xtag = 2 * static_cast<int>(l) + 1;
            gu.hs = e->hs[cur];
            gu.hs_out = e->hs[cur ^ 1];
            gu.vsum = e->partial;
            gu.ss_unrounded = 1;  // rmsnorm_add (rmsnorm.cuh:58-60) squares the unrounded sums
            cur ^= 1;
            Q3_TRY(gemv(r, PRO_RESID_NORM, EPI_SWIGLU, gu, w_gu, 2 * e->il, e->H));
        } else {
            gu.hs = e->hs[0];
            gu.vsum = e->vsum;
            Q3_TRY(gemv(r, PRO_NORM_F32, EPI_SWIGLU, gu, w_gu, 2 * e->il, e->H));
        }
        // ---- down_proj (+ residual add)
        GemvArgs d = base_args(e);
        d.x = e->g;
        if (tp) {
            d.yf = e->partial;
            d.xtag = 2 * static_cast<int>(l) + 2;
            Q3_TRY(gemv(r, PRO_PLAIN, EPI_PARTIAL, d, w_down, e->H, e->il));
            Q3_TRY(allreduce(e, e->partial, e->H));
        } else {
            d.hs = e->hs[0];
            Q3_TRY(gemv(r, PRO_PLAIN, EPI_RESID, d, w_down, e->H, e->il));
        }
    }
    // ---- final RMSNorm + lm_head + argmax (vocab shard)
    const WMat w_lm{e->lm_head, e->f_lm, e->s_lm};
    GemvArgs h = base_args(e);
    h.norm_w = e->final_norm;
    h.y = e->logits;
    h.key_slot = e->key_slot;
    h.done_counter = e->done_counter;
    h.key_out = tp ? e->key_send : e->keys;
    h.pos_inc = e->pos;
    h.vocab_offset = e->voff;
    if (tp) {
        h.xtag = 2 * static_cast<int>(e->layers.size());
        h.hs = e->hs[cur];
        h.hs_out = e->hs[cur ^ 1];
        h.vsum = e->partial;
        h.ss_unrounded = 0;
        Q3_TRY(gemv(r, PRO_RESID_NORM, EPI_ARGMAX, h, w_lm, e->vl, e->H));
        if (!e->peer_mode) {
            if (!e->comm) return fail(Q3_ERR_NCCL, "NCCL communicator aborted");
            Q3_TRY(nccl_check(e, nccl().AllGather(e->key_send, e->keys, 1, ncclUint64, e->comm, e->stream),
                              "ncclAllGather"));
        }
    } else {
        h.hs = e->hs[0];
        Q3_TRY(gemv(r, PRO_NORM, EPI_ARGMAX, h, w_lm, e->vl, e->H));
    }
    return Q3_OK;
}

int build_graph(q3_engine* e) {
    if (e->graph) return Q3_OK;
    if (e->comm_dead) return fail(Q3_ERR_NCCL, "NCCL communicator aborted after a failed exchange");
    if (e->world > 1 && !e->comm && !e->peer_mode)
        return fail(Q3_ERR_INVALID, "tensor-parallel engine needs q3_engine_attach_peers or q3_engine_attach_nccl");
    Recorder r{e, true};
    cudaGraph_t g = nullptr;
    Q3_CUDA(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    int rc = record_step(r, 0);
    cudaError_t st = cudaStreamEndCapture(e->stream, &g);
    if (rc != Q3_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (st != cudaSuccess) return fail(Q3_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(st));
    st = cudaGraphInstantiate(&e->graph, g, 0);
    cudaGraphDestroy(g);
    if (st != cudaSuccess) return fail(Q3_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(st));
    return Q3_OK;
}

int check_device_error(q3_engine* e) {
    uint32_t err = 0;
    Q3_CUDA(cudaMemcpy(&err, e->err, sizeof(err), cudaMemcpyDeviceToHost));
    if (err != 0) {
        static const char* names[] = {"ok", "TMA wait timed out", "peer wait timed out", "token id out of range",
                                      "position out of range", "grid barrier timed out"};
        // clear the error so the engine stays usable
        cudaMemset(e->err, 0, 4);
        return fail(Q3_ERR_DEVICE, std::string("device error: ") + (err < 6 ? names[err] : "unknown"));
    }
    return Q3_OK;
}

// Host rope tables exactly as make_rope_cache (rope_cache.hpp:29-41): fp32,
// inv_freq = 1/pow(theta, 2i/hd), cos/sin(float(p) * inv_freq).
// c and s hold max_pos * hd / 2 floats each.
void rope_tables(size_t max_pos, size_t hd, float theta, float* c, float* s) {
    const size_t half = hd / 2;
    std::vector<float> inv(half);
    for (size_t i = 0; i < half; ++i) {
        const float ex = 2.0F * static_cast<float>(i) / static_cast<float>(hd);
        inv[i] = 1.0F / std::pow(theta, ex);
    }
    for (size_t p = 0; p < max_pos; ++p)
        for (size_t i = 0; i < half; ++i) {
            const float ang = static_cast<float>(p) * inv[i];
            c[p * half + i] = std::cos(ang);
            s[p * half + i] = std::sin(ang);
        }
}

}  // namespace
}  // namespace q3

using namespace q3;

extern "C" {

int q3_engine_create(const q3_model_config* cfg, int device, int tp_rank, int tp_size, q3_engine** out) {
    Q3_CHECK(cfg && out, "q3_engine_create: null argument");
    *out = nullptr;
    const q3_model_config& c = *cfg;
    Q3_CHECK(tp_size >= 1 && tp_rank >= 0 && tp_rank < tp_size, "q3_engine_create: bad tensor-parallel rank");
    Q3_CHECK(tp_size <= kMaxRanks, "q3_engine_create: at most 8 tensor-parallel ranks");
    // peer-exchange tags number the 2 L partial exchanges of a step in 8 bits
    Q3_CHECK(tp_size == 1 || c.layers <= 127, "q3_engine_create: tensor parallelism supports up to 127 layers");
    if (c.head_dim != 128) return fail(Q3_ERR_UNSUPPORTED, "q3_engine_create: head_dim must be 128");
    Q3_CHECK(c.layers > 0 && c.hidden > 0 && c.vocab > 0 && c.capacity > 1, "q3_engine_create: empty config");
    Q3_CHECK(c.kv_heads > 0 && c.q_heads % c.kv_heads == 0, "q3_engine_create: q_heads % kv_heads != 0");
    const uint32_t G = c.q_heads / c.kv_heads;
    if (!(G == 1 || G == 2 || G == 4 || G == 8)) return fail(Q3_ERR_UNSUPPORTED, "GQA group must be 1/2/4/8");
    Q3_CHECK(c.kv_heads % tp_size == 0, "kv_heads must divide by the tensor-parallel size");
    Q3_CHECK(c.inter % tp_size == 0 && (c.inter / tp_size) % 8 == 0, "intermediate/tp must be a multiple of 8");
    Q3_CHECK(c.vocab % tp_size == 0, "vocab must divide by the tensor-parallel size");
    Q3_CHECK(c.hidden % 8 == 0 && c.hidden <= 32768, "hidden must be a multiple of 8 (<= 32768)");
    Q3_CHECK(c.capacity < (1u << 24), "capacity too large");
    Q3_CHECK(c.weight_format == Q3_WEIGHTS_BF16 || c.weight_format == Q3_WEIGHTS_FP8_E4M3 ||
                 c.weight_format == Q3_WEIGHTS_NVFP4,
             "q3_engine_create: unknown weight_format");
    Q3_CHECK(c.weight_format == Q3_WEIGHTS_BF16 || (c.hidden % 64 == 0 && (c.inter / tp_size) % 64 == 0 &&
                                                    (c.q_heads / tp_size * c.head_dim) % 64 == 0),
             "FP8 / NVFP4 weights need hidden, intermediate/tp and q_heads/tp x head_dim multiples of 64");

    auto* e = new q3_engine();
    e->cfg = c;
    e->fp8 = c.weight_format != Q3_WEIGHTS_BF16;
    e->fp4 = c.weight_format == Q3_WEIGHTS_NVFP4;
    e->device = device;
    e->rank = tp_rank;
    e->world = tp_size;
    int rc = Q3_OK;
    auto bail = [&](int code) {
        q3_engine_destroy(e);
        return code;
    };
    if (cudaSetDevice(device) != cudaSuccess) return bail(fail(Q3_ERR_CUDA, "cudaSetDevice failed"));
    e->sms = num_sms(device);
    if (configure_kernels() != cudaSuccess) return bail(fail(Q3_ERR_CUDA, "kernel attribute setup failed"));
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(Q3_ERR_CUDA, "cudaStreamCreate failed"));

    e->H = static_cast<int>(c.hidden);
    e->qh = static_cast<int>(c.q_heads / tp_size);
    e->kvh = static_cast<int>(c.kv_heads / tp_size);
    e->qd = e->qh * 128;
    e->kd = e->kvh * 128;
    e->il = static_cast<int>(c.inter / tp_size);
    e->vl = static_cast<int>(c.vocab / tp_size);
    e->voff = static_cast<uint32_t>(e->vl) * static_cast<uint32_t>(tp_rank);
    const size_t H = e->H;

    // ---- weights
    if ((rc = dalloc_t(e, &e->embed, static_cast<size_t>(c.vocab) * H)) != Q3_OK) return bail(rc);
    if (e->fp8) {
        // the embedding stays BF16 for the lookup; lm_head gets its own E4M3 copy
        if ((rc = dalloc_zero(e, &e->f_lm, packed_bytes(e, e->vl, e->H))) != Q3_OK) return bail(rc);
        if ((rc = dalloc_t(e, &e->s_lm, static_cast<size_t>(e->vl))) != Q3_OK) return bail(rc);
    } else if (c.tied) {
        e->lm_head = e->embed + static_cast<size_t>(e->voff) * H;
    } else if ((rc = dalloc_t(e, &e->lm_head, static_cast<size_t>(e->vl) * H)) != Q3_OK) {
        return bail(rc);
    }
    if ((rc = dalloc_t(e, &e->final_norm, H)) != Q3_OK) return bail(rc);
    e->n_pages = static_cast<int>((c.capacity + kPageSize - 1) / kPageSize);
    const size_t page_elems = static_cast<size_t>(e->n_pages) * e->kvh * kPageSize * 128;
    e->layers.resize(c.layers);
    const size_t rows_qkv = static_cast<size_t>(e->qd + 2 * e->kd), rows_gu = 2 * static_cast<size_t>(e->il);
    for (auto& L : e->layers) {
        L = LayerW{};
        if (e->fp8) {
            // packed layouts (packed_bytes), zero so the column padding is zero
            if ((rc = dalloc_zero(e, &L.f_qkv, packed_bytes(e, static_cast<int>(rows_qkv), e->H))) != Q3_OK) return bail(rc);
            if ((rc = dalloc_zero(e, &L.f_o, packed_bytes(e, e->H, e->qd))) != Q3_OK) return bail(rc);
            if ((rc = dalloc_zero(e, &L.f_gu, packed_bytes(e, static_cast<int>(rows_gu), e->H))) != Q3_OK) return bail(rc);
            if ((rc = dalloc_zero(e, &L.f_down, packed_bytes(e, e->H, e->il))) != Q3_OK) return bail(rc);
            if ((rc = dalloc_t(e, &L.s_qkv, rows_qkv)) != Q3_OK) return bail(rc);
            if ((rc = dalloc_t(e, &L.s_o, H)) != Q3_OK) return bail(rc);
            if ((rc = dalloc_t(e, &L.s_gu, rows_gu)) != Q3_OK) return bail(rc);
            if ((rc = dalloc_t(e, &L.s_down, H)) != Q3_OK) return bail(rc);
        } else {
            if ((rc = dalloc_t(e, &L.w_qkv, rows_qkv * H)) != Q3_OK) return bail(rc);
            if ((rc = dalloc_t(e, &L.w_o, H * e->qd)) != Q3_OK) return bail(rc);
            if ((rc = dalloc_t(e, &L.w_gu, rows_gu * H)) != Q3_OK) return bail(rc);
            if ((rc = dalloc_t(e, &L.w_down, H * e->il)) != Q3_OK) return bail(rc);
        }
        if ((rc = dalloc_t(e, &L.in_norm, H)) != Q3_OK) return bail(rc);
        if ((rc = dalloc_t(e, &L.post_norm, H)) != Q3_OK) return bail(rc);
        if ((rc = dalloc_t(e, &L.q_norm, 128)) != Q3_OK) return bail(rc);
        if ((rc = dalloc_t(e, &L.k_norm, 128)) != Q3_OK) return bail(rc);
        if ((rc = dalloc_t(e, &L.k_pages, page_elems)) != Q3_OK) return bail(rc);
        if ((rc = dalloc_t(e, &L.v_pages, page_elems)) != Q3_OK) return bail(rc);
        if (cudaMemset(L.k_pages, 0, page_elems * 2) != cudaSuccess ||
            cudaMemset(L.v_pages, 0, page_elems * 2) != cudaSuccess)
            return bail(fail(Q3_ERR_CUDA, "KV cache memset failed"));
    }
    // bytes streamed per decode step by this rank (weights read by the GEMVs + norms + one embedding row)
    // (FP8: one byte per weight plus a 4-byte scale per row; NVFP4: half a byte plus a block scale per
    // 16 weights and a 4-byte scale per row)
    const size_t mat_elems = rows_qkv * H + H * e->qd + rows_gu * H + H * e->il;
    const size_t mat_rows = rows_qkv + H + rows_gu + H;
    auto packed_weights = [&](size_t elems) { return e->fp4 ? elems / 2 + elems / 16 : elems; };
    const size_t per_layer = e->fp8 ? packed_weights(mat_elems) + mat_rows * 4 + (2 * H + 256) * 2
                                    : (mat_elems + 2 * H + 256) * 2;
    const size_t lm_bytes = e->fp8 ? packed_weights(static_cast<size_t>(e->vl) * H) + static_cast<size_t>(e->vl) * 4
                                   : static_cast<size_t>(e->vl) * H * 2;
    e->weight_bytes = per_layer * c.layers + lm_bytes + H * 2 + H * 2;

    // ---- page table (identity for a single sequence) and RoPE tables
    std::vector<int32_t> pt(e->n_pages);
    for (int i = 0; i < e->n_pages; ++i) pt[i] = i;
    if ((rc = dalloc_t(e, &e->page_table, pt.size())) != Q3_OK) return bail(rc);
    if (cudaMemcpy(e->page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return bail(fail(Q3_ERR_CUDA, "page table upload failed"));
    std::vector<float> cs(static_cast<size_t>(c.capacity) * 64), sn(cs.size());
    rope_tables(c.capacity, 128, c.theta, cs.data(), sn.data());
    if ((rc = dalloc_t(e, &e->rope_cos, cs.size())) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->rope_sin, sn.size())) != Q3_OK) return bail(rc);
    if (cudaMemcpy(e->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(e->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return bail(fail(Q3_ERR_CUDA, "rope table upload failed"));

    // ---- activations and control
    if ((rc = dalloc_t(e, &e->hs[0], H)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->hs[1], H)) != Q3_OK) return bail(rc);
    // q, then this step's raw key rows (the attention kernel normalises them)
    if ((rc = dalloc_t(e, &e->q, static_cast<size_t>(e->qd) + e->kd)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->attn, e->qd)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->g, e->il)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->logits, e->vl)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->vsum, H)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->partial, H)) != Q3_OK) return bail(rc);
    cudaError_t setup = cudaSuccess;  // the first failure of the set-up copies below
    auto note = [&setup](cudaError_t st) {
        if (setup == cudaSuccess) setup = st;
    };
    if (tp_size > 1) {
        // exchange buffer (xbuf_layout): decode pairs, flags and keys, then the prefill slots
        const size_t pf_rows = std::min<size_t>(kPrefillRows, c.capacity);
        const XbufLayout xl = xbuf_layout(static_cast<size_t>(tp_size), static_cast<size_t>(H), pf_rows);
        e->xbuf_bytes = xl.total;
        e->tpx.slot_floats = pf_rows * static_cast<size_t>(H);
        e->tpx.rank = tp_rank;
        e->tpx.world = tp_size;
        if ((rc = dalloc(e, &e->xbuf, e->xbuf_bytes)) != Q3_OK) return bail(rc);
        note(cudaMemset(e->xbuf, 0, e->xbuf_bytes));
        unsigned long long* seq = nullptr;
        if ((rc = dalloc_t(e, &seq, 2)) != Q3_OK) return bail(rc);
        note(cudaMemset(seq, 0, 16));
        e->links.seq = seq;
        e->links.counter = reinterpret_cast<uint32_t*>(seq + 1);
        e->links.rank = tp_rank;
        e->links.world = tp_size;
        e->links.H = H;
    }
    if ((rc = dalloc_t(e, &e->pos, 4)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->n_forced, 4)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->tokens, c.capacity + 1)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->argmax_hist, c.capacity + 1)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->key_slot, 2)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->key_send, 2)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->keys, static_cast<size_t>(tp_size) + 1)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->done_counter, 4)) != Q3_OK) return bail(rc);
    if ((rc = dalloc_t(e, &e->err, 4)) != Q3_OK) return bail(rc);
    note(cudaMemset(e->pos, 0, 16));
    note(cudaMemset(e->n_forced, 0, 16));
    note(cudaMemset(e->tokens, 0, (c.capacity + 1) * 4));
    note(cudaMemset(e->argmax_hist, 0xFF, (c.capacity + 1) * 4));
    note(cudaMemset(e->key_slot, 0, 16));
    note(cudaMemset(e->key_send, 0, 16));
    note(cudaMemset(e->keys, 0, (tp_size + 1) * 8));
    note(cudaMemset(e->done_counter, 0, 16));
    note(cudaMemset(e->err, 0, 4));

    // ---- attention: splits of the full context merge inside one thread-block cluster
    e->attn_splits = attn_splits(e->kvh, static_cast<int>(c.capacity) - 1, kPageSize, e->sms);
    {
        // decode attention occupies attn_sms_used SMs; the SMs it leaves free start the
        // o_proj GEMV's first CTAs while it runs
        e->o_early = std::max(0, e->sms - attn_sms_used(e->qh, e->kvh, e->attn_splits));
    }

    if (setup != cudaSuccess)
        return bail(fail(Q3_ERR_CUDA, std::string("engine setup copy: ") + cudaGetErrorString(setup)));
    if (cudaDeviceSynchronize() != cudaSuccess) return bail(fail(Q3_ERR_CUDA, "engine setup failed"));
    *out = e;
    return Q3_OK;
}

int q3_engine_destroy(q3_engine* e) {
    if (!e) return Q3_OK;
    cudaSetDevice(e->device);
    if (e->comm && stream_wait(e) != Q3_OK) {
        // a peer is gone: stream_wait aborted the communicator; the stream may still hold
        // a kernel waiting on that peer, so it is not waited for
    } else if (e->stream && !e->comm_dead) {
        cudaStreamSynchronize(e->stream);
    }
    if (e->graph) cudaGraphExecDestroy(e->graph);
    if (e->comm) nccl().CommDestroy(e->comm);
    for (void* p : e->xpeer)
        if (p) cudaIpcCloseMemHandle(p);
    for (void* p : e->allocs) cudaFree(p);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
    return Q3_OK;
}

namespace {

// A temporary device buffer of BF16 weights (FP8 engines quantize from it).
struct Staging {
    bf16* p = nullptr;
    ~Staging() {
        if (p) cudaFree(p);
    }
    int alloc(size_t elems) {
        if (cudaMalloc(&p, elems * 2) != cudaSuccess) {
            p = nullptr;
            return fail(Q3_ERR_OOM, "weight staging buffer: cudaMalloc failed");
        }
        return Q3_OK;
    }
};

int quant(q3_engine* e, const bf16* src, size_t ld_src, size_t rows, size_t full_cols, size_t c0, size_t cols,
          const F8Dst& d) {
    if (d.pack.fmt == 1)
        Q3_CUDA(launch_quantize_nvfp4(src, ld_src, static_cast<int>(rows), static_cast<int>(full_cols),
                                      static_cast<int>(c0), static_cast<int>(cols), d, e->stream));
    else
        Q3_CUDA(launch_quantize_e4m3(src, ld_src, static_cast<int>(rows), static_cast<int>(full_cols),
                                     static_cast<int>(c0), static_cast<int>(cols), d, e->stream));
    return Q3_OK;
}

// The packed matrices as quantize destinations, each in the packed layout of the
// GEMV that reads it (record_step's shapes and epilogues).
F8Pack pack_for(const q3_engine* e, int N, int K, int epi) {
    return e->fp4 ? f4_pack_for(N, K, epi, e->sms) : f8_pack_for(N, K, epi, e->sms);
}
F8Dst dst_qkv(const q3_engine* e, const LayerW& L, int row0) {
    return F8Dst{L.f_qkv, L.s_qkv, pack_for(e, e->qd + 2 * e->kd, e->H, EPI_QKV), row0, 1};
}
F8Dst dst_o(const q3_engine* e, const LayerW& L) {
    return F8Dst{L.f_o, L.s_o, pack_for(e, e->H, e->qd, e->world > 1 ? EPI_PARTIAL : EPI_RESID_F32), 0, 1};
}
F8Dst dst_gu(const q3_engine* e, const LayerW& L, int up) {  // gate row j -> row 2 j, up row j -> 2 j + 1
    return F8Dst{L.f_gu, L.s_gu, pack_for(e, 2 * e->il, e->H, EPI_SWIGLU), up, 2};
}
F8Dst dst_down(const q3_engine* e, const LayerW& L) {
    return F8Dst{L.f_down, L.s_down, pack_for(e, e->H, e->il, e->world > 1 ? EPI_PARTIAL : EPI_RESID), 0, 1};
}
F8Dst dst_lm(const q3_engine* e) {
    return F8Dst{e->f_lm, e->s_lm, pack_for(e, e->vl, e->H, EPI_ARGMAX), 0, 1};
}

// FP8 engines: each GEMV matrix generated at full row width in BF16 (so a
// row-parallel shard is scaled by its full row's maximum), then quantized.
int init_synthetic_fp8(q3_engine* e, uint64_t seed) {
    const q3_model_config& c = e->cfg;
    const size_t H = e->H, qd = e->qd, kd = e->kd, il = e->il, vl = e->vl;
    const size_t qfull = static_cast<size_t>(c.q_heads) * 128, inter = c.inter;
    cudaStream_t s = e->stream;
    Staging st;
    size_t need = std::max({qd * H, H * qfull, il * H, H * inter});
    if (!c.tied) need = std::max(need, vl * H);
    Q3_TRY(st.alloc(need));
    Q3_CUDA(launch_fill_normal(e->embed, seed, 1, c.vocab, H, 0, 0, H, H, s));
    if (c.tied) {
        Q3_TRY(quant(e, e->embed + static_cast<size_t>(e->voff) * H, H, vl, H, 0, H, dst_lm(e)));
    } else {
        Q3_CUDA(launch_fill_normal(st.p, seed, 2, vl, H, e->voff, 0, H, H, s));
        Q3_TRY(quant(e, st.p, H, vl, H, 0, H, dst_lm(e)));
    }
    Q3_CUDA(launch_fill_const(e->final_norm, H, 1.0f, s));
    for (size_t l = 0; l < e->layers.size(); ++l) {
        const LayerW& L = e->layers[l];
        const uint64_t b = 16 + 16 * l;
        const size_t qr0 = static_cast<size_t>(e->rank) * qd, kr0 = static_cast<size_t>(e->rank) * kd;
        const size_t ir0 = static_cast<size_t>(e->rank) * il;
        Q3_CUDA(launch_fill_normal(st.p, seed, b + 0, qd, H, qr0, 0, H, H, s));
        Q3_TRY(quant(e, st.p, H, qd, H, 0, H, dst_qkv(e, L, 0)));
        Q3_CUDA(launch_fill_normal(st.p, seed, b + 1, kd, H, kr0, 0, H, H, s));
        Q3_TRY(quant(e, st.p, H, kd, H, 0, H, dst_qkv(e, L, static_cast<int>(qd))));
        Q3_CUDA(launch_fill_normal(st.p, seed, b + 2, kd, H, kr0, 0, H, H, s));
        Q3_TRY(quant(e, st.p, H, kd, H, 0, H, dst_qkv(e, L, static_cast<int>(qd + kd))));
        Q3_CUDA(launch_fill_normal(st.p, seed, b + 3, H, qfull, 0, 0, qfull, qfull, s));
        Q3_TRY(quant(e, st.p, qfull, H, qfull, qr0, qd, dst_o(e, L)));
        Q3_CUDA(launch_fill_normal(st.p, seed, b + 4, il, H, ir0, 0, H, H, s));
        Q3_TRY(quant(e, st.p, H, il, H, 0, H, dst_gu(e, L, 0)));
        Q3_CUDA(launch_fill_normal(st.p, seed, b + 5, il, H, ir0, 0, H, H, s));
        Q3_TRY(quant(e, st.p, H, il, H, 0, H, dst_gu(e, L, 1)));
        Q3_CUDA(launch_fill_normal(st.p, seed, b + 6, H, inter, 0, 0, inter, inter, s));
        Q3_TRY(quant(e, st.p, inter, H, inter, ir0, il, dst_down(e, L)));
        Q3_CUDA(launch_fill_const(L.in_norm, H, 1.0f, s));
        Q3_CUDA(launch_fill_const(L.post_norm, H, 1.0f, s));
        Q3_CUDA(launch_fill_const(L.q_norm, 128, 1.0f, s));
        Q3_CUDA(launch_fill_const(L.k_norm, 128, 1.0f, s));
    }
    Q3_CUDA(cudaStreamSynchronize(s));
    return Q3_OK;
}

// FP8 engines: `rows` full host rows (full_cols wide) to the device, then
// columns [c0, c0 + cols) of each quantized into dst.
int set_matrix_fp8(q3_engine* e, const uint16_t* host, size_t rows, size_t full_cols, size_t c0, size_t cols,
                   const F8Dst& d) {
    Staging st;
    Q3_TRY(st.alloc(rows * full_cols));
    // stream-ordered before the quantize kernel (a pageable cudaMemcpy may return before its DMA lands)
    Q3_CUDA(cudaMemcpyAsync(st.p, host, rows * full_cols * 2, cudaMemcpyHostToDevice, e->stream));
    Q3_TRY(quant(e, st.p, full_cols, rows, full_cols, c0, cols, d));
    Q3_TRY(stream_wait(e));
    return Q3_OK;
}

}  // namespace

int q3_engine_init_synthetic(q3_engine* e, uint64_t seed) {
    Q3_CHECK(e, "null engine");
    Q3_CUDA(cudaSetDevice(e->device));
    if (e->fp8) return init_synthetic_fp8(e, seed);
    const q3_model_config& c = e->cfg;
    const size_t H = e->H;
    cudaStream_t s = e->stream;
    const size_t qfull = static_cast<size_t>(c.q_heads) * 128;
    const size_t kfull = static_cast<size_t>(c.kv_heads) * 128;
    // tensor ids: embed 1, lm_head 2, layer l: 16 + 16 l + {q,k,v,o,gate,up,down}
    Q3_CUDA(launch_fill_normal(e->embed, seed, 1, c.vocab, H, 0, 0, H, H, s));
    if (!c.tied) Q3_CUDA(launch_fill_normal(e->lm_head, seed, 2, e->vl, H, e->voff, 0, H, H, s));
    Q3_CUDA(launch_fill_const(e->final_norm, H, 1.0f, s));
    for (size_t l = 0; l < e->layers.size(); ++l) {
        const LayerW& L = e->layers[l];
        const uint64_t b = 16 + 16 * l;
        const size_t qr0 = static_cast<size_t>(e->rank) * e->qd, kr0 = static_cast<size_t>(e->rank) * e->kd;
        Q3_CUDA(launch_fill_normal(L.w_qkv, seed, b + 0, e->qd, H, qr0, 0, H, H, s));
        Q3_CUDA(launch_fill_normal(L.w_qkv + e->qd * H, seed, b + 1, e->kd, H, kr0, 0, H, H, s));
        Q3_CUDA(launch_fill_normal(L.w_qkv + (e->qd + e->kd) * H, seed, b + 2, e->kd, H, kr0, 0, H, H, s));
        Q3_CUDA(launch_fill_normal(L.w_o, seed, b + 3, H, e->qd, 0, qr0, qfull, e->qd, s));
        const size_t ir0 = static_cast<size_t>(e->rank) * e->il;
        Q3_CUDA(launch_fill_normal(L.w_gu, seed, b + 4, e->il, H, ir0, 0, H, 2 * H, s));
        Q3_CUDA(launch_fill_normal(L.w_gu + H, seed, b + 5, e->il, H, ir0, 0, H, 2 * H, s));
        Q3_CUDA(launch_fill_normal(L.w_down, seed, b + 6, H, e->il, 0, ir0, c.inter, e->il, s));
        Q3_CUDA(launch_fill_const(L.in_norm, H, 1.0f, s));
        Q3_CUDA(launch_fill_const(L.post_norm, H, 1.0f, s));
        Q3_CUDA(launch_fill_const(L.q_norm, 128, 1.0f, s));
        Q3_CUDA(launch_fill_const(L.k_norm, 128, 1.0f, s));
        (void)kfull;
    }
    Q3_CUDA(cudaStreamSynchronize(s));
    return Q3_OK;
}

int q3_engine_set_weight(q3_engine* e, const char* name, const uint16_t* host, size_t rows, size_t cols) {
    Q3_CHECK(e && name && host, "q3_engine_set_weight: null argument");
    Q3_CUDA(cudaSetDevice(e->device));
    const q3_model_config& c = e->cfg;
    const std::string n(name);
    const size_t H = e->H;
    auto expect = [&](size_t r, size_t cc) { return rows == r && cols == cc; };
    auto copy2d = [&](void* dst, size_t dpitch_elems, const uint16_t* src, size_t spitch_elems, size_t width_elems,
                      size_t height) -> int {
        // on the engine's stream and complete before returning: a host-to-device copy from
        // pageable memory may still be in flight when a plain cudaMemcpy2D returns
        Q3_CUDA(cudaMemcpy2DAsync(dst, dpitch_elems * 2, src, spitch_elems * 2, width_elems * 2, height,
                                  cudaMemcpyHostToDevice, e->stream));
        Q3_TRY(stream_wait(e));
        return Q3_OK;
    };
    if (n == "model.embed_tokens.weight") {
        Q3_CHECK(expect(c.vocab, H), "embed_tokens shape");
        Q3_TRY(copy2d(e->embed, H, host, H, H, c.vocab));
        if (e->fp8 && c.tied) {
            Q3_TRY(quant(e, e->embed + static_cast<size_t>(e->voff) * H, H, e->vl, H, 0, H, dst_lm(e)));
            Q3_TRY(stream_wait(e));
        }
        return Q3_OK;
    }
    if (n == "lm_head.weight") {
        Q3_CHECK(expect(c.vocab, H), "lm_head shape");
        if (c.tied) return fail(Q3_ERR_INVALID, "lm_head.weight given for a tied-embedding model");
        if (e->fp8)
            return set_matrix_fp8(e, host + static_cast<size_t>(e->voff) * H, e->vl, H, 0, H, dst_lm(e));
        return copy2d(e->lm_head, H, host + static_cast<size_t>(e->voff) * H, H, H, e->vl);
    }
    if (n == "model.norm.weight") {
        Q3_CHECK(expect(1, H) || expect(H, 1), "norm shape");
        return copy2d(e->final_norm, H, host, H, H, 1);
    }
    const std::string pre = "model.layers.";
    Q3_CHECK(n.rfind(pre, 0) == 0, "unknown weight name: " + n);
    size_t dot = n.find('.', pre.size());
    Q3_CHECK(dot != std::string::npos, "bad weight name: " + n);
    const size_t l = std::stoul(n.substr(pre.size(), dot - pre.size()));
    Q3_CHECK(l < e->layers.size(), "layer index out of range: " + n);
    const std::string leaf = n.substr(dot + 1);
    const LayerW& L = e->layers[l];
    const size_t qfull = static_cast<size_t>(c.q_heads) * 128, kfull = static_cast<size_t>(c.kv_heads) * 128;
    const size_t qr0 = static_cast<size_t>(e->rank) * e->qd, kr0 = static_cast<size_t>(e->rank) * e->kd;
    const size_t ir0 = static_cast<size_t>(e->rank) * e->il;
    const size_t qd = e->qd, kd = e->kd, il = e->il;
    if (leaf == "self_attn.q_proj.weight") {
        Q3_CHECK(expect(qfull, H), "q_proj shape");
        if (e->fp8) return set_matrix_fp8(e, host + qr0 * H, qd, H, 0, H, dst_qkv(e, L, 0));
        return copy2d(L.w_qkv, H, host + qr0 * H, H, H, qd);
    }
    if (leaf == "self_attn.k_proj.weight") {
        Q3_CHECK(expect(kfull, H), "k_proj shape");
        if (e->fp8) return set_matrix_fp8(e, host + kr0 * H, kd, H, 0, H, dst_qkv(e, L, static_cast<int>(qd)));
        return copy2d(L.w_qkv + qd * H, H, host + kr0 * H, H, H, kd);
    }
    if (leaf == "self_attn.v_proj.weight") {
        Q3_CHECK(expect(kfull, H), "v_proj shape");
        if (e->fp8) return set_matrix_fp8(e, host + kr0 * H, kd, H, 0, H, dst_qkv(e, L, static_cast<int>(qd + kd)));
        return copy2d(L.w_qkv + (qd + kd) * H, H, host + kr0 * H, H, H, kd);
    }
    if (leaf == "self_attn.o_proj.weight") {
        Q3_CHECK(expect(H, qfull), "o_proj shape");
        if (e->fp8) return set_matrix_fp8(e, host, H, qfull, qr0, qd, dst_o(e, L));
        return copy2d(L.w_o, qd, host + qr0, qfull, qd, H);
    }
    if (leaf == "mlp.gate_proj.weight" || leaf == "mlp.up_proj.weight") {
        Q3_CHECK(expect(c.inter, H), "gate/up shape");
        const size_t up = leaf == "mlp.up_proj.weight" ? 1 : 0;
        if (e->fp8) return set_matrix_fp8(e, host + ir0 * H, il, H, 0, H, dst_gu(e, L, static_cast<int>(up)));
        return copy2d(L.w_gu + up * H, 2 * H, host + ir0 * H, H, H, il);
    }
    if (leaf == "mlp.down_proj.weight") {
        Q3_CHECK(expect(H, c.inter), "down_proj shape");
        if (e->fp8) return set_matrix_fp8(e, host, H, c.inter, ir0, il, dst_down(e, L));
        return copy2d(L.w_down, il, host + ir0, c.inter, il, H);
    }
    auto vec = [&](bf16* dst, size_t len) -> int {
        Q3_CHECK(rows * cols == len, "norm weight shape: " + n);
        Q3_CUDA(cudaMemcpyAsync(dst, host, len * 2, cudaMemcpyHostToDevice, e->stream));
        Q3_TRY(stream_wait(e));
        return Q3_OK;
    };
    if (leaf == "input_layernorm.weight") return vec(L.in_norm, H);
    if (leaf == "post_attention_layernorm.weight") return vec(L.post_norm, H);
    if (leaf == "self_attn.q_norm.weight") return vec(L.q_norm, 128);
    if (leaf == "self_attn.k_norm.weight") return vec(L.k_norm, 128);
    return fail(Q3_ERR_INVALID, "unknown weight name: " + n);
}

int q3_engine_reset(q3_engine* e) {
    Q3_CHECK(e, "null engine");
    Q3_CUDA(cudaSetDevice(e->device));
    Q3_CUDA(cudaMemsetAsync(e->pos, 0, 4, e->stream));
    Q3_CUDA(cudaMemsetAsync(e->n_forced, 0, 4, e->stream));
    Q3_CUDA(cudaMemsetAsync(e->argmax_hist, 0xFF, (e->cfg.capacity + 1) * 4, e->stream));
    e->host_pos = 0;
    e->host_forced = 0;
    e->host_max_pos = 0;
    return Q3_OK;
}

int q3_engine_set_tokens(q3_engine* e, const uint32_t* ids, size_t n) {
    Q3_CHECK(e && (ids || n == 0), "q3_engine_set_tokens: null argument");
    Q3_CHECK(n <= e->cfg.capacity, "q3_engine_set_tokens: more tokens than KV capacity");
    for (size_t i = 0; i < n; ++i) Q3_CHECK(ids[i] < e->cfg.vocab, "q3_engine_set_tokens: token id >= vocab");
    Q3_CUDA(cudaSetDevice(e->device));
    if (n) Q3_CUDA(cudaMemcpyAsync(e->tokens, ids, n * 4, cudaMemcpyHostToDevice, e->stream));
    const int32_t nf = static_cast<int32_t>(n);
    Q3_CUDA(cudaMemcpyAsync(e->n_forced, &nf, 4, cudaMemcpyHostToDevice, e->stream));
    Q3_TRY(stream_wait(e));
    e->host_forced = n;
    return Q3_OK;
}

int q3_engine_step(q3_engine* e, size_t n) {
    Q3_CHECK(e, "null engine");
    if (n == 0) return Q3_OK;
    Q3_CHECK(e->host_forced >= 1 || e->host_pos >= 1, "q3_engine_step: no input token (set_tokens first)");
    if (e->host_pos + n > e->cfg.capacity)
        return fail(Q3_ERR_INVALID, "q3_engine_step: KV cache capacity exceeded");
    Q3_CUDA(cudaSetDevice(e->device));
    Q3_TRY(build_graph(e));
    for (size_t i = 0; i < n; ++i) Q3_CUDA(cudaGraphLaunch(e->graph, e->stream));
    e->queued_steps += n;
    e->host_pos += n;
    if (e->host_pos > e->host_max_pos) e->host_max_pos = e->host_pos;
    return Q3_OK;
}

namespace {

int ensure_rows_impl(q3_engine* e) {
    if (e->prefill_rows) return Q3_OK;
    const int H = e->H, qd = e->qd, kd = e->kd, il = e->il;
    const int ldqkv = qd + 2 * kd;
    const int rows = kPrefillRows;
    int rc;
    if ((rc = dalloc_t(e, &e->px, static_cast<size_t>(rows) * H)) != Q3_OK) return rc;
    if ((rc = dalloc_t(e, &e->pxn, static_cast<size_t>(rows) * H)) != Q3_OK) return rc;
    if ((rc = dalloc_t(e, &e->pqkv, static_cast<size_t>(rows) * ldqkv)) != Q3_OK) return rc;
    if ((rc = dalloc_t(e, &e->pattn, static_cast<size_t>(rows) * qd)) != Q3_OK) return rc;
    if ((rc = dalloc_t(e, &e->pg, static_cast<size_t>(rows) * il)) != Q3_OK) return rc;
    if ((rc = dalloc_t(e, &e->pvsum, static_cast<size_t>(rows) * H)) != Q3_OK) return rc;
    // splits x output tiles <= SMs, output tiles >= N / 256: at most 128 x sms x 256 partials
    e->split_ws_floats = static_cast<size_t>(128) * e->sms * 256;
    if ((rc = dalloc_t(e, &e->split_ws, e->split_ws_floats)) != Q3_OK) return rc;
    e->prefill_rows = rows;
    return Q3_OK;
}

// Per layer: row RMSNorm, QKV GEMM (tcgen05), q/k norm + RoPE with the cache
// writes, attention over each row's prefix, then O (+ residual), RMSNorm of the
// fp32 sums, gate/up (SwiGLU epilogue) and down (+ residual).  Without logits
// the last layer stops after its attention (its output only feeds logits that
// the prefill discards); with them the last layer completes and the final
// RMSNorm and the lm_head GEMM follow.
int forward_rows_impl(q3_engine* e, const RowsSpec& R) {
    const bool tp = e->world > 1;
    const int H = e->H, qd = e->qd, kd = e->kd, il = e->il;
    const int ldqkv = qd + 2 * kd;
    const int t = R.n;
    Q3_CHECK(t > 0 && t <= kPrefillRows, "forward_rows: row count");
    if (R.logits && (tp || e->fp8 || e->vl % 128 != 0))
        return fail(Q3_ERR_UNSUPPORTED, "batched logits need a single-GPU BF16 engine with vocab % 128 == 0");
    Q3_TRY(ensure_rows_impl(e));
    if (e->fp8 && !e->pw) {
        const size_t most = std::max({static_cast<size_t>(ldqkv) * H, static_cast<size_t>(H) * qd,
                                      static_cast<size_t>(2 * il) * H, static_cast<size_t>(H) * il});
        int rc;
        if ((rc = dalloc_t(e, &e->pw, most)) != Q3_OK) return rc;
    }
    const float eps = e->cfg.eps;
    cudaStream_t s = e->stream;
    const int L = static_cast<int>(e->layers.size());
    // The BF16 matrix a prefill GEMM reads: the engine's own, or (FP8 engines) the
    // packed E4M3 matrix expanded into pw -- exactly the FP8 model's weights.  One
    // buffer serves every GEMM: stream order keeps an expansion after the GEMM
    // that read the previous one.
    auto weight = [&](const bf16* w, const F8Dst& d, const bf16** out) -> int {
        *out = w;
        if (!e->fp8) return Q3_OK;
        if (d.pack.fmt == 1)
            Q3_CUDA(launch_dequant_nvfp4(d.base, d.scale, d.pack, e->pw, s));
        else
            Q3_CUDA(launch_dequant_e4m3(d.base, d.scale, d.pack, e->pw, s));
        *out = e->pw;
        return Q3_OK;
    };
    auto gemm = [&](const bf16* x, const bf16* w, bf16* y, float* vs, int m, int nn, int k, int ldy, int epi) {
        GemmArgs g{};
        g.x = x;
        g.w = w;
        g.y = y;
        g.vsum = vs;
        g.M = m;
        g.N = nn;
        g.K = k;
        g.ldy = ldy;
        g.epi = epi;
        g.bn = gemm_tile_n(m, nn, e->sms);
        g.err = e->err;
        g.ws = e->split_ws;
        g.ws_floats = e->split_ws_floats;
        g.sms = e->sms;
        return launch_gemm(g, s);
    };
    // Tensor parallel: the row-parallel GEMMs (o_proj, down_proj) write fp32 partial
    // rows (GEMM_F32) into this rank's slot, and every rank adds the sum over all
    // ranks' slots, in rank order, to its replicated residual rows (peer memory:
    // flags + reads over NVLink; NCCL: an allreduce of the slot, then the same add).
    float* pf_mine = nullptr;
    TpExchange xnccl{};
    if (tp) {
        const XbufLayout xl = xbuf_layout(static_cast<size_t>(e->world), static_cast<size_t>(H),
                                          e->tpx.slot_floats / static_cast<size_t>(H));
        pf_mine = reinterpret_cast<float*>(static_cast<uint8_t*>(e->xbuf) + xl.pf_part_off);
        xnccl.part[0] = pf_mine;
        xnccl.slot_floats = e->tpx.slot_floats;
        xnccl.rank = 0;
        xnccl.world = 1;
    }
    auto tp_partial = [&](const bf16* x, const bf16* w, int m, int k, float* vs) -> int {
        const uint32_t seq = ++e->tp_seq;
        float* slot = pf_mine + (seq & 1u) * e->tpx.slot_floats;
        GemmArgs g{};
        g.x = x;
        g.w = w;
        g.yf = slot;
        g.M = m;
        g.N = H;
        g.K = k;
        g.ldy = H;
        g.epi = GEMM_F32;
        g.bn = gemm_tile_n(m, H, e->sms);
        g.err = e->err;
        Q3_CUDA(launch_gemm(g, s));
        if (e->peer_mode) {
            Q3_CUDA(launch_tp_signal(e->tpx, seq, s));
            Q3_CUDA(launch_tp_resid_rows(e->tpx, seq, m, H, e->px, vs, e->err, e->sms, s));
        } else {
            if (!e->comm) return fail(Q3_ERR_NCCL, "NCCL communicator aborted");
            Q3_TRY(nccl_check(e, nccl().AllReduce(slot, slot, static_cast<size_t>(m) * H, ncclFloat32, ncclSum,
                                                  e->comm, s), "ncclAllReduce"));
            Q3_CUDA(launch_tp_resid_rows(xnccl, seq, m, H, e->px, vs, e->err, e->sms, s));
        }
        return Q3_OK;
    };
    Q3_CUDA(launch_embed_rows(e->embed, R.tokens, R.p0, t, static_cast<int>(e->cfg.vocab), H, e->px, e->err, s,
                              R.row_tokens));
    const int pool = R.k_pools ? R.pool_pages : e->n_pages;
    for (int l = 0; l < L; ++l) {
        const LayerW& W = e->layers[l];
        bf16* kp = R.k_pools ? R.k_pools[l] : W.k_pages;
        bf16* vp = R.v_pools ? R.v_pools[l] : W.v_pages;
        Q3_CUDA(launch_rmsnorm_rows(e->px, nullptr, W.in_norm, e->pxn, t, H, eps, s));
        const bf16* wm = nullptr;
        Q3_TRY(weight(W.w_qkv, dst_qkv(e, W, 0), &wm));
        Q3_CUDA(gemm(e->pxn, wm, e->pqkv, nullptr, t, ldqkv, H, ldqkv, GEMM_STORE));
        PrefillQkvArgs qa{};
        qa.qkv = e->pqkv;
        qa.ld = ldqkv;
        qa.q_heads = e->qh;
        qa.kv_heads = e->kvh;
        qa.p0 = R.p0;
        qa.q_norm = W.q_norm;
        qa.k_norm = W.k_norm;
        qa.rope_cos = e->rope_cos;
        qa.rope_sin = e->rope_sin;
        qa.k_pages = kp;
        qa.v_pages = vp;
        qa.page_table = R.page_table;
        qa.row_pos = R.row_pos;
        qa.pt_stride = R.pt_stride;
        qa.eps = eps;
        Q3_CUDA(launch_qkv_rows(qa, t, s));
        AttnArgs aa{};
        aa.q = e->pqkv;
        aa.k = kp;
        aa.v = vp;
        aa.page_table = R.page_table;
        aa.row_pos = R.row_pos;
        aa.pt_stride = R.pt_stride;
        aa.out = e->pattn;
        aa.q_heads = e->qh;
        aa.kv_heads = e->kvh;
        aa.page_size = kPageSize;
        aa.paged = 1;
        aa.pool = pool;
        aa.pos_host = R.p0;
        // many queries already fill the GPU: a split gets at least 8 pages
        const int pages = R.max_pos / kPageSize + 1;
        aa.splits = R.attn_splits ? R.attn_splits
                                  : attn_splits(e->kvh, ((pages + 7) / 8) * kPageSize - 1, kPageSize, e->sms);
        aa.err = e->err;
        aa.n_queries = t;
        aa.q_stride = ldqkv;
        aa.out_stride = qd;
        Q3_CUDA(launch_attention(aa, s, false));
        if (l == L - 1 && !R.logits) break;
        Q3_TRY(weight(W.w_o, dst_o(e, W), &wm));
        if (tp)
            Q3_TRY(tp_partial(e->pattn, wm, t, qd, e->pvsum));
        else
            Q3_CUDA(gemm(e->pattn, wm, e->px, e->pvsum, t, H, qd, H, GEMM_RESID));
        Q3_CUDA(launch_rmsnorm_rows(e->px, e->pvsum, W.post_norm, e->pxn, t, H, eps, s));
        Q3_TRY(weight(W.w_gu, dst_gu(e, W, 0), &wm));
        Q3_CUDA(gemm(e->pxn, wm, e->pg, nullptr, t, 2 * il, H, il, GEMM_SWIGLU));
        Q3_TRY(weight(W.w_down, dst_down(e, W), &wm));
        if (tp)
            Q3_TRY(tp_partial(e->pg, wm, t, il, nullptr));
        else
            Q3_CUDA(gemm(e->pg, wm, e->px, nullptr, t, H, il, H, GEMM_RESID));
    }
    if (R.logits) {
        // qwen3.hpp:161-163: final RMSNorm, lm_head
        Q3_CUDA(launch_rmsnorm_rows(e->px, nullptr, e->final_norm, e->pxn, t, H, eps, s));
        Q3_CUDA(gemm(e->pxn, e->lm_head, R.logits, nullptr, t, e->vl, H, e->vl, GEMM_STORE));
    }
    return Q3_OK;
}

}  // namespace

// Batched prefill (qwen3.hpp:168-173 runs one decode forward per prompt token,
// logits discarded): the K/V of the set tokens at positions [pos, pos + n), up
// to kPrefillRows tokens per forward_rows chunk.
int q3_engine_prefill(q3_engine* e, size_t n) {
    Q3_CHECK(e, "null engine");
    if (n == 0) return Q3_OK;
    const size_t p0 = e->host_pos;
    Q3_CHECK(p0 + n <= e->host_forced, "q3_engine_prefill: tokens not set (set_tokens first)");
    if (p0 + n >= e->cfg.capacity) return fail(Q3_ERR_INVALID, "q3_engine_prefill: KV cache capacity exceeded");
    Q3_CUDA(cudaSetDevice(e->device));
    const bool tp = e->world > 1;
    if ((e->fp8 && !(e->tune & Q3_TUNE_FP8_PREFILL)) ||
        (tp && !((e->tune & Q3_TUNE_TP_PREFILL) && (e->peer_mode || e->comm)))) {
        // FP8-weight engines unless Q3_TUNE_FP8_PREFILL is set, and tensor-parallel ones
        // unless Q3_TUNE_TP_PREFILL is, prefill through the per-token decode step
        return q3_engine_step(e, n);
    }
    for (size_t done = 0; done < n;) {
        RowsSpec R;
        R.n = static_cast<int>(std::min<size_t>(n - done, static_cast<size_t>(kPrefillRows)));
        R.tokens = e->tokens;
        R.p0 = static_cast<int>(p0 + done);
        R.page_table = e->page_table;
        R.max_pos = R.p0 + R.n - 1;
        Q3_TRY(forward_rows_impl(e, R));
        done += static_cast<size_t>(R.n);
    }
    const int32_t np = static_cast<int32_t>(p0 + n);
    Q3_CUDA(cudaMemcpyAsync(e->pos, &np, 4, cudaMemcpyHostToDevice, e->stream));
    e->host_pos = p0 + n;
    if (e->host_pos > e->host_max_pos) e->host_max_pos = e->host_pos;
    return Q3_OK;
}

int q3_engine_sync(q3_engine* e) {
    Q3_CHECK(e, "null engine");
    Q3_CUDA(cudaSetDevice(e->device));
    Q3_TRY(stream_wait(e));
    return check_device_error(e);
}

static int finish_last(q3_engine* e) {
    if (e->peer_mode)
        Q3_CUDA(launch_peer_keys(e->links, reinterpret_cast<unsigned long long*>(e->keys), e->err, e->stream));
    Q3_CUDA(launch_resolve_tokens(e->keys, e->world, e->tokens, e->argmax_hist, e->pos, e->n_forced,
                                  static_cast<int>(e->cfg.vocab), e->err, e->stream));
    return Q3_OK;
}

int q3_engine_forward(q3_engine* e, uint32_t token, uint32_t* next_token) {
    Q3_CHECK(e && next_token, "q3_engine_forward: null argument");
    Q3_CHECK(token < e->cfg.vocab, "q3_engine_forward: token id >= vocab");
    Q3_CUDA(cudaSetDevice(e->device));
    const size_t p = e->host_pos;
    Q3_CHECK(p < e->cfg.capacity, "q3_engine_forward: KV cache full");
    const int32_t t = static_cast<int32_t>(token), nf = static_cast<int32_t>(p + 1);
    Q3_CUDA(cudaMemcpyAsync(e->tokens + p, &t, 4, cudaMemcpyHostToDevice, e->stream));
    Q3_CUDA(cudaMemcpyAsync(e->n_forced, &nf, 4, cudaMemcpyHostToDevice, e->stream));
    e->host_forced = p + 1;
    Q3_TRY(q3_engine_step(e, 1));
    Q3_TRY(finish_last(e));
    std::vector<uint64_t> k(e->world);
    Q3_CUDA(cudaMemcpyAsync(k.data(), e->keys, 8 * e->world, cudaMemcpyDeviceToHost, e->stream));
    Q3_TRY(q3_engine_sync(e));
    uint64_t best = 0;
    for (uint64_t v : k) best = v > best ? v : best;
    *next_token = 0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull);
    return Q3_OK;
}

int q3_engine_generate(q3_engine* e, const uint32_t* prompt, size_t n_prompt, size_t max_new, int stop_at_eos,
                       uint32_t* out, size_t* n_out) {
    Q3_CHECK(e && prompt && out && n_out, "q3_engine_generate: null argument");
    Q3_CHECK(n_prompt >= 1, "q3_engine_generate: empty prompt");
    // generator.cpp:42-44
    if (n_prompt >= e->cfg.capacity) return fail(Q3_ERR_INVALID, "prompt does not fit in the model context");
    Q3_TRY(q3_engine_reset(e));
    Q3_TRY(q3_engine_set_tokens(e, prompt, n_prompt));
    // prefill forwards every prompt id but the last (qwen3.hpp:168-173); the
    // loop then runs while token_count + 1 < capacity (generator.cpp:49).
    const size_t room = e->cfg.capacity - n_prompt;
    const size_t n_gen = max_new < room ? max_new : room;
    const size_t steps = n_prompt - 1 + n_gen;
    Q3_TRY(q3_engine_prefill(e, n_prompt - 1));
    if (!stop_at_eos) {
        Q3_TRY(q3_engine_step(e, n_gen));
    } else {
        // EOS needs the host to look at tokens: run in chunks.
        size_t done = n_prompt - 1;
        const size_t chunk = 32;
        while (done < steps) {
            const size_t k = (steps - done) < chunk ? (steps - done) : chunk;
            Q3_TRY(q3_engine_step(e, k));
            done += k;
            if (done >= n_prompt) {
                Q3_TRY(finish_last(e));
                std::vector<int32_t> t(done + 1);
                Q3_CUDA(cudaMemcpyAsync(t.data(), e->tokens, (done + 1) * 4, cudaMemcpyDeviceToHost, e->stream));
                Q3_TRY(q3_engine_sync(e));
                bool eos = false;
                for (size_t i = n_prompt; i <= done; ++i)
                    if (static_cast<uint32_t>(t[i]) == e->cfg.eos) eos = true;
                if (eos) break;
            }
        }
        const size_t produced = done + 1 - n_prompt;
        std::vector<int32_t> t(done + 1);
        Q3_TRY(finish_last(e));
        Q3_CUDA(cudaMemcpyAsync(t.data(), e->tokens, (done + 1) * 4, cudaMemcpyDeviceToHost, e->stream));
        Q3_TRY(q3_engine_sync(e));
        size_t k = 0;
        for (; k < produced && k < n_gen; ++k) {
            const uint32_t v = static_cast<uint32_t>(t[n_prompt + k]);
            if (v == e->cfg.eos) break;  // generator.cpp:52-54: EOS is not emitted
            out[k] = v;
        }
        *n_out = k;
        return Q3_OK;
    }
    Q3_TRY(finish_last(e));
    Q3_CUDA(cudaMemcpyAsync(out, e->tokens + n_prompt, n_gen * 4, cudaMemcpyDeviceToHost, e->stream));
    Q3_TRY(q3_engine_sync(e));
    *n_out = n_gen;
    return Q3_OK;
}

int q3_engine_set_position(q3_engine* e, size_t pos) {
    Q3_CHECK(e, "null engine");
    const size_t reached = e->host_max_pos > e->host_pos ? e->host_max_pos : e->host_pos;
    Q3_CHECK(pos <= reached && pos < e->cfg.capacity, "q3_engine_set_position: position not reached yet");
    Q3_CUDA(cudaSetDevice(e->device));
    const int32_t p = static_cast<int32_t>(pos);
    Q3_CUDA(cudaMemcpyAsync(e->pos, &p, 4, cudaMemcpyHostToDevice, e->stream));
    Q3_TRY(stream_wait(e));
    e->host_max_pos = reached;
    e->host_pos = pos;
    return Q3_OK;
}

int q3_engine_set_tuning(q3_engine* e, uint32_t flags) {
    Q3_CHECK(e, "null engine");
    Q3_CHECK((flags & ~Q3_TUNE_ALL) == 0u, "q3_engine_set_tuning: unknown flag bits");
    if (flags == e->tune) return Q3_OK;
    Q3_CUDA(cudaSetDevice(e->device));
    if (e->graph) {
        // the step graph holds the launch arguments: record it again at the next step
        Q3_TRY(stream_wait(e));
        Q3_CUDA(cudaGraphExecDestroy(e->graph));
        e->graph = nullptr;
    }
    e->tune = flags;
    return Q3_OK;
}

int q3_engine_tuning(q3_engine* e, uint32_t* flags) {
    Q3_CHECK(e && flags, "q3_engine_tuning: null argument");
    *flags = e->tune;
    return Q3_OK;
}

namespace {

// The CUDA-graph path's timeline: every launch of the step records per CTA;
// toggling it re-records the graph with or without the trace buffer.
int graph_trace(q3_engine* e, int enable, uint64_t* out_host, size_t capacity, size_t* n_phases, size_t* n_ctas) {
    const size_t phases = e->layers.size() * 5 + 1;
    // attention launches splits x kv heads x query-head blocks CTAs (at most one per q head)
    const int ctas = std::max(e->sms, e->attn_splits * e->qh);
    const size_t n = static_cast<size_t>(ctas) * phases * kTraceWords;
    *n_phases = phases;
    *n_ctas = static_cast<size_t>(ctas);
    if (enable && !e->d_gtrace) {
        int rc = dalloc_t(e, &e->d_gtrace, n);
        if (rc != Q3_OK) return rc;
        Q3_CUDA(cudaMemset(e->d_gtrace, 0, n * 8));
    }
    e->gtrace_ctas = ctas;
    if (static_cast<bool>(enable) != e->gtrace) {
        Q3_TRY(stream_wait(e));
        if (e->graph) {
            cudaGraphExecDestroy(e->graph);
            e->graph = nullptr;
        }
        e->gtrace = enable != 0;
    }
    if (out_host && e->d_gtrace) {
        Q3_CHECK(capacity >= n, "q3_engine_trace: output buffer too small");
        Q3_TRY(stream_wait(e));
        Q3_CUDA(cudaMemcpy(out_host, e->d_gtrace, n * 8, cudaMemcpyDeviceToHost));
    }
    return Q3_OK;
}

}  // namespace

int q3_engine_trace(q3_engine* e, int enable, uint64_t* out_host, size_t capacity, size_t* n_phases, size_t* n_ctas) {
    Q3_CHECK(e && n_phases && n_ctas, "null argument");
    Q3_CUDA(cudaSetDevice(e->device));
    return graph_trace(e, enable, out_host, capacity, n_phases, n_ctas);
}

int q3_engine_position(q3_engine* e, size_t* pos) {
    Q3_CHECK(e && pos, "null argument");
    *pos = e->host_pos;
    return Q3_OK;
}

int q3_engine_logits(q3_engine* e, uint16_t* out) {
    Q3_CHECK(e && out, "null argument");
    Q3_CUDA(cudaSetDevice(e->device));
    Q3_CUDA(cudaMemcpyAsync(out, e->logits, static_cast<size_t>(e->vl) * 2, cudaMemcpyDeviceToHost, e->stream));
    return q3_engine_sync(e);
}

int q3_engine_argmax_history(q3_engine* e, uint32_t* out, size_t n) {
    Q3_CHECK(e && out, "null argument");
    Q3_CHECK(n <= e->cfg.capacity, "argmax history longer than capacity");
    Q3_CUDA(cudaSetDevice(e->device));
    Q3_TRY(finish_last(e));
    Q3_CUDA(cudaMemcpyAsync(out, e->argmax_hist, n * 4, cudaMemcpyDeviceToHost, e->stream));
    return q3_engine_sync(e);
}

int q3_engine_kv_slot(q3_engine* e, size_t layer, size_t pos, uint16_t* k_out, uint16_t* v_out) {
    Q3_CHECK(e && k_out && v_out, "null argument");
    Q3_CHECK(layer < e->layers.size() && pos < e->cfg.capacity, "kv slot out of range");
    Q3_CUDA(cudaSetDevice(e->device));
    Q3_TRY(stream_wait(e));  // the legacy-stream copies below do not wait for it
    int32_t page = 0;
    Q3_CUDA(cudaMemcpy(&page, e->page_table + pos / kPageSize, 4, cudaMemcpyDeviceToHost));
    const LayerW& L = e->layers[layer];
    for (int h = 0; h < e->kvh; ++h) {
        const size_t off = ((static_cast<size_t>(page) * e->kvh + h) * kPageSize + pos % kPageSize) * 128;
        Q3_CUDA(cudaMemcpy(k_out + h * 128, L.k_pages + off, 256, cudaMemcpyDeviceToHost));
        Q3_CUDA(cudaMemcpy(v_out + h * 128, L.v_pages + off, 256, cudaMemcpyDeviceToHost));
    }
    return Q3_OK;
}

// Slots [pos0, pos0 + n) of one layer between the paged cache and host arrays
// in the reference layout [n][kv_heads][128]: one strided copy per (page, head).
static int kv_range_copy(q3_engine* e, size_t layer, size_t pos0, size_t n, uint16_t* k_host, uint16_t* v_host,
                         bool to_device) {
    Q3_CHECK(e && k_host && v_host, "null argument");
    Q3_CHECK(layer < e->layers.size() && pos0 <= e->cfg.capacity && n <= e->cfg.capacity - pos0,
             "kv range out of range");
    Q3_CUDA(cudaSetDevice(e->device));
    Q3_TRY(stream_wait(e));
    std::vector<int32_t> table((e->cfg.capacity + kPageSize - 1) / kPageSize);
    Q3_CUDA(cudaMemcpy(table.data(), e->page_table, table.size() * 4, cudaMemcpyDeviceToHost));
    const q3::LayerW& L = e->layers[layer];
    const size_t row = 128 * sizeof(uint16_t), host_pitch = static_cast<size_t>(e->kvh) * row;
    for (size_t p = pos0; p < pos0 + n;) {
        const size_t in_page = std::min<size_t>(kPageSize - p % kPageSize, pos0 + n - p);
        const int32_t page = table[p / kPageSize];
        for (int h = 0; h < e->kvh; ++h) {
            const size_t off = ((static_cast<size_t>(page) * e->kvh + h) * kPageSize + p % kPageSize) * 128;
            const size_t hoff = ((p - pos0) * e->kvh + h) * 128;
            for (int which = 0; which < 2; ++which) {
                q3::bf16* d = (which ? L.v_pages : L.k_pages) + off;
                uint16_t* hp = (which ? v_host : k_host) + hoff;
                if (to_device)
                    Q3_CUDA(cudaMemcpy2DAsync(d, row, hp, host_pitch, row, in_page, cudaMemcpyHostToDevice, e->stream));
                else
                    Q3_CUDA(cudaMemcpy2DAsync(hp, host_pitch, d, row, row, in_page, cudaMemcpyDeviceToHost, e->stream));
            }
        }
        p += in_page;
    }
    Q3_TRY(stream_wait(e));
    return Q3_OK;
}

int q3_engine_kv_read(q3_engine* e, size_t layer, size_t pos0, size_t n, uint16_t* k_host, uint16_t* v_host) {
    return kv_range_copy(e, layer, pos0, n, k_host, v_host, false);
}

int q3_engine_kv_write(q3_engine* e, size_t layer, size_t pos0, size_t n, const uint16_t* k_host,
                       const uint16_t* v_host) {
    Q3_TRY(kv_range_copy(e, layer, pos0, n, const_cast<uint16_t*>(k_host), const_cast<uint16_t*>(v_host), true));
    // the written slots count as computed: set_position may move the cursor up to them
    if (pos0 + n > e->host_max_pos) e->host_max_pos = pos0 + n;
    return Q3_OK;
}

int q3_engine_fill_kv(q3_engine* e, size_t upto, uint64_t seed) {
    Q3_CHECK(e, "null engine");
    Q3_CHECK(upto < e->cfg.capacity, "q3_engine_fill_kv: upto must be < capacity");
    Q3_CUDA(cudaSetDevice(e->device));
    const size_t pages = (upto + kPageSize - 1) / kPageSize;
    const size_t rows = pages * e->kvh * kPageSize;
    for (size_t l = 0; l < e->layers.size(); ++l) {
        if (rows == 0) break;
        Q3_CUDA(launch_fill_normal(e->layers[l].k_pages, seed, 0x4B00 + 2 * l, rows, 128, 0, 0, 128, 128, e->stream));
        Q3_CUDA(launch_fill_normal(e->layers[l].v_pages, seed, 0x4B01 + 2 * l, rows, 128, 0, 0, 128, 128, e->stream));
    }
    const int32_t p = static_cast<int32_t>(upto);
    Q3_CUDA(cudaMemcpyAsync(e->pos, &p, 4, cudaMemcpyHostToDevice, e->stream));
    Q3_TRY(stream_wait(e));
    e->host_pos = upto;
    if (upto > e->host_max_pos) e->host_max_pos = upto;
    return Q3_OK;
}

int q3_engine_stream(q3_engine* e, void** stream) {
    Q3_CHECK(e && stream, "null argument");
    *stream = e->stream;
    return Q3_OK;
}

size_t q3_engine_weight_bytes(q3_engine* e) { return e ? e->weight_bytes : 0; }

size_t q3_engine_kv_bytes_per_position(q3_engine* e) {
    return e ? e->layers.size() * 2 * static_cast<size_t>(e->kvh) * 128 * 2 : 0;
}

int q3_engine_profile_step(q3_engine* e, int klass, double* ms, size_t* launches, double* bytes) {
    Q3_CHECK(e && ms && launches && bytes, "null argument");
    Q3_CHECK(e->host_pos < e->cfg.capacity, "q3_engine_profile_step: KV cache full");
    Q3_CHECK(e->host_forced >= 1 || e->host_pos >= 1, "q3_engine_profile_step: no input token");
    if (e->comm_dead) return fail(Q3_ERR_NCCL, "NCCL communicator aborted after a failed exchange");
    if (e->world > 1 && !e->comm && !e->peer_mode)
        return fail(Q3_ERR_INVALID, "tensor-parallel engine needs q3_engine_attach_peers or q3_engine_attach_nccl");
    Q3_CUDA(cudaSetDevice(e->device));
    std::vector<cudaEvent_t> ev;
    double b = 0;
    Recorder r{e, false, klass, &ev, &b};
    Q3_TRY(record_step(r, e->host_pos));
    e->host_pos += 1;
    if (e->host_pos > e->host_max_pos) e->host_max_pos = e->host_pos;
    Q3_TRY(stream_wait(e));
    double total = 0;
    for (size_t i = 0; i + 1 < ev.size(); i += 2) {
        float t = 0;
        cudaEventElapsedTime(&t, ev[i], ev[i + 1]);
        total += t;
    }
    for (auto x : ev) cudaEventDestroy(x);
    *ms = total;
    *launches = r.launches;
    *bytes = b;
    return check_device_error(e);
}

int q3_rope_tables(size_t max_pos, size_t head_dim, float theta, float* cos_host, float* sin_host) {
    Q3_CHECK(cos_host && sin_host && head_dim % 2 == 0 && head_dim <= 65536, "q3_rope_tables: bad argument");
    rope_tables(max_pos, head_dim, theta, cos_host, sin_host);
    return Q3_OK;
}

int q3_nccl_unique_id(void* id_out) {
    Q3_CHECK(id_out, "null argument");
    if (!nccl().ok) return fail(Q3_ERR_NCCL, nccl().error);
    ncclUniqueId id;
    ncclResult_t nr = nccl().GetUniqueId(&id);
    if (nr != ncclSuccess) return fail(Q3_ERR_NCCL, std::string("ncclGetUniqueId: ") + nccl().GetErrorString(nr));
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
    std::memcpy(id_out, &id, sizeof(id));
    return Q3_OK;
}

int q3_engine_peer_handle(q3_engine* e, void* handle_out) {
    Q3_CHECK(e && handle_out, "null argument");
    Q3_CHECK(e->xbuf, "q3_engine_peer_handle: not a tensor-parallel engine");
    Q3_CUDA(cudaSetDevice(e->device));
    cudaIpcMemHandle_t h;
    Q3_CUDA(cudaIpcGetMemHandle(&h, e->xbuf));
    static_assert(sizeof(h) == Q3_PEER_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle_out, &h, sizeof(h));
    return Q3_OK;
}

int q3_engine_attach_peers(q3_engine* e, const void* handles, size_t n) {
    Q3_CHECK(e && handles, "null argument");
    Q3_CHECK(e->xbuf, "q3_engine_attach_peers: not a tensor-parallel engine");
    Q3_CHECK(n == static_cast<size_t>(e->world), "q3_engine_attach_peers: one handle per rank expected");
    Q3_CHECK(!e->peer_mode, "q3_engine_attach_peers: already attached");
    Q3_CUDA(cudaSetDevice(e->device));
    const size_t H = static_cast<size_t>(e->H), W = static_cast<size_t>(e->world);
    const XbufLayout xl = xbuf_layout(W, H, e->tpx.slot_floats / H);
    const size_t flags_off = xl.flags_off, keys_off = xl.keys_off;
    for (int j = 0; j < e->world; ++j) {
        void* base = nullptr;
        if (j == e->rank) {
            base = e->xbuf;
        } else {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(j) * Q3_PEER_HANDLE_BYTES,
                        sizeof(h));
            Q3_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
            e->xpeer[j] = base;
        }
        e->links.recv[j] = static_cast<unsigned long long*>(base);
        e->links.flags[j] = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(base) + flags_off);
        e->links.keys[j] = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(base) + keys_off);
        e->tpx.part[j] = reinterpret_cast<const float*>(static_cast<uint8_t*>(base) + xl.pf_part_off);
        e->tpx.flags[j] = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(base) + xl.pf_flags_off);
    }
    e->peer_mode = true;
    if (e->graph) {
        cudaGraphExecDestroy(e->graph);
        e->graph = nullptr;
    }
    return Q3_OK;
}

int q3_engine_set_comm_timeout(q3_engine* e, double seconds) {
    Q3_CHECK(e, "null engine");
    Q3_CHECK(seconds > 0.0 && seconds <= 86400.0, "q3_engine_set_comm_timeout: seconds must be in (0, 86400]");
    e->comm_timeout_s = seconds;
    return Q3_OK;
}

int q3_engine_attach_nccl(q3_engine* e, const void* id_in) {
    Q3_CHECK(e && id_in, "null argument");
    if (e->world == 1) return Q3_OK;
    Q3_CUDA(cudaSetDevice(e->device));
    ncclUniqueId id;
    std::memcpy(&id, id_in, sizeof(id));
    if (!nccl().ok) return fail(Q3_ERR_NCCL, nccl().error);
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;  // every wait on peers is bounded by the engine (stream_wait, nccl_settle)
    ncclResult_t nr = nccl().CommInitRankConfig(&e->comm, e->world, id, e->rank, &config);
    if (nr != ncclSuccess && nr != ncclInProgress) {
        e->comm = nullptr;
        return fail(Q3_ERR_NCCL, std::string("ncclCommInitRankConfig: ") + nccl().GetErrorString(nr));
    }
    e->comm_dead = false;
    Q3_TRY(nccl_settle(e, "ncclCommInitRankConfig"));
    if (e->graph) {
        cudaGraphExecDestroy(e->graph);
        e->graph = nullptr;
    }
    return Q3_OK;
}

}  // extern "C"

namespace q3 {
int forward_rows(q3_engine* e, const RowsSpec& r) { return forward_rows_impl(e, r); }
int ensure_rows(q3_engine* e) { return ensure_rows_impl(e); }
}  // namespace q3

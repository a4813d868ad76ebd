// batch.cu -- batched decode: several sequences decoding together on one
// engine's weights, each with its own position and KV pages (batch > 1, which
// the reference does not support: README.md:14).
//
// One step of B live sequences is one forward of B rows through the batched
// kernels (engine.cu forward_rows: tcgen05 GEMMs read every weight matrix once
// for all rows, per-row q/k norm + RoPE + cache writes, split-KV attention with
// each row's own position and page table), then the final RMSNorm, the lm_head
// GEMM and a per-row greedy argmax.  Token histories, positions and page tables
// live in device memory, so a step of B rows is one CUDA graph (captured once
// per B; the attention split count comes from B and the capacity, not from the
// positions) and steps run back to back with no host round trip.
//
// KV memory is a pool of 64-position pages per layer shared by all sequences.
// A sequence owns ceil(max_len / 64) page-table entries; q3_batch_fork starts a
// sequence from another's history by referencing its full pages (they are never
// written again: a sequence writes only at its own position, past them) and
// copying the partial page.  Pages carry a reference count and return to the
// pool when their last sequence is released.
#include <algorithm>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "engine_state.hpp"
#include "page_pool.hpp"

namespace q3 {
namespace {

// Row r of the step: its sequence's position, input token and page table.
__global__ void batch_prepare_kernel(const int32_t* __restrict__ row_seq, int rows, const int32_t* __restrict__ kv_len,
                                     const int32_t* __restrict__ tok, int cap, const int32_t* __restrict__ tables,
                                     int max_pages, int32_t* __restrict__ row_pos, int32_t* __restrict__ row_tok,
                                     int32_t* __restrict__ row_pt) {
    const int r = blockIdx.x;
    if (r >= rows) return;
    const int s = row_seq[r];
    const int p = kv_len[s];
    if (threadIdx.x == 0) {
        row_pos[r] = p;
        row_tok[r] = tok[static_cast<size_t>(s) * cap + p];
    }
    for (int i = threadIdx.x; i < max_pages; i += blockDim.x)
        row_pt[static_cast<size_t>(r) * max_pages + i] = tables[static_cast<size_t>(s) * max_pages + i];
}

// After the step: each row's sequence advances one position; the greedy token
// becomes the next input unless a forced token is already there.
__global__ void batch_advance_kernel(const int32_t* __restrict__ row_seq, int rows, int32_t* __restrict__ kv_len,
                                     const int32_t* __restrict__ forced, int32_t* __restrict__ tok, int cap,
                                     const int32_t* __restrict__ arg) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const int s = row_seq[r];
    const int p = kv_len[s] + 1;
    if (p >= forced[s] && p < cap) tok[static_cast<size_t>(s) * cap + p] = arg[r];
    kv_len[s] = p;
}

}  // namespace
}  // namespace q3

struct q3_batch {
    q3_engine* e = nullptr;
    int max_seqs = 0, pool_pages = 0, max_pages = 0, cap = 0;
    std::vector<q3::bf16*> k_pools, v_pools;  // per layer
    size_t page_elems = 0;                    // BF16 elements of one page of one layer (kv_heads x 64 x 128)
    // device state
    int32_t *tables = nullptr, *row_pt = nullptr, *tok = nullptr, *kv_len = nullptr, *forced = nullptr;
    int32_t *row_seq = nullptr, *row_pos = nullptr, *row_tok = nullptr, *arg = nullptr;
    q3::bf16* logits = nullptr;
    std::vector<void*> allocs;
    // host state
    struct Seq {
        bool live = false;
        std::vector<int32_t> pages;  // physical page of each logical page
        int kv_len = 0;              // positions in the cache = index of the next input token
        int forced = 0;              // tokens given by the caller (prompt, appended)
        int max_len = 0;             // tokens the sequence may hold (its KV capacity)
        int row = -1;                // its row in the last step (logits), -1 if none
    };
    std::vector<Seq> seqs;
    q3::PagePool pool{0};
    std::vector<int32_t> rows_host;  // the rows of the last uploaded step
    std::map<int, cudaGraphExec_t> graphs;  // one step of B rows, by B
};

namespace q3 {
namespace {

int balloc(q3_batch* b, void** p, size_t bytes) {
    cudaError_t st = cudaMalloc(p, bytes ? bytes : 16);
    if (st != cudaSuccess) {
        set_error(std::string("cudaMalloc(") + std::to_string(bytes) + "): " + cudaGetErrorString(st));
        return st == cudaErrorMemoryAllocation ? Q3_ERR_OOM : Q3_ERR_CUDA;
    }
    b->allocs.push_back(*p);
    return Q3_OK;
}
template <class T>
int balloc_t(q3_batch* b, T** p, size_t n) {
    return balloc(b, reinterpret_cast<void**>(p), n * sizeof(T));
}

void free_all(q3_batch* b) {
    for (auto& g : b->graphs) cudaGraphExecDestroy(g.second);
    b->graphs.clear();
    for (void* p : b->allocs) cudaFree(p);
    b->allocs.clear();
}

// One step of B rows (row_seq uploaded): prepare, the rows' forward, argmax, advance.
int record_step(q3_batch* b, int B) {
    q3_engine* e = b->e;
    cudaStream_t s = e->stream;
    batch_prepare_kernel<<<B, 128, 0, s>>>(b->row_seq, B, b->kv_len, b->tok, b->cap, b->tables, b->max_pages,
                                           b->row_pos, b->row_tok, b->row_pt);
    Q3_CUDA(cudaGetLastError());
    RowsSpec R;
    R.n = B;
    R.row_tokens = b->row_tok;
    R.row_pos = b->row_pos;
    R.page_table = b->row_pt;
    R.pt_stride = b->max_pages;
    R.k_pools = b->k_pools.data();
    R.v_pools = b->v_pools.data();
    R.pool_pages = b->pool_pages;
    R.max_pos = b->cap - 1;
    // one graph serves every position: splits from the rows alone, about two waves of
    // CTAs (B rows x kv heads x splits), no more than the capacity's pages
    {
        const int G = e->qh / e->kvh;
        const int per_split = B * e->kvh * (G / attn_heads_per_cta(G));
        const int want = std::max(1, 2 * e->sms / per_split);
        int sp = 1;
        while (sp * 2 <= want && sp * 2 <= 16 && sp * 2 <= b->max_pages) sp *= 2;
        R.attn_splits = std::min(sp, attn_splits(e->kvh, b->cap - 1, kPageSize, e->sms));
    }
    R.logits = b->logits;
    Q3_TRY_STATUS(forward_rows(e, R));
    Q3_CUDA(launch_argmax_rows(b->logits, B, e->vl, e->vl, b->arg, s));
    batch_advance_kernel<<<(B + 127) / 128, 128, 0, s>>>(b->row_seq, B, b->kv_len, b->forced, b->tok, b->cap, b->arg);
    Q3_CUDA(cudaGetLastError());
    return Q3_OK;
}

int step_graph(q3_batch* b, int B, cudaGraphExec_t* out) {
    auto it = b->graphs.find(B);
    if (it != b->graphs.end()) {
        *out = it->second;
        return Q3_OK;
    }
    cudaStream_t s = b->e->stream;
    cudaGraph_t g = nullptr;
    Q3_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    const int rc = record_step(b, B);
    const cudaError_t st = cudaStreamEndCapture(s, &g);
    if (rc != Q3_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (st != cudaSuccess) return fail(Q3_ERR_CUDA, std::string("batch graph capture: ") + cudaGetErrorString(st));
    cudaGraphExec_t x = nullptr;
    const cudaError_t si = cudaGraphInstantiate(&x, g, 0);
    cudaGraphDestroy(g);
    if (si != cudaSuccess) return fail(Q3_ERR_CUDA, std::string("batch graph instantiate: ") + cudaGetErrorString(si));
    b->graphs[B] = x;
    *out = x;
    return Q3_OK;
}

int seq_slot(q3_batch* b, uint32_t id, q3_batch::Seq** out) {
    if (id >= b->seqs.size() || !b->seqs[id].live) return fail(Q3_ERR_INVALID, "q3_batch: no such sequence");
    *out = &b->seqs[id];
    return Q3_OK;
}

int free_slot(q3_batch* b, uint32_t* id) {
    for (size_t i = 0; i < b->seqs.size(); ++i)
        if (!b->seqs[i].live) {
            *id = static_cast<uint32_t>(i);
            return Q3_OK;
        }
    return fail(Q3_ERR_INVALID, "q3_batch: every sequence slot is in use");
}

int upload_state(q3_batch* b, uint32_t id) {
    const q3_batch::Seq& q = b->seqs[id];
    cudaStream_t s = b->e->stream;
    std::vector<int32_t> table(b->max_pages, 0);
    std::copy(q.pages.begin(), q.pages.end(), table.begin());
    Q3_CUDA(cudaMemcpyAsync(b->tables + static_cast<size_t>(id) * b->max_pages, table.data(), b->max_pages * 4,
                            cudaMemcpyHostToDevice, s));
    const int32_t kv = q.kv_len, fo = q.forced;
    // pageable sources: each call returns once its source has been staged
    Q3_CUDA(cudaMemcpyAsync(b->kv_len + id, &kv, 4, cudaMemcpyHostToDevice, s));
    Q3_CUDA(cudaMemcpyAsync(b->forced + id, &fo, 4, cudaMemcpyHostToDevice, s));
    return Q3_OK;
}

}  // namespace
}  // namespace q3

using namespace q3;

extern "C" {

int q3_batch_create(q3_engine* e, uint32_t max_seqs, uint32_t pool_pages, q3_batch** out) {
    Q3_CHECK(e && out, "q3_batch_create: null argument");
    *out = nullptr;
    Q3_CHECK(max_seqs >= 1 && max_seqs <= static_cast<uint32_t>(kPrefillRows), "q3_batch_create: max_seqs");
    Q3_CHECK(pool_pages >= 1, "q3_batch_create: empty page pool");
    if (e->world > 1 || e->fp8 || e->vl % 128 != 0)
        return fail(Q3_ERR_UNSUPPORTED, "q3_batch: a single-GPU BF16 engine with vocab % 128 == 0");
    Q3_CUDA(cudaSetDevice(e->device));
    auto* b = new q3_batch();
    b->e = e;
    b->max_seqs = static_cast<int>(max_seqs);
    b->pool_pages = static_cast<int>(pool_pages);
    b->cap = static_cast<int>(e->cfg.capacity);
    b->max_pages = (b->cap + kPageSize - 1) / kPageSize;
    b->page_elems = static_cast<size_t>(e->kvh) * kPageSize * 128;
    auto bail = [&](int rc) {
        free_all(b);
        delete b;
        return rc;
    };
    int rc;
    const size_t L = e->layers.size();
    b->k_pools.resize(L);
    b->v_pools.resize(L);
    for (size_t l = 0; l < L; ++l) {
        if ((rc = balloc_t(b, &b->k_pools[l], pool_pages * b->page_elems)) != Q3_OK) return bail(rc);
        if ((rc = balloc_t(b, &b->v_pools[l], pool_pages * b->page_elems)) != Q3_OK) return bail(rc);
    }
    const size_t S = max_seqs;
    if ((rc = balloc_t(b, &b->tables, S * b->max_pages)) != Q3_OK) return bail(rc);
    if ((rc = balloc_t(b, &b->row_pt, S * b->max_pages)) != Q3_OK) return bail(rc);
    if ((rc = balloc_t(b, &b->tok, S * b->cap)) != Q3_OK) return bail(rc);
    if ((rc = balloc_t(b, &b->kv_len, S)) != Q3_OK) return bail(rc);
    if ((rc = balloc_t(b, &b->forced, S)) != Q3_OK) return bail(rc);
    if ((rc = balloc_t(b, &b->row_seq, S)) != Q3_OK) return bail(rc);
    if ((rc = balloc_t(b, &b->row_pos, S)) != Q3_OK) return bail(rc);
    if ((rc = balloc_t(b, &b->row_tok, S)) != Q3_OK) return bail(rc);
    if ((rc = balloc_t(b, &b->arg, S)) != Q3_OK) return bail(rc);
    if ((rc = balloc_t(b, &b->logits, S * e->vl)) != Q3_OK) return bail(rc);
    if ((rc = ensure_rows(e)) != Q3_OK) return bail(rc);
    if (cudaMemset(b->tables, 0, S * b->max_pages * 4) != cudaSuccess ||
        cudaMemset(b->tok, 0, S * b->cap * 4) != cudaSuccess)
        return bail(fail(Q3_ERR_CUDA, "q3_batch_create: cudaMemset failed"));
    b->seqs.resize(S);
    b->pool = PagePool(static_cast<int>(pool_pages));
    *out = b;
    return Q3_OK;
}

int q3_batch_destroy(q3_batch* b) {
    if (!b) return Q3_OK;
    cudaSetDevice(b->e->device);
    cudaStreamSynchronize(b->e->stream);
    free_all(b);
    delete b;
    return Q3_OK;
}

int q3_batch_add(q3_batch* b, const uint32_t* prompt, size_t n, size_t max_len, uint32_t* id) {
    Q3_CHECK(b && prompt && id, "q3_batch_add: null argument");
    Q3_CHECK(n >= 1, "q3_batch_add: empty prompt");
    if (max_len == 0) max_len = static_cast<size_t>(b->cap);
    Q3_CHECK(max_len <= static_cast<size_t>(b->cap), "q3_batch_add: max_len exceeds the engine's capacity");
    // generator.cpp:42-44
    if (n >= max_len) return fail(Q3_ERR_INVALID, "prompt does not fit in the model context");
    for (size_t i = 0; i < n; ++i) Q3_CHECK(prompt[i] < b->e->cfg.vocab, "q3_batch_add: token id >= vocab");
    q3_engine* e = b->e;
    Q3_CUDA(cudaSetDevice(e->device));
    uint32_t slot = 0;
    Q3_TRY_STATUS(free_slot(b, &slot));
    q3_batch::Seq q;
    const int pages = static_cast<int>((max_len + kPageSize - 1) / kPageSize);
    if (!b->pool.take_n(pages, q.pages)) return fail(Q3_ERR_OOM, "q3_batch: KV page pool exhausted");
    q.live = true;
    q.kv_len = static_cast<int>(n) - 1;
    q.forced = static_cast<int>(n);
    q.max_len = static_cast<int>(max_len);
    b->seqs[slot] = q;
    std::vector<int32_t> ids(prompt, prompt + n);
    int32_t* tok_row = b->tok + static_cast<size_t>(slot) * b->cap;
    // a failure below leaves no sequence behind: the slot is freed and its pages returned
    auto undo = [&](int rc) {
        b->pool.drop_all(b->seqs[slot].pages);
        b->seqs[slot] = q3_batch::Seq();
        return rc;
    };
    const cudaError_t up = cudaMemcpyAsync(tok_row, ids.data(), n * 4, cudaMemcpyHostToDevice, e->stream);
    if (up != cudaSuccess) return undo(fail(Q3_ERR_CUDA, std::string("q3_batch_add: ") + cudaGetErrorString(up)));
    int rc = upload_state(b, slot);
    if (rc != Q3_OK) return undo(rc);
    // Model::prefill (qwen3.hpp:168-173): positions [0, n - 1) through the batched rows
    for (int done = 0; done < static_cast<int>(n) - 1;) {
        RowsSpec R;
        R.n = std::min(static_cast<int>(n) - 1 - done, kPrefillRows);
        R.tokens = tok_row;
        R.p0 = done;
        R.page_table = b->tables + static_cast<size_t>(slot) * b->max_pages;
        R.k_pools = b->k_pools.data();
        R.v_pools = b->v_pools.data();
        R.pool_pages = b->pool_pages;
        R.max_pos = done + R.n - 1;
        if ((rc = forward_rows(e, R)) != Q3_OK) {
            cudaStreamSynchronize(e->stream);  // launches already queued may still write its pages
            return undo(rc);
        }
        done += R.n;
    }
    *id = slot;
    return Q3_OK;
}

int q3_batch_fork(q3_batch* b, uint32_t src, uint32_t* id) {
    Q3_CHECK(b && id, "q3_batch_fork: null argument");
    q3_batch::Seq* from = nullptr;
    Q3_TRY_STATUS(seq_slot(b, src, &from));
    q3_engine* e = b->e;
    Q3_CUDA(cudaSetDevice(e->device));
    uint32_t slot = 0;
    Q3_TRY_STATUS(free_slot(b, &slot));
    q3_batch::Seq q;
    q.live = true;
    q.kv_len = from->kv_len;
    q.forced = std::max(from->forced, from->kv_len + 1);
    q.max_len = from->max_len;
    // pages entirely before the position: shared, never written again; the rest fresh
    int copy = -1;
    if (!b->pool.fork(from->pages, from->kv_len, kPageSize, q.pages, &copy))
        return fail(Q3_ERR_OOM, "q3_batch: KV page pool exhausted");
    b->seqs[slot] = q;
    // a failure below leaves no sequence behind: the slot is freed and its references dropped
    auto undo = [&](int rc) {
        cudaStreamSynchronize(e->stream);
        b->pool.drop_all(b->seqs[slot].pages);
        b->seqs[slot] = q3_batch::Seq();
        return rc;
    };
    cudaError_t st = cudaSuccess;
    // the partial page (its positions before kv_len) is copied, every layer
    if (copy >= 0) {
        const size_t bytes = b->page_elems * 2;
        for (size_t l = 0; l < e->layers.size() && st == cudaSuccess; ++l) {
            st = cudaMemcpyAsync(b->k_pools[l] + q.pages[copy] * b->page_elems,
                                 b->k_pools[l] + from->pages[copy] * b->page_elems, bytes, cudaMemcpyDeviceToDevice,
                                 e->stream);
            if (st == cudaSuccess)
                st = cudaMemcpyAsync(b->v_pools[l] + q.pages[copy] * b->page_elems,
                                     b->v_pools[l] + from->pages[copy] * b->page_elems, bytes,
                                     cudaMemcpyDeviceToDevice, e->stream);
        }
    }
    if (st == cudaSuccess)
        st = cudaMemcpyAsync(b->tok + static_cast<size_t>(slot) * b->cap, b->tok + static_cast<size_t>(src) * b->cap,
                             static_cast<size_t>(b->cap) * 4, cudaMemcpyDeviceToDevice, e->stream);
    if (st != cudaSuccess) return undo(fail(Q3_ERR_CUDA, std::string("q3_batch_fork: ") + cudaGetErrorString(st)));
    const int rc = upload_state(b, slot);
    if (rc != Q3_OK) return undo(rc);
    if ((st = cudaStreamSynchronize(e->stream)) != cudaSuccess)
        return undo(fail(Q3_ERR_CUDA, std::string("q3_batch_fork: ") + cudaGetErrorString(st)));
    *id = slot;
    return Q3_OK;
}

int q3_batch_append(q3_batch* b, uint32_t id, const uint32_t* ids, size_t n) {
    Q3_CHECK(b && (ids || n == 0), "q3_batch_append: null argument");
    q3_batch::Seq* q = nullptr;
    Q3_TRY_STATUS(seq_slot(b, id, &q));
    if (n == 0) return Q3_OK;
    const int at = std::max(q->forced, q->kv_len + 1);  // after every token already determined
    Q3_CHECK(static_cast<size_t>(at) + n <= static_cast<size_t>(q->max_len), "q3_batch_append: past max_len");
    for (size_t i = 0; i < n; ++i) Q3_CHECK(ids[i] < b->e->cfg.vocab, "q3_batch_append: token id >= vocab");
    Q3_CUDA(cudaSetDevice(b->e->device));
    std::vector<int32_t> v(ids, ids + n);
    Q3_CUDA(cudaMemcpyAsync(b->tok + static_cast<size_t>(id) * b->cap + at, v.data(), n * 4, cudaMemcpyHostToDevice,
                            b->e->stream));
    q->forced = at + static_cast<int>(n);
    Q3_TRY_STATUS(upload_state(b, id));
    Q3_CUDA(cudaStreamSynchronize(b->e->stream));
    return Q3_OK;
}

int q3_batch_release(q3_batch* b, uint32_t id) {
    Q3_CHECK(b, "q3_batch_release: null argument");
    q3_batch::Seq* q = nullptr;
    Q3_TRY_STATUS(seq_slot(b, id, &q));
    Q3_CUDA(cudaSetDevice(b->e->device));
    // steps in flight may still read its pages
    Q3_CUDA(cudaStreamSynchronize(b->e->stream));
    b->pool.drop_all(q->pages);
    *q = q3_batch::Seq();
    return Q3_OK;
}

int q3_batch_step(q3_batch* b, size_t n) {
    Q3_CHECK(b, "q3_batch_step: null argument");
    q3_engine* e = b->e;
    Q3_CUDA(cudaSetDevice(e->device));
    cudaStream_t s = e->stream;
    for (size_t step = 0; step < n; ++step) {
        // the sequences with room for one more token
        std::vector<int32_t> rows;
        for (size_t i = 0; i < b->seqs.size(); ++i) {
            b->seqs[i].row = -1;
            const q3_batch::Seq& q = b->seqs[i];
            if (q.live && q.kv_len + 1 < q.max_len) rows.push_back(static_cast<int32_t>(i));
        }
        if (rows.empty()) break;
        const int B = static_cast<int>(rows.size());
        if (rows != b->rows_host) {
            // a pageable source: the call returns once it has been staged
            Q3_CUDA(cudaMemcpyAsync(b->row_seq, rows.data(), B * 4, cudaMemcpyHostToDevice, s));
            b->rows_host = rows;
        }
        cudaGraphExec_t graph = nullptr;
        Q3_TRY_STATUS(step_graph(b, B, &graph));
        Q3_CUDA(cudaGraphLaunch(graph, s));
        for (int r = 0; r < B; ++r) {
            q3_batch::Seq& q = b->seqs[rows[r]];
            q.row = r;
            ++q.kv_len;
        }
    }
    return Q3_OK;
}

int q3_batch_tokens(q3_batch* b, uint32_t id, uint32_t* out, size_t capacity, size_t* n) {
    Q3_CHECK(b && n, "q3_batch_tokens: null argument");
    q3_batch::Seq* q = nullptr;
    Q3_TRY_STATUS(seq_slot(b, id, &q));
    const size_t have = static_cast<size_t>(std::max(q->forced, q->kv_len + 1));
    *n = have;
    if (!out) return Q3_OK;
    Q3_CHECK(capacity >= have, "q3_batch_tokens: output buffer too small");
    Q3_CUDA(cudaSetDevice(b->e->device));
    Q3_TRY_STATUS(q3_engine_sync(b->e));
    Q3_CUDA(cudaMemcpy(out, b->tok + static_cast<size_t>(id) * b->cap, have * 4, cudaMemcpyDeviceToHost));
    return Q3_OK;
}

int q3_batch_logits(q3_batch* b, uint32_t id, uint16_t* out) {
    Q3_CHECK(b && out, "q3_batch_logits: null argument");
    q3_batch::Seq* q = nullptr;
    Q3_TRY_STATUS(seq_slot(b, id, &q));
    if (q->row < 0) return fail(Q3_ERR_INVALID, "q3_batch_logits: the sequence was not in the last step");
    Q3_CUDA(cudaSetDevice(b->e->device));
    Q3_TRY_STATUS(q3_engine_sync(b->e));
    Q3_CUDA(cudaMemcpy(out, b->logits + static_cast<size_t>(q->row) * b->e->vl, static_cast<size_t>(b->e->vl) * 2,
                       cudaMemcpyDeviceToHost));
    return Q3_OK;
}

int q3_batch_info(q3_batch* b, uint32_t id, size_t* position, size_t* free_pages) {
    Q3_CHECK(b, "q3_batch_info: null argument");
    if (free_pages) *free_pages = static_cast<size_t>(b->pool.free_count());
    if (position) {
        q3_batch::Seq* q = nullptr;
        Q3_TRY_STATUS(seq_slot(b, id, &q));
        *position = static_cast<size_t>(q->kv_len);
    }
    return Q3_OK;
}

}  // extern "C"

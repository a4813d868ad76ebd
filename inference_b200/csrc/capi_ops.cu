// capi_ops.cu -- the op-level C ABI: one entry point per reference Backend op
// (src/lib/backend/backend.hpp:26-36).  Each validates shapes and alignment on
// the host, launches the sm_100a kernel on the caller's stream and returns a
// status; nothing here synchronises.
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "host_util.hpp"
#include "kernels.cuh"

namespace q3 {

namespace {
thread_local std::string g_error;

// SM count of the current device; configures the kernels on first use of a device.
int current_sms() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    static std::mutex mu;
    static std::unordered_map<int, int> cache;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(dev);
    if (it != cache.end()) return it->second;
    const int n = num_sms(dev);
    configure_kernels();
    cache[dev] = n;
    return n;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return Q3_OK;
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return Q3_ERR_CUDA;
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }
const bf16* cb(const uint16_t* p) { return reinterpret_cast<const bf16*>(p); }
bf16* mb(uint16_t* p) { return reinterpret_cast<bf16*>(p); }

// Per-thread scratch word for the standalone argmax.
uint64_t* argmax_scratch() {
    thread_local uint64_t* p = nullptr;
    thread_local int dev_of_p = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (p == nullptr || dev_of_p != dev) {
        if (cudaMalloc(&p, 64) != cudaSuccess) return nullptr;
        dev_of_p = dev;
    }
    return p;
}
}  // namespace

void set_error(const std::string& msg) { g_error = msg; }

cudaError_t configure_kernels() {
    cudaError_t e = configure_gemv_kernels();
    if (e == cudaSuccess) e = configure_attention_kernels();
    if (e == cudaSuccess) e = configure_gemm_kernels();
    return e;
}

}  // namespace q3

using namespace q3;

extern "C" {

const char* q3_last_error(void) { return g_error.c_str(); }
int q3_version(void) { return 1; }

int q3_embedding(const uint16_t* table, size_t vocab, size_t hidden, uint32_t token, uint16_t* out, void* stream) {
    Q3_CHECK(table && out, "q3_embedding: null pointer");
    Q3_CHECK(token < vocab, "q3_embedding: token id out of range");
    return launch_status(launch_embedding(cb(table), static_cast<int>(hidden), token, mb(out), as_stream(stream)),
                         "q3_embedding");
}

int q3_gemv(const uint16_t* x, const uint16_t* w, uint16_t* y, size_t n_out, size_t n_in, void* stream) {
    Q3_CHECK(x && w && y, "q3_gemv: null pointer");
    Q3_CHECK(n_out > 0 && n_in > 0, "q3_gemv: empty shape");
    Q3_CHECK(n_in % 8 == 0, "q3_gemv: n_in must be a multiple of 8 (16-byte rows)");
    Q3_CHECK(n_in <= 32768 && n_out < (1u << 30), "q3_gemv: shape too large");
    Q3_CHECK(aligned16(x) && aligned16(w), "q3_gemv: x and W must be 16-byte aligned");
    GemvArgs a{};
    a.W = cb(w);
    a.N = static_cast<int>(n_out);
    a.K = static_cast<int>(n_in);
    a.plan = plan_gemv(a.N, a.K, EPI_STORE, current_sms());
    a.x = cb(x);
    a.y = mb(y);
    return launch_status(launch_gemv(PRO_PLAIN, EPI_STORE, a, as_stream(stream), false), "q3_gemv");
}

int q3_quantize_e4m3(const uint16_t* w, size_t rows, size_t full_cols, size_t c0, size_t cols, uint8_t* q,
                     float* scale, void* stream) {
    Q3_CHECK(w && q && scale, "q3_quantize_e4m3: null pointer");
    Q3_CHECK(rows < (1u << 30) && full_cols < (1u << 30), "q3_quantize_e4m3: shape too large");
    Q3_CHECK(c0 + cols <= full_cols && (c0 % 2) == 0 && (cols % 2) == 0, "q3_quantize_e4m3: bad column range");
    Q3_CHECK(reinterpret_cast<uintptr_t>(q) % 2 == 0, "q3_quantize_e4m3: q must be 2-byte aligned");
    if (rows == 0) return Q3_OK;
    const F8Dst d{q, scale, F8Pack{0, static_cast<int>(cols), 0, 0, 0}, 0, 1};  // row-major, pitch cols
    return launch_status(launch_quantize_e4m3(cb(w), full_cols, static_cast<int>(rows), static_cast<int>(full_cols),
                                              static_cast<int>(c0), static_cast<int>(cols), d, as_stream(stream)),
                         "q3_quantize_e4m3");
}

size_t q3_e4m3_packed_bytes(size_t n_out, size_t n_in) {
    if (n_out == 0 || n_in == 0 || n_out >= (1u << 30) || n_in > 32768) return 0;
    return f8_packed_bytes(static_cast<int>(n_out), static_cast<int>(n_in));
}

size_t q3_e4m3_packed_offset(size_t n_out, size_t n_in, int num_sms, size_t row, size_t col) {
    if (n_out == 0 || n_in == 0 || n_in % 64 != 0 || n_in > 32768 || n_out >= (1u << 30) || num_sms <= 0 ||
        row >= n_out || col >= n_in)
        return SIZE_MAX;
    const F8Pack L = f8_pack_for(static_cast<int>(n_out), static_cast<int>(n_in), EPI_STORE, num_sms);
    return f8_offset(L, static_cast<int>(row), static_cast<int>(col));
}

int q3_pack_e4m3(const uint8_t* q, size_t n_out, size_t n_in, uint8_t* packed, void* stream) {
    Q3_CHECK(q && packed, "q3_pack_e4m3: null pointer");
    Q3_CHECK(n_out > 0 && n_in > 0 && n_in % 64 == 0, "q3_pack_e4m3: n_in must be a positive multiple of 64");
    Q3_CHECK(n_in <= 32768 && n_out < (1u << 30), "q3_pack_e4m3: shape too large");
    Q3_CHECK(aligned16(q) && aligned16(packed), "q3_pack_e4m3: 16-byte aligned buffers required");
    const F8Pack L = f8_pack_for(static_cast<int>(n_out), static_cast<int>(n_in), EPI_STORE, current_sms());
    return launch_status(launch_pack_e4m3(q, L, packed, as_stream(stream)), "q3_pack_e4m3");
}

int q3_gemv_e4m3(const uint16_t* x, const uint8_t* w8, const float* scale, uint16_t* y, size_t n_out, size_t n_in,
                 void* stream) {
    Q3_CHECK(x && w8 && scale && y, "q3_gemv_e4m3: null pointer");
    Q3_CHECK(n_out > 0 && n_in > 0, "q3_gemv_e4m3: empty shape");
    Q3_CHECK(n_in % 64 == 0, "q3_gemv_e4m3: n_in must be a multiple of 64");
    Q3_CHECK(n_in <= 32768 && n_out < (1u << 30), "q3_gemv_e4m3: shape too large");
    Q3_CHECK(aligned16(x) && aligned16(w8), "q3_gemv_e4m3: x and W8 must be 16-byte aligned");
    GemvArgs a{};
    a.W8 = w8;
    a.wscale = scale;
    a.N = static_cast<int>(n_out);
    a.K = static_cast<int>(n_in);
    a.plan = plan_gemv(a.N, a.K, EPI_STORE, current_sms(), 1);
    a.x = cb(x);
    a.y = mb(y);
    return launch_status(launch_gemv(PRO_PLAIN, EPI_STORE, a, as_stream(stream), false), "q3_gemv_e4m3");
}

size_t q3_nvfp4_packed_bytes(size_t n_out, size_t n_in) {
    if (n_out == 0 || n_in == 0 || n_in % 64 != 0 || n_out >= (1u << 30) || n_in > 32768) return 0;
    return f4_packed_bytes(static_cast<int>(n_out), static_cast<int>(n_in));
}

size_t q3_nvfp4_packed_offset(size_t n_out, size_t n_in, int num_sms, size_t row, size_t col, int scale) {
    if (n_out == 0 || n_in == 0 || n_in % 64 != 0 || n_in > 32768 || n_out >= (1u << 30) || num_sms <= 0 ||
        row >= n_out || col >= n_in)
        return SIZE_MAX;
    const F8Pack L = f4_pack_for(static_cast<int>(n_out), static_cast<int>(n_in), EPI_STORE, num_sms);
    return scale ? f4_scale_offset(L, static_cast<int>(row), static_cast<int>(col))
                 : f4_nibble_offset(L, static_cast<int>(row), static_cast<int>(col));
}

int q3_quantize_nvfp4(const uint16_t* w, size_t n_out, size_t n_in, uint8_t* packed, float* row_scale,
                      void* stream) {
    Q3_CHECK(w && packed && row_scale, "q3_quantize_nvfp4: null pointer");
    Q3_CHECK(n_out > 0 && n_in > 0 && n_in % 64 == 0, "q3_quantize_nvfp4: n_in must be a positive multiple of 64");
    Q3_CHECK(n_in <= 32768 && n_out < (1u << 30), "q3_quantize_nvfp4: shape too large");
    Q3_CHECK(aligned16(packed), "q3_quantize_nvfp4: packed must be 16-byte aligned");
    const F8Dst d{packed, row_scale, f4_pack_for(static_cast<int>(n_out), static_cast<int>(n_in), EPI_STORE,
                                                 current_sms()), 0, 1};
    return launch_status(launch_quantize_nvfp4(cb(w), n_in, static_cast<int>(n_out), static_cast<int>(n_in), 0,
                                               static_cast<int>(n_in), d, as_stream(stream)),
                         "q3_quantize_nvfp4");
}

int q3_dequant_nvfp4(const uint8_t* packed, const float* row_scale, size_t n_out, size_t n_in, uint16_t* out,
                     void* stream) {
    Q3_CHECK(packed && row_scale && out, "q3_dequant_nvfp4: null pointer");
    Q3_CHECK(n_out > 0 && n_in > 0 && n_in % 64 == 0, "q3_dequant_nvfp4: n_in must be a positive multiple of 64");
    Q3_CHECK(n_in <= 32768 && n_out < (1u << 30), "q3_dequant_nvfp4: shape too large");
    Q3_CHECK(aligned16(packed) && aligned16(out), "q3_dequant_nvfp4: 16-byte aligned buffers required");
    const F8Pack L = f4_pack_for(static_cast<int>(n_out), static_cast<int>(n_in), EPI_STORE, current_sms());
    return launch_status(launch_dequant_nvfp4(packed, row_scale, L, mb(out), as_stream(stream)), "q3_dequant_nvfp4");
}

int q3_gemv_nvfp4(const uint16_t* x, const uint8_t* packed, const float* row_scale, uint16_t* y, size_t n_out,
                  size_t n_in, void* stream) {
    Q3_CHECK(x && packed && row_scale && y, "q3_gemv_nvfp4: null pointer");
    Q3_CHECK(n_out > 0 && n_in > 0 && n_in % 64 == 0, "q3_gemv_nvfp4: n_in must be a positive multiple of 64");
    Q3_CHECK(n_in <= 32768 && n_out < (1u << 30), "q3_gemv_nvfp4: shape too large");
    Q3_CHECK(aligned16(x) && aligned16(packed), "q3_gemv_nvfp4: x and the packed weights must be 16-byte aligned");
    GemvArgs a{};
    a.W8 = packed;
    a.wscale = row_scale;
    a.N = static_cast<int>(n_out);
    a.K = static_cast<int>(n_in);
    a.plan = plan_gemv(a.N, a.K, EPI_STORE, current_sms(), 0);
    a.x = cb(x);
    a.y = mb(y);
    return launch_status(launch_gemv(PRO_PLAIN, EPI_STORE, a, as_stream(stream), false), "q3_gemv_nvfp4");
}

int q3_gemm(const uint16_t* x, const uint16_t* w, uint16_t* y, size_t m, size_t n, size_t k, void* stream) {
    Q3_CHECK(x && w && y, "q3_gemm: null pointer");
    Q3_CHECK(m > 0 && n > 0 && k > 0, "q3_gemm: empty shape");
    Q3_CHECK(n % 128 == 0, "q3_gemm: n must be a multiple of 128");
    Q3_CHECK(k % 64 == 0, "q3_gemm: k must be a multiple of 64");
    Q3_CHECK(m < (1u << 24) && n < (1u << 24) && k < (1u << 20), "q3_gemm: shape too large");
    Q3_CHECK(aligned16(x) && aligned16(w) && aligned16(y), "q3_gemm: x, W and y must be 16-byte aligned");
    current_sms();
    GemmArgs a{};
    a.x = cb(x);
    a.w = cb(w);
    a.y = mb(y);
    a.M = static_cast<int>(m);
    a.N = static_cast<int>(n);
    a.K = static_cast<int>(k);
    a.ldy = a.N;
    a.epi = GEMM_STORE;
    return launch_status(launch_gemm(a, as_stream(stream)), "q3_gemm");
}

int q3_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* out, size_t n, float eps, void* stream) {
    Q3_CHECK(x && w && out && n > 0, "q3_rmsnorm: bad argument");
    return launch_status(launch_rmsnorm(cb(x), cb(w), mb(out), static_cast<int>(n), eps, as_stream(stream)),
                         "q3_rmsnorm");
}

int q3_rmsnorm_add(uint16_t* res, const uint16_t* upd, const uint16_t* w, uint16_t* out, size_t n, float eps,
                   void* stream) {
    Q3_CHECK(res && upd && w && out && n > 0, "q3_rmsnorm_add: bad argument");
    return launch_status(
        launch_rmsnorm_add(mb(res), cb(upd), cb(w), mb(out), static_cast<int>(n), eps, as_stream(stream)),
        "q3_rmsnorm_add");
}

int q3_rope(uint16_t* v, const float* cos_t, const float* sin_t, size_t heads, size_t head_dim, size_t pos,
            void* stream) {
    Q3_CHECK(v && cos_t && sin_t && head_dim % 2 == 0, "q3_rope: bad argument");
    return launch_status(launch_rope(mb(v), cos_t, sin_t, static_cast<int>(heads), static_cast<int>(head_dim),
                                     static_cast<int>(pos), as_stream(stream)),
                         "q3_rope");
}

int q3_qk_norm_rope(uint16_t* q, uint16_t* k, const uint16_t* qn, const uint16_t* kn, const float* cos_t,
                    const float* sin_t, size_t q_heads, size_t kv_heads, size_t head_dim, size_t pos, float eps,
                    void* stream) {
    Q3_CHECK(q && k && qn && kn && cos_t && sin_t, "q3_qk_norm_rope: null pointer");
    // the reference asserts head_dim 128 too (cuda/backend.cu:117)
    if (head_dim != 128) return fail(Q3_ERR_UNSUPPORTED, "q3_qk_norm_rope: head_dim must be 128");
    return launch_status(launch_qk_norm_rope(mb(q), mb(k), cb(qn), cb(kn), cos_t, sin_t, static_cast<int>(q_heads),
                                             static_cast<int>(kv_heads), static_cast<int>(pos), eps,
                                             as_stream(stream)),
                         "q3_qk_norm_rope");
}

size_t q3_attention_workspace_bytes(size_t q_heads, size_t kv_heads, size_t max_positions) {
    if (kv_heads == 0 || q_heads % kv_heads) return 0;
    const int splits = attn_splits(static_cast<int>(kv_heads), static_cast<int>(max_positions), 64, current_sms());
    return attn_workspace_bytes(static_cast<int>(q_heads), static_cast<int>(kv_heads), splits);
}

static int attention_common(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int32_t* page_table,
                            uint16_t* out, size_t q_heads, size_t kv_heads, size_t head_dim, size_t page_size,
                            size_t pos, void* ws, size_t ws_bytes, void* stream, int paged) {
    Q3_CHECK(q && k && v && out, "q3_attention: null pointer");
    (void)ws;
    (void)ws_bytes;  // splits merge in distributed shared memory; the workspace is unused
    if (head_dim != 128) return fail(Q3_ERR_UNSUPPORTED, "q3_attention: head_dim must be 128");
    Q3_CHECK(kv_heads > 0 && q_heads % kv_heads == 0, "q3_attention: q_heads must be a multiple of kv_heads");
    const size_t G = q_heads / kv_heads;
    if (!(G == 1 || G == 2 || G == 4 || G == 8)) return fail(Q3_ERR_UNSUPPORTED, "q3_attention: GQA group 1/2/4/8");
    if (paged) Q3_CHECK(page_size == 64 && page_table, "q3_attention_paged: page_size must be 64");
    Q3_CHECK(aligned16(k) && aligned16(v) && aligned16(q), "q3_attention: 16-byte alignment required");
    Q3_CHECK(pos < (1u << 24), "q3_attention: position too large");
    const int splits = attn_splits(static_cast<int>(kv_heads), static_cast<int>(pos), 64, current_sms());
    AttnArgs a{};
    a.q = cb(q);
    a.k = cb(k);
    a.v = cb(v);
    a.page_table = page_table;
    a.out = mb(out);
    a.q_heads = static_cast<int>(q_heads);
    a.kv_heads = static_cast<int>(kv_heads);
    a.page_size = 64;
    a.paged = paged;
    a.pos_ptr = nullptr;
    a.pos_host = static_cast<int>(pos);
    a.splits = splits;
    a.err = nullptr;
    cudaStream_t s = as_stream(stream);
    return launch_status(launch_attention(a, s, false), "q3_attention");
}

int q3_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, size_t q_heads,
                 size_t kv_heads, size_t head_dim, size_t pos, void* ws, size_t ws_bytes, void* stream) {
    return attention_common(q, k, v, nullptr, out, q_heads, kv_heads, head_dim, 64, pos, ws, ws_bytes, stream, 0);
}

int q3_attention_paged(const uint16_t* q, const uint16_t* k_pages, const uint16_t* v_pages, const int32_t* page_table,
                       uint16_t* out, size_t q_heads, size_t kv_heads, size_t head_dim, size_t page_size, size_t pos,
                       void* ws, size_t ws_bytes, void* stream) {
    return attention_common(q, k_pages, v_pages, page_table, out, q_heads, kv_heads, head_dim, page_size, pos, ws,
                            ws_bytes, stream, 1);
}

int q3_add(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n, void* stream) {
    Q3_CHECK(a && b && out, "q3_add: null pointer");
    if (n == 0) return Q3_OK;
    return launch_status(launch_add(cb(a), cb(b), mb(out), n, as_stream(stream)), "q3_add");
}

int q3_silu_mul(const uint16_t* g, const uint16_t* u, uint16_t* out, size_t n, void* stream) {
    Q3_CHECK(g && u && out, "q3_silu_mul: null pointer");
    if (n == 0) return Q3_OK;
    return launch_status(launch_silu_mul(cb(g), cb(u), mb(out), n, as_stream(stream)), "q3_silu_mul");
}

int q3_argmax(const uint16_t* logits, size_t n, uint32_t* index, void* stream) {
    Q3_CHECK(logits && index && n > 0, "q3_argmax: bad argument");
    Q3_CHECK(n < 0xFFFFFFFFull, "q3_argmax: too many logits");
    uint64_t* scratch = argmax_scratch();
    if (!scratch) return fail(Q3_ERR_OOM, "q3_argmax: scratch allocation failed");
    return launch_status(launch_argmax(cb(logits), n, index, scratch, as_stream(stream)), "q3_argmax");
}

int q3_fill_normal(uint16_t* dst, uint64_t seed, uint64_t tensor_id, size_t rows, size_t cols, size_t row0,
                   size_t col0, size_t full_cols, size_t dst_row_stride, void* stream) {
    Q3_CHECK(dst, "q3_fill_normal: null pointer");
    if (rows == 0 || cols == 0) return Q3_OK;
    return launch_status(launch_fill_normal(mb(dst), seed, tensor_id, rows, cols, row0, col0, full_cols,
                                            dst_row_stride ? dst_row_stride : cols, as_stream(stream)),
                         "q3_fill_normal");
}

void q3_prompt_ids(uint32_t* dst, size_t n, uint64_t seed, uint32_t vocab) {
    const uint64_t key = seed_key(seed);
    for (size_t i = 0; i < n; ++i) {
        uint64_t z = key ^ (0xFFull << 56) ^ static_cast<uint64_t>(i);
        z += 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z ^= z >> 31;
        dst[i] = static_cast<uint32_t>(((z >> 32) * static_cast<uint64_t>(vocab)) >> 32);
    }
}

}  // extern "C"

// ref_harness.cpp -- a C-ABI driver around the UNMODIFIED reference code.
// TEST INFRASTRUCTURE ONLY: built by oracle/build_ref.py from the reference's
// own sources into oracle/_ref/ (never committed, never part of the product).
//
// It drives the reference's Backend ops (src/lib/backend/backend.hpp:16-36)
// and its Qwen3 Model::build / Model::forward (src/lib/model/qwen3/qwen3.hpp:
// 105-166) with in-memory weights, exactly as Generator::load/generate do
// (src/lib/inference/generator.cpp:26-56) minus the tokenizer and file
// loading.  Compiled once against the CPU backend (libref_cpu.so) and, when
// CCCL 3.x headers are available, once against the CUDA backend
// (libref_cuda.so, -DREF_CUDA).
#include "backend/backend.hpp"
#include "backend/util/rope_cache.hpp"
#include "kv_cache/kv_cache.hpp"
#include "model/qwen3/config.hpp"
#include "model/qwen3/qwen3.hpp"
#include "model/weights.hpp"
#include "tensor/tensor.hpp"

#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <optional>
#include <string>
#include <vector>

#ifdef REF_CUDA
#include <cuda_runtime_api.h>
#endif

using namespace inference;

extern "C" void q3o_fill_normal(std::uint16_t* dst, std::uint64_t seed, std::uint64_t tensor_id, std::size_t rows,
                                std::size_t cols, std::size_t row0, std::size_t col0, std::size_t full_cols);

namespace {
    thread_local std::string g_error;

#ifdef REF_CUDA
    constexpr auto kDevice = types::Device::CUDA;
#else
    constexpr auto kDevice = types::Device::CPU;
#endif

    Backend& be() { return Backend::get_backend<kDevice>(); }

    Tensor upload(const void* src, const TensorShape& shape, types::DType dt = types::DType::BF16) {
        const auto bytes = shape.size() * types::dtype_byte_size(dt);
        return be().make_tensor(std::span{static_cast<const std::byte*>(src), bytes}, shape, dt);
    }

    void download(const Tensor& t, void* dst) {
#ifdef REF_CUDA
        if (cudaDeviceSynchronize() != cudaSuccess) throw std::runtime_error("cudaDeviceSynchronize failed");
        if (cudaMemcpy(dst, t.data<std::byte>(), t.size_bytes(), cudaMemcpyDeviceToHost) != cudaSuccess)
            throw std::runtime_error("cudaMemcpy D2H failed");
#else
        std::memcpy(dst, t.data<std::byte>(), t.size_bytes());
#endif
    }

    void write(Tensor& t, const void* src) {
#ifdef REF_CUDA
        if (cudaMemcpy(t.data<std::byte>(), src, t.size_bytes(), cudaMemcpyHostToDevice) != cudaSuccess)
            throw std::runtime_error("cudaMemcpy H2D failed");
#else
        std::memcpy(t.data<std::byte>(), src, t.size_bytes());
#endif
    }

    template <class F>
    int guarded(F&& f) {
        try {
            f();
            return 0;
        } catch (const std::exception& e) {
            g_error = e.what();
            return -1;
        }
    }
} // namespace

struct ref_config {
    std::size_t hidden, inter, layers, q_heads, kv_heads, head_dim, vocab, capacity;
    float eps, theta;
    int tied;
};

struct RefModel {
    model::qwen3::Model model;
    KVCache kv;
};

extern "C" {

const char* ref_last_error() { return g_error.c_str(); }
int ref_device() { return kDevice == types::Device::CUDA ? 1 : 0; }

// make_rope_cache, src/lib/backend/util/rope_cache.hpp:23-45.
int ref_rope_cache(std::size_t max_pos, std::size_t head_dim, float theta, float* cos_out, float* sin_out) {
    return guarded([&] {
        auto c = backend::make_rope_cache(max_pos, head_dim, theta, be());
        download(c.cosine, cos_out);
        download(c.sine, sin_out);
    });
}

int ref_op_embedding(std::uint32_t token, const std::uint16_t* table, std::size_t vocab, std::size_t hidden,
                     std::uint16_t* out) {
    return guarded([&] {
        auto w = upload(table, {vocab, hidden});
        auto o = Tensor::empty({hidden}, types::DType::BF16, be());
        be().embedding(token, w, o);
        download(o, out);
    });
}

int ref_op_gemv(const std::uint16_t* x, const std::uint16_t* w, std::uint16_t* y, std::size_t n_out, std::size_t n_in) {
    return guarded([&] {
        auto xt = upload(x, {n_in});
        auto wt = upload(w, {n_out, n_in});
        auto yt = Tensor::empty({n_out}, types::DType::BF16, be());
        be().matmul(xt, wt, yt);
        download(yt, y);
    });
}

int ref_op_rmsnorm(const std::uint16_t* x, const std::uint16_t* w, std::uint16_t* out, std::size_t hidden, float eps) {
    return guarded([&] {
        auto xt = upload(x, {hidden});
        auto wt = upload(w, {hidden});
        auto ot = Tensor::empty({hidden}, types::DType::BF16, be());
        be().rmsnorm(xt, wt, ot, eps);
        download(ot, out);
    });
}

int ref_op_rmsnorm_add(std::uint16_t* res, const std::uint16_t* upd, const std::uint16_t* w, std::uint16_t* out,
                       std::size_t hidden, float eps) {
    return guarded([&] {
        auto rt = upload(res, {hidden});
        auto ut = upload(upd, {hidden});
        auto wt = upload(w, {hidden});
        auto ot = Tensor::empty({hidden}, types::DType::BF16, be());
        be().rmsnorm_add(rt, ut, wt, ot, eps);
        download(rt, res);
        download(ot, out);
    });
}

int ref_op_qk_norm_rope(std::uint16_t* q, std::uint16_t* k, const std::uint16_t* qn, const std::uint16_t* kn,
                        std::size_t q_heads, std::size_t kv_heads, std::size_t head_dim, std::size_t pos, float theta,
                        float eps) {
    return guarded([&] {
        auto qt = upload(q, {q_heads, head_dim});
        auto kt = upload(k, {kv_heads, head_dim});
        auto qnt = upload(qn, {head_dim});
        auto knt = upload(kn, {head_dim});
        auto cache = backend::make_rope_cache(pos + 1, head_dim, theta, be());
        be().qk_norm_rope(qt, kt, qnt, knt, cache, pos, eps);
        download(qt, q);
        download(kt, k);
    });
}

int ref_op_attention(const std::uint16_t* q, const std::uint16_t* kc, const std::uint16_t* vc, std::uint16_t* out,
                     std::size_t q_heads, std::size_t kv_heads, std::size_t head_dim, std::size_t capacity,
                     std::size_t pos) {
    return guarded([&] {
        auto qt = upload(q, {q_heads, head_dim});
        auto kt = upload(kc, {capacity, kv_heads, head_dim});
        auto vt = upload(vc, {capacity, kv_heads, head_dim});
        auto ot = Tensor::empty({q_heads, head_dim}, types::DType::BF16, be());
        be().self_attention(qt, kt, vt, ot, pos);
        download(ot, out);
    });
}

int ref_op_silu(const std::uint16_t* g, const std::uint16_t* u, std::uint16_t* out, std::size_t n) {
    return guarded([&] {
        auto gt = upload(g, {n});
        auto ut = upload(u, {n});
        auto ot = Tensor::empty({n}, types::DType::BF16, be());
        be().silu(gt, ut, ot);
        download(ot, out);
    });
}

int ref_op_add(const std::uint16_t* a, const std::uint16_t* b, std::uint16_t* out, std::size_t n) {
    return guarded([&] {
        auto at = upload(a, {n});
        auto bt = upload(b, {n});
        auto ot = Tensor::empty({n}, types::DType::BF16, be());
        be().add(at, bt, ot);
        download(ot, out);
    });
}

long long ref_op_argmax(const std::uint16_t* logits, std::size_t n) {
    long long r = -1;
    if (guarded([&] {
            auto t = upload(logits, {n});
            r = be().argmax(t);
        }) != 0)
        return -1;
    return r;
}

// Model::build + KVCache over synthetic weights named as in the Hugging Face
// checkpoint (qwen3.hpp:17-68,105-128).  Tensor ids match the oracle's
// generator: embed 1, lm_head 2, layer l: 16+16l+{q,k,v,o,gate,up,down}.
void* ref_model_create(const ref_config* c, std::uint64_t seed) {
    RefModel* result = nullptr;
    guarded([&] {
        Weights weights;
        const auto H = c->hidden, I = c->inter, hd = c->head_dim;
        const auto qd = c->q_heads * hd, kd = c->kv_heads * hd;
        std::vector<std::uint16_t> buf;
        auto rand_tensor = [&](std::uint64_t tid, std::size_t rows, std::size_t cols) {
            buf.resize(rows * cols);
            q3o_fill_normal(buf.data(), seed, tid, rows, cols, 0, 0, cols);
            return upload(buf.data(), {rows, cols});
        };
        auto ones = [&](std::size_t n) {
            std::vector<std::uint16_t> one(n, 0x3F80);
            return upload(one.data(), {n});
        };
        weights.insert("model.embed_tokens.weight", rand_tensor(1, c->vocab, H));
        if (!c->tied) weights.insert("lm_head.weight", rand_tensor(2, c->vocab, H));
        weights.insert("model.norm.weight", ones(H));
        for (std::size_t l = 0; l < c->layers; ++l) {
            const auto p = "model.layers." + std::to_string(l) + ".";
            const std::uint64_t b = 16 + 16 * l;
            weights.insert(p + "self_attn.q_proj.weight", rand_tensor(b + 0, qd, H));
            weights.insert(p + "self_attn.k_proj.weight", rand_tensor(b + 1, kd, H));
            weights.insert(p + "self_attn.v_proj.weight", rand_tensor(b + 2, kd, H));
            weights.insert(p + "self_attn.o_proj.weight", rand_tensor(b + 3, H, qd));
            weights.insert(p + "mlp.gate_proj.weight", rand_tensor(b + 4, I, H));
            weights.insert(p + "mlp.up_proj.weight", rand_tensor(b + 5, I, H));
            weights.insert(p + "mlp.down_proj.weight", rand_tensor(b + 6, H, I));
            weights.insert(p + "input_layernorm.weight", ones(H));
            weights.insert(p + "post_attention_layernorm.weight", ones(H));
            weights.insert(p + "self_attn.q_norm.weight", ones(hd));
            weights.insert(p + "self_attn.k_norm.weight", ones(hd));
        }
        model::qwen3::Config config{
            .model_type = "qwen3",
            .eos_token_id = 151645,
            .head_dim = hd,
            .hidden_size = H,
            .intermediate_size = I,
            .max_position_embeddings = c->capacity,
            .dtype = types::DType::BF16,
            .num_attention_heads = c->q_heads,
            .num_hidden_layers = c->layers,
            .num_key_value_heads = c->kv_heads,
            .rms_norm_eps = c->eps,
            .rope_theta = c->theta,
            .tie_word_embeddings = c->tied != 0,
            .vocab_size = c->vocab,
        };
        auto kv = KVCache(c->layers, c->kv_heads, hd, c->capacity, types::DType::BF16, be());
        auto m = model::qwen3::Model::build(config, std::move(weights), c->capacity, be());
        result = new RefModel{std::move(m), std::move(kv)};
    });
    return result;
}

void ref_model_destroy(void* h) { delete static_cast<RefModel*>(h); }

// One Model::forward call (qwen3.hpp:131-166); returns the greedy token or -1.
long long ref_model_forward(void* h, std::uint32_t token) {
    auto* r = static_cast<RefModel*>(h);
    long long next = -1;
    if (guarded([&] { next = r->model.forward(token, be(), r->kv); }) != 0) return -1;
    return next;
}

int ref_model_logits(void* h, std::uint16_t* out) {
    auto* r = static_cast<RefModel*>(h);
    return guarded([&] { download(r->model.scratch.logits, out); });
}

int ref_model_kv_slot(void* h, std::size_t layer, std::size_t pos, std::uint16_t* k_out, std::uint16_t* v_out) {
    auto* r = static_cast<RefModel*>(h);
    return guarded([&] {
        auto k = r->kv.layers.at(layer).key.select(pos);
        auto v = r->kv.layers.at(layer).value.select(pos);
        download(k, k_out);
        download(v, v_out);
    });
}

// Slots [pos0, pos0 + n) of one layer's key / value caches (layout [capacity,
// kv_heads, head_dim], kv_cache.hpp:6-24) to / from host arrays [n][kv_heads][hd].
int ref_model_kv_range(void* h, std::size_t layer, std::size_t pos0, std::size_t n, std::uint16_t* k, std::uint16_t* v,
                       int to_model) {
    auto* r = static_cast<RefModel*>(h);
    return guarded([&] {
        auto& layer_kv = r->kv.layers.at(layer);
        const auto per = layer_kv.key.size() / r->kv.capacity;  // kv_heads * head_dim
        if (pos0 > r->kv.capacity || n > r->kv.capacity - pos0) throw std::out_of_range("kv range");
        const auto off = pos0 * per * sizeof(std::uint16_t), bytes = n * per * sizeof(std::uint16_t);
        auto* kd = layer_kv.key.data<std::byte>() + off;
        auto* vd = layer_kv.value.data<std::byte>() + off;
#ifdef REF_CUDA
        const auto dir = to_model ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost;
        if (cudaDeviceSynchronize() != cudaSuccess) throw std::runtime_error("cudaDeviceSynchronize failed");
        if (cudaMemcpy(to_model ? static_cast<void*>(kd) : static_cast<void*>(k), to_model ? static_cast<const void*>(k)
                       : static_cast<const void*>(kd), bytes, dir) != cudaSuccess ||
            cudaMemcpy(to_model ? static_cast<void*>(vd) : static_cast<void*>(v), to_model ? static_cast<const void*>(v)
                       : static_cast<const void*>(vd), bytes, dir) != cudaSuccess)
            throw std::runtime_error("cudaMemcpy of the KV range failed");
#else
        if (to_model) {
            std::memcpy(kd, k, bytes);
            std::memcpy(vd, v, bytes);
        } else {
            std::memcpy(k, kd, bytes);
            std::memcpy(v, vd, bytes);
        }
#endif
    });
}

std::size_t ref_model_token_count(void* h) { return static_cast<RefModel*>(h)->kv.token_count; }
void ref_model_set_token_count(void* h, std::size_t n) { static_cast<RefModel*>(h)->kv.token_count = n; }

// Fill KV slots [0, upto) of every layer with synthetic N(0, 0.02)-shaped
// values and move the cursor to `upto`, so a decode step can be timed at a
// given context without running the prompt through the model first.
int ref_model_fill_kv(void* h, std::size_t upto, std::uint64_t seed) {
    auto* r = static_cast<RefModel*>(h);
    return guarded([&] {
        for (std::size_t l = 0; l < r->kv.layers.size(); ++l) {
            auto& layer = r->kv.layers[l];
            const auto per = layer.key.size() / r->kv.capacity;
            std::vector<std::uint16_t> buf(r->kv.capacity * per, 0);
            q3o_fill_normal(buf.data(), seed, 0x4B00 + 2 * l, upto, per, 0, 0, per);
            write(layer.key, buf.data());
            q3o_fill_normal(buf.data(), seed, 0x4B01 + 2 * l, upto, per, 0, 0, per);
            write(layer.value, buf.data());
        }
        r->kv.token_count = upto;
    });
}

} // extern "C"

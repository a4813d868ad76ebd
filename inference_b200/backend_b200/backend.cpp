// backend.cpp -- the reference's Backend interface (src/lib/backend/backend.hpp:
// 16-42) implemented on libq3_sm100a.so: a drop-in for the reference's cuBLAS
// CUDA backend (src/lib/backend/cuda/backend.cu:24-155), which it replaces at
// link time -- its get_backend<Device::CUDA> specialisation is this one.
//
// A maintainer adds this file to the reference tree as
// src/lib/backend/b200/backend.cpp and links it, with libq3_sm100a.so and the
// CUDA runtime, in place of backend_cuda.  It includes the reference's own
// headers, so it compiles only against that tree (the library itself does
// not).
//
// Every op is one C-ABI call on this backend's stream, with the reference's
// semantics and aliasing (out == query for self_attention, out == update for
// rmsnorm_add, out == gate for silu, matmul into a KV-cache slot view).  As in
// the reference, only make_tensor and argmax synchronise with the host.
// Memory: plain cudaMalloc / cudaFree (the reference uses a stream-ordered
// pool; cudaFree waits for the device, so a tensor is never freed under a
// running kernel).  The stream is a blocking one, so the legacy default
// stream -- which callers such as tests use for their own copies -- stays
// ordered with it.
#include "backend/backend.hpp"
#include "backend/util/rope_cache.hpp"
#include "tensor/tensor.hpp"
#include "types/device.hpp"

#include "q3_sm100a.h"

#include <cuda_runtime_api.h>

#include <cstdint>
#include <new>
#include <stdexcept>
#include <string>

namespace inference::b200 {
    namespace {
        void check(const int status, const char* what) {
            if (status != Q3_OK) throw std::runtime_error(std::string(what) + ": " + q3_last_error());
        }

        void check_cuda(const cudaError_t error, const char* what) {
            if (error != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(error));
        }

        // BF16 tensors cross the C ABI as their bit patterns.
        const std::uint16_t* bits(const Tensor& t) { return t.data<std::uint16_t>(); }
        std::uint16_t* bits(Tensor& t) { return t.data<std::uint16_t>(); }
        const float* f32(const Tensor& t) { return t.data<float>(); }
    } // namespace

    class B200Backend final : public Backend {
    public:
        B200Backend() { check_cuda(cudaStreamCreate(&stream_), "cudaStreamCreate"); }

        ~B200Backend() override {
            if (index_ != nullptr) cudaFree(index_);
            if (stream_ != nullptr) cudaStreamDestroy(stream_);
        }

        B200Backend(const B200Backend&) = delete;
        B200Backend& operator=(const B200Backend&) = delete;

        [[nodiscard]] types::Device device() const override { return types::Device::CUDA; }

        [[nodiscard]] void* allocate(const std::size_t size_bytes) override {
            void* p = nullptr;
            if (cudaMalloc(&p, size_bytes == 0 ? 16 : size_bytes) != cudaSuccess) throw std::bad_alloc();
            return p;
        }

        void deallocate(void* pointer, std::size_t) noexcept override { cudaFree(pointer); }

        [[nodiscard]] Tensor make_tensor(const std::span<const std::byte> source, const TensorShape& shape,
                                         const types::DType dtype) override {
            // cuda/backend.cu make_tensor: the bytes must match the shape
            if (source.size_bytes() != shape.size() * types::dtype_byte_size(dtype))
                throw std::invalid_argument("b200::backend: tensor shape and dtype do not match the supplied data size");
            auto tensor = Tensor::empty(shape, dtype, *this);
            if (!source.empty()) {
                check_cuda(cudaMemcpyAsync(tensor.data<std::byte>(), source.data(), source.size_bytes(),
                                           cudaMemcpyHostToDevice, stream_),
                           "make_tensor upload");
                check_cuda(cudaStreamSynchronize(stream_), "make_tensor upload");
            }
            return tensor;
        }

        void embedding(const types::TokenId token_id, const Tensor& weights, Tensor& output) override {
            check(q3_embedding(bits(weights), weights.shape().dim(0), weights.shape().dim(1), token_id, bits(output),
                               stream_),
                  "embedding");
        }

        void matmul(const Tensor& input, const Tensor& weights, Tensor& output) override {
            check(q3_gemv(bits(input), bits(weights), bits(output), weights.shape().dim(0), weights.shape().dim(1),
                          stream_),
                  "matmul");
        }

        void rmsnorm(Tensor& input, const Tensor& weight, Tensor& output, const float epsilon) override {
            check(q3_rmsnorm(bits(input), bits(weight), bits(output), input.size(), epsilon, stream_), "rmsnorm");
        }

        void rmsnorm_add(Tensor& residual, const Tensor& residual_update, const Tensor& weight, Tensor& output,
                         const float epsilon) override {
            check(q3_rmsnorm_add(bits(residual), bits(residual_update), bits(weight), bits(output), residual.size(),
                                 epsilon, stream_),
                  "rmsnorm_add");
        }

        void rope(Tensor& values, const backend::RopeCache& cache, const std::size_t position) override {
            check(q3_rope(bits(values), f32(cache.cosine), f32(cache.sine), values.shape().dim(0),
                          values.shape().dim(1), position, stream_),
                  "rope");
        }

        void self_attention(const Tensor& query, const Tensor& key, const Tensor& value, Tensor& output,
                            const std::size_t position) override {
            // key / value: the layer's cache, [capacity, kv_heads, head_dim] (kv_cache.hpp:6-29);
            // the splits merge on chip, so no scratch tensor is kept (cuda/backend.cu:86-95 keeps one)
            check(q3_attention(bits(query), bits(key), bits(value), bits(output), query.shape().dim(0),
                               key.shape().dim(1), query.shape().dim(1), position, nullptr, 0, stream_),
                  "self_attention");
        }

        void add(const Tensor& left, const Tensor& right, Tensor& output) override {
            check(q3_add(bits(left), bits(right), bits(output), output.size(), stream_), "add");
        }

        void silu(const Tensor& gate, const Tensor& up, Tensor& output) override {
            check(q3_silu_mul(bits(gate), bits(up), bits(output), output.size(), stream_), "silu");
        }

        void qk_norm_rope(Tensor& query, Tensor& key, const Tensor& q_norm, const Tensor& k_norm,
                          const backend::RopeCache& cache, const std::size_t token_pos, const float eps) override {
            check(q3_qk_norm_rope(bits(query), bits(key), bits(q_norm), bits(k_norm), f32(cache.cosine),
                                  f32(cache.sine), query.shape().dim(0), key.shape().dim(0), query.shape().dim(1),
                                  token_pos, eps, stream_),
                  "qk_norm_rope");
        }

        [[nodiscard]] types::TokenId argmax(const Tensor& logits) override {
            // first index of the largest logit, returned to the host (cuda/backend.cu:107-112)
            if (index_ == nullptr) {
                void* p = nullptr;
                check_cuda(cudaMalloc(&p, sizeof(std::uint32_t)), "argmax scratch");
                index_ = static_cast<std::uint32_t*>(p);
            }
            check(q3_argmax(bits(logits), logits.size(), index_, stream_), "argmax");
            std::uint32_t host = 0;
            check_cuda(cudaMemcpyAsync(&host, index_, sizeof(host), cudaMemcpyDeviceToHost, stream_), "argmax");
            check_cuda(cudaStreamSynchronize(stream_), "argmax");
            return host;
        }

    private:
        cudaStream_t stream_ = nullptr;
        std::uint32_t* index_ = nullptr;
    };
} // namespace inference::b200

template <>
inference::Backend& inference::Backend::get_backend<inference::types::Device::CUDA>() {
    static inference::b200::B200Backend backend;
    return backend;
}

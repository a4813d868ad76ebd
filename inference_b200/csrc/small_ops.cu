// small_ops.cu -- the reference Backend's small ops as standalone kernels
// (used by the op-level C ABI, i.e. the drop-in Backend), plus the synthetic
// weight generator.  Inside the decode engine these ops are fused into the
// GEMV prologues/epilogues (gemv.cu) instead.
#include <algorithm>

#include "kernels.cuh"

namespace q3 {

namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// embedding.cuh:9-30
__global__ void embedding_kernel(const bf16* __restrict__ table, int hidden, uint32_t token, bf16* __restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < hidden) out[i] = table[static_cast<size_t>(token) * hidden + i];
}

__device__ float block_sum_1024(float v, float* sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float t = 0.f;
    const int nw = blockDim.x >> 5;
    for (int w = 0; w < nw; ++w) t += sh[w];
    __syncthreads();
    return t;
}

// rmsnorm.cuh:12-46 (one CTA; the op-level path is not the engine's hot path)
__global__ void rmsnorm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, bf16* __restrict__ out, int n,
                               float eps) {
    __shared__ float sh[32];
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = bf2f(x[i]);
        ss += v * v;
    }
    ss = block_sum_1024(ss, sh);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = f2bf(bf2f(x[i]) * scale * bf2f(w[i]));
}

// rmsnorm.cuh:48-80: res = bf16(res + upd); sum of squares of the unrounded
// sums; out from the rounded residual.  upd may alias out.
__global__ void rmsnorm_add_kernel(bf16* __restrict__ res, const bf16* upd, const bf16* __restrict__ w, bf16* out,
                                   int n, float eps) {
    __shared__ float sh[32];
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = bf2f(res[i]) + bf2f(upd[i]);
        res[i] = f2bf(v);
        ss += v * v;
    }
    ss = block_sum_1024(ss, sh);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = f2bf(bf2f(res[i]) * scale * bf2f(w[i]));
}

// qk_norm_rope.cuh:14-90: one warp per head, head_dim 128.
__global__ void qk_norm_rope_kernel(bf16* q, bf16* k, const bf16* __restrict__ qn, const bf16* __restrict__ kn,
                                    const float* __restrict__ cos_t, const float* __restrict__ sin_t, int q_heads,
                                    int kv_heads, int pos, float eps) {
    const int head = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (head >= q_heads + kv_heads) return;
    const bool is_q = head < q_heads;
    bf16* base = is_q ? q + static_cast<size_t>(head) * 128 : k + static_cast<size_t>(head - q_heads) * 128;
    const bf16* nw = is_q ? qn : kn;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = bf2f(base[lane + 32 * j]);
    const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
    const float scale = 1.0f / sqrtf(ss / 128.0f + eps);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int i = lane + 32 * j;
        const float c = cos_t[static_cast<size_t>(pos) * 64 + i];
        const float s = sin_t[static_cast<size_t>(pos) * 64 + i];
        const float x = v[j] * bf2f(nw[i]) * scale;
        const float y = v[j + 2] * bf2f(nw[i + 64]) * scale;
        base[i] = f2bf(x * c - y * s);
        base[i + 64] = f2bf(y * c + x * s);
    }
}

// rope.cuh:10-58
__global__ void rope_kernel(bf16* v, const float* __restrict__ cos_t, const float* __restrict__ sin_t, int heads,
                            int head_dim, int pos) {
    const int half = head_dim / 2;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= heads * half) return;
    const int h = idx / half, i = idx % half;
    const float c = cos_t[static_cast<size_t>(pos) * half + i];
    const float s = sin_t[static_cast<size_t>(pos) * half + i];
    bf16* base = v + static_cast<size_t>(h) * head_dim;
    const float x = bf2f(base[i]), y = bf2f(base[half + i]);
    base[i] = f2bf(x * c - y * s);
    base[half + i] = f2bf(x * s + y * c);
}

// add.cuh:10-31
__global__ void add_kernel(const bf16* a, const bf16* b, bf16* out, size_t n) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = f2bf(bf2f(a[i]) + bf2f(b[i]));
}

// silu.cuh:9-32
__global__ void silu_mul_kernel(const bf16* g, const bf16* u, bf16* out, size_t n) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float gv = bf2f(g[i]);
        out[i] = f2bf(gv / (1.0f + expf(-gv)) * bf2f(u[i]));
    }
}

// backend.cu:107-112 (thrust::max_element): first index of the maximum.
__global__ void argmax_partial_kernel(const bf16* __restrict__ logits, size_t n, unsigned long long* key) {
    __shared__ unsigned long long best;
    if (threadIdx.x == 0) best = 0ull;
    __syncthreads();
    unsigned long long mine = 0ull;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const unsigned long long k = argmax_key(bf2f(logits[i]), static_cast<uint32_t>(i));
        mine = mine > k ? mine : k;
    }
    atomicMax(&best, mine);
    __syncthreads();
    if (threadIdx.x == 0) atomicMax(key, best);
}

__global__ void argmax_final_kernel(const unsigned long long* key, uint32_t* index) {
    *index = argmax_key_index(*key);
}

// Synthetic N(0, 0.02) weights: Irwin-Hall sum of four 16-bit uniforms from
// one SplitMix64 hash of (tensor_id << 40 | flat index), one fp32 multiply,
// BF16 round-to-nearest-even -- the same bits as q3o_fill_normal on the host.
__global__ void fill_normal_kernel(bf16* dst, uint64_t key, uint64_t tensor_id, size_t rows, size_t cols, size_t row0,
                                   size_t col0, size_t full_cols, size_t dst_row_stride) {
    const size_t total = rows * cols;
    for (size_t e = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = e / cols, c = e % cols;
        const uint64_t flat = static_cast<uint64_t>(row0 + r) * full_cols + (col0 + c);
        const uint64_t h = mix64(key ^ ((tensor_id << 40) | flat));
        const int s = static_cast<int>(h & 0xFFFF) + static_cast<int>((h >> 16) & 0xFFFF) +
                      static_cast<int>((h >> 32) & 0xFFFF) + static_cast<int>((h >> 48) & 0xFFFF) - 131070;
        dst[r * dst_row_stride + c] = __float2bfloat16_rn(__fmul_rn(static_cast<float>(s), 0x1.1bc77ap-21f));
    }
}

__global__ void fill_const_kernel(bf16* dst, size_t n, float v) {
    const bf16 b = __float2bfloat16_rn(v);
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        dst[i] = b;
}

// Resolve the greedy token of the step that just ran from the per-rank
// argmax keys (used after the final step of a run, when no following step
// consumes the keys): argmax_hist[pos - 1] and, past the forced prefix,
// tokens[pos].
__global__ void resolve_tokens_kernel(const unsigned long long* keys, int n_keys, int32_t* tokens,
                                      int32_t* argmax_hist, const int32_t* pos_ptr, const int32_t* n_forced, int vocab,
                                      uint32_t* err) {
    const int pos = *pos_ptr;
    unsigned long long best = 0ull;
    for (int r = 0; r < n_keys; ++r) best = best > keys[r] ? best : keys[r];
    const uint32_t idx = argmax_key_index(best);
    if (pos < 1) return;
    if (idx >= static_cast<uint32_t>(vocab)) {
        record_error(err, DEV_BAD_TOKEN);
        return;
    }
    argmax_hist[pos - 1] = static_cast<int32_t>(idx);
    if (pos >= *n_forced) tokens[pos] = static_cast<int32_t>(idx);
}

int grid_for(size_t n, int block) {
    const size_t g = (n + block - 1) / block;
    return static_cast<int>(std::min<size_t>(g, 148 * 16));
}

}  // namespace

uint64_t seed_key(uint64_t seed) {
    uint64_t z = seed ^ 0x51A3D0F1B200ull;
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

int num_sms(int device) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
    return n;
}

cudaError_t launch_embedding(const bf16* table, int hidden, uint32_t token, bf16* out, cudaStream_t s) {
    embedding_kernel<<<(hidden + 255) / 256, 256, 0, s>>>(table, hidden, token, out);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const bf16* x, const bf16* w, bf16* out, int n, float eps, cudaStream_t s) {
    rmsnorm_kernel<<<1, 1024, 0, s>>>(x, w, out, n, eps);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm_add(bf16* res, const bf16* upd, const bf16* w, bf16* out, int n, float eps,
                               cudaStream_t s) {
    rmsnorm_add_kernel<<<1, 1024, 0, s>>>(res, upd, w, out, n, eps);
    return cudaGetLastError();
}

cudaError_t launch_qk_norm_rope(bf16* q, bf16* k, const bf16* qn, const bf16* kn, const float* cos_t,
                                const float* sin_t, int q_heads, int kv_heads, int pos, float eps, cudaStream_t s) {
    const int heads = q_heads + kv_heads;
    qk_norm_rope_kernel<<<(heads + 3) / 4, 128, 0, s>>>(q, k, qn, kn, cos_t, sin_t, q_heads, kv_heads, pos, eps);
    return cudaGetLastError();
}

cudaError_t launch_rope(bf16* v, const float* cos_t, const float* sin_t, int heads, int head_dim, int pos,
                        cudaStream_t s) {
    const int n = heads * head_dim / 2;
    rope_kernel<<<(n + 255) / 256, 256, 0, s>>>(v, cos_t, sin_t, heads, head_dim, pos);
    return cudaGetLastError();
}

cudaError_t launch_add(const bf16* a, const bf16* b, bf16* out, size_t n, cudaStream_t s) {
    add_kernel<<<grid_for(n, 256), 256, 0, s>>>(a, b, out, n);
    return cudaGetLastError();
}

cudaError_t launch_silu_mul(const bf16* g, const bf16* u, bf16* out, size_t n, cudaStream_t s) {
    silu_mul_kernel<<<grid_for(n, 256), 256, 0, s>>>(g, u, out, n);
    return cudaGetLastError();
}

cudaError_t launch_argmax(const bf16* logits, size_t n, uint32_t* index, uint64_t* scratch, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(uint64_t), s);
    if (e != cudaSuccess) return e;
    argmax_partial_kernel<<<std::min(grid_for(n, 256), 296), 256, 0, s>>>(
        logits, n, reinterpret_cast<unsigned long long*>(scratch));
    argmax_final_kernel<<<1, 1, 0, s>>>(reinterpret_cast<const unsigned long long*>(scratch), index);
    return cudaGetLastError();
}

cudaError_t launch_fill_normal(bf16* dst, uint64_t seed, uint64_t tensor_id, size_t rows, size_t cols, size_t row0,
                               size_t col0, size_t full_cols, size_t dst_row_stride, cudaStream_t s) {
    fill_normal_kernel<<<grid_for(rows * cols, 256), 256, 0, s>>>(dst, seed_key(seed), tensor_id, rows, cols, row0,
                                                                  col0, full_cols, dst_row_stride);
    return cudaGetLastError();
}

cudaError_t launch_fill_const(bf16* dst, size_t n, float value, cudaStream_t s) {
    fill_const_kernel<<<grid_for(n, 256), 256, 0, s>>>(dst, n, value);
    return cudaGetLastError();
}

cudaError_t launch_resolve_tokens(const uint64_t* keys, int n_keys, int32_t* tokens, int32_t* argmax_hist,
                                  const int32_t* pos_ptr, const int32_t* n_forced, int vocab, uint32_t* err,
                                  cudaStream_t s) {
    resolve_tokens_kernel<<<1, 1, 0, s>>>(reinterpret_cast<const unsigned long long*>(keys), n_keys, tokens,
                                          argmax_hist, pos_ptr, n_forced, vocab, err);
    return cudaGetLastError();
}

}  // namespace q3

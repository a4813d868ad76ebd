// prefill.cu -- the row-wise kernels of the batched prefill (one row = one
// prompt token).  The GEMMs are gemm.cu's; attention is attention.cu's with a
// batch of query positions.  Arithmetic per row is the decode path's:
//   embedding      embedding.cuh:9-30
//   rmsnorm        rmsnorm.cuh:12-46 (x * scale * w rounded once)
//   rmsnorm_add    rmsnorm.cuh:58-60 (squares of the unrounded fp32 sums)
//   qk_norm_rope   qk_norm_rope.cuh:14-90 (rounded once, after the rotation)
#include "kernels.cuh"

namespace q3 {

namespace {

constexpr int kRowThreads = 256;

__global__ void __launch_bounds__(128) embed_rows_kernel(const bf16* __restrict__ table, const int32_t* __restrict__ tokens,
                                                       int p0, int vocab, int H, bf16* __restrict__ x,
                                                       uint32_t* err, const int32_t* __restrict__ row_tokens) {
    const int row = blockIdx.x;
    int t = row_tokens ? row_tokens[row] : tokens[p0 + row];
    if (t < 0 || t >= vocab) {
        if (threadIdx.x == 0) record_error(err, DEV_BAD_TOKEN);
        t = 0;
    }
    const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(t) * H);
    uint4* dst = reinterpret_cast<uint4*>(x + static_cast<size_t>(row) * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// xn[row] = rmsnorm(x[row]) with weights w; with vsum the sum of squares runs
// over vsum[row] (the unrounded residual sums).
__global__ void __launch_bounds__(kRowThreads) rmsnorm_rows_kernel(const bf16* __restrict__ x,
                                                                 const float* __restrict__ vsum,
                                                                 const bf16* __restrict__ w, bf16* __restrict__ xn,
                                                                 int H, float eps) {
    __shared__ float red[kRowThreads / 32];
    const int row = blockIdx.x, tid = threadIdx.x;
    const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * H);
    float ss = 0.f;
    for (int i = tid; i < H / 8; i += kRowThreads) {
        if (vsum) {
            const float4* vr = reinterpret_cast<const float4*>(vsum + static_cast<size_t>(row) * H);
            const float4 v0 = vr[2 * i], v1 = vr[2 * i + 1];
            ss += v0.x * v0.x + v0.y * v0.y + v0.z * v0.z + v0.w * v0.w;
            ss += v1.x * v1.x + v1.y * v1.y + v1.z * v1.z + v1.w * v1.w;
        } else {
            const uint4 h = xr[i];
            const uint32_t* hw = reinterpret_cast<const uint32_t*>(&h);
#pragma unroll
            for (int e = 0; e < 4; ++e) ss += bf_lo(hw[e]) * bf_lo(hw[e]) + bf_hi(hw[e]) * bf_hi(hw[e]);
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < kRowThreads / 32; ++i) tot += red[i];
    const float scale = 1.0f / sqrtf(tot / static_cast<float>(H) + eps);
    uint4* out = reinterpret_cast<uint4*>(xn + static_cast<size_t>(row) * H);
    for (int i = tid; i < H / 8; i += kRowThreads) {
        const uint4 h = xr[i];
        const uint4 wv = reinterpret_cast<const uint4*>(w)[i];
        const uint32_t* hw = reinterpret_cast<const uint32_t*>(&h);
        const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const bf16 b0 = f2bf(bf_lo(hw[e]) * scale * bf_lo(ww[e]));
            const bf16 b1 = f2bf(bf_hi(hw[e]) * scale * bf_hi(ww[e]));
            ow[e] = static_cast<uint32_t>(__bfloat16_as_ushort(b0)) |
                    (static_cast<uint32_t>(__bfloat16_as_ushort(b1)) << 16);
        }
        out[i] = o;
    }
}

// One CTA per prompt token at position p0 + row: q heads normalised and
// rotated in place in the QKV row, k heads normalised and rotated into the
// cache slot, v heads copied to theirs.  Warp w handles heads w, w + 8, ...
__global__ void __launch_bounds__(kRowThreads) qkv_rows_kernel(PrefillQkvArgs a) {
    const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = a.row_pos ? a.row_pos[row] : a.p0 + row;
    bf16* qkv = a.qkv + static_cast<size_t>(row) * a.ld;
    const int page = (a.row_pos ? a.page_table + static_cast<size_t>(row) * a.pt_stride : a.page_table)[pos / 64];
    const int n_heads = a.q_heads + 2 * a.kv_heads;
    for (int h = warp; h < n_heads; h += kRowThreads / 32) {
        if (h >= a.q_heads + a.kv_heads) {
            const int kh = h - a.q_heads - a.kv_heads;
            bf16* dst = a.v_pages + ((static_cast<size_t>(page) * a.kv_heads + kh) * 64 + pos % 64) * 128;
            if (lane < 16)
                reinterpret_cast<uint4*>(dst)[lane] = reinterpret_cast<const uint4*>(qkv + static_cast<size_t>(h) * 128)[lane];
            continue;
        }
        const bool is_q = h < a.q_heads;
        const bf16* src = qkv + static_cast<size_t>(h) * 128;
        const bf16* nw = is_q ? a.q_norm : a.k_norm;
        bf16* dst = is_q ? qkv + static_cast<size_t>(h) * 128
                         : a.k_pages + ((static_cast<size_t>(page) * a.kv_heads + (h - a.q_heads)) * 64 + pos % 64) * 128;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = bf2f(src[lane + 32 * j]);
        const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
        const float scale = 1.0f / sqrtf(ss / 128.0f + a.eps);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int i = lane + 32 * j;
            const float cs = a.rope_cos[static_cast<size_t>(pos) * 64 + i];
            const float sn = a.rope_sin[static_cast<size_t>(pos) * 64 + i];
            const float x = v[j] * bf2f(nw[i]) * scale;
            const float y = v[j + 2] * bf2f(nw[i + 64]) * scale;
            dst[i] = f2bf(x * cs - y * sn);
            dst[i + 64] = f2bf(y * cs + x * sn);
        }
    }
}

// One CTA per row: the first index of the row's largest BF16 value, through the
// order-preserving (value, index) keys of the fused lm_head argmax.
__global__ void __launch_bounds__(kRowThreads) argmax_rows_kernel(const bf16* __restrict__ logits, int n, int ld,
                                                                int32_t* __restrict__ out) {
    __shared__ unsigned long long red[kRowThreads / 32];
    const bf16* row = logits + static_cast<size_t>(blockIdx.x) * ld;
    uint64_t best = 0;
    for (int i = threadIdx.x; i < n; i += kRowThreads) best = max(best, argmax_key(bf2f(row[i]), static_cast<uint32_t>(i)));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
        best = max(best, static_cast<uint64_t>(__shfl_xor_sync(0xffffffffu, static_cast<unsigned long long>(best), off)));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint64_t b = 0;
        for (int w = 0; w < kRowThreads / 32; ++w) b = max(b, static_cast<uint64_t>(red[w]));
        out[blockIdx.x] = static_cast<int32_t>(argmax_key_index(b));
    }
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// This rank's partial rows of exchange `seq` (written by the GEMM launched just
// before on the same stream, so complete) are ready: raise the flag in every
// rank's buffer after a system-scope fence.
__global__ void tp_signal_kernel(TpExchange x, uint32_t seq) {
    if (threadIdx.x != 0) return;
    __threadfence_system();
    const int slot = static_cast<int>(seq & 1u);
    for (int j = 0; j < x.world; ++j)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(x.flags[j] + slot * kMaxRanks + x.rank), "r"(seq)
                     : "memory");
}

// Residual update with the sum of every rank's partial rows, in rank order (the
// same bits on every rank): v = x + bf16(sum); x = bf16(v); vsum = v (the
// unrounded sums the next rmsnorm_add squares, rmsnorm.cuh:58-60).  With flags,
// first waits (bounded) until every rank raised its flag for `seq`.
__global__ void __launch_bounds__(kRowThreads) tp_resid_rows_kernel(TpExchange x, uint32_t seq, size_t n4, bf16* xr,
                                                                  float* vsum, uint32_t* err) {
    const int slot = static_cast<int>(seq & 1u);
    if (x.flags[x.rank]) {
        if (threadIdx.x < static_cast<unsigned>(x.world)) {
            const uint32_t* f = x.flags[x.rank] + slot * kMaxRanks + threadIdx.x;
            for (uint32_t polls = 0; ld_acquire_sys_u32(f) != seq; ++polls) {
                if ((polls & 1023) == 1023 && *reinterpret_cast<volatile uint32_t*>(err)) break;
                if (polls > (1u << 22)) {
                    record_error(err, DEV_PEER_WAIT_TIMEOUT);
                    break;
                }
                __nanosleep(64);
            }
        }
        __syncthreads();
    }
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        float4 p[kMaxRanks];
#pragma unroll
        for (int j = 0; j < kMaxRanks; ++j)
            if (j < x.world) p[j] = __ldcg(reinterpret_cast<const float4*>(x.part[j] + slot * x.slot_floats) + i);
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < kMaxRanks; ++j)
            if (j < x.world) {
                t.x += p[j].x;
                t.y += p[j].y;
                t.z += p[j].z;
                t.w += p[j].w;
            }
        uint2 h = reinterpret_cast<const uint2*>(xr)[i];
        const float v0 = bf_lo(h.x) + round_bf(t.x), v1 = bf_hi(h.x) + round_bf(t.y);
        const float v2 = bf_lo(h.y) + round_bf(t.z), v3 = bf_hi(h.y) + round_bf(t.w);
        h.x = static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(v0))) | (static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(v1))) << 16);
        h.y = static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(v2))) | (static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(v3))) << 16);
        reinterpret_cast<uint2*>(xr)[i] = h;
        if (vsum) reinterpret_cast<float4*>(vsum)[i] = make_float4(v0, v1, v2, v3);
    }
}

}  // namespace

cudaError_t launch_tp_signal(const TpExchange& x, uint32_t seq, cudaStream_t s) {
    tp_signal_kernel<<<1, 32, 0, s>>>(x, seq);
    return cudaGetLastError();
}

cudaError_t launch_tp_resid_rows(const TpExchange& x, uint32_t seq, int n, int H, bf16* xr, float* vsum, uint32_t* err,
                                 int num_sms, cudaStream_t s) {
    if (x.world < 1 || x.world > kMaxRanks || H % 4 != 0 || n <= 0) return cudaErrorInvalidValue;
    if (static_cast<size_t>(n) * H > x.slot_floats) return cudaErrorInvalidValue;
    const size_t n4 = static_cast<size_t>(n) * H / 4;
    const size_t want = (n4 + kRowThreads - 1) / kRowThreads;
    const int grid = static_cast<int>(want < static_cast<size_t>(num_sms) * 8 ? want : static_cast<size_t>(num_sms) * 8);
    tp_resid_rows_kernel<<<grid, kRowThreads, 0, s>>>(x, seq, n4, xr, vsum, err);
    return cudaGetLastError();
}

cudaError_t launch_embed_rows(const bf16* table, const int32_t* tokens, int p0, int n, int vocab, int H, bf16* x,
                              uint32_t* err, cudaStream_t s, const int32_t* row_tokens) {
    embed_rows_kernel<<<n, 128, 0, s>>>(table, tokens, p0, vocab, H, x, err, row_tokens);
    return cudaGetLastError();
}

cudaError_t launch_argmax_rows(const bf16* logits, int rows, int n, int ld, int32_t* out, cudaStream_t s) {
    if (rows <= 0 || n <= 0 || ld < n) return cudaErrorInvalidValue;
    argmax_rows_kernel<<<rows, kRowThreads, 0, s>>>(logits, n, ld, out);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm_rows(const bf16* x, const float* vsum, const bf16* w, bf16* xn, int n, int H, float eps,
                                cudaStream_t s) {
    rmsnorm_rows_kernel<<<n, kRowThreads, 0, s>>>(x, vsum, w, xn, H, eps);
    return cudaGetLastError();
}

cudaError_t launch_qkv_rows(const PrefillQkvArgs& a, int n, cudaStream_t s) {
    qkv_rows_kernel<<<n, kRowThreads, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace q3

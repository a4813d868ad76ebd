// fp8.cu -- packed weight storage for the decode GEMVs.  FP8 E4M3: row-wise
// quantization with power-of-two scales.  NVFP4 (below): E2M1 weights with an
// E4M3 scale per 16-column block and a power-of-two scale per row.  The reference stores BF16 weights only (README.md:13); this is the
// build's optional weight format, halving the bytes the decode GEMVs stream.
// A power-of-two scale keeps every dequantized weight q * 2^e an exact BF16
// value (at most four significant bits), so an FP8 engine computes exactly the
// BF16 model whose weights are those round trips, and the GEMV applies the
// scale to the fp32 row sum (an exact power-of-two multiply).
#include "kernels.cuh"

namespace q3 {

namespace {

constexpr int kQThreads = 256;

__global__ void __launch_bounds__(kQThreads) quantize_e4m3_kernel(const bf16* __restrict__ src, size_t ld_src,
                                                                 int full_cols, int c0, int cols, const F8Dst d) {
    __shared__ float red[kQThreads / 32];
    const int row = blockIdx.x, tid = threadIdx.x;
    const bf16* s = src + static_cast<size_t>(row) * ld_src;
    float mx = 0.f;
    for (int c = tid; c < full_cols; c += kQThreads) mx = fmaxf(mx, fabsf(bf2f(s[c])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = 0.f;
    for (int i = 0; i < kQThreads / 32; ++i) mx = fmaxf(mx, red[i]);
    // mx = f * 2^k, f in [0.5, 1); 448 = 0.875 * 2^9
    int e = 0;
    if (mx > 0.f) {
        int k;
        const float f = frexpf(mx, &k);
        e = (f <= 0.875f) ? k - 9 : k - 8;
    }
    const int drow = d.row0 + row * d.row_step;
    if (tid == 0) d.scale[drow] = ldexpf(1.0f, e);
    const bf16* sc = s + c0;
    for (int c = 2 * tid; c < cols; c += 2 * kQThreads) {
        const float2 v = make_float2(ldexpf(bf2f(sc[c]), -e), ldexpf(bf2f(sc[c + 1]), -e));
        const __nv_fp8x2_storage_t q = __nv_cvt_float2_to_fp8x2(v, __NV_SATFINITE, __NV_E4M3);
        // an even column and the next share a 16-byte group in either layout
        *reinterpret_cast<uint16_t*>(d.base + f8_offset(d.pack, drow, c)) = static_cast<uint16_t>(q);
    }
}

// One thread per 16-byte group of the row-major matrix (groups past K: zeros).
__global__ void pack_e4m3_kernel(const uint8_t* __restrict__ q, const F8Pack L, uint8_t* __restrict__ packed) {
    const int groups = L.nch * (kF8TileCols / 16);
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<long long>(L.N) * groups) return;
    const int row = static_cast<int>(i / groups), col = static_cast<int>(i % groups) * 16;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (col < L.K) v = *reinterpret_cast<const uint4*>(q + static_cast<size_t>(row) * L.K + col);
    *reinterpret_cast<uint4*>(packed + f8_offset(L, row, col)) = v;
}

// The exact BF16 values of a packed E4M3 matrix: out[row, col] =
// E4M3(row, col) * scale[row], row-major [N, K] (K % 16 == 0).  Each product
// has at most four significant bits and a power-of-two factor, so every step
// (E4M3 -> f16 -> f32, the scaling, f32 -> BF16) is exact.  One thread per
// 16-byte group: the group's bytes are contiguous in the packed layout too.
__global__ void dequant_e4m3_kernel(const uint8_t* __restrict__ packed, const float* __restrict__ scale,
                                    const F8Pack L, bf16* __restrict__ out) {
    const int groups = L.K / 16;
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<long long>(L.N) * groups) return;
    const int row = static_cast<int>(i / groups), col = static_cast<int>(i % groups) * 16;
    const uint4 v = *reinterpret_cast<const uint4*>(packed + f8_offset(L, row, col));
    const float sc = scale[row];
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
    uint4 o[2];
    uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t word = w[j / 2] >> (16 * (j & 1));
        const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(word & 0xFFFFu), __NV_E4M3);
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
        ow[j] = static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(f.x * sc))) |
                (static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(f.y * sc))) << 16);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * L.K + col);
    dst[0] = o[0];
    dst[1] = o[1];
}

// ---------------------------------------------------------------- NVFP4
// E2M1 code of x: nearest of 0, 0.5, 1, 1.5, 2, 3, 4, 6 (ties to the even code),
// saturating at 6; bit 3 the sign.
__device__ __forceinline__ uint32_t e2m1_code(float x) {
    const uint32_t s = (__float_as_uint(x) >> 31) << 3;
    const float a = fabsf(x);
    uint32_t c;
    if (a <= 0.25f) c = 0;
    else if (a < 0.75f) c = 1;
    else if (a <= 1.25f) c = 2;
    else if (a < 1.75f) c = 3;
    else if (a <= 2.5f) c = 4;
    else if (a < 3.5f) c = 5;
    else if (a <= 5.0f) c = 6;
    else c = 7;
    return s | c;
}

__device__ __forceinline__ float e2m1_value(uint32_t c) {
    const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    const float v = mag[c & 7];
    return (c & 8) ? -v : v;
}

__device__ __forceinline__ float e4m3_value(uint8_t q) {
    const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(q), __NV_E4M3);
    return __half2float(*reinterpret_cast<const __half*>(&h));
}

// One CTA per source row: the row scale from the whole row (full_cols), then one
// thread per 16-column block of [c0, c0 + cols): its E4M3 scale and 16 nibbles.
__global__ void __launch_bounds__(kQThreads) quantize_nvfp4_kernel(const bf16* __restrict__ src, size_t ld_src,
                                                                  int full_cols, int c0, int cols, const F8Dst d) {
    __shared__ float red[kQThreads / 32];
    const int row = blockIdx.x, tid = threadIdx.x;
    const bf16* s = src + static_cast<size_t>(row) * ld_src;
    float mx = 0.f;
    for (int c = tid; c < full_cols; c += kQThreads) mx = fmaxf(mx, fabsf(bf2f(s[c])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = 0.f;
    for (int i = 0; i < kQThreads / 32; ++i) mx = fmaxf(mx, red[i]);
    // mx = f * 2^k, f in [0.5, 1); 6 * 448 = 2688 = 0.65625 * 2^12
    int e = 0;
    if (mx > 0.f) {
        int k;
        const float f = frexpf(mx, &k);
        e = (f <= 0.65625f) ? k - 12 : k - 11;
    }
    const int drow = d.row0 + row * d.row_step;
    if (tid == 0) d.scale[drow] = ldexpf(1.0f, e);
    for (int b = tid; b < cols / 16; b += kQThreads) {
        const bf16* blk = s + c0 + 16 * b;
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(bf2f(blk[j])));
        const uint8_t sc =
            static_cast<uint8_t>(__nv_cvt_float_to_fp8(ldexpf(amax / 6.0f, -e), __NV_SATFINITE, __NV_E4M3));
        const float sv = e4m3_value(sc);
        uint32_t lo = 0, hi = 0;  // 16 nibbles, column 2 i in the low nibble of byte i
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float x = bf2f(blk[j]);
            const uint32_t q = sv > 0.f ? e2m1_code(ldexpf(x, -e) / sv) : ((__float_as_uint(x) >> 31) << 3);
            if (j < 8) lo |= q << (4 * j);
            else hi |= q << (4 * (j - 8));
        }
        *reinterpret_cast<uint2*>(d.base + f4_nibble_offset(d.pack, drow, 16 * b)) = make_uint2(lo, hi);
        d.base[f4_scale_offset(d.pack, drow, 16 * b)] = sc;
    }
}

// One thread per 16-column block: its 16 exact BF16 values.
__global__ void dequant_nvfp4_kernel(const uint8_t* __restrict__ packed, const float* __restrict__ scale,
                                     const F8Pack L, bf16* __restrict__ out) {
    const int blocks = L.K / 16;
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<long long>(L.N) * blocks) return;
    const int row = static_cast<int>(i / blocks), col = static_cast<int>(i % blocks) * 16;
    const uint2 v = *reinterpret_cast<const uint2*>(packed + f4_nibble_offset(L, row, col));
    const float sc = e4m3_value(packed[f4_scale_offset(L, row, col)]) * scale[row];
    bf16* dst = out + static_cast<size_t>(row) * L.K + col;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const uint32_t word = j < 8 ? v.x : v.y;
        dst[j] = f2bf(e2m1_value((word >> (4 * (j & 7))) & 0xF) * sc);
    }
}

}  // namespace

cudaError_t launch_quantize_nvfp4(const bf16* src, size_t ld_src, int rows, int full_cols, int c0, int cols,
                                  const F8Dst& dst, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    if (dst.pack.fmt != 1 || (cols % 16) || (c0 % 16) || c0 + cols > full_cols || cols > dst.pack.K ||
        dst.pack.N <= 0)
        return cudaErrorInvalidValue;
    quantize_nvfp4_kernel<<<rows, kQThreads, 0, s>>>(src, ld_src, full_cols, c0, cols, dst);
    return cudaGetLastError();
}

cudaError_t launch_dequant_nvfp4(const uint8_t* packed, const float* scale, const F8Pack& pack, bf16* out,
                                 cudaStream_t s) {
    if (pack.fmt != 1 || pack.N <= 0 || pack.K % 16 != 0) return cudaErrorInvalidValue;
    const long long n = static_cast<long long>(pack.N) * (pack.K / 16);
    dequant_nvfp4_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(packed, scale, pack, out);
    return cudaGetLastError();
}

cudaError_t launch_dequant_e4m3(const uint8_t* packed, const float* scale, const F8Pack& pack, bf16* out,
                                cudaStream_t s) {
    if (pack.N <= 0 || pack.K % 16 != 0) return cudaErrorInvalidValue;
    const long long n = static_cast<long long>(pack.N) * (pack.K / 16);
    dequant_e4m3_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(packed, scale, pack, out);
    return cudaGetLastError();
}

cudaError_t launch_quantize_e4m3(const bf16* src, size_t ld_src, int rows, int full_cols, int c0, int cols,
                                 const F8Dst& dst, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    if ((cols & 1) || (c0 & 1) || (dst.pack.K & 1) || c0 + cols > full_cols || cols > dst.pack.K)
        return cudaErrorInvalidValue;
    quantize_e4m3_kernel<<<rows, kQThreads, 0, s>>>(src, ld_src, full_cols, c0, cols, dst);
    return cudaGetLastError();
}

cudaError_t launch_pack_e4m3(const uint8_t* q, const F8Pack& pack, uint8_t* packed, cudaStream_t s) {
    if (pack.N <= 0 || pack.K % 16 != 0) return cudaErrorInvalidValue;
    const long long n = static_cast<long long>(pack.N) * pack.nch * (kF8TileCols / 16);
    pack_e4m3_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(q, pack, packed);
    return cudaGetLastError();
}

}  // namespace q3

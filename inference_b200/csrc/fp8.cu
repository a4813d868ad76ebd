// fp8.cu -- FP8 E4M3 weight storage: row-wise quantization with power-of-two
// scales.  The reference stores BF16 weights only (README.md:13); this is the
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

}  // namespace

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

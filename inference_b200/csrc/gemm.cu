// gemm.cu -- Y[M, N] = X[M, K] W[N, K]^T on the 5th-generation tensor cores,
// for the batched prefill (all prompt tokens of a layer in one GEMM).
//
// The reference prefills by running the decode step once per prompt token
// (src/lib/model/qwen3/qwen3.hpp:168-173), i.e. P cuBLAS GEMVs per weight
// matrix.  Here every weight matrix is read once per 128 prompt tokens:
//   * one CTA per (128-row token tile, BN-column output tile), BN = 128 or 256;
//   * warp 0 streams 128 x 64 tiles of X and BN x 64 tiles of W into a
//     kStages-deep shared-memory ring with 2-D TMA (128-byte swizzle; both
//     operands K-major, exactly as they sit in memory);
//   * one thread of warp 1 issues tcgen05.mma (kind::f16, BF16 x BF16 -> FP32)
//     into a BN-column TMEM accumulator, four K=16 steps per stage, and frees
//     each stage with tcgen05.commit on its "empty" mbarrier;
//   * warps 2-5 (one per 32-lane TMEM quarter) read the accumulator with
//     tcgen05.ld after the final commit, round to BF16 and apply the epilogue:
//     store, residual add (keeping the unrounded fp32 sums the next
//     rmsnorm_add squares), or SwiGLU of interleaved gate/up columns.
// Numerics follow the GEMV: fp32 accumulation of exact BF16 products, one
// rounding to BF16 per output (cuBLAS GemmEx in the reference, matmul.cuh:8-18).
// Every mbarrier wait is bounded; on a timeout the kernel records the error,
// lets its copies and MMAs drain, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <atomic>
#include <mutex>

#include "kernels.cuh"

namespace q3 {

namespace {

constexpr int kBM = 128;          // token rows per tile (TMEM lanes)
constexpr int kBK = 64;           // K per stage: one 128-byte swizzle atom of BF16
constexpr int kGemmThreads = 192; // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr int kATile = kBM * kBK * 2;  // 16 KB

template <int BN>
struct GemmCfg {
    static constexpr int kStages = BN == 256 ? 4 : 6;
    static constexpr int kBTile = BN * kBK * 2;
    static constexpr int kStage = kATile + kBTile;
    static constexpr int kSmem = kStages * kStage + 1024 /* barriers */ + 1024 /* alignment */;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major tile with 128-byte swizzle:
// rows of 128 B, 8-row atoms 1024 B apart (stride byte offset), version 1.
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
    const uint64_t addr = smem_u32(tile);
    return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

// Instruction descriptor: D fp32, A and B BF16, both K-major, M = 128, N = BN.
template <int BN>
__device__ __forceinline__ uint32_t mma_idesc() {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
           (static_cast<uint32_t>(kBM >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 16 consecutive fp32 columns of TMEM: this thread's row, columns col..col+15.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                const __grid_constant__ GemmArgs a) {
    using Cfg = GemmCfg<BN>;
    constexpr int S = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    // SWIZZLE_128B tiles want 1024-byte alignment
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStage);
    uint64_t* empty = full + S;
    uint64_t* accum = empty + S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN;
    // split-K (blockIdx.z): this CTA's k-tiles [kt0, kt0 + KT)
    const int kt0 = a.kt_per ? static_cast<int>(blockIdx.z) * a.kt_per : 0;
    const int KT = a.kt_per ? min(a.kt_per, a.K / kBK - kt0) : a.K / kBK;
    float* const yf = a.yf ? a.yf + blockIdx.z * a.yf_split : nullptr;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer
            int issued = 0;
            for (int kt = 0; kt < KT; ++kt) {
                const int s = kt % S;
                if (kt >= S && !mbar_wait(&empty[s], ((kt / S) - 1) & 1, a.err, DEV_TMA_WAIT_TIMEOUT)) break;
                uint8_t* st = smem + s * Cfg::kStage;
                mbar_arrive_expect_tx(&full[s], Cfg::kStage);
                tma_load_2d(st, &tmap_x, (kt0 + kt) * kBK, m0, &full[s]);
                tma_load_2d(st + kATile, &tmap_w, (kt0 + kt) * kBK, n0, &full[s]);
                issued = kt + 1;
            }
            // leave no copy in flight: the last round issued into every stage must land
            for (int kt = (issued > S ? issued - S : 0); kt < issued; ++kt)
                mbar_wait(&full[kt % S], (kt / S) & 1, nullptr, 0);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer
            const uint32_t idesc = mma_idesc<BN>();
            for (int kt = 0; kt < KT; ++kt) {
                const int s = kt % S;
                const bool ok = mbar_wait(&full[s], (kt / S) & 1, a.err, DEV_TMA_WAIT_TIMEOUT);
                tc_fence_after();
                if (ok) {
                    const uint8_t* st = smem + s * Cfg::kStage;
                    const uint64_t ad = sw128_desc(st), bd = sw128_desc(st + kATile);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)  // K = 16 per MMA: +32 bytes in the swizzled row
                        umma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (kt | kk) != 0);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(accum);
            // TMEM is freed below only after every MMA has landed
            mbar_wait(accum, 0, a.err, DEV_TMA_WAIT_TIMEOUT);
        }
        __syncwarp();
    } else {
        // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31, one token row per thread
        const int quarter = warp & 3;
        const int row = m0 + quarter * 32 + lane;
        const bool ok = mbar_wait(accum, 0, a.err, DEV_TMA_WAIT_TIMEOUT);
        tc_fence_after();
        if (ok) {
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                float v[16];
                tmem_ld16(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + c0, v);
                if (row >= a.M) continue;
                const int n = n0 + c0;
                if constexpr (EPI == GEMM_STORE) {
                    uint4 o[2];
                    uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        ow[i] = static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(v[2 * i]))) |
                                (static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(v[2 * i + 1]))) << 16);
                    uint4* dst = reinterpret_cast<uint4*>(a.y + static_cast<size_t>(row) * a.ldy + n);
                    dst[0] = o[0];
                    dst[1] = o[1];
                } else if constexpr (EPI == GEMM_SWIGLU) {
                    // columns (2j, 2j + 1) = (gate_j, up_j); qwen3.hpp:154-156 -> silu.cuh:18-20
                    uint4 o;
                    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float r[2];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const float gv = round_bf(v[4 * i + 2 * h]), uv = round_bf(v[4 * i + 2 * h + 1]);
                            r[h] = gv / (1.0f + expf(-gv)) * uv;
                        }
                        ow[i] = static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(r[0]))) |
                                (static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(r[1]))) << 16);
                    }
                    *reinterpret_cast<uint4*>(a.y + static_cast<size_t>(row) * a.ldy + n / 2) = o;
                } else if constexpr (EPI == GEMM_F32) {
                    // a row-parallel shard's partial: summed over the ranks, then rounded once
                    float4* dst = reinterpret_cast<float4*>(yf + static_cast<size_t>(row) * a.ldy + n);
#pragma unroll
                    for (int i = 0; i < 4; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                } else {
                    // residual: hs = bf16(hs + bf16(acc)) (qwen3.hpp:151-152, 158-159); the fp32
                    // sums feed the next rmsnorm_add (rmsnorm.cuh:58-60)
                    bf16* h = a.y + static_cast<size_t>(row) * a.ldy + n;
                    uint4 hv[2];
                    hv[0] = reinterpret_cast<const uint4*>(h)[0];
                    hv[1] = reinterpret_cast<const uint4*>(h)[1];
                    uint32_t* hw = reinterpret_cast<uint32_t*>(hv);
                    float s[16];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        s[2 * i] = bf_lo(hw[i]) + round_bf(v[2 * i]);
                        s[2 * i + 1] = bf_hi(hw[i]) + round_bf(v[2 * i + 1]);
                        hw[i] = static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(s[2 * i]))) |
                                (static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(s[2 * i + 1]))) << 16);
                    }
                    reinterpret_cast<uint4*>(h)[0] = hv[0];
                    reinterpret_cast<uint4*>(h)[1] = hv[1];
                    if (a.vsum) {
                        float4* vs = reinterpret_cast<float4*>(a.vsum + static_cast<size_t>(row) * a.ldy + n);
#pragma unroll
                        for (int i = 0; i < 4; ++i) vs[i] = make_float4(s[4 * i], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
    }
}

// Row-major [rows, K] BF16 matrix, box = box_rows x 64 columns, 128-byte swizzle.
bool make_tmap(CUtensorMap* map, const bf16* base, int rows, int K, int box_rows) {
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<bf16*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int EPI>
cudaError_t launch_bn(const GemmArgs& a, const CUtensorMap& tx, const CUtensorMap& tw, cudaStream_t s, int splits) {
    auto* fn = gemm_kernel<BN, EPI>;
    // the shared-memory opt-in once per device (not per launch: launches may be captured into a graph)
    static std::atomic<uint32_t> configured{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint32_t bit = 1u << (dev & 31);
    if (!(configured.load() & bit)) {
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN>::kSmem);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    const dim3 grid((a.M + kBM - 1) / kBM, a.N / BN, splits);
    fn<<<grid, kGemmThreads, GemmCfg<BN>::kSmem, s>>>(tx, tw, a);
    return cudaGetLastError();
}

// Split-K: the splits' fp32 partial tiles ws[split][M][N] summed in split order,
// then the requested epilogue on the sums (the same arithmetic as the GEMM's own
// epilogues).  One thread per 8 consecutive output columns of a row.
__global__ void gemm_split_reduce_kernel(GemmArgs a, const float* __restrict__ ws, int splits) {
    const int per_row = a.N / 8;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.M * per_row) return;
    const int row = i / per_row, n = (i % per_row) * 8;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int z = 0; z < splits; ++z) {
        const float4* src = reinterpret_cast<const float4*>(ws + (static_cast<size_t>(z) * a.M + row) * a.N + n);
        const float4 p0 = src[0], p1 = src[1];
        v[0] += p0.x, v[1] += p0.y, v[2] += p0.z, v[3] += p0.w;
        v[4] += p1.x, v[5] += p1.y, v[6] += p1.z, v[7] += p1.w;
    }
    if (a.epi == GEMM_STORE) {
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
        for (int k = 0; k < 4; ++k)
            ow[k] = static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(v[2 * k]))) |
                    (static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(v[2 * k + 1]))) << 16);
        *reinterpret_cast<uint4*>(a.y + static_cast<size_t>(row) * a.ldy + n) = o;
    } else if (a.epi == GEMM_SWIGLU) {
        uint2 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
        for (int k = 0; k < 2; ++k) {
            float r[2];
            for (int h = 0; h < 2; ++h) {
                const float gv = round_bf(v[4 * k + 2 * h]), uv = round_bf(v[4 * k + 2 * h + 1]);
                r[h] = gv / (1.0f + expf(-gv)) * uv;
            }
            ow[k] = static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(r[0]))) |
                    (static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(r[1]))) << 16);
        }
        *reinterpret_cast<uint2*>(a.y + static_cast<size_t>(row) * a.ldy + n / 2) = o;
    } else if (a.epi == GEMM_F32) {
        float4* dst = reinterpret_cast<float4*>(a.yf + static_cast<size_t>(row) * a.ldy + n);
        dst[0] = make_float4(v[0], v[1], v[2], v[3]);
        dst[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        bf16* h = a.y + static_cast<size_t>(row) * a.ldy + n;
        uint4 hv = *reinterpret_cast<const uint4*>(h);
        uint32_t* hw = reinterpret_cast<uint32_t*>(&hv);
        float sm[8];
        for (int k = 0; k < 4; ++k) {
            sm[2 * k] = bf_lo(hw[k]) + round_bf(v[2 * k]);
            sm[2 * k + 1] = bf_hi(hw[k]) + round_bf(v[2 * k + 1]);
            hw[k] = static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(sm[2 * k]))) |
                    (static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(sm[2 * k + 1]))) << 16);
        }
        *reinterpret_cast<uint4*>(h) = hv;
        if (a.vsum) {
            float4* vs = reinterpret_cast<float4*>(a.vsum + static_cast<size_t>(row) * a.ldy + n);
            vs[0] = make_float4(sm[0], sm[1], sm[2], sm[3]);
            vs[1] = make_float4(sm[4], sm[5], sm[6], sm[7]);
        }
    }
}

}  // namespace

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// The shared-memory opt-in of every GEMM variant on the current device, ahead of
// any stream capture.
cudaError_t configure_gemm_kernels() {
    cudaError_t e = cudaSuccess;
    auto set = [&](const void* fn, int bytes) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    };
    set(reinterpret_cast<const void*>(gemm_kernel<128, GEMM_STORE>), GemmCfg<128>::kSmem);
    set(reinterpret_cast<const void*>(gemm_kernel<256, GEMM_STORE>), GemmCfg<256>::kSmem);
    set(reinterpret_cast<const void*>(gemm_kernel<128, GEMM_SWIGLU>), GemmCfg<128>::kSmem);
    set(reinterpret_cast<const void*>(gemm_kernel<256, GEMM_SWIGLU>), GemmCfg<256>::kSmem);
    set(reinterpret_cast<const void*>(gemm_kernel<128, GEMM_RESID>), GemmCfg<128>::kSmem);
    set(reinterpret_cast<const void*>(gemm_kernel<256, GEMM_RESID>), GemmCfg<256>::kSmem);
    set(reinterpret_cast<const void*>(gemm_kernel<128, GEMM_F32>), GemmCfg<128>::kSmem);
    set(reinterpret_cast<const void*>(gemm_kernel<256, GEMM_F32>), GemmCfg<256>::kSmem);
    return e;
}

// BN = 256 when that still gives at least one wave of CTAs, else 128.
int gemm_tile_n(int M, int N, int sms) {
    const int mt = (M + kBM - 1) / kBM;
    return (N % 256 == 0 && mt * (N / 256) >= sms) ? 256 : 128;
}

cudaError_t launch_gemm(const GemmArgs& args, cudaStream_t s) {
    GemmArgs a = args;
    if (a.M <= 0 || a.N % 128 || a.K % kBK || a.K <= 0) return cudaErrorInvalidValue;
    if (a.epi == GEMM_F32 && (!a.yf || a.ldy % 4 != 0 || a.ldy < a.N)) return cudaErrorInvalidValue;
    const int BN = a.bn ? a.bn : gemm_tile_n(a.M, a.N, 148);
    if (BN != 128 && BN != 256) return cudaErrorInvalidValue;
    if (a.N % BN) return cudaErrorInvalidValue;
    CUtensorMap tx, tw;
    if (!make_tmap(&tx, a.x, a.M, a.K, kBM) || !make_tmap(&tw, a.w, a.N, a.K, BN)) return cudaErrorInvalidValue;
    // Split-K for one row tile (a batch of decode rows: the weights stream once and the
    // output tiles alone would leave SMs idle or a ragged last wave): the split count
    // whose CTAs fill whole waves best (fewer splits on a tie), every split keeping at
    // least 4 k-tiles and the partials fitting the workspace
    int splits = 1;
    const int tiles = a.N / BN, KT = a.K / kBK, sms = a.sms > 0 ? a.sms : 148;
    if (a.ws && a.M <= kBM) {
        auto fill = [&](int sp) {
            const double waves = static_cast<double>(tiles) * sp / sms;
            return waves / std::ceil(waves);
        };
        double best = fill(1);
        for (int sp = 2; sp <= 16 && KT / sp >= 4; ++sp) {
            if (static_cast<size_t>(sp) * a.M * a.N > a.ws_floats) break;
            if (fill(sp) > best + 0.05) {
                best = fill(sp);
                splits = sp;
            }
        }
    }
    if (splits > 1) {
        a.kt_per = (KT + splits - 1) / splits;
        splits = (KT + a.kt_per - 1) / a.kt_per;
        GemmArgs p = a;  // the splits' partial tiles, [split][M][N] fp32
        p.epi = GEMM_F32;
        p.yf = a.ws;
        p.ldy = a.N;
        p.yf_split = static_cast<size_t>(a.M) * a.N;
        const cudaError_t e = BN == 256 ? launch_bn<256, GEMM_F32>(p, tx, tw, s, splits)
                                        : launch_bn<128, GEMM_F32>(p, tx, tw, s, splits);
        if (e != cudaSuccess) return e;
        const int threads = a.M * (a.N / 8);
        gemm_split_reduce_kernel<<<(threads + 63) / 64, 64, 0, s>>>(a, a.ws, splits);
        return cudaGetLastError();
    }
    a.kt_per = 0;
    a.yf_split = 0;
    switch (a.epi * 2 + (BN == 256)) {
        case GEMM_STORE * 2: return launch_bn<128, GEMM_STORE>(a, tx, tw, s, 1);
        case GEMM_STORE * 2 + 1: return launch_bn<256, GEMM_STORE>(a, tx, tw, s, 1);
        case GEMM_SWIGLU * 2: return launch_bn<128, GEMM_SWIGLU>(a, tx, tw, s, 1);
        case GEMM_SWIGLU * 2 + 1: return launch_bn<256, GEMM_SWIGLU>(a, tx, tw, s, 1);
        case GEMM_RESID * 2: return launch_bn<128, GEMM_RESID>(a, tx, tw, s, 1);
        case GEMM_RESID * 2 + 1: return launch_bn<256, GEMM_RESID>(a, tx, tw, s, 1);
        case GEMM_F32 * 2: return launch_bn<128, GEMM_F32>(a, tx, tw, s, 1);
        case GEMM_F32 * 2 + 1: return launch_bn<256, GEMM_F32>(a, tx, tw, s, 1);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace q3

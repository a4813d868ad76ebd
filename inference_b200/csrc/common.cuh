// common.cuh -- device helpers shared by the sm_100a decode kernels.
//
// Everything here is plain inline PTX for sm_100a: mbarriers, the 1-D bulk
// tensor-memory-accelerator copy (cp.async.bulk, into this CTA only),
// programmatic dependent launch (griddepcontrol) and L2 cache policies.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/q3_sm100a.h"

namespace q3 {

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------------ errors
// A device-side error word the host reads after a step.  Kernels never trap:
// a wait that runs out of budget records its code here and returns.
enum DeviceError : uint32_t {
    DEV_OK = 0,
    DEV_TMA_WAIT_TIMEOUT = 1,
    DEV_PEER_WAIT_TIMEOUT = 2,
    DEV_BAD_TOKEN = 3,
    DEV_BAD_POSITION = 4,
    DEV_GRID_TIMEOUT = 5,
};

// Upper bound on mbarrier polls before a kernel gives up (each try_wait
// blocks for a hardware-chosen interval of up to about a microsecond): far
// beyond any real copy latency, short of a hang.
constexpr uint32_t kMaxPolls = 1u << 20;

__device__ __forceinline__ void record_error(uint32_t* err, uint32_t code) {
    if (err) atomicCAS(err, 0u, code);
}

// ------------------------------------------------------------------ bf16
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float bf2f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ bf16 f2bf(float v) { return __float2bfloat16_rn(v); }
__device__ __forceinline__ float round_bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// 8 products of a 16-byte vector pair (8 bf16 each), accumulated in fp32.
__device__ __forceinline__ float dot8(const uint4& a, const uint4& b, float acc) {
    acc = fmaf(bf_lo(a.x), bf_lo(b.x), acc);
    acc = fmaf(bf_hi(a.x), bf_hi(b.x), acc);
    acc = fmaf(bf_lo(a.y), bf_lo(b.y), acc);
    acc = fmaf(bf_hi(a.y), bf_hi(b.y), acc);
    acc = fmaf(bf_lo(a.z), bf_lo(b.z), acc);
    acc = fmaf(bf_hi(a.z), bf_hi(b.z), acc);
    acc = fmaf(bf_lo(a.w), bf_lo(b.w), acc);
    acc = fmaf(bf_hi(a.w), bf_hi(b.w), acc);
    return acc;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t sm_id() {
    uint32_t s;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(s));
    return s;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ------------------------------------------------------------------ smem / PTX
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records `code`) if
// the phase did not complete within kMaxPolls polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t code) {
    for (uint32_t i = 0; i < kMaxPolls; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    record_error(err, code);
    return false;
}

// L2 eviction-priority policies for bulk copies.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 1-D bulk copy global -> this CTA's shared memory, completion counted in
// bytes on `bar`.  Both addresses 16-byte aligned, size a multiple of 16.
// Each copy lands in the issuing CTA only.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// ------------------------------------------------------------------ clusters
// The cluster barrier in split phases (every thread of every CTA of the cluster
// takes part): arrive without memory ordering, arrive releasing this thread's
// earlier writes (shared::cluster stores included), wait acquiring the others'.
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// The generic address of `p` (this CTA's shared memory) in cluster CTA `rank`.
__device__ __forceinline__ void* map_cluster_rank(void* p, uint32_t rank) {
    uint64_t out;
    asm volatile("mapa.u64 %0, %1, %2;" : "=l"(out) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
    return reinterpret_cast<void*>(out);
}

// ------------------------------------------------------------------ PDL
// Programmatic dependent launch.  Without the launch attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Named barrier over the first `threads` threads of the CTA (id 0 is __syncthreads).
__device__ __forceinline__ void named_bar(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------------ argmax keys
// (value, index) packed so that a larger key means a larger BF16 value and,
// on equal values, a SMALLER index -- first-index-of-maximum semantics.
__device__ __forceinline__ uint64_t argmax_key(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<uint64_t>(b) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t argmax_key_index(uint64_t k) {
    return 0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull);
}

}  // namespace q3

// noalloc.cu -- q3_argmax_noalloc: the greedy argmax with no device allocation.
//
// q3_argmax keeps its reduction word in device memory it allocates on first
// use.  Some callers cannot let a library allocate: serving runtimes that plan
// every byte of device memory up front and hand libraries only buffers they
// own, and latency-critical loops that cannot absorb cudaMalloc's implicit
// device synchronisation.  This variant keeps its scratch in a fixed array
// compiled into the library instead.
//
// Scratch: kSegments keys of 8 bytes (32 KB), one per 4096-logit segment, so
// the largest input is kSegments * kSegment = 16,777,216 logits; larger inputs
// are rejected.  Every GPU that loads the library holds the array until the
// process exits.  All calls share it: each call overwrites the keys of the
// segments it uses before reading them (nothing has to start at zero), and
// calls that overlap on the GPU (different streams, no ordering between
// them) race on it.
//
// The array's host-side name is not a device address.  The first call on each
// device, with that device current, resolves the address once with
// cudaGetSymbolAddress.  The address is cached for the life of the process: the library must not be used
// across a cudaDeviceReset of that device (the reset frees the module's
// memory, and later calls would launch with the stale address).
#include <mutex>
#include <string>

#include "host_util.hpp"
#include "kernels.cuh"

namespace q3 {
namespace {

constexpr unsigned kSegment = 4096;      // logits per first-pass block
constexpr unsigned kSegments = 4096;     // keys the static scratch holds
constexpr unsigned kThreads = 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned long long g_noalloc_keys[kSegments];

// Pass 1: block b writes the (value, first index) key of its segment.
__global__ void __launch_bounds__(kThreads) argmax_segments_kernel(const bf16* __restrict__ logits, size_t n,
                                                                   unsigned long long* keys) {
    __shared__ unsigned long long best;
    if (threadIdx.x == 0) best = 0ull;
    __syncthreads();
    const size_t begin = static_cast<size_t>(blockIdx.x) * kSegment;
    const size_t end = begin + kSegment < n ? begin + kSegment : n;
    unsigned long long mine = 0ull;
    for (size_t i = begin + threadIdx.x; i < end; i += kThreads) {
        const unsigned long long k = argmax_key(bf2f(logits[i]), static_cast<uint32_t>(i));
        mine = mine > k ? mine : k;
    }
    atomicMax(&best, mine);
    __syncthreads();
    if (threadIdx.x == 0) keys[blockIdx.x] = best;
}

// Pass 2: one block reduces the segment keys and writes the index.
__global__ void __launch_bounds__(kThreads) argmax_keys_kernel(const unsigned long long* keys, unsigned nseg,
                                                               uint32_t* index) {
    __shared__ unsigned long long best;
    if (threadIdx.x == 0) best = 0ull;
    __syncthreads();
    unsigned long long mine = 0ull;
    for (unsigned i = threadIdx.x; i < nseg; i += kThreads) mine = mine > keys[i] ? mine : keys[i];
    atomicMax(&best, mine);
    __syncthreads();
    if (threadIdx.x == 0) *index = argmax_key_index(best);
}

std::mutex g_mu;
unsigned long long* g_keys_addr[kMaxDevices] = {};

// Device address of the static scratch for the current device, resolved once.
int scratch_for_current_device(unsigned long long** out) {
    int dev = 0;
    Q3_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(Q3_ERR_UNSUPPORTED, "q3_argmax_noalloc: device index too large");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_keys_addr[dev]) {
        void* p = nullptr;
        Q3_CUDA(cudaGetSymbolAddress(&p, g_noalloc_keys));
        g_keys_addr[dev] = static_cast<unsigned long long*>(p);
    }
    *out = g_keys_addr[dev];
    return Q3_OK;
}

}  // namespace
}  // namespace q3

using namespace q3;

extern "C" int q3_argmax_noalloc(const uint16_t* logits_dev, size_t n, uint32_t* index_dev, void* stream) {
    Q3_CHECK(logits_dev && index_dev, "q3_argmax_noalloc: null pointer");
    Q3_CHECK(n > 0, "q3_argmax_noalloc: empty input");
    if (n > static_cast<size_t>(kSegment) * kSegments)
        return fail(Q3_ERR_INVALID, "q3_argmax_noalloc: " + std::to_string(n) +
                                        " logits exceed the 16777216-logit maximum of its static scratch");
    unsigned long long* keys = nullptr;
    const int rc = scratch_for_current_device(&keys);
    if (rc != Q3_OK) return rc;
    const unsigned nseg = static_cast<unsigned>((n + kSegment - 1) / kSegment);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    argmax_segments_kernel<<<nseg, kThreads, 0, s>>>(reinterpret_cast<const bf16*>(logits_dev), n, keys);
    argmax_keys_kernel<<<1, kThreads, 0, s>>>(keys, nseg, index_dev);
    Q3_CUDA(cudaGetLastError());
    return Q3_OK;
}

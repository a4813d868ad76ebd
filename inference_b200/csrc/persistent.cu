// persistent.cu -- the whole decode loop as one persistent kernel.
//
// The reference runs ~14 kernels per layer plus a host sync per token
// (src/lib/model/qwen3/qwen3.hpp:131-166, src/lib/backend/cuda/backend.cu).
// Here one cooperative launch runs n decode steps with one CTA per SM.  Every
// byte the steps read -- the weights of every GEMV of every layer, then the
// KV pages of every attention -- streams through one ring of 8 KB shared
// memory slots with 1-D TMA bulk copies, in the exact order it is used.  The
// consumer warps walk the phases
//   QKV -> attention (+ split merge) -> O -> gate/up -> down   (per layer)
//   lm_head                                                    (per step)
// separated by a grid-wide barrier, and keep the ring full themselves: the
// warp (or, for KV pages, the attention group) that consumes item g issues
// item g + S into the same slot.  Weights and pages older than the current
// position do not depend on the phase before them, so the ring refills while
// the CTAs wait at a barrier; the one K/V row produced inside a step (the
// current position) is patched into the ring during the attention phase.
//
// Ring protocol: S = 2 W slots for W warps.  Item g lives in slot g % S; a
// GEMV item g is consumed by warp g % W.  A slot's round r + 1 is issued only
// after round r was consumed, so a waiter never meets a barrier two phases
// ahead (an mbarrier wait sees only the phase parity).
//
// Numerics follow the kernel-per-op path (gemv.cu, attention.cu): fp32
// accumulation, BF16 rounding where the reference rounds, fixed-order
// reductions.  Every wait is bounded (kMaxPolls for a slot, kGridPolls for the
// grid barrier); a wait that runs out records its code and raises the abort
// word, and every CTA leaves at its next barrier after its copies land.
#include <algorithm>
#include <cstring>

#include "kernels.cuh"

namespace q3 {

namespace {

constexpr int kSlot = 8192;             // ring slot: 8 KB of a weight band, or half a K or V page of a head
constexpr int kBufs = 2;                // ring slots per warp
constexpr int kMaxW = 12;               // warps per CTA
constexpr int kMaxThreads = kMaxW * 32;
constexpr int kAttWarps = 8;            // warps that run attention: 16 half-warps x 4 tokens of a page
constexpr int kPage = 64;
constexpr int kPhasesPerLayer = 5;      // QKV, attention, O, gate/up, down
constexpr uint32_t kGridPolls = 1u << 22;
constexpr float kLog2e = 1.4426950408889634f;

enum Phase : int { PH_QKV = 0, PH_ATT = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_LM = 5 };

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
    return *reinterpret_cast<const volatile uint32_t*>(p);
}
__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Generic-proxy accesses to global memory (the K/V rows written by earlier
// phases) before the async-proxy copies this thread issues next.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
// This CTA's generic-proxy reads of a ring slot before the async refill of it.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Phase timeline of the first step of a launch, kTraceWords words per (CTA,
// phase): [0] / [1] %globaltimer ns at phase start / end (comparable across
// CTAs), [2] / [3] clock64 at phase start / end (cycles per ns), then SM
// cycles of thread 0's view of the phase: GEMV [4] input ready, [5] waiting
// for items, [6] issuing refills, [7] input ready -> dot products done;
// attention [4] q/k norm, [5] page loop, [6] waiting for pages, [7] split
// merge and publish, [9] computing on pages; [8] the SM the CTA runs on.
__device__ __forceinline__ unsigned long long* trace_at(const PersistentArgs& a, int step, int phase) {
    return (a.trace && step == 0 && phase < a.trace_phases)
               ? a.trace + (static_cast<size_t>(blockIdx.x) * a.trace_phases + phase) * kTraceWords
               : nullptr;
}
__device__ __forceinline__ void trace_edge(const PersistentArgs& a, int step, int phase, int end) {
    if (unsigned long long* t = trace_at(a, step, phase)) {
        t[end] = now_ns();
        t[2 + end] = clock64();
        if (!end) {
            uint32_t sm;
            asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
            t[8] = sm;
        }
    }
}
__device__ __forceinline__ void trace_put(const PersistentArgs& a, int step, int phase, int what,
                                          unsigned long long v) {
    if (unsigned long long* t = trace_at(a, step, phase)) t[what] = v;
}

// ----------------------------------------------------------------- work split
struct Band {
    int r0, r1;
};
// (cta + 1) x units stays below 2^32: the plan checks rows x grid.
__device__ __forceinline__ Band band(int N, int row_gran, int cta, int ncta) {
    const uint32_t units = static_cast<uint32_t>(N / row_gran);
    const uint32_t u0 = static_cast<uint32_t>(cta) * units / static_cast<uint32_t>(ncta);
    const uint32_t u1 = static_cast<uint32_t>(cta + 1) * units / static_cast<uint32_t>(ncta);
    return {static_cast<int>(u0) * row_gran, static_cast<int>(u1) * row_gran};
}
// A CTA's band of rows [r0, r1) of a row-major [N, K] matrix is one contiguous
// byte range; it streams as 8 KB items (the last one may be shorter).
__device__ __forceinline__ uint32_t band_items(const Band& b, int K) {
    return static_cast<uint32_t>((static_cast<size_t>(b.r1 - b.r0) * K * 2 + kSlot - 1) / kSlot);
}
// Partial sums per row: one per item the row touches (summed in item order).
__host__ __device__ __forceinline__ int pieces_per_row(int K) { return (K * 2 + kSlot - 1) / kSlot + 1; }

// Attention unit of a CTA: (kv head, block of HG query heads, split of the
// pages).  The first four fields are fixed for the launch (kept in shared
// memory); the page range [pb, pe) follows the position.
struct AttUnit {
    int valid, kvh, qb, split, pb, pe;
};
__device__ __forceinline__ AttUnit att_static(const PersistentArgs& a, int cta) {
    AttUnit u{};
    if (cta >= a.kvh * a.nqb * a.splits) return u;
    u.valid = 1;
    u.split = cta % a.splits;
    const int kq = cta / a.splits;
    u.kvh = kq / a.nqb;
    u.qb = kq % a.nqb;
    return u;
}
__device__ __forceinline__ AttUnit att_unit(const PersistentArgs& a, const AttUnit& st, int pos) {
    AttUnit u = st;
    const uint32_t n_pages = static_cast<uint32_t>(pos) / kPage + 1;
    u.pb = static_cast<int>(static_cast<uint32_t>(u.split) * n_pages / static_cast<uint32_t>(a.splits));
    u.pe = static_cast<int>(static_cast<uint32_t>(u.split + 1) * n_pages / static_cast<uint32_t>(a.splits));
    return u;
}

// Layer pointers, in PersistentLayer order (kLayerPtrs per layer).
enum Field : int { F_QKV = 0, F_O, F_GU, F_DOWN, F_IN_NORM, F_POST_NORM, F_Q_NORM, F_K_NORM, F_K_PAGES, F_V_PAGES };

// ----------------------------------------------------------------- the item sequence
// This CTA's band of one GEMV kind: byte offset into the matrix, bytes, items.
struct Geom {
    unsigned long long off;
    uint32_t bytes, items;
};

// Phase p of a launch = step * (5 L + 1) + phase of the step; items(p) = this
// CTA's items in it.  The GEMV bands are the same in every layer and step
// (geo[], filled once); only the attention unit's pages move with the position.
struct Seq {
    const PersistentArgs* a;
    const Geom* geo;      // [PH_LM + 1] in shared memory (PH_ATT unused)
    const uint32_t* lt;   // [layers][kLayerPtrs] layer pointer offsets, shared memory
    const int32_t* pt;    // page table, shared memory
    const AttUnit* ast;   // this CTA's attention unit (fixed part), shared memory
    int pos0;
    uint32_t per_step;
    int total;  // phases in the launch

    template <class T = bf16>
    __device__ __forceinline__ T* ptr(int layer, int field) const {
        return reinterpret_cast<T*>(a->layer_base +
                                    (static_cast<unsigned long long>(lt[layer * kLayerPtrs + field]) << 8));
    }
    __device__ __forceinline__ void locate(int p, int* step, int* layer, int* kind) const {
        const uint32_t st = static_cast<uint32_t>(p) / per_step;
        const uint32_t lp = static_cast<uint32_t>(p) - st * per_step;
        *step = static_cast<int>(st);
        if (lp == per_step - 1) {
            *layer = a->layers;
            *kind = PH_LM;
        } else {
            *layer = static_cast<int>(lp / kPhasesPerLayer);
            *kind = static_cast<int>(lp - *layer * kPhasesPerLayer);
        }
    }
    __device__ __forceinline__ const bf16* weight(int layer, int kind) const {
        if (kind == PH_LM) return a->lm_head;
        return ptr(layer, kind == PH_QKV ? F_QKV : kind == PH_O ? F_O : kind == PH_GU ? F_GU : F_DOWN);
    }
    __device__ __forceinline__ uint32_t items(int p) const {
        int step, layer, kind;
        locate(p, &step, &layer, &kind);
        if (kind == PH_ATT) {
            const AttUnit u = att_unit(*a, *ast, pos0 + step);
            return u.valid ? 4u * static_cast<uint32_t>(u.pe - u.pb) : 0u;
        }
        return geo[kind].items;
    }
    // Source and size of item k of phase p; true for a KV page item.  A page
    // is four items: the low and high 32 tokens of its K block, then of its V block.
    __device__ __forceinline__ bool desc(int p, uint32_t k, const void** src, uint32_t* bytes) const {
        int step, layer, kind;
        locate(p, &step, &layer, &kind);
        if (kind == PH_ATT) {
            const AttUnit u = att_unit(*a, *ast, pos0 + step);
            const int page = u.pb + static_cast<int>(k >> 2);
            const int q = static_cast<int>(k & 3);
            const size_t base = (static_cast<size_t>(pt[page]) * a->kvh + u.kvh) * kPage * 128 +
                                static_cast<size_t>(q & 1) * (kPage / 2) * 128;
            *src = ptr(layer, q < 2 ? F_K_PAGES : F_V_PAGES) + base;
            *bytes = kSlot;
            return true;
        }
        const Geom& g = geo[kind];
        const uint32_t off = k * kSlot;
        *src = reinterpret_cast<const uint8_t*>(weight(layer, kind)) + g.off + off;
        *bytes = min(static_cast<uint32_t>(kSlot), g.bytes - off);
        return false;
    }
    // (p, k) moved n items on; false if that runs past the launch.
    __device__ __forceinline__ bool advance(int* p, uint32_t* k, uint32_t n) const {
        *k += n;
        while (*p < total) {
            const uint32_t m = items(*p);
            if (*k < m) return true;
            *k -= m;
            ++*p;
        }
        return false;
    }
};

struct Smem {
    uint8_t* ring;
    uint64_t* full;
    uint32_t* issued;  // copies issued into each slot (for the final drain)
    bf16* x;           // GEMV input vector
    float* part;       // per-(row, item) partial sums
    uint8_t* att;      // attention scratch
    float* red;        // 32 floats
    uint32_t* flags;   // [0] barrier outcome, [1] last split
    unsigned long long* key;
    Geom* geo;         // [PH_LM + 1]
    AttUnit* ast;      // this CTA's attention unit (fixed part)
    uint32_t* lt;      // layer pointer offsets
    int32_t* pt;       // page table
};

struct Ctx {
    const PersistentArgs* a;
    Seq seq;
    Smem s;
    int tid, warp, lane, nw, nt;
    uint32_t S;                // ring slots
    uint32_t gi;               // global index of the current phase's first item
    unsigned long long nsync;  // grid barriers passed (thread 0)
    int tstep, tph;            // step and phase of the step (timeline)
    unsigned long long tc0;    // clock64 at the phase start (thread 0, timeline)
};

// thread 0: cycles since the phase began (for the inner trace words)
__device__ __forceinline__ unsigned long long tcyc(const Ctx& c) { return clock64() - c.tc0; }

__device__ __forceinline__ void cbar(int id, int n) { named_bar(id, n); }

// Copy `bytes` from src into `slot` (whose previous item this CTA consumed).
__device__ __forceinline__ void issue_copy(Ctx& c, uint32_t slot, const void* src, uint32_t bytes, bool kv) {
    fence_proxy_async_smem();
    if (kv) fence_proxy_async_global();
    atomicAdd(&c.s.issued[slot], 1u);
    mbar_arrive_expect_tx(&c.s.full[slot], bytes);
    bulk_g2s(c.s.ring + static_cast<size_t>(slot) * kSlot, src, bytes, &c.s.full[slot], policy_evict_first());
}
// Issue item k of phase p into `slot`.
__device__ __forceinline__ void issue(Ctx& c, int p, uint32_t k, uint32_t slot) {
    const void* src;
    uint32_t bytes;
    const bool kv = c.seq.desc(p, k, &src, &bytes);
    issue_copy(c, slot, src, bytes, kv);
}

// The item S after (p, k), if the launch has one, goes into `slot`.
__device__ __forceinline__ void refill(Ctx& c, int p, uint32_t k, uint32_t slot) {
    if (c.seq.advance(&p, &k, c.S)) issue(c, p, k, slot);
}

// Bounded wait for a ring slot.  It also stops (false) once another wait of
// the launch has failed; that word is read only every 64 polls.
__device__ __forceinline__ bool slot_wait(const PersistentArgs& a, uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kMaxPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 63 && ld_volatile(a.abort)) return false;
    }
    record_error(a.err, DEV_TMA_WAIT_TIMEOUT);
    atomicExch(a.abort, 1u);
    return false;
}

// Grid barrier: a monotonic arrival count (zeroed before each launch); the
// n-th barrier completes when it reaches n x grid.  False: the kernel stops.
__device__ bool grid_sync(Ctx& c) {
    const PersistentArgs& a = *c.a;
    cbar(1, c.nt);
    if (c.tid == 0) {
        uint32_t ok = 1;
        const unsigned long long target = (++c.nsync) * gridDim.x;
        red_release_add(a.gsync, 1ull);
        uint32_t polls = 0;
        while (ld_acquire_u64(a.gsync) < target) {
            if ((++polls & 255) == 0 && ld_volatile(a.abort)) {
                ok = 0;
                break;
            }
            if (polls > kGridPolls) {
                record_error(a.err, DEV_GRID_TIMEOUT);
                atomicExch(a.abort, 1u);
                ok = 0;
                break;
            }
        }
        __threadfence();
        c.s.flags[0] = ok;
    }
    cbar(1, c.nt);
    return c.s.flags[0] != 0;
}

__device__ __forceinline__ float csum(Ctx& c, float v) {
    v = warp_sum(v);
    if (c.lane == 0) c.s.red[c.warp] = v;
    cbar(1, c.nt);
    float t = 0.f;
    for (int w = 0; w < c.nw; ++w) t += c.s.red[w];
    cbar(1, c.nt);
    return t;
}

__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
    return static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(lo))) |
           (static_cast<uint32_t>(__bfloat16_as_ushort(f2bf(hi))) << 16);
}

// x = rmsnorm(src) into shared memory (rmsnorm.cuh:12-46).  With vsum the sum
// of squares runs over the unrounded fp32 sums (rmsnorm_add, rmsnorm.cuh:58-60).
// CTA 0 copies src to hs_out when given.  Source, fp32 sums and weights are
// loaded together (one memory round trip); the weights wait in x[K, 2K).
__device__ void prologue_norm(Ctx& c, const bf16* src, const float* vsum, const bf16* w, int K, bf16* hs_out) {
    const PersistentArgs& a = *c.a;
    const int k8 = K / 8;
    uint4* xs = reinterpret_cast<uint4*>(c.s.x);
    float ss = 0.f;
#pragma unroll 2
    for (int i = c.tid; i < k8; i += c.nt) {
        const uint4 h = __ldcg(reinterpret_cast<const uint4*>(src) + i);
        const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w) + i);
        if (vsum) {
            const float4 v0 = __ldcg(reinterpret_cast<const float4*>(vsum) + 2 * i);
            const float4 v1 = __ldcg(reinterpret_cast<const float4*>(vsum) + 2 * i + 1);
            ss += v0.x * v0.x + v0.y * v0.y + v0.z * v0.z + v0.w * v0.w;
            ss += v1.x * v1.x + v1.y * v1.y + v1.z * v1.z + v1.w * v1.w;
        } else {
            const uint32_t* hw = reinterpret_cast<const uint32_t*>(&h);
#pragma unroll
            for (int e = 0; e < 4; ++e) ss += bf_lo(hw[e]) * bf_lo(hw[e]) + bf_hi(hw[e]) * bf_hi(hw[e]);
        }
        if (hs_out && blockIdx.x == 0) reinterpret_cast<uint4*>(hs_out)[i] = h;
        xs[i] = h;
        xs[k8 + i] = wv;
    }
    ss = csum(c, ss);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(K) + a.eps);
    for (int i = c.tid; i < k8; i += c.nt) {
        const uint4 h = xs[i], wv = xs[k8 + i];
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
        const uint32_t* hw = reinterpret_cast<const uint32_t*>(&h);
        const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
#pragma unroll
        for (int e = 0; e < 4; ++e)
            ow[e] = pack_bf2(bf_lo(hw[e]) * scale * bf_lo(ww[e]), bf_hi(hw[e]) * scale * bf_hi(ww[e]));
        xs[i] = o;
    }
    cbar(1, c.nt);
}

__device__ void prologue_copy(Ctx& c, const bf16* src, int K) {
    for (int i = c.tid; i < K / 8; i += c.nt)
        reinterpret_cast<uint4*>(c.s.x)[i] = __ldcg(reinterpret_cast<const uint4*>(src) + i);
    cbar(1, c.nt);
}

// Dot every item of this CTA's band with x.  Item k covers band bytes
// [k * 8 KB, ...), i.e. one or more row segments; since K is a multiple of
// 256 every segment is a whole number of 512-byte warp groups.  The partial
// of (row, item) goes to part[row * P + (k - first item of the row)].
__device__ Band gemv_consume(Ctx& c, int p, int N, int K, int row_gran) {
    const PersistentArgs& a = *c.a;
    const Band b = band(N, row_gran, blockIdx.x, gridDim.x);
    const uint32_t n_items = band_items(b, K);
    const int P = pieces_per_row(K);
    const int nrows = b.r1 - b.r0;
    for (int i = c.tid; i < nrows * P; i += c.nt) c.s.part[i] = 0.f;
    cbar(1, c.nt);
    const bool tw = a.trace && c.tid == 0;
    const unsigned long long t_ready = tw ? tcyc(c) : 0ull;
    const uint32_t vpr = static_cast<uint32_t>(K) / 8;  // 16-byte vectors per row
    const uint32_t vtot = static_cast<uint32_t>(nrows) * vpr;
    const uint32_t nw = static_cast<uint32_t>(c.nw);
    const uint32_t k0 = (static_cast<uint32_t>(c.warp) + nw - c.gi % nw) % nw;
    const uint4* xv = reinterpret_cast<const uint4*>(c.s.x);
    // refills that stay inside this phase need no sequence walk
    int step_, layer_, kind_;
    c.seq.locate(p, &step_, &layer_, &kind_);
    const Geom geo = c.s.geo[kind_];
    const uint8_t* wsrc = reinterpret_cast<const uint8_t*>(c.seq.weight(layer_, kind_)) + geo.off;
    unsigned long long t_wait = 0, t_refill = 0;
    for (uint32_t k = k0; k < n_items; k += nw) {
        const uint32_t g = c.gi + k;
        const uint32_t slot = g % c.S;
        const unsigned long long w0 = tw ? clock64() : 0ull;
        const bool ok = slot_wait(a, &c.s.full[slot], (g / c.S) & 1);
        if (tw) t_wait += clock64() - w0;
        const uint32_t v0 = k * (kSlot / 16);
        const uint32_t v1 = min(vtot, v0 + kSlot / 16);
        const uint4* wv = reinterpret_cast<const uint4*>(c.s.ring + static_cast<size_t>(slot) * kSlot) - v0;
        uint32_t row = v0 / vpr;
        for (uint32_t sg = v0; sg < v1; ++row) {
            const uint32_t e = min(v1, (row + 1) * vpr);
            const uint4* w = wv + sg;
            const uint4* x = xv + (sg - row * vpr);
            const int n = static_cast<int>(e - sg);
            float acc0 = 0.f, acc1 = 0.f;
            if (ok) {
                int v = c.lane;
                for (; v + 32 < n; v += 64) {
                    acc0 = dot8(w[v], x[v], acc0);
                    acc1 = dot8(w[v + 32], x[v + 32], acc1);
                }
                if (v < n) acc0 = dot8(w[v], x[v], acc0);
            }
            const float sum = warp_sum(acc0 + acc1);
            if (c.lane == 0) c.s.part[row * P + (k - (row * vpr * 16) / kSlot)] = sum;
            sg = e;
        }
        __syncwarp();
        if (c.lane == 0 && ok) {
            const unsigned long long r0 = tw ? clock64() : 0ull;
            const uint32_t kn = k + c.S;
            if (kn < n_items)
                issue_copy(c, slot, wsrc + static_cast<size_t>(kn) * kSlot, min(static_cast<uint32_t>(kSlot), geo.bytes - kn * kSlot), false);
            else
                refill(c, p, k, slot);
            if (tw) t_refill += clock64() - r0;
        }
    }
    if (tw) {
        trace_put(a, c.tstep, c.tph, 4, t_ready);
        trace_put(a, c.tstep, c.tph, 5, t_wait);
        trace_put(a, c.tstep, c.tph, 6, t_refill);
    }
    c.gi += n_items;
    cbar(1, c.nt);
    if (tw) trace_put(a, c.tstep, c.tph, 7, tcyc(c) - t_ready);
    return b;
}

__device__ __forceinline__ float row_sum(Ctx& c, int rl, int P) {
    float r = 0.f;
    for (int q = 0; q < P; ++q) r += c.s.part[rl * P + q];
    return r;
}

__device__ __forceinline__ size_t kv_slot(const Ctx& c, int pos, int head) {
    const int page = c.s.pt[pos / kPage];
    return ((static_cast<size_t>(page) * c.a->kvh + head) * kPage + (pos % kPage)) * 128;
}

// ----------------------------------------------------------------- phases
// q = x Wq, k = x Wk, v = x Wv of this position (qwen3.hpp:139-144): q and the
// raw k rows to the q buffer (q[qd + ...]), v straight to its cache slot.  q/k
// norm and RoPE run in the attention phase.
__device__ void phase_qkv(Ctx& c, int p, int l, int pos) {
    const PersistentArgs& a = *c.a;
    if (l == 0) {
        // embedding (embedding.cuh:9-30) of the token at this position
        int token = __ldcg(a.tokens + pos);
        if (token < 0 || token >= a.vocab) {
            if (c.tid == 0) record_error(a.err, DEV_BAD_TOKEN);
            token = 0;
        }
        prologue_norm(c, a.embed + static_cast<size_t>(token) * a.H, nullptr, c.seq.ptr(l, F_IN_NORM), a.H, a.hs);
    } else {
        prologue_norm(c, a.hs, nullptr, c.seq.ptr(l, F_IN_NORM), a.H, nullptr);
    }
    const Band b = gemv_consume(c, p, a.qd + 2 * a.kd, a.H, 1);
    const int P = pieces_per_row(a.H);
    for (int rl = c.tid; rl < b.r1 - b.r0; rl += c.nt) {
        const int gr = b.r0 + rl;
        const bf16 v = f2bf(row_sum(c, rl, P));
        if (gr < a.qd + a.kd) {
            a.q[gr] = v;
        } else {
            const int k = gr - a.qd - a.kd;
            c.seq.ptr(l, F_V_PAGES)[kv_slot(c, pos, k >> 7) + (k & 127)] = v;
        }
    }
}

// q_norm / k_norm + RoPE of one 128-wide head by one warp (qk_norm_rope.cuh:14-90):
// lane holds elements lane + 32 j; output rounded to BF16 once, after the rotation.
__device__ __forceinline__ void head_norm_rope(const PersistentArgs& a, const bf16* src, const bf16* nw, int pos,
                                               int lane, bf16* dst, bf16* dst2) {
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
        v[j] = __uint_as_float(
            static_cast<uint32_t>(__ldcg(reinterpret_cast<const unsigned short*>(src) + lane + 32 * j)) << 16);
    float cs[2], sn[2], w0[2], w1[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int i = lane + 32 * j;
        cs[j] = __ldg(a.rope_cos + static_cast<size_t>(pos) * 64 + i);
        sn[j] = __ldg(a.rope_sin + static_cast<size_t>(pos) * 64 + i);
        w0[j] = bf2f(nw[i]);
        w1[j] = bf2f(nw[i + 64]);
    }
    const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
    const float scale = 1.0f / sqrtf(ss / 128.0f + a.eps);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int i = lane + 32 * j;
        const float x = v[j] * w0[j] * scale;
        const float y = v[j + 2] * w1[j] * scale;
        const bf16 o0 = f2bf(x * cs[j] - y * sn[j]);
        const bf16 o1 = f2bf(y * cs[j] + x * sn[j]);
        dst[i] = o0;
        dst[i + 64] = o1;
        if (dst2) {
            dst2[i] = o0;
            dst2[i + 64] = o1;
        }
    }
}

// Split-KV flash decode for this CTA's (kv head, query block, split) unit,
// then the merge of the splits by the CTA that finishes its group last.
template <int HG>
__device__ void phase_attention(Ctx& c, int p, int layer, int pos) {
    const PersistentArgs& a = *c.a;
    const AttUnit u = att_unit(a, *c.s.ast, pos);
    const int np = u.valid ? u.pe - u.pb : 0;
    const int live_page = pos / kPage;
    const bool live_unit = u.valid && u.pe - 1 == live_page;
    // scratch: qn[HG][128] bf16 | krow[128] bf16 | vrow[128] bf16 | S[8][HG][kAttRecord] f32
    bf16* qn = reinterpret_cast<bf16*>(c.s.att);
    bf16* krow = qn + HG * 128;
    bf16* vrow = krow + 128;
    float* S = reinterpret_cast<float*>(vrow + 128);
    const int G = a.qh / a.kvh;
    const int qh0 = u.kvh * G + u.qb * HG;
    if (u.valid) {
        if (c.warp < HG) {
            head_norm_rope(a, a.q + static_cast<size_t>(qh0 + c.warp) * 128, c.seq.ptr(layer, F_Q_NORM), pos, c.lane,
                           qn + c.warp * 128, nullptr);
        } else if (c.warp == HG && live_unit) {
            // this step's key, normalised and rotated; query block 0 stores it in the cache
            head_norm_rope(a, a.q + a.qd + u.kvh * 128, c.seq.ptr(layer, F_K_NORM), pos, c.lane, krow,
                           u.qb == 0 ? c.seq.ptr(layer, F_K_PAGES) + kv_slot(c, pos, u.kvh) : nullptr);
        } else if (c.warp == HG + 1 && live_unit && c.lane < 16) {
            reinterpret_cast<uint4*>(vrow)[c.lane] =
                __ldcg(reinterpret_cast<const uint4*>(c.seq.ptr(layer, F_V_PAGES) + kv_slot(c, pos, u.kvh)) + c.lane);
        }
    }
    cbar(1, c.nt);
    const bool att_warp = c.warp < kAttWarps;
    const int hw = c.tid >> 4, hl = c.tid & 15;  // half-warp 0..15 of the attention warps
    float q[HG][8], m[HG], l[HG], acc[HG][8];
    if (att_warp && u.valid) {
#pragma unroll
        for (int g = 0; g < HG; ++g) {
            const uint4 v = reinterpret_cast<const uint4*>(qn + g * 128)[hl];
            const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                q[g][2 * j] = bf_lo(w[j]);
                q[g][2 * j + 1] = bf_hi(w[j]);
            }
            m[g] = -INFINITY;
            l[g] = 0.f;
#pragma unroll
            for (int d = 0; d < 8; ++d) acc[g][d] = 0.f;
        }
    }
    const float qscale = (1.0f / sqrtf(128.0f)) * kLog2e;
    unsigned long long t_wait = 0;
    const unsigned long long t_pages = c.tid == 0 ? tcyc(c) : 0ull;
    unsigned long long t_bar = 0;
    for (int i = 0; i < np && att_warp; ++i) {
        const uint32_t g0 = c.gi + 4 * i;
        bool ok = true;
        const unsigned long long w0 = c.tid == 0 && a.trace ? clock64() : 0ull;
        for (int qq = 0; qq < 4; ++qq) ok = slot_wait(a, &c.s.full[(g0 + qq) % c.S], ((g0 + qq) / c.S) & 1) && ok;
        if (c.tid == 0 && a.trace) t_wait += clock64() - w0;
        const int page = u.pb + i;
        if (page == live_page && c.warp == 0) {
            // the current position's row was written after this page's copy was issued
            const int j = pos % kPage;
            const int which = c.lane >> 4;  // 0: K, 1: V
            const uint32_t slot = (g0 + which * 2 + (j >> 5)) % c.S;
            uint4* dst = reinterpret_cast<uint4*>(c.s.ring + static_cast<size_t>(slot) * kSlot + (j & 31) * 256);
            dst[c.lane & 15] = reinterpret_cast<const uint4*>(which ? vrow : krow)[c.lane & 15];
        }
        cbar(2, kAttWarps * 32);
        const unsigned long long b0 = c.tid == 0 && a.trace ? clock64() : 0ull;
        const int valid = min(kPage, pos + 1 - page * kPage);
        const int j0 = hw * 4;  // 4 consecutive tokens, all in half j0 / 32 of the page
        const uint32_t kslot = (g0 + (j0 >> 5)) % c.S, vslot = (g0 + 2 + (j0 >> 5)) % c.S;
        const uint4* kt = reinterpret_cast<const uint4*>(c.s.ring + static_cast<size_t>(kslot) * kSlot);
        const uint4* vt = reinterpret_cast<const uint4*>(c.s.ring + static_cast<size_t>(vslot) * kSlot);
        float sc[4][HG];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int j = j0 + t;
            const uint4 kv = kt[(j & 31) * 16 + hl];
            const uint32_t* w = reinterpret_cast<const uint32_t*>(&kv);
#pragma unroll
            for (int g = 0; g < HG; ++g) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    d = fmaf(q[g][2 * e], bf_lo(w[e]), d);
                    d = fmaf(q[g][2 * e + 1], bf_hi(w[e]), d);
                }
                d += __shfl_xor_sync(0xffffffffu, d, 8);
                d += __shfl_xor_sync(0xffffffffu, d, 4);
                d += __shfl_xor_sync(0xffffffffu, d, 2);
                d += __shfl_xor_sync(0xffffffffu, d, 1);
                sc[t][g] = (ok && j < valid) ? d * qscale : -INFINITY;
            }
        }
#pragma unroll
        for (int g = 0; g < HG; ++g) {
            const float mx = fmaxf(fmaxf(sc[0][g], sc[1][g]), fmaxf(sc[2][g], sc[3][g]));
            const float mn = fmaxf(m[g], mx);
            if (mn == -INFINITY) continue;
            const float corr = exp2f(m[g] - mn);
            m[g] = mn;
            l[g] *= corr;
#pragma unroll
            for (int d = 0; d < 8; ++d) acc[g][d] *= corr;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float pr = exp2f(sc[t][g] - mn);
                sc[t][g] = pr;
                l[g] += pr;
            }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int j = j0 + t;
            if (!ok || j >= valid) continue;
            const uint4 vv = vt[(j & 31) * 16 + hl];
            const uint32_t* w = reinterpret_cast<const uint32_t*>(&vv);
            float vf[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                vf[2 * e] = bf_lo(w[e]);
                vf[2 * e + 1] = bf_hi(w[e]);
            }
#pragma unroll
            for (int g = 0; g < HG; ++g) {
                const float pr = (m[g] == -INFINITY) ? 0.f : sc[t][g];
#pragma unroll
                for (int d = 0; d < 8; ++d) acc[g][d] = fmaf(pr, vf[d], acc[g][d]);
            }
        }
        if (c.tid == 0 && a.trace) t_bar += clock64() - b0;
        // every attention warp is done with the page: warps 0-3 refill its four slots
        cbar(2, kAttWarps * 32);
        if (c.lane == 0 && c.warp < 4 && ok) refill(c, p, static_cast<uint32_t>(4 * i + c.warp), (g0 + c.warp) % c.S);
    }
    c.gi += 4 * np;
    const unsigned long long t_done = c.tid == 0 ? tcyc(c) : 0ull;
    if (c.tid == 0) {
        trace_put(a, c.tstep, c.tph, 4, t_pages);
        trace_put(a, c.tstep, c.tph, 5, t_done - t_pages);
        trace_put(a, c.tstep, c.tph, 6, t_wait);
        trace_put(a, c.tstep, c.tph, 9, t_bar);
    }
    if (!u.valid) return;
    // ---- this split's state: half-warp pairs by shuffle, then the 8 warps in shared memory
    if (att_warp) {
#pragma unroll
        for (int g = 0; g < HG; ++g) {
            const float mo = __shfl_xor_sync(0xffffffffu, m[g], 16);
            const float lo = __shfl_xor_sync(0xffffffffu, l[g], 16);
            const float M = fmaxf(m[g], mo);
            const float f0 = (M == -INFINITY) ? 0.f : exp2f(m[g] - M);
            const float f1 = (M == -INFINITY) ? 0.f : exp2f(mo - M);
            float* Sw = S + (c.warp * HG + g) * kAttRecord;
#pragma unroll
            for (int d = 0; d < 8; ++d) {
                const float ao = __shfl_xor_sync(0xffffffffu, acc[g][d], 16);
                if (c.lane < 16) Sw[4 + 8 * hl + d] = acc[g][d] * f0 + ao * f1;
            }
            if (c.lane == 0) {
                Sw[0] = M;
                Sw[1] = l[g] * f0 + lo * f1;
            }
        }
    }
    cbar(1, c.nt);
    const int kq = u.kvh * a.nqb + u.qb;
    float* grp = a.att_part + static_cast<size_t>(kq) * a.splits * HG * kAttRecord;
    float* dst = grp + static_cast<size_t>(u.split) * HG * kAttRecord;
    for (int o = c.tid; o < HG * 128; o += c.nt) {
        const int g = o >> 7, d = o & 127;
        float M = -INFINITY;
        for (int w = 0; w < kAttWarps; ++w) M = fmaxf(M, S[(w * HG + g) * kAttRecord]);
        float Ls = 0.f, A = 0.f;
        if (M != -INFINITY)
            for (int w = 0; w < kAttWarps; ++w) {
                const float* Sw = S + (w * HG + g) * kAttRecord;
                const float f = exp2f(Sw[0] - M);
                Ls += Sw[1] * f;
                A += Sw[4 + d] * f;
            }
        dst[g * kAttRecord + 4 + d] = A;
        if (d == 0) {
            dst[g * kAttRecord] = M;
            dst[g * kAttRecord + 1] = Ls;
        }
    }
    // publish: the CTA barrier orders every thread's stores before thread 0's
    // release; the last split's acquire makes all partials visible to its CTA
    cbar(1, c.nt);
    if (c.tid == 0) {
        const uint32_t old = atom_add_acq_rel(&a.att_counters[kq], 1u);
        c.s.flags[1] = (old == static_cast<uint32_t>(a.splits - 1)) ? 1u : 0u;
    }
    cbar(1, c.nt);
    if (c.tid == 0) trace_put(a, c.tstep, c.tph, 7, tcyc(c) - t_done);
    if (!c.s.flags[1]) return;
    // ---- last split of the group: merge all splits (rows of att_part) in parallel
    // One round trip: every (m, l) to shared memory, and each thread's share
    // of the accumulators (column cl = (head, 4 dims); R threads stripe the
    // splits) with their m into registers, loaded together.
    const int SG = a.splits * HG;
    float* msh = S;          // [splits][HG] m
    float* lsh = msh + SG;   // [splits][HG] l
    float* Mg = lsh + SG;    // [HG]
    float* Lg = Mg + 4;      // [HG]
    float4* red = reinterpret_cast<float4*>(S + ((2 * SG + 8 + 3) & ~3));  // [threads]
    constexpr int C = HG * 32;
    constexpr int kRegSplits = 6;
    const int R = c.nt / C;
    const bool comb = c.tid < R * C;
    const int cl = c.tid % C, r = c.tid / C;
    const int g = cl >> 5, d4 = cl & 31;
    float4 va[kRegSplits];
    float ma[kRegSplits];
#pragma unroll
    for (int j = 0; j < kRegSplits; ++j) {
        const int sp = r + j * R;
        ma[j] = -INFINITY;
        if (comb && sp < a.splits) {
            const float* e = grp + static_cast<size_t>(sp * HG + g) * kAttRecord;
            ma[j] = __ldcg(e);
            va[j] = __ldcg(reinterpret_cast<const float4*>(e + 4) + d4);
        }
    }
    for (int i = c.tid; i < SG; i += c.nt) {
        msh[i] = __ldcg(grp + static_cast<size_t>(i) * kAttRecord);
        lsh[i] = __ldcg(grp + static_cast<size_t>(i) * kAttRecord + 1);
    }
    cbar(1, c.nt);
    if (c.tid < HG) {
        float M = -INFINITY;
        for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, msh[sp * HG + c.tid]);
        float Ls = 0.f;
        for (int sp = 0; sp < a.splits; ++sp) {
            const float ms = msh[sp * HG + c.tid];
            if (ms != -INFINITY) Ls += lsh[sp * HG + c.tid] * exp2f(ms - M);
        }
        Mg[c.tid] = M;
        Lg[c.tid] = Ls;
    }
    cbar(1, c.nt);
    if (comb) {
        const float M = Mg[g];
        float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < kRegSplits; ++j) {
            if (ma[j] == -INFINITY) continue;
            const float f = exp2f(ma[j] - M);
            s4.x = fmaf(va[j].x, f, s4.x);
            s4.y = fmaf(va[j].y, f, s4.y);
            s4.z = fmaf(va[j].z, f, s4.z);
            s4.w = fmaf(va[j].w, f, s4.w);
        }
        // more splits than registers hold: the rest in a second pass
        for (int sp = r + kRegSplits * R; sp < a.splits; sp += R) {
            const float* e = grp + static_cast<size_t>(sp * HG + g) * kAttRecord;
            const float ms = __ldcg(e);
            if (ms == -INFINITY) continue;
            const float f = exp2f(ms - M);
            const float4 v = __ldcg(reinterpret_cast<const float4*>(e + 4) + d4);
            s4.x = fmaf(v.x, f, s4.x);
            s4.y = fmaf(v.y, f, s4.y);
            s4.z = fmaf(v.z, f, s4.z);
            s4.w = fmaf(v.w, f, s4.w);
        }
        red[c.tid] = s4;
    }
    cbar(1, c.nt);
    if (c.tid < C) {
        float4 s4 = red[c.tid];
        for (int rr = 1; rr < R; ++rr) {
            const float4 v = red[rr * C + c.tid];
            s4.x += v.x;
            s4.y += v.y;
            s4.z += v.z;
            s4.w += v.w;
        }
        const float L = Lg[g];
        uint2 o;
        o.x = pack_bf2(s4.x / L, s4.y / L);
        o.y = pack_bf2(s4.z / L, s4.w / L);
        reinterpret_cast<uint2*>(a.attn + static_cast<size_t>(qh0 + g) * 128)[d4] = o;
    }
    if (c.tid == 0) a.att_counters[kq] = 0u;
}

__device__ void phase_o(Ctx& c, int p) {
    const PersistentArgs& a = *c.a;
    const Band b0 = band(a.H, 1, blockIdx.x, gridDim.x);
    const float res = (c.tid < b0.r1 - b0.r0) ? bf2f(__ldcg(a.hs + b0.r0 + c.tid)) : 0.f;
    prologue_copy(c, a.attn, a.qd);
    const Band b = gemv_consume(c, p, a.H, a.qd, 1);
    const int P = pieces_per_row(a.qd);
    for (int rl = c.tid; rl < b.r1 - b.r0; rl += c.nt) {
        const int gr = b.r0 + rl;
        // qwen3.hpp:151-152 -> rmsnorm.cuh:58-60: keep the fp32 sum for the next norm
        const float v = (rl == c.tid ? res : bf2f(__ldcg(a.hs + gr))) + round_bf(row_sum(c, rl, P));
        a.hs[gr] = f2bf(v);
        a.vsum[gr] = v;
    }
}

__device__ void phase_gu(Ctx& c, int p, int l) {
    const PersistentArgs& a = *c.a;
    prologue_norm(c, a.hs, a.vsum, c.seq.ptr(l, F_POST_NORM), a.H, nullptr);
    const Band b = gemv_consume(c, p, 2 * a.il, a.H, 2);
    const int P = pieces_per_row(a.H);
    for (int m = c.tid; m < (b.r1 - b.r0) / 2; m += c.nt) {
        // qwen3.hpp:154-156 -> silu.cuh:18-20 on the BF16-rounded matmul outputs
        const float gv = round_bf(row_sum(c, 2 * m, P)), uv = round_bf(row_sum(c, 2 * m + 1, P));
        a.g[(b.r0 >> 1) + m] = f2bf(gv / (1.0f + expf(-gv)) * uv);
    }
}

__device__ void phase_down(Ctx& c, int p) {
    const PersistentArgs& a = *c.a;
    const Band b0 = band(a.H, 1, blockIdx.x, gridDim.x);
    const float res = (c.tid < b0.r1 - b0.r0) ? bf2f(__ldcg(a.hs + b0.r0 + c.tid)) : 0.f;
    prologue_copy(c, a.g, a.il);
    const Band b = gemv_consume(c, p, a.H, a.il, 1);
    const int P = pieces_per_row(a.il);
    for (int rl = c.tid; rl < b.r1 - b.r0; rl += c.nt) {
        const int gr = b.r0 + rl;
        // qwen3.hpp:158-159
        a.hs[gr] = f2bf((rl == c.tid ? res : bf2f(__ldcg(a.hs + gr))) + round_bf(row_sum(c, rl, P)));
    }
}

__device__ void phase_lm(Ctx& c, int p, int pos, int nf) {
    const PersistentArgs& a = *c.a;
    prologue_norm(c, a.hs, nullptr, a.final_norm, a.H, nullptr);
    if (c.tid == 0) *c.s.key = 0ull;
    const Band b = gemv_consume(c, p, a.vl, a.H, 1);
    const int P = pieces_per_row(a.H);
    unsigned long long best = 0ull;
    for (int rl = c.tid; rl < b.r1 - b.r0; rl += c.nt) {
        const int gr = b.r0 + rl;
        const bf16 v = f2bf(row_sum(c, rl, P));
        a.logits[gr] = v;
        const unsigned long long k = argmax_key(bf2f(v), static_cast<uint32_t>(gr) + a.voff);
        best = best > k ? best : k;
    }
    if (best) atomicMax(c.s.key, best);
    cbar(1, c.nt);
    if (c.tid == 0) {
        atomicMax(a.key_slot, *c.s.key);
        __threadfence();
        const uint32_t old = atomicAdd(a.done_counter, 1u);
        if (old == gridDim.x - 1) {
            // backend.cu:107-112 + generator.cpp:49-56: the greedy token feeds the next step
            __threadfence();
            const unsigned long long k = atomicExch(a.key_slot, 0ull);
            const uint32_t idx = argmax_key_index(k);
            *a.key_out = k;
            a.argmax_hist[pos] = static_cast<int32_t>(idx);
            if (pos + 1 >= nf && pos + 1 <= a.capacity) a.tokens[pos + 1] = static_cast<int32_t>(idx);
            *a.done_counter = 0u;
            __threadfence();
            atomicAdd(a.pos, 1);
        }
    }
}

template <int HG>
__global__ void __launch_bounds__(kMaxThreads, 1) persistent_decode_kernel(const __grid_constant__ PersistentArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    Ctx c;
    c.a = &a;
    c.tid = threadIdx.x;
    c.warp = c.tid >> 5;
    c.lane = c.tid & 31;
    c.nw = static_cast<int>(blockDim.x >> 5);
    c.nt = static_cast<int>(blockDim.x);
    c.S = a.ring_slots;
    c.gi = 0;
    c.nsync = 0;
    c.s.ring = smem;
    c.s.full = reinterpret_cast<uint64_t*>(smem + a.off_bars);
    c.s.issued = reinterpret_cast<uint32_t*>(c.s.full + a.ring_slots);
    c.s.x = reinterpret_cast<bf16*>(smem + a.off_x);
    c.s.part = reinterpret_cast<float*>(smem + a.off_part);
    c.s.att = smem + a.off_att;
    c.s.red = reinterpret_cast<float*>(smem + a.off_misc);
    c.s.flags = reinterpret_cast<uint32_t*>(smem + a.off_misc + 128);
    c.s.key = reinterpret_cast<unsigned long long*>(smem + a.off_misc + 168);
    c.s.geo = reinterpret_cast<Geom*>(smem + a.off_misc + 176);
    c.s.ast = reinterpret_cast<AttUnit*>(smem + a.off_misc + 272);
    c.s.lt = reinterpret_cast<uint32_t*>(smem + a.off_tab);
    c.s.pt = reinterpret_cast<int32_t*>(c.s.lt + a.layers * kLayerPtrs);
    const int pos0 = *reinterpret_cast<volatile int32_t*>(a.pos);
    const int per_step = a.layers * kPhasesPerLayer + 1;
    c.seq = Seq{&a, c.s.geo, c.s.lt, c.s.pt, c.s.ast, pos0, static_cast<uint32_t>(per_step), per_step * a.n_steps};

    // launch constants into shared memory: layer pointers, page table, attention unit
    for (int i = c.tid; i < a.layers * kLayerPtrs; i += c.nt) c.s.lt[i] = __ldg(a.layer_tab + i);
    for (int i = c.tid; i < a.n_pages; i += c.nt) c.s.pt[i] = __ldg(a.page_table + i);
    if (c.tid == 32) *c.s.ast = att_static(a, blockIdx.x);
    if (c.tid <= PH_LM && c.tid != PH_ATT) {
        const int kind = c.tid;
        const int N = kind == PH_QKV ? a.qd + 2 * a.kd : kind == PH_GU ? 2 * a.il : kind == PH_LM ? a.vl : a.H;
        const int K = kind == PH_O ? a.qd : kind == PH_DOWN ? a.il : a.H;
        const Band b = band(N, kind == PH_GU ? 2 : 1, blockIdx.x, gridDim.x);
        Geom g;
        g.off = static_cast<unsigned long long>(b.r0) * K * 2;
        g.bytes = static_cast<uint32_t>(b.r1 - b.r0) * static_cast<uint32_t>(K) * 2u;
        g.items = band_items(b, K);
        c.s.geo[kind] = g;
    }
    if (c.tid == 0) {
        for (uint32_t s = 0; s < c.S; ++s) {
            mbar_init(&c.s.full[s], 1);
            c.s.issued[s] = 0u;
        }
        fence_barrier_init();
    }
    __syncthreads();
    // Prime the ring: slot s takes item s, issued by the warp that consumes it.
    if (c.lane == 0) {
        for (uint32_t s = static_cast<uint32_t>(c.warp); s < c.S; s += c.nw) {
            int p = 0;
            uint32_t k = 0;
            if (c.seq.advance(&p, &k, s)) issue(c, p, k, s);
        }
    }

    int p = 0;
    for (int step = 0; step < a.n_steps; ++step) {
        if (step > 0 && !grid_sync(c)) break;
        const int pos = *reinterpret_cast<volatile int32_t*>(a.pos);
        const int nf = *a.n_forced;
        if (pos != pos0 + step || pos < 0 || pos >= a.capacity) {
            if (c.tid == 0) {
                record_error(a.err, DEV_BAD_POSITION);
                atomicExch(a.abort, 1u);
            }
            break;
        }
        bool go = true;
        int ph = 0;  // phase within the step (timeline)
        const bool t0 = c.tid == 0;
        c.tstep = step;
        auto begin = [&]() {
            c.tph = ph;
            if (t0) {
                c.tc0 = clock64();
                trace_edge(a, step, ph, 0);
            }
        };
        auto end = [&]() {
            if (t0) trace_edge(a, step, ph, 1);
            ++ph;
        };
        for (int l = 0; l < a.layers && go; ++l) {
            if (l > 0 && !(go = grid_sync(c))) break;
            begin();
            phase_qkv(c, p++, l, pos);
            end();
            if (!(go = grid_sync(c))) break;
            begin();
            phase_attention<HG>(c, p++, l, pos);
            end();
            if (!(go = grid_sync(c))) break;
            begin();
            phase_o(c, p++);
            end();
            if (!(go = grid_sync(c))) break;
            begin();
            phase_gu(c, p++, l);
            end();
            if (!(go = grid_sync(c))) break;
            begin();
            phase_down(c, p++);
            end();
        }
        if (!go || !grid_sync(c)) break;
        begin();
        phase_lm(c, p++, pos, nf);
        end();
    }
    // Leave no copy in flight: the last round issued into each slot must land
    // (it is the only one that can be outstanding; bounded wait).
    __syncthreads();
    if (c.lane == 0) {
        for (uint32_t s = static_cast<uint32_t>(c.warp); s < c.S; s += c.nw) {
            const uint32_t n = c.s.issued[s];
            if (n == 0) continue;
            for (uint32_t polls = 0; polls < (1u << 20) && !mbar_try_wait(&c.s.full[s], (n - 1) & 1); ++polls) {
            }
        }
    }
    __syncthreads();
}

template <int HG>
cudaError_t launch_hg(const PersistentArgs& a, cudaStream_t s) {
    auto* fn = persistent_decode_kernel<HG>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(a.smem));
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(a.gsync, 0, sizeof(unsigned long long), s);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.grid);
    cfg.blockDim = dim3(a.ring_slots / kBufs * 32);
    cfg.dynamicSmemBytes = a.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, a);
}

}  // namespace

// Shared-memory plan and attention split count for the persistent kernel.
// Returns false if the model does not fit it (the engine then replays the
// CUDA graph of fused kernels instead).
bool plan_persistent(PersistentArgs& a, int sms, size_t smem_limit) {
    // every GEMV row must be a whole number of 512-byte warp groups
    if (a.H % 256 || a.qd % 256 || a.il % 256 || a.kd % 128) return false;
    // band arithmetic is 32-bit: rows x (grid + 1) < 2^32
    const long long max_rows = std::max({a.vl, 2 * a.il, a.qd + 2 * a.kd, a.H});
    if (max_rows * (sms + 1) >= (1ll << 32)) return false;
    a.grid = sms;
    const int HG = attention_head_group(a.qh, a.kvh);
    a.nqb = (a.qh / a.kvh) / HG;
    a.splits = std::max(1, sms / (a.kvh * a.nqb));
    // x holds the largest GEMV input, and a norm's input plus its weights
    const int kmax = std::max({a.qd, a.il, 2 * a.H});
    // partial sums: the largest (rows x pieces) band of any GEMV phase
    auto items = [&](int N, int K, int rg) {
        const int units = N / rg;
        const int rows = (units + sms - 1) / sms * rg;
        return rows * pieces_per_row(K);
    };
    const int max_items = std::max({items(a.qd + 2 * a.kd, a.H, 1), items(a.H, a.qd, 1), items(2 * a.il, a.H, 2),
                                    items(a.H, a.il, 1), items(a.vl, a.H, 1)});
    auto up = [](size_t n) { return (n + 127) / 128 * 128; };
    const size_t x_bytes = up(static_cast<size_t>(kmax) * 2);
    const size_t part_bytes = up(static_cast<size_t>(max_items) * 4);
    // attention: q, key and value rows + per-warp states; the merge reuses the states' space
    const size_t att_state = (static_cast<size_t>(HG) * 128 + 256) * 2 + static_cast<size_t>(kAttWarps) * HG * kAttRecord * 4;
    const size_t att_merge = (static_cast<size_t>(HG) * 128 + 256) * 2 +
                             (static_cast<size_t>(a.splits) * HG * 2 + 16) * 4 + static_cast<size_t>(kMaxThreads) * 16;
    const size_t att_bytes = up(std::max(att_state, att_merge));
    // the attention phase uses no GEMV buffer: its scratch shares their region
    const size_t region = std::max(x_bytes + part_bytes, att_bytes);
    const size_t misc = 384;  // reduction words, flags, argmax key, band geometry, attention unit
    // slots fill the rest (8 KB + 8-byte barrier + 4-byte count each), kBufs per warp
    // launch constants: layer pointer offsets and the page table
    a.n_pages = (a.capacity + kPage - 1) / kPage;
    const size_t tab_bytes = (static_cast<size_t>(a.layers) * kLayerPtrs + a.n_pages) * 4;
    const long fixed = static_cast<long>(region + misc + (tab_bytes + 15) / 16 * 16);
    long warps = (static_cast<long>(smem_limit) - fixed - 256) / (kBufs * (kSlot + 12));
    if (warps < kAttWarps) return false;
    warps = std::min(warps, static_cast<long>(kMaxW));
    const long slots = warps * kBufs;
    a.ring_slots = static_cast<uint32_t>(slots);
    a.off_bars = static_cast<size_t>(slots) * kSlot;
    a.off_x = a.off_bars + up(static_cast<size_t>(slots) * 12);
    a.off_part = a.off_x + x_bytes;
    a.off_att = a.off_x;
    a.off_misc = a.off_x + region;
    a.off_tab = a.off_misc + misc;
    a.smem = a.off_tab + tab_bytes;
    return a.smem <= smem_limit;
}

cudaError_t launch_persistent(const PersistentArgs& a, cudaStream_t s) {
    switch (attention_head_group(a.qh, a.kvh)) {
        case 1: return launch_hg<1>(a, s);
        case 2: return launch_hg<2>(a, s);
        default: return launch_hg<4>(a, s);
    }
}

}  // namespace q3

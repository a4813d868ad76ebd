// persistent.cu -- the whole decode loop as one persistent kernel.
//
// The reference runs ~14 kernels per layer plus a host sync per token
// (src/lib/model/qwen3/qwen3.hpp:131-166, src/lib/backend/cuda/backend.cu).
// Here one cooperative launch runs n decode steps: one CTA per SM, a producer
// warp that streams every byte the steps read -- weights of every GEMV of
// every layer, then the KV pages of every attention -- through one ring of
// 4 KB shared-memory slots with 1-D TMA bulk copies, in the exact order the
// consumers use them, and up to 12 consumer warps that walk the phases
//   QKV -> attention -> O -> gate/up -> down   (per layer), lm_head (per step)
// separated by a grid-wide barrier.  The producer never waits at a phase
// boundary (weights and pages older than the current position do not depend
// on the previous phase), so HBM stays busy while the consumers synchronise;
// the only K/V row produced inside a step (the current position) is patched
// into the ring by the consumers after the QKV phase.
//
// Numerics are those of the kernel-per-op path (gemv.cu, attention.cu): fp32
// accumulation, BF16 rounding where the reference rounds, fixed-order
// reductions (per-(row, chunk) partials summed in order; attention split
// states merged in split order).
//
// Every wait is bounded: mbarrier waits by kMaxPolls, the grid barrier by
// kGridPolls.  A grid barrier that runs out records DEV_GRID_TIMEOUT and
// raises the abort word; every CTA then leaves at its next barrier, after
// its producer has drained the copies it issued.
#include <algorithm>
#include <cstring>

#include "kernels.cuh"

namespace q3 {

namespace {

// Ring of kBufs slots per consumer warp (at most kMaxCW warps): item g lands in
// slot g % S and GEMV item g is consumed by warp g % W (S = kBufs * W), so
// every slot's rounds are consumed in program order by one warp.  (An
// mbarrier wait sees only the phase parity: a warp must never wait on a
// slot's next round while another warp still holds the current one.)
constexpr int kMaxCW = 12;
constexpr int kMaxThreads = (kMaxCW + 1) * 32;
constexpr int kSlot = 8192;             // ring slot bytes: half a K or V page of a head, or 8 KB of a weight band
constexpr int kBufs = 2;                // ring slots per consumer warp (double buffering)
constexpr int kAttWarps = 8;            // warps that run attention (16 half-warps x 4 tokens)
constexpr int kPage = 64;
constexpr uint32_t kGridPolls = 1u << 22;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
    return *reinterpret_cast<const volatile uint32_t*>(p);
}
__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Phase timeline (first step of a launch only): slot 0/1 consumer start/end,
// 2/3 producer first/last issue of the phase.
__device__ __forceinline__ void trace_mark(const PersistentArgs& a, int step, int phase, int what) {
    if (a.trace && step == 0 && phase < a.trace_phases)
        a.trace[(static_cast<size_t>(blockIdx.x) * a.trace_phases + phase) * 4 + what] = now_ns();
}

struct Smem {
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    bf16* x;
    float* part;
    float* att;      // attention merge scratch (aliases x/part)
    float* red;      // 32 floats
    uint32_t* flags; // [0] abort seen, [1] last-arriver, [2] token
    unsigned long long* key;
};

struct Ctx {
    const PersistentArgs* a;
    Smem s;
    int tid, warp, lane;
    uint32_t gi;  // global item counter (consumers)
    int nw;       // consumer warps (= ring slots)
    int nt;       // consumer threads
};

// ----------------------------------------------------------------- work split
struct Band {
    int r0, r1;
};
__device__ __forceinline__ Band band(int N, int row_gran, int cta, int ncta) {
    const int units = N / row_gran;
    const int u0 = static_cast<int>(static_cast<long long>(cta) * units / ncta);
    const int u1 = static_cast<int>(static_cast<long long>(cta + 1) * units / ncta);
    return {u0 * row_gran, u1 * row_gran};
}
// A CTA's band of rows [r0, r1) of a row-major [N, K] matrix is one
// contiguous byte range; it streams as 16 KB items (the last one shorter).
__device__ __forceinline__ size_t band_bytes(const Band& b, int K) {
    return static_cast<size_t>(b.r1 - b.r0) * K * 2;
}
__device__ __forceinline__ int band_items(const Band& b, int K) {
    return static_cast<int>((band_bytes(b, K) + kSlot - 1) / kSlot);
}
// Partial sums per row: one per item the row touches (fixed order).
__device__ __forceinline__ int pieces_per_row(int K) { return (K * 2 + kSlot - 1) / kSlot + 1; }

struct AttUnit {
    bool valid;
    int kvh, qb, split, pb, pe;
};
__device__ __forceinline__ AttUnit att_unit(const PersistentArgs& a, int cta, int pos) {
    AttUnit u{};
    const int n_units = a.kvh * a.nqb * a.splits;
    if (cta >= n_units) return u;
    u.valid = true;
    u.split = cta % a.splits;
    const int kq = cta / a.splits;
    u.kvh = kq / a.nqb;
    u.qb = kq % a.nqb;
    const int n_pages = pos / kPage + 1;
    u.pb = static_cast<int>(static_cast<long long>(u.split) * n_pages / a.splits);
    u.pe = static_cast<int>(static_cast<long long>(u.split + 1) * n_pages / a.splits);
    return u;
}

// ----------------------------------------------------------------- producer
struct Producer {
    const PersistentArgs* a;
    Smem s;
    uint32_t gi = 0;      // items issued
    uint32_t slot = 0;    // gi % ring_slots
    uint32_t round = 0;   // gi / ring_slots
    uint64_t pol = 0;
    bool aborted = false;

    __device__ void issue(const void* src, uint32_t bytes) {
        if (aborted) return;
        if (round > 0) {
            const uint32_t parity = (round - 1) & 1;
            uint32_t polls = 0;
            while (!mbar_try_wait(&s.empty[slot], parity)) {
                if ((++polls & 1023) == 0 && ld_volatile(a->abort)) {
                    aborted = true;
                    return;
                }
                if (polls > kMaxPolls * 4) {
                    record_error(a->err, DEV_TMA_WAIT_TIMEOUT);
                    atomicExch(a->abort, 1u);
                    aborted = true;
                    return;
                }
            }
        }
        mbar_arrive_expect_tx(&s.full[slot], bytes);
        bulk_g2s(s.ring + static_cast<size_t>(slot) * kSlot, src, bytes, &s.full[slot], pol);
        ++gi;
        if (++slot == a->ring_slots) {
            slot = 0;
            ++round;
        }
    }

    __device__ void gemv(const bf16* W, int N, int K, int row_gran) {
        const Band b = band(N, row_gran, blockIdx.x, gridDim.x);
        const size_t total = band_bytes(b, K);
        const uint8_t* base = reinterpret_cast<const uint8_t*>(W + static_cast<size_t>(b.r0) * K);
        for (size_t off = 0; off < total; off += kSlot) {
            const size_t n = total - off < static_cast<size_t>(kSlot) ? total - off : static_cast<size_t>(kSlot);
            issue(base + off, static_cast<uint32_t>(n));
        }
    }

    // Pages older than this step's position are final only once every CTA
    // finished the previous step; the consumers publish entering a step.
    __device__ bool wait_step(int step) {
        const volatile uint32_t* cur = s.flags + 3;
        for (uint32_t polls = 0; static_cast<int>(*cur) < step; ++polls) {
            if ((polls & 1023) == 1023 && ld_volatile(a->abort)) return false;
            if (polls > kMaxPolls * 4) return false;
            __nanosleep(64);
        }
        return true;
    }

    __device__ void attention(const PersistentLayer& L, int pos) {
        const AttUnit u = att_unit(*a, blockIdx.x, pos);
        if (!u.valid) return;
        for (int page = u.pb; page < u.pe; ++page) {
            const size_t base = (static_cast<size_t>(a->page_table[page]) * a->kvh + u.kvh) * kPage * 128;
            issue(L.k_pages + base, kSlot);
            issue(L.k_pages + base + kPage * 64, kSlot);
            issue(L.v_pages + base, kSlot);
            issue(L.v_pages + base + kPage * 64, kSlot);
        }
    }

    __device__ void run(int pos0) {
        pol = policy_evict_first();
        for (int step = 0; step < a->n_steps && !aborted; ++step) {
            const int pos = pos0 + step;
            int ph = 0;
            for (int l = 0; l < a->layers && !aborted; ++l) {
                const PersistentLayer& L = a->L[l];
                trace_mark(*a, step, ph, 2);
                gemv(L.w_qkv, a->qd + 2 * a->kd, a->H, 1);
                trace_mark(*a, step, ph++, 3);
                if (l == 0 && !wait_step(step)) {
                    aborted = true;
                    break;
                }
                trace_mark(*a, step, ph, 2);
                attention(L, pos);
                trace_mark(*a, step, ph++, 3);
                trace_mark(*a, step, ph, 2);
                gemv(L.w_o, a->H, a->qd, 1);
                trace_mark(*a, step, ph++, 3);
                trace_mark(*a, step, ph, 2);
                gemv(L.w_gu, 2 * a->il, a->H, 2);
                trace_mark(*a, step, ph++, 3);
                trace_mark(*a, step, ph, 2);
                gemv(L.w_down, a->H, a->il, 1);
                trace_mark(*a, step, ph++, 3);
            }
            trace_mark(*a, step, ph, 2);
            gemv(a->lm_head, a->vl, a->H, 1);
            trace_mark(*a, step, ph, 3);
        }
        // Leave no copy in flight: wait (bounded) for the last slots issued.
        const uint32_t first = gi > a->ring_slots ? gi - a->ring_slots : 0;
        for (uint32_t g = first; g < gi; ++g) {
            const uint32_t slot = g % a->ring_slots;
            for (uint32_t p = 0; p < (1u << 16) && !mbar_try_wait(&s.full[slot], (g / a->ring_slots) & 1); ++p) {
            }
        }
    }
};

// ----------------------------------------------------------------- consumers
__device__ __forceinline__ void cbar(int id, int n) { named_bar(id, n); }

// Bounded wait for a ring slot.  After any failure (here or in another CTA)
// it stops waiting at once, so a broken pipeline unwinds in one poll budget.
__device__ __forceinline__ bool slot_wait(const PersistentArgs& a, uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    if (ld_volatile(a.abort)) return false;
    if (mbar_wait(bar, parity, a.err, DEV_TMA_WAIT_TIMEOUT)) return true;
    atomicExch(a.abort, 1u);
    return false;
}

// Grid barrier among the consumer threads of all CTAs.  Returns false when the
// kernel must stop (a barrier ran out of polls here or elsewhere).
__device__ bool grid_sync(Ctx& c) {
    const PersistentArgs& a = *c.a;
    cbar(1, c.nt);
    if (c.tid == 0) {
        uint32_t ok = 1;
        const uint32_t gen = ld_volatile(&a.gsync[1]);
        __threadfence();
        const uint32_t arrived = atomicAdd(&a.gsync[0], 1u);
        if (arrived == gridDim.x - 1) {
            a.gsync[0] = 0;
            __threadfence();
            atomicAdd(&a.gsync[1], 1u);
        } else {
            uint32_t polls = 0;
            while (ld_acquire(&a.gsync[1]) == gen) {
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
        }
        __threadfence();
        if (ld_volatile(a.abort)) ok = 0;
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

// x = rmsnorm(src) into shared memory; optionally the fp32 sums for the
// sum of squares (rmsnorm_add semantics); optionally write src to hs_out.
__device__ void prologue_norm(Ctx& c, const bf16* src, const float* vsum, const bf16* w, int K, bf16* hs_out) {
    const PersistentArgs& a = *c.a;
    float ss = 0.f;
    const int k8 = K / 8;
    for (int i = c.tid; i < k8; i += c.nt) {
        const uint4 h = reinterpret_cast<const uint4*>(src)[i];
        if (vsum) {
            const float4 v0 = reinterpret_cast<const float4*>(vsum)[2 * i];
            const float4 v1 = reinterpret_cast<const float4*>(vsum)[2 * i + 1];
            ss += v0.x * v0.x + v0.y * v0.y + v0.z * v0.z + v0.w * v0.w;
            ss += v1.x * v1.x + v1.y * v1.y + v1.z * v1.z + v1.w * v1.w;
        } else {
            const uint32_t* hw = reinterpret_cast<const uint32_t*>(&h);
#pragma unroll
            for (int j = 0; j < 4; ++j) ss += bf_lo(hw[j]) * bf_lo(hw[j]) + bf_hi(hw[j]) * bf_hi(hw[j]);
        }
        reinterpret_cast<uint4*>(c.s.x)[i] = h;
        if (hs_out && blockIdx.x == 0) reinterpret_cast<uint4*>(hs_out)[i] = h;
    }
    ss = csum(c, ss);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(K) + a.eps);
    for (int i = c.tid; i < k8; i += c.nt) {
        uint4 h = reinterpret_cast<uint4*>(c.s.x)[i];
        const uint4 wv = reinterpret_cast<const uint4*>(w)[i];
        uint32_t* hw = reinterpret_cast<uint32_t*>(&h);
        const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const bf16 b0 = f2bf(bf_lo(hw[j]) * scale * bf_lo(ww[j]));
            const bf16 b1 = f2bf(bf_hi(hw[j]) * scale * bf_hi(ww[j]));
            hw[j] = static_cast<uint32_t>(__bfloat16_as_ushort(b0)) |
                    (static_cast<uint32_t>(__bfloat16_as_ushort(b1)) << 16);
        }
        reinterpret_cast<uint4*>(c.s.x)[i] = h;
    }
    cbar(1, c.nt);
}

__device__ void prologue_copy(Ctx& c, const bf16* src, int K) {
    for (int i = c.tid; i < K / 8; i += c.nt)
        reinterpret_cast<uint4*>(c.s.x)[i] = reinterpret_cast<const uint4*>(src)[i];
    cbar(1, c.nt);
}

// Dot every item of this CTA's band with x.  Item i covers band bytes
// [i * 16 KB, ...); a warp walks it in 512-byte groups (32 lanes x 16 B), and
// since K is a multiple of 256 a group never straddles two rows.  The partial
// of (row, item) goes to part[row * P + (item - first item of the row)].
__device__ Band gemv_consume(Ctx& c, int N, int K, int row_gran) {
    const PersistentArgs& a = *c.a;
    const Band b = band(N, row_gran, blockIdx.x, gridDim.x);
    const int n_items = band_items(b, K);
    const int P = pieces_per_row(K);
    const int nrows = b.r1 - b.r0;
    for (int i = c.tid; i < nrows * P; i += c.nt) c.s.part[i] = 0.f;
    cbar(1, c.nt);
    const uint32_t vpr = static_cast<uint32_t>(K) / 8;          // 16-byte vectors per row
    const uint32_t vtot = static_cast<uint32_t>(nrows) * vpr;
    const uint32_t rows_per_item_bytes = kSlot;                  // for first-item arithmetic
    // this warp's first item of the phase: the one that lands in its slot
    const uint32_t nw = static_cast<uint32_t>(c.nw);
    const int k0 = static_cast<int>((static_cast<uint32_t>(c.warp) + nw - c.gi % nw) % nw);
    for (int k = k0; k < n_items; k += c.nw) {
        const uint32_t g = c.gi + k;
        const uint32_t slot = g % a.ring_slots;
        const bool ok = slot_wait(a, &c.s.full[slot], (g / a.ring_slots) & 1);
        const uint32_t v0 = static_cast<uint32_t>(k) * (kSlot / 16);
        const uint32_t v1 = min(vtot, v0 + kSlot / 16);
        const uint4* wv = reinterpret_cast<const uint4*>(c.s.ring + static_cast<size_t>(slot) * kSlot);
        const uint4* xv = reinterpret_cast<const uint4*>(c.s.x);
        uint32_t row = v0 / vpr;
        uint32_t col = v0 - row * vpr;
        float acc0 = 0.f, acc1 = 0.f;
        for (uint32_t v = v0; v < v1; v += 32) {
            if (ok) {
                if ((v - v0) & 32) acc1 = dot8(wv[v - v0 + c.lane], xv[col + c.lane], acc1);
                else acc0 = dot8(wv[v - v0 + c.lane], xv[col + c.lane], acc0);
            }
            col += 32;
            if (col == vpr || v + 32 >= v1) {
                const float sum = warp_sum(acc0 + acc1);
                acc0 = acc1 = 0.f;
                if (c.lane == 0) {
                    const uint32_t first = (row * vpr * 16) / rows_per_item_bytes;
                    c.s.part[row * P + (static_cast<uint32_t>(k) - first)] = sum;
                }
                if (col == vpr) {
                    col = 0;
                    ++row;
                }
            }
        }
        __syncwarp();
        if (c.lane == 0) mbar_arrive(&c.s.empty[slot]);
    }
    c.gi += n_items;
    cbar(1, c.nt);
    return b;
}

__device__ __forceinline__ float row_sum(Ctx& c, int rl, int P) {
    float r = 0.f;
    for (int p = 0; p < P; ++p) r += c.s.part[rl * P + p];
    return r;
}

__device__ __forceinline__ size_t kv_slot(const PersistentArgs& a, int pos, int head) {
    const int page = a.page_table[pos / kPage];
    return ((static_cast<size_t>(page) * a.kvh + head) * kPage + (pos % kPage)) * 128;
}

// ----------------------------------------------------------------- phases
__device__ void phase_qkv(Ctx& c, const PersistentLayer& L, int l, int pos, int nf) {
    const PersistentArgs& a = *c.a;
    if (l == 0) {
        // embedding (embedding.cuh:9-30) of the token at this position
        int token = a.tokens[pos];
        if (token < 0 || token >= a.vocab) {
            if (c.tid == 0) record_error(a.err, DEV_BAD_TOKEN);
            token = 0;
        }
        (void)nf;
        prologue_norm(c, a.embed + static_cast<size_t>(token) * a.H, nullptr, L.in_norm, a.H, a.hs);
    } else {
        prologue_norm(c, a.hs, nullptr, L.in_norm, a.H, nullptr);
    }
    const int N = a.qd + 2 * a.kd;
    const Band b = gemv_consume(c, N, a.H, 1);
    const int nch = pieces_per_row(a.H);
    for (int rl = c.tid; rl < b.r1 - b.r0; rl += c.nt) {
        const int gr = b.r0 + rl;
        const bf16 v = f2bf(row_sum(c, rl, nch));
        if (gr < a.qd) {
            a.q[gr] = v;
        } else if (gr < a.qd + a.kd) {
            const int k = gr - a.qd;
            L.k_pages[kv_slot(a, pos, k >> 7) + (k & 127)] = v;
        } else {
            const int k = gr - a.qd - a.kd;
            L.v_pages[kv_slot(a, pos, k >> 7) + (k & 127)] = v;
        }
    }
    // qk_norm_rope (qk_norm_rope.cuh:14-90) by the CTA that completes a head
    __threadfence();
    cbar(1, c.nt);
    if (c.warp == 0) {
        const int nqk = a.qd + a.kd;
        const int hi_row = min(b.r1, nqk);
        for (int h = b.r0 / 128; h * 128 < hi_row; ++h) {
            const int lo = max(b.r0, h * 128), hi = min(hi_row, (h + 1) * 128);
            if (hi <= lo) continue;
            uint32_t old = 0;
            if (c.lane == 0) old = atomicAdd(&a.head_counters[h], static_cast<uint32_t>(hi - lo));
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old + static_cast<uint32_t>(hi - lo) != 128u) continue;
            __threadfence();
            const bool is_q = h * 128 < a.qd;
            bf16* base = is_q ? a.q + h * 128 : L.k_pages + kv_slot(a, pos, h - a.qd / 128);
            const bf16* nw = is_q ? L.q_norm : L.k_norm;
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                v[j] = __uint_as_float(
                    static_cast<uint32_t>(__ldcg(reinterpret_cast<const unsigned short*>(base) + c.lane + 32 * j))
                    << 16);
            const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
            const float scale = 1.0f / sqrtf(ss / 128.0f + a.eps);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int i = c.lane + 32 * j;
                const float cs = a.rope_cos[static_cast<size_t>(pos) * 64 + i];
                const float sn = a.rope_sin[static_cast<size_t>(pos) * 64 + i];
                const float x = v[j] * bf2f(nw[i]) * scale;
                const float y = v[j + 2] * bf2f(nw[i + 64]) * scale;
                base[i] = f2bf(x * cs - y * sn);
                base[i + 64] = f2bf(y * cs + x * sn);
            }
            if (c.lane == 0) a.head_counters[h] = 0u;
        }
    }
}

template <int HG>
__device__ void phase_attention(Ctx& c, const PersistentLayer& L, int pos) {
    const PersistentArgs& a = *c.a;
    const AttUnit u = att_unit(a, blockIdx.x, pos);
    const int np = u.valid ? u.pe - u.pb : 0;
    float* S = c.s.att;  // [8 warps][HG][130]: m, l, acc[128]
    const bool att_warp = c.warp < kAttWarps;
    const int hw = c.tid >> 4, hl = c.tid & 15;  // half-warp 0..15 for attention warps
    const int G = a.qh / a.kvh;
    const int qh0 = u.kvh * G + u.qb * HG;
    float q[HG][8], m[HG], l[HG], acc[HG][8];
    if (att_warp && u.valid) {
#pragma unroll
        for (int g = 0; g < HG; ++g) {
            const uint4 v = reinterpret_cast<const uint4*>(a.q + static_cast<size_t>(qh0 + g) * 128)[hl];
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
    const int live_page = pos / kPage;
    for (int i = 0; i < np; ++i) {
        const uint32_t g0 = c.gi + 4 * i;
        if (att_warp) {
            bool ok = true;
            for (int q = 0; q < 4; ++q)
                ok = slot_wait(a, &c.s.full[(g0 + q) % a.ring_slots], ((g0 + q) / a.ring_slots) & 1) && ok;
            const int page = u.pb + i;
            if (page == live_page && c.warp == 0) {
                // this step's K/V row was written by the QKV phase after the copy was issued
                const int j = pos % kPage;
                const int which = c.lane >> 4;  // 0: K, 1: V
                const uint32_t slot = (g0 + which * 2 + (j >> 5)) % a.ring_slots;
                const bf16* src = (which ? L.v_pages : L.k_pages) + kv_slot(a, pos, u.kvh);
                uint4* dst = reinterpret_cast<uint4*>(c.s.ring + static_cast<size_t>(slot) * kSlot + (j & 31) * 256);
                dst[c.lane & 15] = __ldcg(reinterpret_cast<const uint4*>(src) + (c.lane & 15));
            }
            cbar(2, kAttWarps * 32);
            const int valid = min(kPage, pos + 1 - page * kPage);
            const int j0 = hw * 4;  // 4 consecutive tokens of the page, all in half (j0 / 32) of it
            const uint32_t kslot = (g0 + (j0 >> 5)) % a.ring_slots, vslot = (g0 + 2 + (j0 >> 5)) % a.ring_slots;
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
                float mx = fmaxf(fmaxf(sc[0][g], sc[1][g]), fmaxf(sc[2][g], sc[3][g]));
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
            cbar(2, kAttWarps * 32);
            if (c.tid == 0)
                for (int q = 0; q < 4; ++q) mbar_arrive(&c.s.empty[(g0 + q) % a.ring_slots]);
        }
    }
    c.gi += 4 * np;
    // ---- merge: half-warp pairs by shuffle, then the 8 warp states in shared memory
    if (att_warp && u.valid) {
#pragma unroll
        for (int g = 0; g < HG; ++g) {
            const float mo = __shfl_xor_sync(0xffffffffu, m[g], 16);
            const float lo = __shfl_xor_sync(0xffffffffu, l[g], 16);
            const float M = fmaxf(m[g], mo);
            const float f0 = (M == -INFINITY) ? 0.f : exp2f(m[g] - M);
            const float f1 = (M == -INFINITY) ? 0.f : exp2f(mo - M);
            const float L2 = l[g] * f0 + lo * f1;
            float* Sw = S + (c.warp * HG + g) * 130;
#pragma unroll
            for (int d = 0; d < 8; ++d) {
                const float ao = __shfl_xor_sync(0xffffffffu, acc[g][d], 16);
                // lanes 0-15 (the lower half-warp) hold dims 8 hl .. 8 hl + 7 after the pair merge
                if (c.lane < 16) Sw[2 + 8 * hl + d] = acc[g][d] * f0 + ao * f1;
            }
            if (c.lane == 0) {
                Sw[0] = M;
                Sw[1] = L2;
            }
        }
    }
    cbar(1, c.nt);
    const int n_out = HG * 128;
    const int kq = u.kvh * a.nqb + u.qb;
    if (u.valid) {
        float* dst = a.att_part + (static_cast<size_t>(kq) * a.splits + u.split) * HG * 130;
        for (int o = c.tid; o < n_out; o += c.nt) {
            const int g = o / 128, d = o % 128;
            float M = -INFINITY;
            for (int w = 0; w < kAttWarps; ++w) M = fmaxf(M, S[(w * HG + g) * 130]);
            float Ls = 0.f, A = 0.f;
            if (M != -INFINITY)
                for (int w = 0; w < kAttWarps; ++w) {
                    const float* Sw = S + (w * HG + g) * 130;
                    const float f = exp2f(Sw[0] - M);
                    Ls += Sw[1] * f;
                    A += Sw[2 + d] * f;
                }
            dst[g * 130 + 2 + d] = A;
            if (d == 0) {
                dst[g * 130] = M;
                dst[g * 130 + 1] = Ls;
            }
        }
        __threadfence();
        cbar(1, c.nt);
        if (c.tid == 0) {
            const uint32_t old = atomicAdd(&a.att_counters[kq], 1u);
            c.s.flags[1] = (old == static_cast<uint32_t>(a.splits - 1)) ? 1u : 0u;
        }
        cbar(1, c.nt);
        if (c.s.flags[1]) {
            // last split of this (kv head, block): merge the splits in order
            __threadfence();
            const float* src = a.att_part + static_cast<size_t>(kq) * a.splits * HG * 130;
            float* ml = S;  // [splits][HG] scale factors, then L per head
            for (int i = c.tid; i < a.splits * HG; i += c.nt) ml[i] = __ldcg(src + (i / HG) * HG * 130 + (i % HG) * 130);
            cbar(1, c.nt);
            float* Mg = S + a.splits * HG;
            float* Lg = Mg + HG;
            if (c.tid < HG) {
                float M = -INFINITY;
                for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, ml[sp * HG + c.tid]);
                float Ls = 0.f;
                for (int sp = 0; sp < a.splits; ++sp) {
                    const float ms = ml[sp * HG + c.tid];
                    if (ms != -INFINITY) Ls += __ldcg(src + (sp * HG + c.tid) * 130 + 1) * exp2f(ms - M);
                }
                Mg[c.tid] = M;
                Lg[c.tid] = Ls;
            }
            cbar(1, c.nt);
            for (int o = c.tid; o < n_out; o += c.nt) {
                const int g = o / 128, d = o % 128;
                float A = 0.f;
                for (int sp = 0; sp < a.splits; ++sp) {
                    const float ms = ml[sp * HG + g];
                    if (ms == -INFINITY) continue;
                    A += __ldcg(src + (sp * HG + g) * 130 + 2 + d) * exp2f(ms - Mg[g]);
                }
                a.attn[static_cast<size_t>(qh0 + g) * 128 + d] = f2bf(A / Lg[g]);
            }
            if (c.tid == 0) a.att_counters[kq] = 0u;
        }
    }
}

__device__ void phase_o(Ctx& c, const PersistentLayer& L) {
    const PersistentArgs& a = *c.a;
    prologue_copy(c, a.attn, a.qd);
    const Band b = gemv_consume(c, a.H, a.qd, 1);
    const int nch = pieces_per_row(a.qd);
    for (int rl = c.tid; rl < b.r1 - b.r0; rl += c.nt) {
        const int gr = b.r0 + rl;
        // qwen3.hpp:151-152 -> rmsnorm.cuh:58-60
        const float v = bf2f(a.hs[gr]) + round_bf(row_sum(c, rl, nch));
        a.hs[gr] = f2bf(v);
        a.vsum[gr] = v;
    }
    (void)L;
}

__device__ void phase_gu(Ctx& c, const PersistentLayer& L) {
    const PersistentArgs& a = *c.a;
    prologue_norm(c, a.hs, a.vsum, L.post_norm, a.H, nullptr);
    const Band b = gemv_consume(c, 2 * a.il, a.H, 2);
    const int nch = pieces_per_row(a.H);
    for (int m = c.tid; m < (b.r1 - b.r0) / 2; m += c.nt) {
        // qwen3.hpp:154-156 -> silu.cuh:18-20 on the BF16-rounded matmul outputs
        const float gv = round_bf(row_sum(c, 2 * m, nch)), uv = round_bf(row_sum(c, 2 * m + 1, nch));
        a.g[(b.r0 >> 1) + m] = f2bf(gv / (1.0f + expf(-gv)) * uv);
    }
}

__device__ void phase_down(Ctx& c) {
    const PersistentArgs& a = *c.a;
    prologue_copy(c, a.g, a.il);
    const Band b = gemv_consume(c, a.H, a.il, 1);
    const int nch = pieces_per_row(a.il);
    for (int rl = c.tid; rl < b.r1 - b.r0; rl += c.nt) {
        const int gr = b.r0 + rl;
        // qwen3.hpp:158-159
        a.hs[gr] = f2bf(bf2f(a.hs[gr]) + round_bf(row_sum(c, rl, nch)));
    }
}

__device__ void phase_lm(Ctx& c, int pos, int nf) {
    const PersistentArgs& a = *c.a;
    prologue_norm(c, a.hs, nullptr, a.final_norm, a.H, nullptr);
    const Band b = gemv_consume(c, a.vl, a.H, 1);
    const int nch = pieces_per_row(a.H);
    if (c.tid == 0) *c.s.key = 0ull;
    cbar(1, c.nt);
    unsigned long long best = 0ull;
    for (int rl = c.tid; rl < b.r1 - b.r0; rl += c.nt) {
        const int gr = b.r0 + rl;
        const bf16 v = f2bf(row_sum(c, rl, nch));
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
    c.gi = 0;
    c.nw = static_cast<int>(a.ring_slots) / kBufs;
    c.nt = c.nw * 32;
    // shared memory carve-up (offsets computed on the host, see PersistentArgs)
    c.s.ring = smem;
    c.s.full = reinterpret_cast<uint64_t*>(smem + a.off_bars);
    c.s.empty = c.s.full + a.ring_slots;
    c.s.x = reinterpret_cast<bf16*>(smem + a.off_x);
    c.s.part = reinterpret_cast<float*>(smem + a.off_part);
    c.s.att = reinterpret_cast<float*>(smem + a.off_x);
    c.s.red = reinterpret_cast<float*>(smem + a.off_misc);
    c.s.flags = reinterpret_cast<uint32_t*>(smem + a.off_misc + 128);
    c.s.key = reinterpret_cast<unsigned long long*>(smem + a.off_misc + 160);

    if (c.tid == 0) {
        for (uint32_t s = 0; s < a.ring_slots; ++s) {
            mbar_init(&c.s.full[s], 1);
            mbar_init(&c.s.empty[s], 1);
        }
        c.s.flags[3] = 0;
        fence_barrier_init();
    }
    __syncthreads();
    const int pos0 = *a.pos;

    if (c.warp == c.nw) {
        if (c.lane == 0) {
            Producer p{&a, c.s};
            p.run(pos0);
        }
    } else {
        for (int step = 0; step < a.n_steps; ++step) {
            if (step > 0 && !grid_sync(c)) break;
            if (c.tid == 0) {
                *reinterpret_cast<volatile uint32_t*>(c.s.flags + 3) = static_cast<uint32_t>(step);
                __threadfence_block();
            }
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
            int ph = 0;
            const bool t0 = c.tid == 0;
            for (int l = 0; l < a.layers && go; ++l) {
                const PersistentLayer& L = a.L[l];
                if (l > 0 && !(go = grid_sync(c))) break;
                if (t0) trace_mark(a, step, ph, 0);
                phase_qkv(c, L, l, pos, nf);
                if (t0) trace_mark(a, step, ph++, 1);
                if (!(go = grid_sync(c))) break;
                if (t0) trace_mark(a, step, ph, 0);
                phase_attention<HG>(c, L, pos);
                if (t0) trace_mark(a, step, ph++, 1);
                if (!(go = grid_sync(c))) break;
                if (t0) trace_mark(a, step, ph, 0);
                phase_o(c, L);
                if (t0) trace_mark(a, step, ph++, 1);
                if (!(go = grid_sync(c))) break;
                if (t0) trace_mark(a, step, ph, 0);
                phase_gu(c, L);
                if (t0) trace_mark(a, step, ph++, 1);
                if (!(go = grid_sync(c))) break;
                if (t0) trace_mark(a, step, ph, 0);
                phase_down(c);
                if (t0) trace_mark(a, step, ph++, 1);
            }
            if (!go || !grid_sync(c)) break;
            if (t0) trace_mark(a, step, ph, 0);
            phase_lm(c, pos, nf);
            if (t0) trace_mark(a, step, ph, 1);
        }
    }
    __syncthreads();
}

template <int HG>
cudaError_t launch_hg(const PersistentArgs& a, cudaStream_t s) {
    auto* fn = persistent_decode_kernel<HG>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(a.smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.grid);
    cfg.blockDim = dim3((a.ring_slots / kBufs + 1) * 32);
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
// Returns false if the model does not fit the per-CTA budget.
bool plan_persistent(PersistentArgs& a, int sms, size_t smem_limit) {
    // every GEMV row must be a whole number of 512-byte warp groups
    if (a.H % 256 || a.qd % 256 || a.il % 256) return false;
    a.grid = sms;
    const int HG = (a.qh / a.kvh) >= 4 ? 4 : (a.qh / a.kvh);
    a.nqb = (a.qh / a.kvh) / HG;
    a.splits = std::max(1, sms / (a.kvh * a.nqb));
    const int kmax = std::max(std::max(a.H, a.qd), a.il);
    // partial sums: the largest (rows x pieces) band of any GEMV phase
    auto items = [&](int N, int K, int rg) {
        const int units = N / rg;
        const int rows = (units + sms - 1) / sms * rg;
        return rows * ((K * 2 + kSlot - 1) / kSlot + 1);
    };
    int max_items = std::max({items(a.qd + 2 * a.kd, a.H, 1), items(a.H, a.qd, 1), items(2 * a.il, a.H, 2),
                              items(a.H, a.il, 1), items(a.vl, a.H, 1)});
    const size_t x_bytes = (static_cast<size_t>(kmax) * 2 + 127) / 128 * 128;
    const size_t part_bytes = (static_cast<size_t>(max_items) * 4 + 127) / 128 * 128;
    const size_t att_bytes = static_cast<size_t>(kAttWarps) * HG * 130 * 4 + static_cast<size_t>(a.splits) * HG * 4 + 64;
    const size_t region = std::max(x_bytes + part_bytes, (att_bytes + 127) / 128 * 128);
    const size_t misc = 256;
    // slots fill what is left (each 8 KB + two 8-byte barriers), kBufs per consumer warp
    const long rest = static_cast<long>(smem_limit) - static_cast<long>(region + misc);
    long warps = rest / (kBufs * (kSlot + 16));
    if (warps < kAttWarps) return false;
    warps = std::min(warps, static_cast<long>(kMaxCW));
    const long slots = warps * kBufs;
    a.ring_slots = static_cast<uint32_t>(slots);
    a.off_bars = slots * kSlot;
    a.off_x = a.off_bars + (slots * 16 + 127) / 128 * 128;
    a.off_part = a.off_x + x_bytes;
    a.off_misc = a.off_x + region;
    a.smem = a.off_misc + misc;
    return a.smem <= smem_limit;
}

cudaError_t launch_persistent(const PersistentArgs& a, cudaStream_t s) {
    const int G = a.qh / a.kvh;
    const int HG = G >= 4 ? 4 : G;
    switch (HG) {
        case 1: return launch_hg<1>(a, s);
        case 2: return launch_hg<2>(a, s);
        default: return launch_hg<4>(a, s);
    }
}

}  // namespace q3

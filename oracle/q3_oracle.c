/*
 * q3_oracle.c -- CPU restatement of the reference's Qwen3 batch-1 decode step.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load it.  The
 * product library (inference_b200/) never links, loads or calls it.
 *
 * Every function restates one operation of pind0s/inference and cites the
 * reference file:line it follows (paths relative to the reference project).
 * Arithmetic follows the reference: BF16 storage between ops, fp32 inside an
 * op, BF16 round-to-nearest-even at the end of every op.  Dot products use
 * the reference CPU backend's accumulation shape: 16 fp32 lanes, each lane
 * taking an (odd, even) BF16 pair per 32-element block the way
 * _mm512_dpbf16_ps does, then a lane sum.
 *
 * Parity of this oracle is pinned against the reference CPU backend compiled
 * from its own sources (oracle/build_ref.py -> oracle/_ref/libref_cpu.so) on
 * the golden fixtures under tests/golden/.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define Q3O_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------- bf16 */

/* bf16 -> fp32: src/lib/backend/cpu/bf16.hpp:18-20 (upper 16 bits). */
static inline float bf2f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* fp32 -> bf16, round to nearest even, NaN quieted:
 * src/lib/backend/cpu/bf16.hpp:27-41. */
static inline uint16_t f2bf(float f) {
    uint32_t bits;
    memcpy(&bits, &f, 4);
    if ((bits & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((bits >> 16) | 0x0040u);
    bits += 0x7FFFu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}

Q3O_API float q3o_bf16_to_f32(uint16_t b) { return bf2f(b); }
Q3O_API uint16_t q3o_f32_to_bf16(float f) { return f2bf(f); }

/* Dot product of two BF16 vectors in the reference CPU backend's lane shape:
 * src/lib/backend/cpu/kernels/matmul.hpp:22-30 with avx.hpp:46-48
 * (_mm512_dpbf16_ps: lane j adds element 2j+1's product, then element 2j's)
 * and avx.hpp:59-61 (horizontal add of the 16 lanes).  n % 32 == 0 is the
 * reference's own precondition (cpu/backend.cpp:52-58); a ragged tail is
 * accumulated into lane 0 so the oracle also covers odd sizes. */
static float dot_bf16(const uint16_t* a, const uint16_t* b, size_t n) {
    float lane[16] = {0};
    size_t blocks = n / 32;
    for (size_t blk = 0; blk < blocks; ++blk) {
        const uint16_t* pa = a + blk * 32;
        const uint16_t* pb = b + blk * 32;
        for (int j = 0; j < 16; ++j) {
            lane[j] += bf2f(pa[2 * j + 1]) * bf2f(pb[2 * j + 1]);
            lane[j] += bf2f(pa[2 * j]) * bf2f(pb[2 * j]);
        }
    }
    for (size_t i = blocks * 32; i < n; ++i) lane[0] += bf2f(a[i]) * bf2f(b[i]);
    /* _mm512_reduce_add_ps halves the vector: 16 -> 8 -> 4 -> 2 -> 1. */
    for (int w = 8; w >= 1; w >>= 1)
        for (int j = 0; j < w; ++j) lane[j] = lane[j] + lane[j + w];
    return lane[0];
}

/* --------------------------------------------------- deterministic inputs */

/* SplitMix64 finaliser (Steele, Lea, Flood 2014). */
static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Synthetic N(0, 0.02) BF16 weights, bit-reproducible on any IEEE machine:
 * the sum of four 16-bit uniforms (Irwin-Hall, n = 4) from one counter hash,
 * centred and scaled to standard deviation 0.02 by a single fp32 multiply.
 * Element (r, c) of a tensor with `full_cols` columns uses counter
 * (tensor_id << 40) | (r * full_cols + c), so any row/column slice (a
 * tensor-parallel shard) reproduces the matching part of the full tensor.
 * The GPU generator (fill_normal_kernel, inference_b200/csrc/small_ops.cu)
 * computes the same bits. */
static inline uint16_t normal_bf16(uint64_t key, uint64_t tensor_id, uint64_t flat) {
    uint64_t h = mix64(key ^ ((tensor_id << 40) | flat));
    int32_t s = (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) + (int32_t)((h >> 32) & 0xFFFF) +
                (int32_t)((h >> 48) & 0xFFFF) - 131070;
    return f2bf((float)s * 0x1.1bc77ap-21f);
}

Q3O_API uint64_t q3o_seed_key(uint64_t seed) { return mix64(seed ^ 0x51A3D0F1B200ull); }

Q3O_API void q3o_fill_normal(uint16_t* dst, uint64_t seed, uint64_t tensor_id, size_t rows, size_t cols,
                             size_t row0, size_t col0, size_t full_cols) {
    uint64_t key = q3o_seed_key(seed);
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c)
            dst[r * cols + c] = normal_bf16(key, tensor_id, (uint64_t)(row0 + r) * full_cols + (col0 + c));
}

/* Prompt token ids uniform in [0, vocab): one hash per id, multiply-high. */
Q3O_API void q3o_prompt_ids(uint32_t* dst, size_t n, uint64_t seed, uint32_t vocab) {
    uint64_t key = q3o_seed_key(seed);
    for (size_t i = 0; i < n; ++i) {
        uint64_t h = mix64(key ^ (0xFFull << 56) ^ (uint64_t)i);
        dst[i] = (uint32_t)(((h >> 32) * (uint64_t)vocab) >> 32);
    }
}

/* ------------------------------------------------------------------ ops */

/* RoPE tables: src/lib/backend/util/rope_cache.hpp:23-41.  fp32 host libm,
 * inverse frequency 1/theta^(2i/head_dim), cos/sin of pos * inv_freq. */
Q3O_API void q3o_rope_cache(size_t max_pos, size_t head_dim, float theta, float* cos_out, float* sin_out) {
    size_t half = head_dim / 2;
    float* inv = (float*)malloc(half * sizeof(float));
    for (size_t i = 0; i < half; ++i) {
        float e = 2.0f * (float)i / (float)head_dim;
        inv[i] = 1.0f / powf(theta, e);
    }
    for (size_t p = 0; p < max_pos; ++p)
        for (size_t i = 0; i < half; ++i) {
            float a = (float)p * inv[i];
            cos_out[p * half + i] = cosf(a);
            sin_out[p * half + i] = sinf(a);
        }
    free(inv);
}

/* embedding: src/lib/backend/cpu/kernels/embedding.hpp:7-10 (row copy). */
Q3O_API void q3o_embedding(uint32_t token, const uint16_t* table, uint16_t* out, size_t hidden) {
    memcpy(out, table + (size_t)token * hidden, hidden * sizeof(uint16_t));
}

/* matmul (batch-1 GEMV), y[j] = sum_i x[i] W[j,i], W row-major [n_out, n_in]:
 * src/lib/backend/cpu/kernels/matmul.hpp:8-33; CUDA call site
 * src/lib/backend/cuda/kernels/matmul.cuh:8-18. */
Q3O_API void q3o_gemv(const uint16_t* x, const uint16_t* w, uint16_t* y, size_t n_out, size_t n_in) {
#pragma omp parallel for schedule(static)
    for (size_t j = 0; j < n_out; ++j) y[j] = f2bf(dot_bf16(x, w + j * n_in, n_in));
}

/* rmsnorm: src/lib/backend/cpu/kernels/rmsnorm.hpp:17-29 and
 * src/lib/backend/cuda/kernels/rmsnorm.cuh:12-46: out = bf16(x*scale*w),
 * scale = 1/sqrt(sum(x^2)/H + eps). */
Q3O_API void q3o_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* out, size_t hidden, float eps) {
    float ss = dot_bf16(x, x, hidden);
    float scale = 1.0f / sqrtf(ss / (float)hidden + eps);
    for (size_t i = 0; i < hidden; ++i) out[i] = f2bf(bf2f(x[i]) * scale * bf2f(w[i]));
}

/* rmsnorm_add: src/lib/backend/cpu/kernels/rmsnorm.hpp:31-46 and
 * src/lib/backend/cuda/kernels/rmsnorm.cuh:48-80.  residual = bf16(res+upd)
 * in place; the sum of squares uses the unrounded fp32 sums (both backends);
 * out = bf16(bf16(res) * scale * w).  `upd` may alias `out`. */
Q3O_API void q3o_rmsnorm_add(uint16_t* res, const uint16_t* upd, const uint16_t* w, uint16_t* out, size_t hidden,
                             float eps) {
    float lane[16] = {0};
    for (size_t i = 0; i < hidden; ++i) {
        float v = bf2f(res[i]) + bf2f(upd[i]);
        res[i] = f2bf(v);
        lane[i % 16] += v * v;
    }
    for (int s = 8; s >= 1; s >>= 1)
        for (int j = 0; j < s; ++j) lane[j] = lane[j] + lane[j + s];
    float scale = 1.0f / sqrtf(lane[0] / (float)hidden + eps);
    for (size_t i = 0; i < hidden; ++i) out[i] = f2bf(bf2f(res[i]) * scale * bf2f(w[i]));
}

static void norm_rope_head(uint16_t* v, const uint16_t* nw, size_t hd, const float* c, const float* s, float eps) {
    size_t half = hd / 2;
    float ss = dot_bf16(v, v, hd);
    float scale = 1.0f / sqrtf(ss / (float)hd + eps);
    for (size_t i = 0; i < half; ++i) {
        float x = bf2f(v[i]) * bf2f(nw[i]) * scale;
        float y = bf2f(v[half + i]) * bf2f(nw[half + i]) * scale;
        v[i] = f2bf(x * c[i] - y * s[i]);
        v[half + i] = f2bf(y * c[i] + x * s[i]);
    }
}

/* qk_norm_rope: src/lib/backend/cpu/kernels/qk_norm_rope.hpp:19-61 and
 * src/lib/backend/cuda/kernels/qk_norm_rope.cuh:14-90.  Per head: RMSNorm
 * with the q_norm/k_norm weight (not rounded), then rotate-half RoPE at
 * `pos`, BF16 in place.  cos/sin are rows of the [max_pos, hd/2] tables. */
Q3O_API void q3o_qk_norm_rope(uint16_t* q, uint16_t* k, const uint16_t* q_norm, const uint16_t* k_norm,
                              const float* cos_tab, const float* sin_tab, size_t q_heads, size_t kv_heads,
                              size_t head_dim, size_t pos, float eps) {
    const float* c = cos_tab + pos * (head_dim / 2);
    const float* s = sin_tab + pos * (head_dim / 2);
    for (size_t h = 0; h < q_heads; ++h) norm_rope_head(q + h * head_dim, q_norm, head_dim, c, s, eps);
    for (size_t h = 0; h < kv_heads; ++h) norm_rope_head(k + h * head_dim, k_norm, head_dim, c, s, eps);
}

/* self_attention over positions 0..pos with GQA head map kv = qh/(qH/kvH):
 * src/lib/backend/cpu/kernels/self_attention.hpp:12-74 (scores scaled by
 * 1/sqrt(hd), max-subtracted exp, normalised weights, fp32 weighted V sum)
 * and src/lib/backend/cuda/kernels/flash_attention.cuh:38-156.  K and V are
 * the reference KV-cache layout [capacity, kv_heads, head_dim]
 * (src/lib/kv_cache/kv_cache.hpp:16-24).  `out` may alias `q`. */
Q3O_API void q3o_attention(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, uint16_t* out,
                           size_t q_heads, size_t kv_heads, size_t head_dim, size_t pos) {
    size_t group = q_heads / kv_heads;
    float scale = 1.0f / sqrtf((float)head_dim);
    size_t n = pos + 1;
    uint16_t* result = (uint16_t*)malloc(q_heads * head_dim * sizeof(uint16_t));
#pragma omp parallel for schedule(static)
    for (size_t h = 0; h < q_heads; ++h) {
        size_t kvh = h / group;
        float* sc = (float*)malloc(n * sizeof(float));
        float mx = -INFINITY;
        for (size_t t = 0; t < n; ++t) {
            sc[t] = dot_bf16(q + h * head_dim, kc + (t * kv_heads + kvh) * head_dim, head_dim) * scale;
            if (sc[t] > mx) mx = sc[t];
        }
        float sum = 0.0f;
        for (size_t t = 0; t < n; ++t) {
            sc[t] = expf(sc[t] - mx);
            sum += sc[t];
        }
        for (size_t d = 0; d < head_dim; ++d) {
            float acc = 0.0f;
            for (size_t t = 0; t < n; ++t) acc += bf2f(vc[(t * kv_heads + kvh) * head_dim + d]) * (sc[t] / sum);
            result[h * head_dim + d] = f2bf(acc);
        }
        free(sc);
    }
    memcpy(out, result, q_heads * head_dim * sizeof(uint16_t));
    free(result);
}

/* silu: src/lib/backend/cpu/kernels/silu.hpp:6-13 and
 * src/lib/backend/cuda/kernels/silu.cuh:9-32: bf16(g/(1+exp(-g)) * u). */
Q3O_API void q3o_silu(const uint16_t* gate, const uint16_t* up, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float g = bf2f(gate[i]);
        out[i] = f2bf(g / (1.0f + expf(-g)) * bf2f(up[i]));
    }
}

/* add: src/lib/backend/cpu/kernels/add.hpp:6-19, cuda/kernels/add.cuh:10-31. */
Q3O_API void q3o_add(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = f2bf(bf2f(a[i]) + bf2f(b[i]));
}

/* argmax, first index of the largest BF16 value:
 * testing/reference/sampling.hpp:7-17, cpu/kernels/sampling.hpp:10-41,
 * cuda/backend.cu:107-112 (thrust::max_element keeps the first maximum). */
Q3O_API uint32_t q3o_argmax(const uint16_t* logits, size_t n) {
    size_t best = 0;
    for (size_t i = 1; i < n; ++i)
        if (bf2f(logits[i]) > bf2f(logits[best])) best = i;
    return (uint32_t)best;
}

/* ---------------------------------------------------------------- FP8 weights
 * (the build's optional weight format; no reference counterpart: the
 * reference runs BF16 weights only, README.md:13).  OCP FP8 E4M3: 1 sign,
 * 4 exponent bits (bias 7), 3 mantissa bits, subnormals down to 2^-9, no
 * infinities, largest finite 448.  Encoding rounds to nearest, ties to even,
 * and saturates to +-448 (the PTX cvt.rn.satfinite.e4m3x2.f32 semantics).
 * Each weight row r gets a power-of-two scale 2^e_r, e_r the smallest integer
 * with max|w_r| <= 448 * 2^e_r, so every dequantized weight q * 2^e_r has at
 * most four significant bits and is exactly a BF16 value. */
Q3O_API uint8_t q3o_e4m3(float x) {
    const uint8_t s = signbit(x) ? 0x80 : 0x00;
    if (isnan(x)) return (uint8_t)(s | 0x7F);
    const float a = fabsf(x);
    if (a > 448.0f) return (uint8_t)(s | 0x7E);
    if (a < 0.015625f) {                             /* below 2^-6: subnormal steps of 2^-9 */
        const int q = (int)nearbyintf(ldexpf(a, 9));  /* 0..8; 8 is the smallest normal, code 0x08 */
        return (uint8_t)(s | q);
    }
    int e2;
    frexpf(a, &e2);
    int E = e2 - 1;                                  /* a = 1.f * 2^E, E >= -6 */
    int m = (int)nearbyintf((ldexpf(a, -E) - 1.0f) * 8.0f);
    if (m == 8) {
        m = 0;
        ++E;
    }
    return (uint8_t)(s | ((E + 7) << 3) | m);
}

Q3O_API float q3o_e4m3_value(uint8_t q) {
    const int E = (q >> 3) & 0xF, m = q & 7;
    float v = E ? ldexpf(1.0f + m / 8.0f, E - 7) : ldexpf((float)m, -9);
    if ((q & 0x7F) == 0x7F) v = NAN;
    return (q & 0x80) ? -v : v;
}

/* Row-wise E4M3 with power-of-two scales: q[rows, cols], scale[rows]. */
Q3O_API void q3o_quantize_e4m3(const uint16_t* w, size_t rows, size_t cols, uint8_t* q, float* scale) {
    for (size_t r = 0; r < rows; ++r) {
        const uint16_t* wr = w + r * cols;
        float mx = 0.0f;
        for (size_t c = 0; c < cols; ++c) mx = fmaxf(mx, fabsf(bf2f(wr[c])));
        int e = 0;
        if (mx > 0.0f) {
            int k;
            const float f = frexpf(mx, &k);          /* mx = f * 2^k, 448 = 0.875 * 2^9 */
            e = (f <= 0.875f) ? k - 9 : k - 8;
        }
        scale[r] = ldexpf(1.0f, e);
        for (size_t c = 0; c < cols; ++c) q[r * cols + c] = q3o_e4m3(ldexpf(bf2f(wr[c]), -e));
    }
}

/* In place: w <- bf16(dequant(quant(w))) (exact, see above). */
static void fp8_roundtrip(uint16_t* w, size_t rows, size_t cols) {
    uint8_t* q = (uint8_t*)malloc(cols);
    float sc;
    for (size_t r = 0; r < rows; ++r) {
        q3o_quantize_e4m3(w + r * cols, 1, cols, q, &sc);
        for (size_t c = 0; c < cols; ++c) w[r * cols + c] = f2bf(q3o_e4m3_value(q[c]) * sc);
    }
    free(q);
}

/* ---------------------------------------------------------------- NVFP4 weights
 * (the build's 4-bit weight format; no reference counterpart).  E2M1 values
 * (1 sign, 2 exponent, 1 mantissa bit: 0, 0.5, 1, 1.5, 2, 3, 4, 6) with one
 * E4M3 scale per block of 16 consecutive columns, and per row a power-of-two
 * scale 2^e_r, e_r the smallest integer with max|w_r| / 6 <= 448 * 2^e_r (so
 * every block scale fits E4M3).  Block b of row r: code = E4M3(amax_b / 6 *
 * 2^-e_r) (nearest, ties to even, the FP8 encoder above), s = its value; each
 * weight w -> E2M1(w * 2^-e_r / s) (nearest, ties to even, saturating at
 * +-6; 0 when s is 0).  A dequantized weight E2M1 * s * 2^e_r has at most six
 * significant bits: exactly a BF16 value. */
Q3O_API uint8_t q3o_e2m1(float x) {
    const uint8_t s = signbit(x) ? 0x8 : 0x0;
    const float a = fabsf(x);
    uint8_t c;
    if (a <= 0.25f) c = 0;          /* the ties go to the even code */
    else if (a < 0.75f) c = 1;
    else if (a <= 1.25f) c = 2;
    else if (a < 1.75f) c = 3;
    else if (a <= 2.5f) c = 4;
    else if (a < 3.5f) c = 5;
    else if (a <= 5.0f) c = 6;
    else c = 7;                     /* 6, saturating */
    return (uint8_t)(s | c);
}

Q3O_API float q3o_e2m1_value(uint8_t q) {
    static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    const float v = mag[q & 7];
    return (q & 8) ? -v : v;
}

/* Row r: q[r, c] E2M1 codes (one per byte), bscale[r, c / 16] E4M3 codes,
 * rscale[r] = 2^e_r.  cols % 16 == 0. */
Q3O_API void q3o_quantize_nvfp4(const uint16_t* w, size_t rows, size_t cols, uint8_t* q, uint8_t* bscale,
                                float* rscale) {
    for (size_t r = 0; r < rows; ++r) {
        const uint16_t* wr = w + r * cols;
        float mx = 0.0f;
        for (size_t c = 0; c < cols; ++c) mx = fmaxf(mx, fabsf(bf2f(wr[c])));
        int e = 0;
        if (mx > 0.0f) {
            int k;
            const float f = frexpf(mx, &k);          /* mx = f * 2^k; 6 * 448 = 2688 = 0.65625 * 2^12 */
            e = (f <= 0.65625f) ? k - 12 : k - 11;
        }
        rscale[r] = ldexpf(1.0f, e);
        for (size_t b = 0; b < cols / 16; ++b) {
            float amax = 0.0f;
            for (size_t j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(bf2f(wr[16 * b + j])));
            const uint8_t sc = q3o_e4m3(ldexpf(amax / 6.0f, -e));
            const float sv = q3o_e4m3_value(sc);
            bscale[r * (cols / 16) + b] = sc;
            for (size_t j = 0; j < 16; ++j) {
                const float x = bf2f(wr[16 * b + j]);
                q[r * cols + 16 * b + j] = sv > 0.0f ? q3o_e2m1(ldexpf(x, -e) / sv) : (uint8_t)(signbit(x) ? 8 : 0);
            }
        }
    }
}

/* In place: w <- bf16(dequant(quant(w))) (exact, see above). */
static void nvfp4_roundtrip(uint16_t* w, size_t rows, size_t cols) {
    uint8_t* q = (uint8_t*)malloc(cols);
    uint8_t* bs = (uint8_t*)malloc(cols / 16);
    float rs;
    for (size_t r = 0; r < rows; ++r) {
        q3o_quantize_nvfp4(w + r * cols, 1, cols, q, bs, &rs);
        for (size_t c = 0; c < cols; ++c)
            w[r * cols + c] = f2bf(q3o_e2m1_value(q[c]) * q3o_e4m3_value(bs[c / 16]) * rs);
    }
    free(q);
    free(bs);
}

/* ---------------------------------------------------------------- model */

typedef struct {
    size_t hidden, inter, layers, q_heads, kv_heads, head_dim, vocab, capacity;
    float eps, theta;
    int tied;
} q3o_config;

typedef struct {
    uint16_t *q_proj, *k_proj, *v_proj, *o_proj, *gate, *up, *down;
    uint16_t *in_norm, *post_norm, *q_norm, *k_norm;
} q3o_layer;

typedef struct {
    q3o_config cfg;
    uint16_t *embed, *lm_head, *final_norm;
    q3o_layer* layer;
    uint16_t **kcache, **vcache; /* per layer [capacity, kv_heads, head_dim] */
    float *cos_tab, *sin_tab;
    uint16_t *hs, *hidden, *query, *gate_buf, *up_buf, *logits;
    size_t token_count;
} q3o_model;

/* Tensor ids of the synthetic weight generator.  Layer l uses
 * 16 + 16*l + {0..6} for q, k, v, o, gate, up, down. */
enum { Q3_TID_EMBED = 1, Q3_TID_LM_HEAD = 2, Q3_TID_LAYER0 = 16 };

static uint16_t* ones(size_t n) {
    uint16_t* p = (uint16_t*)malloc(n * 2);
    for (size_t i = 0; i < n; ++i) p[i] = 0x3F80; /* 1.0 */
    return p;
}

static uint16_t* rand_mat(uint64_t seed, uint64_t tid, size_t rows, size_t cols) {
    uint16_t* p = (uint16_t*)malloc(rows * cols * 2);
    q3o_fill_normal(p, seed, tid, rows, cols, 0, 0, cols);
    return p;
}

/* Model::build (src/lib/model/qwen3/qwen3.hpp:105-128) over synthetic
 * weights; KVCache (src/lib/kv_cache/kv_cache.hpp:16-24); rope cache sized to
 * the context (qwen3.hpp:125). */
Q3O_API q3o_model* q3o_model_create(const q3o_config* cfg, uint64_t seed) {
    q3o_model* m = (q3o_model*)calloc(1, sizeof(q3o_model));
    m->cfg = *cfg;
    size_t H = cfg->hidden, I = cfg->inter, hd = cfg->head_dim;
    size_t qd = cfg->q_heads * hd, kd = cfg->kv_heads * hd;
    m->embed = rand_mat(seed, Q3_TID_EMBED, cfg->vocab, H);
    m->lm_head = cfg->tied ? m->embed : rand_mat(seed, Q3_TID_LM_HEAD, cfg->vocab, H);
    m->final_norm = ones(H);
    m->layer = (q3o_layer*)calloc(cfg->layers, sizeof(q3o_layer));
    m->kcache = (uint16_t**)calloc(cfg->layers, sizeof(uint16_t*));
    m->vcache = (uint16_t**)calloc(cfg->layers, sizeof(uint16_t*));
    for (size_t l = 0; l < cfg->layers; ++l) {
        uint64_t b = Q3_TID_LAYER0 + 16 * l;
        q3o_layer* L = &m->layer[l];
        L->q_proj = rand_mat(seed, b + 0, qd, H);
        L->k_proj = rand_mat(seed, b + 1, kd, H);
        L->v_proj = rand_mat(seed, b + 2, kd, H);
        L->o_proj = rand_mat(seed, b + 3, H, qd);
        L->gate = rand_mat(seed, b + 4, I, H);
        L->up = rand_mat(seed, b + 5, I, H);
        L->down = rand_mat(seed, b + 6, H, I);
        L->in_norm = ones(H);
        L->post_norm = ones(H);
        L->q_norm = ones(hd);
        L->k_norm = ones(hd);
        m->kcache[l] = (uint16_t*)calloc(cfg->capacity * kd, 2);
        m->vcache[l] = (uint16_t*)calloc(cfg->capacity * kd, 2);
    }
    m->cos_tab = (float*)malloc(cfg->capacity * hd / 2 * sizeof(float));
    m->sin_tab = (float*)malloc(cfg->capacity * hd / 2 * sizeof(float));
    q3o_rope_cache(cfg->capacity, hd, cfg->theta, m->cos_tab, m->sin_tab);
    m->hs = (uint16_t*)calloc(H, 2);
    m->hidden = (uint16_t*)calloc(H, 2);
    m->query = (uint16_t*)calloc(qd, 2);
    m->gate_buf = (uint16_t*)calloc(I, 2);
    m->up_buf = (uint16_t*)calloc(I, 2);
    m->logits = (uint16_t*)calloc(cfg->vocab, 2);
    return m;
}

/* The model an FP8-weight engine computes: every GEMV matrix (q, k, v, o,
 * gate, up, down, lm_head) replaced by its E4M3 round trip; the embedding
 * lookup keeps the BF16 table (a tied model gets its own lm_head copy). */
Q3O_API void q3o_model_quantize_fp8(q3o_model* m) {
    const q3o_config* c = &m->cfg;
    size_t H = c->hidden, I = c->inter, hd = c->head_dim;
    size_t qd = c->q_heads * hd, kd = c->kv_heads * hd;
    if (m->lm_head == m->embed) {
        m->lm_head = (uint16_t*)malloc(c->vocab * H * 2);
        memcpy(m->lm_head, m->embed, c->vocab * H * 2);
    }
    fp8_roundtrip(m->lm_head, c->vocab, H);
    for (size_t l = 0; l < c->layers; ++l) {
        q3o_layer* L = &m->layer[l];
        fp8_roundtrip(L->q_proj, qd, H);
        fp8_roundtrip(L->k_proj, kd, H);
        fp8_roundtrip(L->v_proj, kd, H);
        fp8_roundtrip(L->o_proj, H, qd);
        fp8_roundtrip(L->gate, I, H);
        fp8_roundtrip(L->up, I, H);
        fp8_roundtrip(L->down, H, I);
    }
}

/* The model an NVFP4-weight engine computes: every GEMV matrix replaced by its
 * NVFP4 round trip (the embedding lookup keeps the BF16 table). */
Q3O_API void q3o_model_quantize_nvfp4(q3o_model* m) {
    const q3o_config* c = &m->cfg;
    size_t H = c->hidden, I = c->inter, hd = c->head_dim;
    size_t qd = c->q_heads * hd, kd = c->kv_heads * hd;
    if (m->lm_head == m->embed) {
        m->lm_head = (uint16_t*)malloc(c->vocab * H * 2);
        memcpy(m->lm_head, m->embed, c->vocab * H * 2);
    }
    nvfp4_roundtrip(m->lm_head, c->vocab, H);
    for (size_t l = 0; l < c->layers; ++l) {
        q3o_layer* L = &m->layer[l];
        nvfp4_roundtrip(L->q_proj, qd, H);
        nvfp4_roundtrip(L->k_proj, kd, H);
        nvfp4_roundtrip(L->v_proj, kd, H);
        nvfp4_roundtrip(L->o_proj, H, qd);
        nvfp4_roundtrip(L->gate, I, H);
        nvfp4_roundtrip(L->up, I, H);
        nvfp4_roundtrip(L->down, H, I);
    }
}

Q3O_API void q3o_model_destroy(q3o_model* m) {
    if (!m) return;
    for (size_t l = 0; l < m->cfg.layers; ++l) {
        q3o_layer* L = &m->layer[l];
        free(L->q_proj); free(L->k_proj); free(L->v_proj); free(L->o_proj);
        free(L->gate); free(L->up); free(L->down);
        free(L->in_norm); free(L->post_norm); free(L->q_norm); free(L->k_norm);
        free(m->kcache[l]); free(m->vcache[l]);
    }
    if (m->lm_head != m->embed) free(m->lm_head);
    free(m->embed); free(m->final_norm); free(m->layer); free(m->kcache); free(m->vcache);
    free(m->cos_tab); free(m->sin_tab);
    free(m->hs); free(m->hidden); free(m->query); free(m->gate_buf); free(m->up_buf); free(m->logits);
    free(m);
}

/* Model::forward: src/lib/model/qwen3/qwen3.hpp:131-166, op for op. */
Q3O_API uint32_t q3o_model_forward(q3o_model* m, uint32_t token) {
    const q3o_config* c = &m->cfg;
    size_t H = c->hidden, I = c->inter, hd = c->head_dim, kd = c->kv_heads * hd, qd = c->q_heads * hd;
    size_t pos = m->token_count;
    q3o_embedding(token, m->embed, m->hs, H);
    for (size_t l = 0; l < c->layers; ++l) {
        q3o_layer* L = &m->layer[l];
        uint16_t* key = m->kcache[l] + pos * kd;
        uint16_t* value = m->vcache[l] + pos * kd;
        q3o_rmsnorm(m->hs, L->in_norm, m->hidden, H, c->eps);
        q3o_gemv(m->hidden, L->q_proj, m->query, qd, H);
        q3o_gemv(m->hidden, L->k_proj, key, kd, H);
        q3o_gemv(m->hidden, L->v_proj, value, kd, H);
        q3o_qk_norm_rope(m->query, key, L->q_norm, L->k_norm, m->cos_tab, m->sin_tab, c->q_heads, c->kv_heads, hd,
                         pos, c->eps);
        q3o_attention(m->query, m->kcache[l], m->vcache[l], m->query, c->q_heads, c->kv_heads, hd, pos);
        q3o_gemv(m->query, L->o_proj, m->hidden, H, qd);
        q3o_rmsnorm_add(m->hs, m->hidden, L->post_norm, m->hidden, H, c->eps);
        q3o_gemv(m->hidden, L->gate, m->gate_buf, I, H);
        q3o_gemv(m->hidden, L->up, m->up_buf, I, H);
        q3o_silu(m->gate_buf, m->up_buf, m->gate_buf, I);
        q3o_gemv(m->gate_buf, L->down, m->hidden, H, I);
        q3o_add(m->hs, m->hidden, m->hs, H);
    }
    q3o_rmsnorm(m->hs, m->final_norm, m->hidden, H, c->eps);
    q3o_gemv(m->hidden, m->lm_head, m->logits, c->vocab, H);
    m->token_count++;
    return q3o_argmax(m->logits, c->vocab);
}

Q3O_API const uint16_t* q3o_model_logits(q3o_model* m) { return m->logits; }
Q3O_API size_t q3o_model_token_count(q3o_model* m) { return m->token_count; }
Q3O_API void q3o_model_set_token_count(q3o_model* m, size_t n) { m->token_count = n; }
/* Copy one KV-cache slot (layer, position) as [kv_heads, head_dim] BF16. */
Q3O_API void q3o_model_kv_slot(q3o_model* m, size_t layer, size_t pos, uint16_t* k_out, uint16_t* v_out) {
    size_t kd = m->cfg.kv_heads * m->cfg.head_dim;
    memcpy(k_out, m->kcache[layer] + pos * kd, kd * 2);
    memcpy(v_out, m->vcache[layer] + pos * kd, kd * 2);
}
/* Host weight pointers, for handing identical bytes to another implementation. */
Q3O_API const uint16_t* q3o_model_weight(q3o_model* m, int layer, int which) {
    if (layer < 0) return which == 0 ? m->embed : which == 1 ? m->lm_head : m->final_norm;
    q3o_layer* L = &m->layer[layer];
    const uint16_t* t[] = {L->q_proj, L->k_proj, L->v_proj, L->o_proj, L->gate, L->up, L->down,
                           L->in_norm, L->post_norm, L->q_norm, L->k_norm};
    return (which >= 0 && which < 11) ? t[which] : NULL;
}

/*
 * q3_sm100a.h -- C ABI of the B200 (sm_100a) Qwen3 batch-1 decode library
 * (libq3_sm100a.so).
 *
 * Plain pointers and sizes only.  BF16 tensors are passed as `uint16_t*`
 * holding bfloat16 bit patterns; every pointer named *_dev is device memory.
 * Every call returns a q3_status; q3_last_error() describes the last failure
 * on the calling thread.  Streams are `cudaStream_t` passed as `void*`
 * (NULL = the legacy default stream).
 *
 * Each entry point names the reference interface it replaces
 * (pind0s/inference, paths relative to that project).
 */
#ifndef Q3_SM100A_H
#define Q3_SM100A_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define Q3_API __attribute__((visibility("default")))
#else
#define Q3_API
#endif

typedef enum q3_status {
    Q3_OK = 0,
    Q3_ERR_INVALID = 1,     /* bad shape, alignment or argument */
    Q3_ERR_CUDA = 2,        /* a CUDA runtime call failed */
    Q3_ERR_UNSUPPORTED = 3, /* valid request this build does not handle */
    Q3_ERR_OOM = 4,         /* device (or host) allocation failed */
    Q3_ERR_DEVICE = 5,      /* a kernel recorded an error (e.g. a bounded wait ran out) */
    Q3_ERR_NCCL = 6,        /* a NCCL call failed */
} q3_status;

Q3_API const char* q3_last_error(void);
Q3_API int q3_version(void);

/* ------------------------------------------------------------------------
 * Op-level entry points: one per reference Backend op
 * (src/lib/backend/backend.hpp:26-36), with the reference's semantics and the
 * aliasing it relies on (src/lib/model/qwen3/qwen3.hpp:143-159).  Shapes follow
 * the reference's tensors; all are BF16 except the fp32 RoPE tables.
 * ---------------------------------------------------------------------- */

/* Backend::embedding (backend.hpp:26; cuda/kernels/embedding.cuh:9-30):
 * out[hidden] = table[token, :]. */
Q3_API int q3_embedding(const uint16_t* table_dev, size_t vocab, size_t hidden, uint32_t token, uint16_t* out_dev,
                        void* stream);

/* Backend::matmul (backend.hpp:27; cuda/kernels/matmul.cuh:8-18 cublasGemmEx):
 * y[n_out] = W[n_out, n_in] . x[n_in], fp32 accumulation, BF16 out.
 * n_in % 8 == 0 and 16-byte aligned x, W. */
Q3_API int q3_gemv(const uint16_t* x_dev, const uint16_t* w_dev, uint16_t* y_dev, size_t n_out, size_t n_in,
                   void* stream);

/* FP8 weights (no reference counterpart; the reference stores BF16 only,
 * README.md:13).  q3_quantize_e4m3: for each of `rows` rows of w (BF16,
 * row-major [rows, full_cols]) the scale 2^e with e the smallest integer such
 * that max|row| <= 448 * 2^e goes to scale[r]; columns [c0, c0 + cols) of the
 * row go to q[r, 0..cols) as E4M3(w / 2^e), rounded to nearest even and
 * saturated at +-448.  cols, c0 even.
 * q3_gemv_e4m3: y[n_out] = (W8[n_out, n_in] . x[n_in]) * scale, W8 packed, on the tensor
 * cores (weights exact as f16, x as f16 scaled by a power of two so that
 * max|x| falls in [2^14, 2^15)), fp32 accumulation, BF16 out; n_in % 64 == 0,
 * 16-byte aligned x and W8. */
Q3_API int q3_quantize_e4m3(const uint16_t* w_dev, size_t rows, size_t full_cols, size_t c0, size_t cols,
                            uint8_t* q_dev, float* scale_dev, void* stream);
/* The FP8 GEMV reads its weights in a packed layout (16-row x 256-column
 * tiles of each CTA's row band, contiguous and bank-swizzled; it depends on
 * the device's SM count): q3_pack_e4m3 converts a row-major E4M3 matrix
 * [n_out, n_in] into it (q3_e4m3_packed_bytes(n_out, n_in) bytes, zero
 * padding included); n_in % 64 == 0. */
Q3_API size_t q3_e4m3_packed_bytes(size_t n_out, size_t n_in);
/* Byte offset of weight (row, col) in that layout for a device with num_sms
 * SMs (what q3_pack_e4m3 does on the device, for hosts that pack
 * pre-quantized weights themselves); SIZE_MAX for invalid arguments. */
Q3_API size_t q3_e4m3_packed_offset(size_t n_out, size_t n_in, int num_sms, size_t row, size_t col);
Q3_API int q3_pack_e4m3(const uint8_t* q_dev, size_t n_out, size_t n_in, uint8_t* packed_dev, void* stream);
Q3_API int q3_gemv_e4m3(const uint16_t* x_dev, const uint8_t* w8_dev, const float* scale_dev, uint16_t* y_dev,
                        size_t n_out, size_t n_in, void* stream);

/* NVFP4 weights (Q3_WEIGHTS_NVFP4; no reference counterpart): E2M1 values,
 * an E4M3 scale per 16 columns, a power-of-two scale per row (the smallest
 * 2^e with max|row| / 6 <= 448 * 2^e); block scale E4M3(amax / 6 * 2^-e),
 * weights E2M1(w * 2^-e / scale), both round to nearest-even, saturating.
 * q3_quantize_nvfp4 writes W [n_out, n_in] (BF16, row-major) in the packed
 * layout of the NVFP4 GEMV (q3_nvfp4_packed_bytes bytes, for this device's
 * SM count) and the row scales; q3_dequant_nvfp4 gives back the exact BF16
 * values of the packed matrix; q3_gemv_nvfp4 is y = W x on it.  n_in % 64 == 0. */
Q3_API size_t q3_nvfp4_packed_bytes(size_t n_out, size_t n_in);
/* Byte offset in that layout (for num_sms SMs) of the byte holding weight
 * (row, col) -- the low nibble for an even col -- or, with scale != 0, of
 * the E4M3 scale of col's 16-column block; SIZE_MAX when out of range. */
Q3_API size_t q3_nvfp4_packed_offset(size_t n_out, size_t n_in, int num_sms, size_t row, size_t col, int scale);
Q3_API int q3_quantize_nvfp4(const uint16_t* w_dev, size_t n_out, size_t n_in, uint8_t* packed_dev,
                             float* row_scale_dev, void* stream);
Q3_API int q3_dequant_nvfp4(const uint8_t* packed_dev, const float* row_scale_dev, size_t n_out, size_t n_in,
                            uint16_t* out_dev, void* stream);
Q3_API int q3_gemv_nvfp4(const uint16_t* x_dev, const uint8_t* packed_dev, const float* row_scale_dev, uint16_t* y_dev,
                         size_t n_out, size_t n_in, void* stream);

/* Batched matmul for the prefill (no Backend counterpart: the reference
 * prefills by calling matmul once per prompt token, qwen3.hpp:168-173):
 * y[m, n] = x[m, k] . W[n, k]^T with W as stored (row-major [out, in]),
 * tcgen05 tensor cores, fp32 accumulation, BF16 out.  n % 128 == 0,
 * k % 64 == 0, 16-byte aligned pointers. */
Q3_API int q3_gemm(const uint16_t* x_dev, const uint16_t* w_dev, uint16_t* y_dev, size_t m, size_t n, size_t k,
                   void* stream);

/* Backend::rmsnorm (backend.hpp:28; cuda/kernels/rmsnorm.cuh:12-46,83-89). */
Q3_API int q3_rmsnorm(const uint16_t* x_dev, const uint16_t* w_dev, uint16_t* out_dev, size_t n, float eps,
                      void* stream);

/* Backend::rmsnorm_add (backend.hpp:29; cuda/kernels/rmsnorm.cuh:48-80,91-95):
 * res = bf16(res + upd); out = rmsnorm(res).  `upd` may alias `out`. */
Q3_API int q3_rmsnorm_add(uint16_t* res_dev, const uint16_t* upd_dev, const uint16_t* w_dev, uint16_t* out_dev,
                          size_t n, float eps, void* stream);

/* Backend::rope (backend.hpp:30; cuda/kernels/rope.cuh:10-58): rotate-half
 * RoPE in place on values[heads, head_dim] at `pos`; cos/sin are the
 * [max_pos, head_dim/2] fp32 tables of backend/util/rope_cache.hpp:23-45. */
Q3_API int q3_rope(uint16_t* values_dev, const float* cos_dev, const float* sin_dev, size_t heads, size_t head_dim,
                   size_t pos, void* stream);

/* Backend::qk_norm_rope (backend.hpp:33-34; cuda/kernels/qk_norm_rope.cuh:14-100):
 * per-head RMSNorm with q_norm / k_norm then RoPE at `pos`, in place. */
Q3_API int q3_qk_norm_rope(uint16_t* q_dev, uint16_t* k_dev, const uint16_t* q_norm_dev, const uint16_t* k_norm_dev,
                           const float* cos_dev, const float* sin_dev, size_t q_heads, size_t kv_heads,
                           size_t head_dim, size_t pos, float eps, void* stream);

/* Backend::self_attention (backend.hpp:31; cuda/backend.cu:86-95,124-134;
 * cuda/kernels/flash_attention.cuh:38-184): softmax(q K^T / sqrt(hd)) V over
 * positions 0..pos with the GQA map kv = qh / (q_heads / kv_heads).  K and V
 * use the reference KV layout [capacity, kv_heads, head_dim].  `out` may
 * alias `q`.  head_dim must be 128; q_heads / kv_heads in {1, 2, 4, 8}.
 * The KV splits merge inside a thread-block cluster through distributed
 * shared memory, so no global scratch is needed: `workspace` may be NULL
 * (q3_attention_workspace_bytes() reports the size kept for ABI stability). */
Q3_API size_t q3_attention_workspace_bytes(size_t q_heads, size_t kv_heads, size_t max_positions);
Q3_API int q3_attention(const uint16_t* q_dev, const uint16_t* k_dev, const uint16_t* v_dev, uint16_t* out_dev,
                        size_t q_heads, size_t kv_heads, size_t head_dim, size_t pos, void* workspace_dev,
                        size_t workspace_bytes, void* stream);

/* The same attention over the paged KV layout this library uses:
 * k_pages / v_pages are [num_pages, kv_heads, page_size, head_dim] and
 * page_table maps logical page -> physical page.  page_size is 64. */
Q3_API int q3_attention_paged(const uint16_t* q_dev, const uint16_t* k_pages_dev, const uint16_t* v_pages_dev,
                              const int32_t* page_table_dev, uint16_t* out_dev, size_t q_heads, size_t kv_heads,
                              size_t head_dim, size_t page_size, size_t pos, void* workspace_dev,
                              size_t workspace_bytes, void* stream);

/* Backend::add (backend.hpp:32; cuda/kernels/add.cuh:10-31); out may alias a. */
Q3_API int q3_add(const uint16_t* a_dev, const uint16_t* b_dev, uint16_t* out_dev, size_t n, void* stream);

/* Backend::silu (backend.hpp:33; cuda/kernels/silu.cuh:9-32):
 * out = bf16(g / (1 + exp(-g)) * u); out may alias gate. */
Q3_API int q3_silu_mul(const uint16_t* gate_dev, const uint16_t* up_dev, uint16_t* out_dev, size_t n, void* stream);

/* Backend::argmax (backend.hpp:35; cuda/backend.cu:107-112 thrust::max_element):
 * first index of the largest BF16 logit, written to *index_dev. */
Q3_API int q3_argmax(const uint16_t* logits_dev, size_t n, uint32_t* index_dev, void* stream);

/* q3_argmax without any device allocation (no counterpart in the reference).
 * For callers that must not let the library allocate: serving runtimes that
 * plan all device memory themselves and hand libraries only buffers they own,
 * latency-critical loops that cannot take cudaMalloc's implicit
 * synchronisation.  Its scratch is a 32 KB array compiled into the library
 * (kept by every GPU that loads it until the process exits), so n is limited
 * to 16,777,216 logits; larger inputs return Q3_ERR_INVALID.  The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress) and
 * caches it, so do not use the library across a cudaDeviceReset of the
 * device.  Calls share the array, so calls that
 * overlap on the GPU (unordered streams) race. */
Q3_API int q3_argmax_noalloc(const uint16_t* logits_dev, size_t n, uint32_t* index_dev, void* stream);

/* make_rope_cache (src/lib/backend/util/rope_cache.hpp:23-45) on the host:
 * fp32 cos/sin tables [max_pos, head_dim/2], the same bits the engine uses. */
Q3_API int q3_rope_tables(size_t max_pos, size_t head_dim, float theta, float* cos_host, float* sin_host);

/* ------------------------------------------------------------------------
 * Synthetic inputs (no reference counterpart: the reference loads
 * safetensors).  Bit-identical to oracle/q3_oracle.c q3o_fill_normal /
 * q3o_prompt_ids on any IEEE machine.
 * ---------------------------------------------------------------------- */
Q3_API int q3_fill_normal(uint16_t* dst_dev, uint64_t seed, uint64_t tensor_id, size_t rows, size_t cols,
                          size_t row0, size_t col0, size_t full_cols, size_t dst_row_stride, void* stream);
Q3_API void q3_prompt_ids(uint32_t* dst_host, size_t n, uint64_t seed, uint32_t vocab);

/* ------------------------------------------------------------------------
 * Decode engine: Model + KVCache + Generator loop
 * (src/lib/model/qwen3/qwen3.hpp:105-173, src/lib/kv_cache/kv_cache.hpp:6-29,
 * src/lib/inference/generator.cpp:37-63), one engine per GPU / TP rank.
 * ---------------------------------------------------------------------- */
typedef struct q3_model_config {
    /* src/lib/model/qwen3/config.hpp:8-23 */
    uint32_t hidden;      /* hidden_size */
    uint32_t inter;       /* intermediate_size */
    uint32_t layers;      /* num_hidden_layers */
    uint32_t q_heads;     /* num_attention_heads */
    uint32_t kv_heads;    /* num_key_value_heads */
    uint32_t head_dim;    /* head_dim (128) */
    uint32_t vocab;       /* vocab_size */
    uint32_t tied;        /* tie_word_embeddings */
    float eps;            /* rms_norm_eps */
    float theta;          /* rope_theta */
    uint32_t capacity;    /* KV-cache capacity (context size) */
    uint32_t eos;         /* eos_token_id (used only when stop_at_eos) */
    /* Storage of the GEMV matrices (q, k, v, o, gate, up, down, lm_head):
     * Q3_WEIGHTS_BF16 (0, the reference's format) or Q3_WEIGHTS_FP8_E4M3 (1:
     * E4M3 bytes with one power-of-two scale per row, quantized on the device
     * from the BF16 tensors that init_synthetic / set_weight provide; no
     * reference counterpart), or Q3_WEIGHTS_NVFP4 (2, below).  Embedding and
     * norm weights stay BF16. */
    uint32_t weight_format;
} q3_model_config;

#define Q3_WEIGHTS_BF16 0
#define Q3_WEIGHTS_FP8_E4M3 1
/* NVFP4: E2M1 weights with an E4M3 scale per 16 columns and a power-of-two
 * scale per row (every dequantized weight an exact BF16 value), quantized on
 * the device like FP8; the GEMVs read 4.5 bits per weight. */
#define Q3_WEIGHTS_NVFP4 2

typedef struct q3_engine q3_engine;

/* Tensor-parallel placement: rank `tp_rank` of `tp_size` on CUDA device
 * `device`.  tp_size 1 needs no communicator. */
Q3_API int q3_engine_create(const q3_model_config* cfg, int device, int tp_rank, int tp_size, q3_engine** out);
/* Tensor-parallel engines: peers store into and read from this rank's
 * exchange buffer over NVLink (decode partials, and the batched prefill's
 * partial rows), so every rank calls q3_engine_sync, then the ranks meet at a
 * host barrier, before any rank destroys its engine. */
Q3_API int q3_engine_destroy(q3_engine* e);

/* Weights: synthetic N(0, 0.02) BF16 from `seed` (norm weights 1.0), each
 * rank generating its own shard of the full tensors. */
Q3_API int q3_engine_init_synthetic(q3_engine* e, uint64_t seed);

/* Weights::insert + Backend::make_tensor (src/lib/model/weights.hpp:16-37,
 * cuda/backend.cu:39-50) for one full (unsharded) tensor named as in the
 * Hugging Face checkpoint (model.layers.N.self_attn.q_proj.weight, ...).
 * The engine packs / shards it into its own layout. */
Q3_API int q3_engine_set_weight(q3_engine* e, const char* name, const uint16_t* host, size_t rows, size_t cols);

/* KVCache::reset (kv_cache.hpp:26-28) and prompt installation. */
Q3_API int q3_engine_reset(q3_engine* e);

/* Tokens: installs ids[0..n) as the forced prefix (prompt or a teacher-forced
 * sequence).  Steps at positions < n consume these ids; later steps consume
 * the greedy argmax of the previous step. */
Q3_API int q3_engine_set_tokens(q3_engine* e, const uint32_t* ids_host, size_t n);

/* Runs `n` decode steps (Model::forward each) on the engine's stream without
 * host synchronisation.  Replays one CUDA graph per step. */
Q3_API int q3_engine_step(q3_engine* e, size_t n);

/* Model::prefill (qwen3.hpp:168-173) batched: writes the K/V cache of the set
 * tokens at positions [position, position + n) -- tcgen05 GEMMs over up to
 * 512 tokens at a time instead of n decode steps -- and advances the
 * position by n.  No logits (the reference discards the prefill's).  The
 * tokens must have been given with q3_engine_set_tokens.  Tensor-parallel
 * engines run the n decode steps instead unless Q3_TUNE_TP_PREFILL is set
 * (q3_engine_set_tuning), FP8-weight engines unless Q3_TUNE_FP8_PREFILL is.
 * Asynchronous like step. */
Q3_API int q3_engine_prefill(q3_engine* e, size_t n);

/* Blocks until queued steps finish; returns Q3_ERR_DEVICE if a kernel
 * recorded an error. */
Q3_API int q3_engine_sync(q3_engine* e);

/* Model::forward(token) with a host round trip, as the reference
 * Backend-based loop does (qwen3.hpp:131-166): returns the greedy token. */
Q3_API int q3_engine_forward(q3_engine* e, uint32_t token, uint32_t* next_token);

/* Generator::generate (generator.cpp:37-63) on ids: prefill the prompt, then
 * greedy-decode until the KV cache is full (capacity - 1 positions) or
 * `max_new` tokens; EOS stops it only if stop_at_eos.  Prompt and output are
 * host arrays.  Returns the number of tokens written to out_host. */
Q3_API int q3_engine_generate(q3_engine* e, const uint32_t* prompt_host, size_t n_prompt, size_t max_new,
                              int stop_at_eos, uint32_t* out_host, size_t* n_out);

/* Moves the decode cursor (KVCache::token_count) back to `pos`, which must
 * not exceed the furthest position already computed; KV entries from `pos`
 * on are overwritten by the following steps.  Used to re-run a decode window
 * after one prefill. */
Q3_API int q3_engine_set_position(q3_engine* e, size_t pos);

/* Opt-in variants of the prefill (no counterpart in the reference), as bit
 * flags; 0, the default, prefills tensor-parallel and packed-weight engines
 * through one decode step per prompt token.
 *   Q3_TUNE_TP_PREFILL: tensor-parallel engines prefill with the batched
 *     tcgen05 GEMMs on their shards (row-parallel outputs exchanged as fp32
 *     partials).  This changes the fp32 order of the prefill's sums (GEMM
 *     instead of GEMV), exactly as the single-GPU batched prefill does;
 *   Q3_TUNE_FP8_PREFILL: FP8- and NVFP4-weight engines prefill with the
 *     batched tcgen05 GEMMs too, each matrix first expanded into a BF16
 *     scratch copy (its dequantized values are exact BF16 values, so the
 *     GEMMs see exactly the quantized model's weights).  The same change of
 *     fp32 order as above.
 * Unknown bits return Q3_ERR_INVALID. */
#define Q3_TUNE_TP_PREFILL 0x10u
#define Q3_TUNE_FP8_PREFILL 0x20u
#define Q3_TUNE_ALL 0x30u /* the lower bits are unused (invalid) */
Q3_API int q3_engine_set_tuning(q3_engine* e, uint32_t flags);
Q3_API int q3_engine_tuning(q3_engine* e, uint32_t* flags);

/* Launch timeline (tracing) of the CUDA-graph decode path: with enable = 1
 * every step records, per launch (5 per layer + lm_head) and CTA,
 * Q3_TRACE_WORDS uint64 words: [0] / [1] CTA start / end (%globaltimer ns),
 * [2] / [3] clock64 there, SM cycles of [4] start -> dependency wait
 * returned, [5] prologue (attention: q/k RMSNorm + RoPE), [6] main loop
 * (attention: the page loop), [7] epilogue (attention: warp and split merge),
 * [8] the SM id, [9] for a tensor-parallel GEMV that sums the ranks' partials
 * in its prologue the SM cycles from the dependency release until CTA thread
 * 0 held every rank's partials of its first rows, for attention the cycles
 * after its cluster barrier (toggling re-records the graph).  out_host (if
 * not NULL) receives the last step's record, [ctas][launches][Q3_TRACE_WORDS];
 * capacity counts uint64 words. */
#define Q3_TRACE_WORDS 10
Q3_API int q3_engine_trace(q3_engine* e, int enable, uint64_t* out_host, size_t capacity, size_t* n_phases,
                           size_t* n_ctas);

/* State readers (the reference keeps these as public members). */
Q3_API int q3_engine_position(q3_engine* e, size_t* pos);
Q3_API int q3_engine_logits(q3_engine* e, uint16_t* out_host);  /* this rank's vocab shard */
Q3_API int q3_engine_argmax_history(q3_engine* e, uint32_t* out_host, size_t n);
Q3_API int q3_engine_kv_slot(q3_engine* e, size_t layer, size_t pos, uint16_t* k_host, uint16_t* v_host);
Q3_API int q3_engine_fill_kv(q3_engine* e, size_t upto, uint64_t seed); /* synthetic KV for timing windows */
/* KVCache contents (kv_cache.hpp:6-29: per layer key / value [capacity,
 * kv_heads, head_dim], slot p = key.select(p)) for slots [pos0, pos0 + n) of
 * one layer, as host arrays in that layout [n][kv_heads][128] (this rank's kv
 * heads).  kv_write makes the written slots count as computed, so
 * q3_engine_set_position may move the cursor to pos0 + n: a decode can resume
 * from a KV history produced elsewhere (another engine, the reference). */
Q3_API int q3_engine_kv_read(q3_engine* e, size_t layer, size_t pos0, size_t n, uint16_t* k_host, uint16_t* v_host);
Q3_API int q3_engine_kv_write(q3_engine* e, size_t layer, size_t pos0, size_t n, const uint16_t* k_host,
                              const uint16_t* v_host);

/* Device pointers / sizes for instrumentation and tests. */
Q3_API int q3_engine_stream(q3_engine* e, void** stream);
Q3_API size_t q3_engine_weight_bytes(q3_engine* e);      /* this rank's weight bytes read per step */
Q3_API size_t q3_engine_kv_bytes_per_position(q3_engine* e);

/* Per-kernel-class timing of one eager step with CUDA events (kernel class:
 * 0 all GEMVs, 1 attention, 2 everything).  Reports total milliseconds,
 * launches and algorithmic bytes. */
Q3_API int q3_engine_profile_step(q3_engine* e, int kernel_class, double* ms, size_t* launches, double* bytes);

/* Checkpoints (the reference reads one safetensors file
 * whole, src/lib/model/safetensors.hpp:30-54): `path` is a .safetensors file,
 * a model.safetensors.index.json of a sharded checkpoint, or a directory
 * holding either.  Shards are memory-mapped and every BF16 tensor goes
 * through q3_engine_set_weight (packing and tensor-parallel sharding); the call
 * fails if a tensor is malformed, unknown or missing.  n_loaded (optional)
 * receives the number of tensors loaded. */
Q3_API int q3_engine_load_safetensors(q3_engine* e, const char* path, size_t* n_loaded);

/* The tensors of a checkpoint (same `path` forms) without loading anything
 * and without a GPU: one line per tensor, "name\tdtype\tshape\tfile\toffset\tbytes"
 * (shape as d0xd1, offset absolute in the file).  *needed receives the text
 * size including the terminating zero; out may be NULL to ask for it. */
Q3_API int q3_safetensors_list(const char* path, char* out, size_t capacity, size_t* needed);

/* Tensor parallelism through peer memory (the fast path): every rank exports
 * its exchange buffer as a CUDA IPC handle of Q3_PEER_HANDLE_BYTES bytes,
 * the handles are shared by any means (the tests use torch.distributed), and
 * every rank attaches all of them, its own included, in rank order.  The
 * o_proj / down_proj GEMVs then store their fp32 partial rows straight into
 * every rank's buffer over NVLink, each row as one 8-byte (value, tag) store;
 * the next GEMV reads every rank's rows until all carry the exchange's tag
 * (bounded; Q3_ERR_DEVICE "peer wait timed out" otherwise) and sums the
 * partials in rank order, so every rank holds the same bits.  The argmax keys
 * of lm_head travel with a flag per rank.  Replaces the two allreduces and the
 * allgather per layer that the NCCL path issues.  Requires peer access between
 * the GPUs (NVLink). */
#define Q3_PEER_HANDLE_BYTES 64
Q3_API int q3_engine_peer_handle(q3_engine* e, void* handle_out);
Q3_API int q3_engine_attach_peers(q3_engine* e, const void* handles, size_t n_ranks);

/* Tensor parallelism over NCCL: rank 0 calls q3_nccl_unique_id, the id is
 * shared by the caller (e.g. torch.distributed), then every rank attaches. */
Q3_API int q3_nccl_unique_id(void* id_out_128_bytes);
Q3_API int q3_engine_attach_nccl(q3_engine* e, const void* id_128_bytes);

/* Failure detection on the NCCL path (no counterpart in the reference, which
 * has no multi-GPU path): the communicator is created non-blocking, and every
 * host wait on the engine's stream (q3_engine_sync and the calls that read
 * state back) gives up after `seconds` plus 0.25 s per decode step queued
 * since the last wait.  A rank whose peer has gone -- exited, or never stepped
 * -- then aborts its communicator, reports Q3_ERR_NCCL instead of blocking,
 * and refuses further work; the engine can still be destroyed.  A collective
 * captured in the step graph may keep its kernel waiting on the departed peer
 * after the abort, so the process should then exit (tearing down its CUDA
 * context).  Default 60 s.  Peer-memory engines bound every wait on the device
 * instead (Q3_ERR_DEVICE "peer wait timed out", context usable). */
Q3_API int q3_engine_set_comm_timeout(q3_engine* e, double seconds);

/* ------------------------------------------------------------------------
 * Batched decode (batch > 1; the reference decodes one sequence: README.md:14).
 * Up to max_seqs sequences decode together on one engine's weights (a single-GPU
 * BF16 engine): each step is one forward of all live sequences as rows through
 * the batched tcgen05 GEMMs, with each row's own position and KV pages, then a
 * greedy argmax per row (backend.cu:107-112).  KV memory is a pool of
 * pool_pages pages of 64 positions per layer; a sequence takes
 * ceil(max_len / 64) of them when added.  Steps are asynchronous like
 * q3_engine_step; tokens / logits synchronise.
 * ---------------------------------------------------------------------- */
typedef struct q3_batch q3_batch;

/* A batch holds its own KV pages and token histories and uses the engine's
 * weights, stream and row buffers: destroy it before its engine. */
Q3_API int q3_batch_create(q3_engine* e, uint32_t max_seqs, uint32_t pool_pages, q3_batch** out);
Q3_API int q3_batch_destroy(q3_batch* b);

/* A new sequence: prompt[0..n) and room for max_len tokens in all (0 = the
 * engine's capacity).  Prefills positions [0, n - 1) (Model::prefill,
 * qwen3.hpp:168-173); the last prompt id is its first step's input.
 * Q3_ERR_INVALID "prompt does not fit in the model context" if n >= max_len;
 * Q3_ERR_OOM if the page pool is exhausted. */
Q3_API int q3_batch_add(q3_batch* b, const uint32_t* prompt, size_t n, size_t max_len, uint32_t* seq);

/* Paged-KV sharing: a new sequence continuing from `src` with the same tokens
 * so far.  Its page table references src's full pages (read-only from then on
 * for both) and holds a copy of src's partial page; its later tokens may
 * differ (q3_batch_append). */
Q3_API int q3_batch_fork(q3_batch* b, uint32_t src, uint32_t* seq);

/* Forces ids[0..n) as the sequence's next tokens after every token already
 * determined (teacher forcing); steps consume them instead of greedy picks. */
Q3_API int q3_batch_append(q3_batch* b, uint32_t seq, const uint32_t* ids, size_t n);

/* Releases the sequence's slot and its references to pages. */
Q3_API int q3_batch_release(q3_batch* b, uint32_t seq);

/* n steps of every live sequence with room for another token (a sequence stops
 * at max_len). */
Q3_API int q3_batch_step(q3_batch* b, size_t n);

/* The sequence's tokens (prompt, generated and appended); *n = their count;
 * out NULL only counts. */
Q3_API int q3_batch_tokens(q3_batch* b, uint32_t seq, uint32_t* out, size_t capacity, size_t* n);

/* The BF16 logits [vocab] of the sequence's row in the last step. */
Q3_API int q3_batch_logits(q3_batch* b, uint32_t seq, uint16_t* out);

/* The sequence's position (the index of its next input token) and the pool's
 * free pages (either pointer may be NULL; seq is ignored without position). */
Q3_API int q3_batch_info(q3_batch* b, uint32_t seq, size_t* position, size_t* free_pages);

/* ------------------------------------------------------------------------
 * Tokenizer and text generation (host code): tokenizer::Tokenizer
 * (src/lib/tokenizer/tokenizer.hpp:35-66, tokenizer.cpp:205-265) and
 * Generator::generate on text (src/lib/inference/generator.cpp:37-63).
 * Byte-level BPE of a Qwen3 tokenizer.json: added tokens, NFC, the Qwen2
 * pre-tokenizer pattern, BPE by merge rank.
 * ---------------------------------------------------------------------- */
typedef struct q3_tokenizer q3_tokenizer;

/* Tokenizer(model_path) (tokenizer.cpp:205-215): `path` is a tokenizer.json
 * or a directory holding one.  Q3_ERR_UNSUPPORTED for a model other than BPE
 * or a pre-tokenizer pattern other than Qwen2's. */
Q3_API int q3_tokenizer_load(const char* path, q3_tokenizer** out);
Q3_API int q3_tokenizer_destroy(q3_tokenizer* t);

/* Tokenizer::tokenize (tokenizer.cpp:217-235) of text[0..len) (UTF-8;
 * ill-formed bytes become U+FFFD as in the reference's ICU conversion).
 * Writes the ids to ids[0..capacity) and their count to *n_ids; ids NULL only
 * counts.  Q3_ERR_INVALID if capacity is too small. */
Q3_API int q3_tokenizer_encode(const q3_tokenizer* t, const char* text, size_t len, uint32_t* ids, size_t capacity,
                               size_t* n_ids);

/* Tokenizer::decode (tokenizer.cpp:237-265): the bytes of ids[0..n) as a
 * NUL-terminated string in out[0..capacity); *needed = its size with the NUL.
 * out NULL only sizes.  Q3_ERR_INVALID for an id outside the vocabulary. */
Q3_API int q3_tokenizer_decode(const q3_tokenizer* t, const uint32_t* ids, size_t n, char* out, size_t capacity,
                               size_t* needed);

/* Model::apply_chat_template (src/lib/model/qwen3/qwen3.hpp:97-103) into
 * out, sized like q3_tokenizer_decode. */
Q3_API int q3_chat_template(const char* prompt, size_t len, char* out, size_t capacity, size_t* needed);

/* Generator::generate (generator.cpp:37-63): chat template, tokenize, then
 * q3_engine_generate with EOS stopping and no limit but the KV cache, and the
 * response decoded.  *out receives a NUL-terminated string allocated by the
 * library (free it with q3_string_free) and *out_len its length without the
 * NUL.  Q3_ERR_INVALID ("prompt does not fit in the model context") if the
 * templated prompt has >= capacity tokens, as the reference's
 * std::length_error. */
Q3_API int q3_engine_generate_text(q3_engine* e, const q3_tokenizer* t, const char* prompt, size_t len, char** out,
                                   size_t* out_len);
Q3_API void q3_string_free(char* s);

#ifdef __cplusplus
}
#endif
#endif /* Q3_SM100A_H */

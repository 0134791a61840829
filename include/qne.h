/*
 * qne.h - C ABI of the B200 decode engine for Qwen3.5-shaped hybrid decoders.
 *
 * The model-level entry points replace the public API of the `qwen-kernels` crate
 * (`kernels/src/model.rs`, struct `Model`); the operator-level entry points replace the
 * per-kernel WGSL dispatches of `kernels/src/shaders.rs` that the crate's self-checks
 * (`kernels/src/lib.rs:513-712`) exercise. Every pointer argument of an operator-level
 * entry point is DEVICE memory unless the comment says "host"; every model-level entry
 * point takes HOST buffers.
 *
 * Status codes: 0 on success, a negative QNE_E* code on failure; qne_last_error() returns
 * the message of the last failure on the calling thread. No entry point aborts on bad input.
 * Handles are not thread-safe: one host thread drives one model (as in the reference, where one
 * inference worker owns the `Model`).
 */
#ifndef QNE_H
#define QNE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Symbols of the shared library; everything else in it is hidden. */
#if defined(__GNUC__)
#define QNE_API __attribute__((visibility("default")))
#else
#define QNE_API
#endif

typedef int32_t qne_status;

#define QNE_OK 0
#define QNE_EINVAL (-1)     /* bad argument, null handle, size out of range */
#define QNE_ERANGE_CTX (-2) /* context limit (4096 tokens) reached */
#define QNE_EFORMAT (-3)    /* index.json / weights.bin rejected by validation */
#define QNE_ECUDA (-4)      /* a CUDA call failed */
#define QNE_ETIMEOUT (-5)   /* a device wait ran past its deadline */
#define QNE_ENOSNAP (-6)    /* restore without a snapshot */
#define QNE_ENOMEM (-7)     /* device allocation failed */

/* Upper bound of the attention context, kernels/src/shaders.rs:34 (MAX_CONTEXT). */
#define QNE_MAX_CONTEXT 4096
/* Tokens per KV-cache page. */
#define QNE_PAGE_TOKENS 16

/* Weight storage kinds of one matrix. kernels/src/lib.rs:141-155 (QMat) defines QNE_Q4; the
 * other two are the f16 and group-64 kinds the B200 engine adds. */
#define QNE_KIND_F16 0   /* f16 [rows][k] row-major */
#define QNE_KIND_Q4 1    /* MatMulNBits block 32: u32 w[rows*k/8], u32 s[rows*k/64] (f16 pairs), u32 z[rows*k/256] (4-bit zp) */
#define QNE_KIND_Q4G64 2 /* group 64: u32 w[rows*k/8], f16 s[rows*k/64], f16 z[rows*k/64] */

/* GEMV epilogues, kernels/src/shaders.rs:36-43 (Epilogue). */
#define QNE_EPI_STORE 0      /* y[r] = W x */
#define QNE_EPI_ACCUMULATE 1 /* y[r] += W x (residual stream) */
#define QNE_EPI_SWIGLU 2     /* y[r] = silu(W[r] x) * W[r + rows/2] x */

typedef struct qne_model qne_model;
typedef struct qne_batch qne_batch;

/* One weight matrix in device memory; s and z are unused (NULL) for QNE_KIND_F16. */
typedef struct qne_matrix {
  int32_t kind;
  int32_t rows; /* physical rows (for SwiGLU: gate rows then up rows) */
  int32_t k;
  int32_t pad;
  const void* w;
  const void* s;
  const void* z;
} qne_matrix;

typedef struct qne_model_info {
  int32_t layers;
  int32_t hidden;
  int32_t intermediate;
  int32_t vocab;
  int32_t weight_kind;     /* kind of the layer matrices */
  int32_t embed_kind;      /* kind of the embedding / LM head */
  int32_t tied_lm_head;    /* 1 when lm_head shares the embedding's bytes */
  int32_t device;
  uint64_t weight_bytes;   /* bytes read by one decode token: every matrix once, LM head once */
  uint64_t device_bytes;   /* device memory held by the model */
} qne_model_info;

/* ---------------------------------------------------------------------------------------- */
/* Library                                                                                   */
/* ---------------------------------------------------------------------------------------- */

/* Message of the last failed call on this thread ("" if none). */
QNE_API const char* qne_last_error(void);
QNE_API const char* qne_version(void);
/* Number of kernel launches this library issued on the calling process so far. */
QNE_API uint64_t qne_kernel_launches(void);

/* ---------------------------------------------------------------------------------------- */
/* Model: kernels/src/model.rs (struct Model)                                               */
/* ---------------------------------------------------------------------------------------- */

/* Model::load, kernels/src/model.rs:171. Parses and validates index.json (host, n bytes, not
 * NUL-terminated) against weights (host, weights_len bytes) as Index::validate does
 * (kernels/src/model.rs:51-86), uploads every tensor once per (offset, bytes) pair, and builds
 * the per-token launch graph. The caller may free both host buffers after the call. Like the
 * reference, it accepts only the Qwen3.5-0.8B and -2B architectures (24 layers, attention every
 * 4th, (hidden, intermediate) (1024, 3584) or (2048, 6144), vocab 248320, rope_dim 64, theta 1e7)
 * and rejects others with QNE_EFORMAT and "unsupported model architecture: these kernels require
 * Qwen3.5-0.8B or Qwen3.5-2B". Matrices may be q4 (the reference's kind), f16 or q4g64. */
QNE_API qne_status qne_model_load(const char* index_json, size_t index_len, const void* weights,
                          size_t weights_len, int device, qne_model** out);
/* qne_model_load with flags (no counterpart in the reference). QNE_LOAD_ANY_SHAPE also accepts
 * other layer counts (1..256), attention periods, vocabularies and widths (hidden, intermediate:
 * multiples of 256 up to 8192 / 16384) with the same head geometry, e.g. small test models. */
#define QNE_LOAD_ANY_SHAPE 1u
QNE_API qne_status qne_model_load_ex(const char* index_json, size_t index_len, const void* weights,
                                     size_t weights_len, int device, uint32_t flags, qne_model** out);
QNE_API void qne_model_free(qne_model* m);
QNE_API qne_status qne_model_info_get(const qne_model* m, qne_model_info* out);
/* Runs the model's work on `cuda_stream` (a cudaStream_t of the model's device; NULL = the
 * model's own stream). */
QNE_API qne_status qne_model_set_stream(qne_model* m, void* cuda_stream);
/* Chooses how a token's work is launched: enable = 0 (the default) runs one kernel per operation
 * as kernels/src/model.rs:220-269 dispatches them, chained by programmatic dependent launch;
 * enable = 1 runs each decoder layer as one launch of a fused kernel whose phases are separated
 * by grid barriers. Both compute the same results within the logit tolerance and the same
 * greedy picks. The fused path needs one sequence, f16 weights with k % 256 == 0 and a grid of
 * two CTAs per SM; QNE_EINVAL if it is requested and not available. No counterpart in the
 * reference, whose dispatch granularity is fixed. */
QNE_API qne_status qne_model_set_fused(qne_model* m, int enable);
/* 1 if the fused layer kernels are in use. */
QNE_API int qne_model_fused(const qne_model* m);
/* Launch path of a token (no counterpart in the reference, whose dispatch list is fixed):
 * QNE_PATH_OPERATIONS = one kernel per operation (qne_model_set_fused(m, 0)), QNE_PATH_LAYERS =
 * one fused launch per layer (qne_model_set_fused(m, 1)), QNE_PATH_TOKEN = the token kernel: one
 * launch per stretch of layers between attention mixers (a kernel with one CTA per SM whose
 * producer warp streams every weight of the stretch through a shared-memory ring with bulk copies
 * while the consumer warps run the layers' phases behind grid barriers), the attention mixers as
 * their own kernel in between (13 launches per token for 24 layers). All three compute the same results within the logit tolerance. QNE_PATH_TOKEN
 * needs one sequence and f16 matrices with k % 256 == 0 and k <= 6144; QNE_EINVAL when a path is
 * not available. qne_model_path returns the current one. */
#define QNE_PATH_OPERATIONS 0
#define QNE_PATH_LAYERS 1
#define QNE_PATH_TOKEN 2
QNE_API qne_status qne_model_set_path(qne_model* m, int path);
QNE_API int qne_model_path(const qne_model* m);
/* Diagnostics of the fused path (no counterpart in the reference): with enable = 1 every fused
 * launch records, per CTA, %globaltimer stamps at its phase boundaries (slots 0-7), grid-barrier
 * arrivals (8-15) and releases (16-23) into [layer][cta][32] u64 slots, overwritten each token.
 * qne_model_phase_trace copies up to `cap` slots of the last token and reports how many were
 * written and the grid size. QNE_EINVAL if the fused path is not available or the trace is off. */
QNE_API qne_status qne_model_set_phase_trace(qne_model* m, int enable);
QNE_API qne_status qne_model_phase_trace(qne_model* m, uint64_t* out, size_t cap, size_t* n_out,
                                         size_t* ctas);
/* Test hook of the fused path's bounded waits (no counterpart in the reference): with limit_us > 0
 * every grid barrier of the fused layer kernels also waits for one arrival that never comes, with
 * a limit of limit_us microseconds (at most 2 s), so each token's first barrier wait runs out; the
 * kernels set the timeout flag in the control words and return, and the next call that reads them
 * (qne_last_token, qne_decode) fails with QNE_ETIMEOUT and clears the flag. limit_us = 0 restores
 * the normal barriers. QNE_EINVAL if the fused path is not available. */
QNE_API qne_status qne_model_test_barrier_timeout(qne_model* m, uint32_t limit_us);
/* Model::profile_token, kernels/src/model.rs:305-307 (Gpu::profile, kernels/src/lib.rs:366-396):
 * consumes one greedy token (like qne_decode of one step), launching its kernels one by one with
 * a CUDA event behind each, and reports the milliseconds summed per dispatch label ("gemv_<rows>x
 * <k>_<Store|Accumulate|SwiGlu|Argmax>", "gdn", "attention"), in label order. Writes up to `cap`
 * entries and the number of labels to *n_out. Diagnostic only: the kernels do not overlap as they
 * do in decoding, so the sum exceeds a decoded token's time. */
typedef struct qne_profile_entry {
  char label[48];
  double ms;
  uint32_t dispatches;
  uint32_t pad;
} qne_profile_entry;
QNE_API qne_status qne_profile_token(qne_model* m, qne_profile_entry* out, size_t cap, size_t* n_out);
/* Model::adapter, kernels/src/model.rs:167. */
QNE_API const char* qne_adapter(const qne_model* m);
/* Model::dispatches_per_token, kernels/src/model.rs:309. */
QNE_API size_t qne_dispatches_per_token(const qne_model* m);
/* ModelTiles::validate, kernels/src/model.rs:101-109: accepts the reference's tile-profile
 * JSON for API compatibility (the CUDA kernels choose their own shapes). */
QNE_API qne_status qne_validate_tiles(const char* tiles_json, size_t len);

/* Model::reset, kernels/src/model.rs:314: clears recurrent state, conv windows, KV cache. */
QNE_API qne_status qne_reset(qne_model* m);
/* Model::prefill, kernels/src/model.rs:324: prompt from position 0, one token per step;
 * afterwards logits hold the prediction after the last id and the greedy pick is stored. */
QNE_API qne_status qne_prefill(qne_model* m, const uint32_t* ids, uint32_t n);
/* Model::prefill_chunk, kernels/src/model.rs:349 (prefill_from / prefill_batched are
 * prefill_chunk with finish_logits = 1). Fails when start + n >= QNE_MAX_CONTEXT. The ids run
 * in 64-token chunks (tensor-core GEMMs, chunked GDN scan, causal attention over the appended
 * keys), like the reference's batched prefill list (kernels/src/model.rs:222-259); int4 decoder
 * matrices are decoded to f16 before each GEMM. Decoder matrices with k % 64 != 0 (not produced
 * by the converters) run one token per step, like qne_prefill. Afterwards the
 * control words hold (ids[n-1], start + n - 1), or with finish_logits the logits after the last
 * id and (greedy pick, start + n). */
QNE_API qne_status qne_prefill_chunk(qne_model* m, const uint32_t* ids, uint32_t n, uint32_t start,
                             int finish_logits);
/* 1 if qne_prefill_chunk runs batched chunks on this model, 0 if one token per step. */
QNE_API int qne_prefill_chunk_batched(const qne_model* m);
/* Token sampling on the device (Sampler, src/sampling.rs:30-134, the agent's sampler; the
 * reference samples on the host after reading the logits back). A sampler draws from the model's
 * current logits (after qne_step, qne_prefill or qne_prefill_chunk with finish_logits) and
 * returns only the token: greedy when temperature <= 0, else temperature + top_k (1..256 here;
 * 0 counts as 1) + top_p over the allowed tokens, drawing from the reference's xorshift64
 * generator seeded with `seed`. presence_penalty is subtracted from the logit of every token this
 * sampler already returned, except when a mask is given. Equal logits rank by lower token index.
 * Free every sampler before its model. */
typedef struct qne_sampling {
  float temperature;
  uint32_t top_k;
  float top_p;
  uint64_t seed;
  float presence_penalty;
} qne_sampling;
typedef struct qne_sampler qne_sampler;
QNE_API qne_status qne_sampler_create(qne_model* m, const qne_sampling* opts, qne_sampler** out);
QNE_API void qne_sampler_free(qne_sampler* s);
/* Sampler::try_sample (src/sampling.rs:58-67) with the agent's tool-call bias
 * (agent/src/session.rs:400-404): `bias` is added to logit `bias_token` first (bias 0: none).
 * mask (host, optional): bit (i % 32) of word i / 32 allows token i; tokens at or past
 * mask_tokens are not allowed. Fails with QNE_EINVAL and the reference's messages ("non-finite
 * model logits", "no finite token is allowed by the sampling mask"); a failed draw leaves the
 * generator where it was. */
QNE_API qne_status qne_sampler_sample(qne_sampler* s, const uint32_t* mask, uint32_t mask_tokens, int32_t bias_token,
                              float bias, uint32_t* token_out);
/* The same draw from `logits` (DEVICE, vocab floats of the sampler's model) instead of the
 * model's own logits (operator level: sampling any row, e.g. one sequence of a batch). */
QNE_API qne_status qne_sampler_sample_device(qne_sampler* s, const float* logits, const uint32_t* mask,
                                     uint32_t mask_tokens, int32_t bias_token, float bias, uint32_t* token_out);
/* qne_step (no logits copied to the host) followed by qne_sampler_sample: the agent's per-token
 * loop (agent/src/session.rs:390-420) with 8 bytes of readback instead of vocab floats. */
QNE_API qne_status qne_step_sample(qne_model* m, qne_sampler* s, uint32_t token, uint32_t pos, const uint32_t* mask,
                           uint32_t mask_tokens, int32_t bias_token, float bias, uint32_t* token_out);
/* Model::logits, kernels/src/model.rs:374: copies vocab f32 logits to host `out`. */
QNE_API qne_status qne_logits(qne_model* m, float* out, size_t out_len);
/* Model::step, kernels/src/model.rs:380: feeds `token` at `pos`, returns the next-token logits
 * in host `logits_out` (vocab floats). The stored greedy pick is not updated. */
QNE_API qne_status qne_step(qne_model* m, uint32_t token, uint32_t pos, float* logits_out,
                    size_t out_len);
/* Model::snapshot / restore, kernels/src/model.rs:395-414. */
QNE_API qne_status qne_snapshot(qne_model* m);
QNE_API qne_status qne_restore(qne_model* m);
/* Model::last_token, kernels/src/model.rs:417: greedy pick and next position. */
QNE_API qne_status qne_last_token(qne_model* m, uint32_t* token, uint32_t* pos);
/* Model::decode, kernels/src/model.rs:426: greedy decoding, `window` tokens per host sync;
 * ids_out (host, capacity n) receives the first pick then one id per step (UINT32_MAX inside
 * windows > 1, as in the reference); stops after a stop id. */
QNE_API qne_status qne_decode(qne_model* m, uint32_t n, uint32_t window, const uint32_t* stop,
                      uint32_t nstop, uint32_t* ids_out, uint32_t* n_out);
/* Enqueues `steps` greedy decode steps on the model's stream and returns without waiting
 * (device-resident loop; used to time the engine). Fails if the context would overflow. */
QNE_API qne_status qne_decode_async(qne_model* m, uint32_t steps);
/* Enqueues one host-token step (Model::step without the readback). */
QNE_API qne_status qne_step_async(qne_model* m, uint32_t token, uint32_t pos);
/* Waits for the model's stream, polling with a deadline (QNE_ETIMEOUT after timeout_ms). */
QNE_API qne_status qne_sync(qne_model* m, uint32_t timeout_ms);
/* Device descriptor of a loaded matrix: "embed", "lm_head" or "layer<i>.<mixer_in|mixer_out|
 * gate_up|down>" (the index.json names). */
QNE_API qne_status qne_model_matrix(const qne_model* m, const char* name, qne_matrix* out);
/* Device pointer of a loaded f32 vector: "final_norm", "layer<i>.<input_norm|post_norm|
 * attn_norms|conv_w|gdn_params>". */
QNE_API qne_status qne_model_tensor(const qne_model* m, const char* name, const void** out);
/* Device pointer of the f32 logits buffer (vocab floats). */
QNE_API const float* qne_logits_device(const qne_model* m);

/* ---------------------------------------------------------------------------------------- */
/* Batched decode: independent sequences sharing one weight copy                            */
/* ---------------------------------------------------------------------------------------- */

/* Creates `batch` (1..32) independent sequences, each with its own GDN states and a page table
 * of QNE_MAX_CONTEXT / QNE_PAGE_TOKENS entries into a shared pool of `pool_pages` pages per
 * attention layer (pool_pages >= batch * 256). The default page table maps sequence b's
 * logical page i to physical page b * 256 + i. f16 and int4 weights (an int4 matrix is decoded
 * to an f16 scratch, sized for the largest one, before each of its GEMMs). */
QNE_API qne_status qne_batch_create(qne_model* m, uint32_t batch, uint32_t pool_pages, qne_batch** out);
QNE_API void qne_batch_free(qne_batch* b);
/* Replaces the page tables (host, batch x 256 entries, each < pool_pages). */
QNE_API qne_status qne_batch_set_page_table(qne_batch* b, const uint32_t* table, size_t n);
QNE_API qne_status qne_batch_reset(qne_batch* b);
/* One decode step for every sequence: tokens[i] at pos[i] (host arrays of `batch`).
 * logits_out (host, batch x vocab) and next_out (host, batch greedy picks) may be NULL.
 * Afterwards sequence i stands at (its greedy pick, pos[i] + 1), so qne_batch_decode_async
 * continues from there. */
QNE_API qne_status qne_batch_step(qne_batch* b, const uint32_t* tokens, const uint32_t* pos,
                          float* logits_out, uint32_t* next_out);
/* Enqueues `steps` greedy steps for all sequences (each feeds back its own pick). */
QNE_API qne_status qne_batch_decode_async(qne_batch* b, uint32_t steps);
/* Copies the current (token, pos) pairs to host arrays of `batch`. */
QNE_API qne_status qne_batch_tokens(qne_batch* b, uint32_t* tokens, uint32_t* pos);
/* Writes synthetic history into sequence `seq` for positions [0, len): K/V pages filled from
 * (seed) and GDN states and conv windows from (seed); sets (token, pos) = (token, len). Used by
 * throughput runs whose prompts would take minutes to prefill. */
QNE_API qne_status qne_batch_fill_synthetic(qne_batch* b, uint32_t seq, uint32_t len, uint32_t token,
                                    uint64_t seed);
QNE_API qne_status qne_batch_sync(qne_batch* b, uint32_t timeout_ms);

/* ---------------------------------------------------------------------------------------- */
/* Operators (device pointers; `stream` is a cudaStream_t or NULL for the legacy stream)     */
/* ---------------------------------------------------------------------------------------- */

/* gemv / gemv_f16 / gemv_split_f16 + split_reduce, kernels/src/shaders.rs:48-376:
 * y (= / += / silu-gated) W x for one f32 vector x[k]. For QNE_EPI_SWIGLU, m->rows is the
 * physical row count and y has m->rows / 2 entries. */
QNE_API qne_status qne_gemv(const qne_matrix* m, const float* x, float* y, int epilogue, void* stream);
/* qne_gemv with an explicit kernel variant (the counterpart of the reference's per-matrix Tile
 * choice, kernels/src/lib.rs:39-64): 0 = automatic (f16: pipelined register streaming with
 * rows dealt over all warps; int4: the tensor-core kernel when k % 128 == 0, else the register
 * pipeline), 1 = row-group register streaming, 2 = bulk-copy (TMA) shared-memory ring with a
 * producer warp per CTA (f16, k % 256 == 0, k <= 6144, k <= 4096 for SwiGLU), 3 = tensor-core
 * int4 kernel (int4, k % 128 == 0: mma.sync on nibbles widened in registers, the warp's share of
 * weights, scales and zero points loaded before the dependency wait), 4 = int4 register pipeline
 * (CUDA-core dot products, k % 256 == 0, k <= 8192, 4096 with SwiGLU). ctas_per_sm (1 or 2)
 * sizes the grid of variant 1. */
QNE_API qne_status qne_gemv_ex(const qne_matrix* m, const float* x, float* y, int epilogue, int variant,
                               int ctas_per_sm, void* stream);
/* rmsnorm_width (kernels/src/shaders.rs:380-403) fused in front of the GEMV:
 * x = h * rsqrt(mean(h^2) + eps) * norm_w. */
QNE_API qne_status qne_rmsnorm_gemv(const qne_matrix* m, const float* h, const float* norm_w, float eps,
                            float* y, int epilogue, void* stream);
/* Batched GEMV/GEMM over `batch` (1..64) f32 vectors x[batch][k] -> y[batch][out_rows]. Uses the
 * tensor cores for batch >= 2. `scratch` must hold qne_gemm_scratch_bytes(m, batch) bytes.
 * f16, block-32 int4 (k % 256 == 0) and group-64 int4 (k % 64 == 0) weights; int4 nibbles are
 * widened to f16 ((q - zp) * scale, rounded once, the value the per-token kernels multiply) in
 * shared memory between the tensor-memory-accelerator load and the MMA. */
QNE_API size_t qne_gemm_scratch_bytes(const qne_matrix* m, int batch);
QNE_API qne_status qne_gemm(const qne_matrix* m, const float* x, int batch, float* y, int epilogue,
                    void* scratch, size_t scratch_bytes, void* stream);
/* qne_gemm with the kernel chosen explicitly (no counterpart in the reference; for comparisons):
 * QNE_GEMM_TENSOR_CORE = tcgen05 MMAs with TMA-staged tiles and tensor-memory accumulators (the
 * default of qne_gemm and of the batched decode and prefill paths), QNE_GEMM_MMA_SYNC = warp-level
 * mma.sync with cp.async staging (batch 1..32). Both compute the same sums; only the f32 summation
 * order differs. */
#define QNE_GEMM_TENSOR_CORE 0
#define QNE_GEMM_MMA_SYNC 1
QNE_API qne_status qne_gemm_ex(const qne_matrix* m, const float* x, int batch, float* y, int epilogue,
                       int impl, void* stream);
/* qne_gemm without any device allocation (no counterpart in the reference, whose buffers are
 * all created at model load): the same kernels, with x's hi/lo planes and the SwiGLU
 * intermediate in one static 2 MiB device array instead of a workspace grown with cudaMalloc.
 * For callers whose device memory is fully planned or who cannot afford an allocation's
 * synchronization. batch 1..64 and f16 weights with k % 32 == 0, as qne_gemm. Rejects calls needing
 * more than 2 MiB (2*Bp*k*2 bytes, plus 2*Bp*out_rows*2 with SwiGLU; Bp = batch rounded up to 8)
 * with QNE_EINVAL. The first call on a device sets up
 * the array's address; make it before any stream capture. One array per device: overlapping
 * calls on one device race; serialize them on one stream. */
QNE_API qne_status qne_gemm_noalloc(const qne_matrix* m, const float* x, int batch, float* y, int epilogue,
                                    void* stream);
/* Dequantized rows [row0, row0 + nrows) of m into out[nrows][k] f32, through the same unpack
 * code as the GEMV (QMat layout, kernels/src/lib.rs:484-497 dequant_row). */
QNE_API qne_status qne_dequant_rows(const qne_matrix* m, int row0, int nrows, float* out, void* stream);
/* embed_width, kernels/src/shaders.rs:409-434: h = deq(E[tok[0]]). */
QNE_API qne_status qne_embed(const qne_matrix* e, const uint32_t* tok, float* h, void* stream);
/* argmax_partial + argmax_final, kernels/src/shaders.rs:636-699: tok[0] = index of the
 * largest logit (lowest index among equal maxima, NaN never wins), tok[1] += 1.
 * `scratch` must hold qne_argmax_scratch_bytes(n) bytes. */
QNE_API size_t qne_argmax_scratch_bytes(uint32_t n);
QNE_API qne_status qne_argmax(const float* logits, uint32_t n, uint32_t* tok, void* scratch,
                      size_t scratch_bytes, void* stream);

/* gdn, kernels/src/shaders.rs:445-520, for `batch` sequences. proj[batch][8224]; conv ring
 * conv[batch][4][6144] (slot (count-1)%4 receives this step's input, the three before it are the
 * window); conv_w[6144*4]; state[batch][16][128][128]; params[160] = dt_bias, A_neg_exp,
 * norm_w; counter[batch] = tokens processed including this one (read only).
 * out[batch][2048] receives the gated, normalized output (kernels/src/shaders.rs:512-516). */
QNE_API qne_status qne_gdn_step(const float* proj, float* conv, const float* conv_w, float* state,
                        const float* params, const uint32_t* counter, float* out, int batch,
                        void* stream);

/* attention, kernels/src/shaders.rs:531-633, over a paged f16 KV cache, for `batch`
 * sequences. proj[batch][5120]; norms[512] = q_norm, k_norm; RoPE angles pos * theta^(-2i/64);
 * kv: pool of `pool_pages` pages, each [2 (K,V)][2 kv heads][16 tokens][256] f16;
 * page_table[batch][256] (entries < pool_pages); pos[batch] is the current token's position
 * (its K/V are written to the cache before use). out[batch][2048].
 * `scratch` must hold qne_attention_scratch_bytes(batch) bytes, zero-filled before first use. */
QNE_API size_t qne_attention_scratch_bytes(int batch);
QNE_API qne_status qne_attention_step(const float* proj, const float* norms, double rope_theta, void* kv,
                              uint32_t pool_pages, const uint32_t* page_table, const uint32_t* pos,
                              float* out, int batch, void* scratch, size_t scratch_bytes,
                              void* stream);
/* qne_attention_step with the kernel chosen explicitly (no counterpart in the reference; for
 * comparisons): QNE_ATTN_TENSOR_CORE = scores and PV product with mma.sync (the default of
 * qne_attention_step and of every decode path except the fused layer kernels), QNE_ATTN_CUDA_CORE
 * = per-token dot products reduced across a warp. */
#define QNE_ATTN_TENSOR_CORE 0
#define QNE_ATTN_CUDA_CORE 1
QNE_API qne_status qne_attention_step_ex(const float* proj, const float* norms, double rope_theta, void* kv,
                                 uint32_t pool_pages, const uint32_t* page_table, const uint32_t* pos,
                                 float* out, int batch, void* scratch, size_t scratch_bytes, int impl,
                                 void* stream);
/* Gathers the K and V rows of positions [0, len) of one sequence through its page table into
 * contiguous out_k/out_v [2 kv heads][len][256] f16 (bit copy). */
QNE_API qne_status qne_kv_gather(const void* kv, const uint32_t* page_table, uint32_t len, void* out_k,
                         void* out_v, void* stream);

/* Dispatch-cost probe, the reference's noop kernel and dispatch_cost (kernels/src/shaders.rs:
 * 720-729, kernels/src/lib.rs:718-724): n (1..100000) launches of a one-block kernel that adds 1 to
 * y[0] (device), back to back on `stream`, timed with CUDA events; *us_per_dispatch (host)
 * receives the microseconds per launch. mode: QNE_DISPATCH_PLAIN (stream launches), _GRAPH (the
 * n launches captured as one CUDA graph, replayed once), _PDL (launches with programmatic
 * dependent launch: each kernel releases its successor, then waits for its predecessor), or
 * _GRAPH_PDL (a graph of those, how the decode step runs). Synchronizes the stream. */
#define QNE_DISPATCH_PLAIN 0
#define QNE_DISPATCH_GRAPH 1
#define QNE_DISPATCH_PDL 2
#define QNE_DISPATCH_GRAPH_PDL 3
QNE_API qne_status qne_dispatch_cost(uint32_t n, int mode, float* y, void* stream, double* us_per_dispatch);

/* Streaming-read probe, kernels/src/shaders.rs:703-717: XOR of `bytes` (multiple of 16). */
QNE_API qne_status qne_bandwidth_probe(const void* data, size_t bytes, uint32_t* sink, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* QNE_H */

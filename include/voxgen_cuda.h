/*
 * voxgen_cuda.h — C ABI of the B200 BaseLM (MiniCPM4) per-token decode step.
 *
 * This library stands in for the Vulkan half of VoxGen's BaseLM engine: the
 * `BaseLmEngine` methods in src/baselm.rs and the dispatch surface of
 * src/vulkan.rs that they record into. Every function returns an int status
 * (VG_OK = 0, negative = error); a human-readable message for the last failure
 * on a context is available from vg_last_error(). No C++ exception crosses
 * this boundary and no torch type appears in a signature.
 *
 * Threading: a vg_stream is used by one host thread at a time (the reference
 * wraps each engine in a Mutex, src/runtime.rs:177). Distinct streams, models
 * and contexts may be driven from different threads.
 *
 * Reference citations name files inside the VoxGen project (v0.7.67).
 */
#ifndef VOXGEN_CUDA_H
#define VOXGEN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define VG_OK 0
#define VG_EINVAL -1        /* bad argument (null pointer, zero size, ...)          */
#define VG_EIO -2           /* file could not be opened / read                       */
#define VG_EFORMAT -3       /* malformed GGUF (bad magic, truncated, overflow)       */
#define VG_EUNSUPPORTED -4  /* unsupported dtype / geometry / metadata               */
#define VG_ERANGE -5        /* token id outside the vocabulary, offset overflow      */
#define VG_EFULL -6         /* KV cache full (position == max_context)               */
#define VG_ECUDA -7         /* a CUDA runtime call failed                             */
#define VG_ENOMEM -8        /* device or host allocation failed                       */
#define VG_ETIMEDOUT -9     /* bounded wait expired (vg_stream_sync)                  */
#define VG_EDEVICE -10      /* a kernel reported an error through the device flag    */
#define VG_ESTATE -11       /* call on a destroyed or mismatched handle               */

/* ---- weight formats (GGML type ids, src/gguf.rs:22-33) ------------------ */
#define VG_FORMAT_AUTO 0
#define VG_FORMAT_F16 1
#define VG_FORMAT_Q8_0 8

typedef struct vg_ctx vg_ctx;
typedef struct vg_model vg_model;
typedef struct vg_stream vg_stream;

/* Model geometry and metadata; mirrors BaseLmConfig (src/baselm.rs:35-57). */
typedef struct vg_model_info {
  uint32_t context_length;
  uint32_t embedding_length;
  uint32_t block_count;
  uint32_t feed_forward_length;
  uint32_t vocab_size;
  uint32_t head_count;
  uint32_t head_count_kv;
  uint32_t head_dim;
  uint32_t kv_dim;
  uint32_t rope_original_context_length;
  float rms_epsilon;
  float rope_theta;
  float rope_scaling_factor;   /* rope_scaling_factor(), src/baselm.rs:194-205 */
  float embedding_scale;       /* raw metadata value; 0 means identity            */
  float residual_scale;
  float logit_scale;
  int32_t format;              /* VG_FORMAT_Q8_0 or VG_FORMAT_F16 (primary)       */
  int32_t tied_output;         /* 1 when the LM head is token_embd.weight         */
  int32_t rope_long_factors;   /* 1 when rope_factors_long is the active set      */
  int32_t reserved0;
  uint64_t gguf_data_bytes;    /* bytes of the GGUF data region                   */
  uint64_t layer_weight_bytes; /* GGUF bytes of every matrix read per decode step */
  uint64_t norm_weight_bytes;  /* fp32 norm weights read per decode step          */
  uint64_t device_weight_bytes;/* bytes held in HBM after the repack              */
} vg_model_info;

/* Result of one step as printed by the reference CLI (BaseLmStepResult,
 * src/baselm.rs:404-411; collect_result :1204-1231). */
typedef struct vg_top_logit {
  uint32_t token_id;
  float logit;
} vg_top_logit;

typedef struct vg_step_result {
  uint32_t position;
  uint32_t n_top;
  double final_hidden_checksum;
  double final_hidden_l2;
} vg_step_result;

/* BaseLmBenchmark, src/baselm.rs:413-421. */
typedef struct vg_benchmark_result {
  uint32_t iterations;
  uint32_t token_id;
  double mean_ms;
  double min_ms;
  double max_ms;
  double tokens_per_second;
} vg_benchmark_result;

/* ---- context ------------------------------------------------------------ */
/* Creates a context bound to one CUDA device (replaces VulkanContext::new,
 * src/vulkan.rs:284-467). */
int vg_ctx_create(int device, vg_ctx **out);
int vg_ctx_destroy(vg_ctx *ctx);
/* Message of the last failure on this context ("" if none). Never NULL. */
const char *vg_last_error(const vg_ctx *ctx);
/* Number of SMs of the context's device. */
int vg_ctx_sm_count(const vg_ctx *ctx, int *out);

/* ---- host-only GGUF inspection (no GPU needed) -------------------------- */
/* Parses the GGUF header and tensor table (gguf::load_summary,
 * src/gguf.rs:222-286), detects the primary format (primary_base_format
 * :117-133, validate_baselm :135-148) and validates the BaseLM config
 * (BaseLmConfig::from_gguf, src/baselm.rs:60-180) without the reference's
 * fixed-geometry gate (:102-113). `format` is VG_FORMAT_AUTO or the requested
 * format. On failure the message is written to err (NUL-terminated). */
int vg_gguf_inspect(const char *path, int format, vg_model_info *info,
                    char *err, size_t err_len);

/* KV-cache bytes of a session: layers * max_context * kv_dim * 2 (fp16) * 2
 * (K and V) — BaseLmConfig::kv_cache_bytes, src/baselm.rs:182-192. Host only. */
int vg_kv_cache_bytes(const vg_model_info *info, uint32_t max_context, uint64_t *bytes);
/* top_k_logits (src/baselm.rs:1295-1309): the k largest finite logits in
 * descending order; *n_out receives min(k, number of finite logits). Host only. */
int vg_top_k_logits(const float *logits, uint32_t n, uint32_t k, vg_top_logit *out,
                    uint32_t *n_out);

/* ---- model -------------------------------------------------------------- */
/* Loads, validates, repacks and uploads a BaseLM GGUF (BaseLmEngine::new,
 * src/baselm.rs:451-586 up to the upload at :472-477). Q8_0 matrices are
 * repacked into 16-byte aligned row records for 128-bit / bulk-copy loads. */
int vg_model_load_gguf(vg_ctx *ctx, const char *path, int format, vg_model **out);
int vg_model_info_get(const vg_model *model, vg_model_info *info);
int vg_model_destroy(vg_model *model);

/* ---- stream (one decode session: KV cache, activations, CUDA graphs) ---- */
/* max_context plays the role of --max-context (checked as in
 * BaseLmConfig::from_gguf, src/baselm.rs:67-72). */
int vg_stream_create(vg_model *model, uint32_t max_context, vg_stream **out);
int vg_stream_destroy(vg_stream *stream);
/* Rewinds to position 0 without clearing the cache (BaseLmEngine::reset,
 * src/baselm.rs:616-620). */
int vg_stream_reset(vg_stream *stream);
int vg_stream_position(const vg_stream *stream, uint32_t *position);
/* Moves the decode position to `position` (<= max_context) without touching
 * the cache: the next step attends over rows [0, position] and writes row
 * `position`, whatever rows [0, position) hold. vg_stream_reset is
 * vg_stream_seek(stream, 0) (BaseLmEngine::reset, src/baselm.rs:616-620);
 * other positions serve callers that restore a session whose cache they kept,
 * and benchmarks that time steps at chosen context lengths. */
int vg_stream_seek(vg_stream *stream, uint32_t position);
/* Wall-clock limit of every bounded wait inside this stream's kernels (grid
 * barriers, bulk-copy barriers, attention merge counters), in nanoseconds; 0
 * restores the default of 2 s. A wait that runs out sets a bit in the stream's
 * device error flag and the kernel leaves; the next vg_stream_sync or output
 * copy returns VG_EDEVICE. Enqueued on the stream: it applies to later steps.
 * The reference's fence wait has no limit (src/vulkan.rs:653). */
int vg_stream_set_wait_limit(vg_stream *stream, uint64_t limit_ns);
/* How this stream runs a decode step: 1 = one persistent cooperative kernel
 * per token (all layers, grid barriers between phases), 0 = one kernel per
 * projection / attention / norm (the program the reference records,
 * record_transformer, src/baselm.rs:892-1052). Chosen at vg_stream_create:
 * the persistent kernel needs one weight format for all projections and
 * cooperative launch; the environment variable VOXGEN_STEP_KERNEL=0 selects
 * the per-kernel program, and VOXGEN_STEP_KERNEL=1 makes vg_stream_create
 * fail with VG_EUNSUPPORTED (and the reason) when the persistent kernel
 * cannot be used. */
int vg_stream_kernel_mode(const vg_stream *stream, int *mode);
/* The cudaStream_t every call of this stream is enqueued on. */
int vg_stream_cuda_stream(const vg_stream *stream, void **cuda_stream);
/* Writes fp16 K and V for positions [0, n_positions) of every layer from host
 * arrays laid out as the reference cache, kv[(layer*n_positions + pos)*kv_dim
 * + j] (store_kv.comp:21 with context = n_positions), and sets the position to
 * n_positions. Used to start a session from a prefilled context. */
int vg_stream_write_kv(vg_stream *stream, const uint16_t *k, const uint16_t *v,
                       uint32_t n_positions);
/* Reads back positions [0, n_positions) in the same layout. Synchronous. */
int vg_stream_read_kv(vg_stream *stream, uint16_t *k, uint16_t *v,
                      uint32_t n_positions);

/* One decode step at the current position, then position += 1. All decode
 * calls are asynchronous on the stream's CUDA stream; vg_stream_sync or a copy
 * call waits (bounded).
 *   vg_decode_token:            decode_token / decode_token_gpu_only
 *                               (src/baselm.rs:622-655, :689-721)
 *   vg_decode_embedding:        decode_embedding / decode_embedding_gpu_only
 *                               (:657-681, :766-789), host fp32[H] input
 *   vg_decode_embedding_device: decode_embedding_from_gpu_only (:793-821),
 *                               device fp32[H] input
 * want_logits selects compute_logits (record_transformer :1040-1050). */
int vg_decode_token(vg_stream *stream, uint32_t token, int want_logits);
int vg_decode_embedding(vg_stream *stream, const float *host_embedding,
                        int want_logits);
int vg_decode_embedding_device(vg_stream *stream, const float *device_embedding,
                               int want_logits);

/* ---- ResidualLM + FSQ + fusion (acoustic GGUF) -----------------------------
 * vg_residual_load_gguf replaces ResidualFsqEngine::new (src/acoustic.rs:
 * 435-560) with AcousticConfig::from_gguf's checks (:59-187): the acoustic
 * GGUF's residual_lm.blk.N.* layers, fsq.{in,out}_proj and
 * projections.res_fusion_proj, F16 matrices, against the BaseLM model base
 * (same heads, head_dim, FFN width and epsilon; no RoPE). The result is a
 * vg_model with no token table and no LM head: vg_stream_create gives it a
 * KV cache (max_context <= 8192), vg_stream_output its final normalised
 * hidden state, vg_stream_reset / vg_stream_position work as for BaseLM.
 *   vg_residual_step:      one position, step_record_submit / _gpu_only
 *                          (:851-900): with fsq_applied the LM state is
 *                          FSQ(base) (record_fsq :921-944), else the raw base
 *                          hidden (text prefix); the layers take
 *                          res_fusion_proj([LM state | embed]) + bias
 *                          (record_fusion :946-966; embed NULL = zeros), then
 *                          record_residual_lm (:968-1035). Device fp32[H]
 *                          inputs, read in stream order.
 *   vg_residual_step_host: the same with host inputs; returns once the step
 *                          is enqueued and the inputs are copied.
 *   vg_residual_state:     device fp32[H] buffers of the last step: the FSQ
 *                          output, the fusion output (fusion_snapshot) and the
 *                          LM state (current_lm). The buffers stay valid until
 *                          the stream is destroyed. */
enum {
  VG_RESIDUAL_FSQ_OUTPUT = 0,
  VG_RESIDUAL_FUSED_INPUT = 1,
  VG_RESIDUAL_LM_STATE = 2
};
int vg_residual_load_gguf(vg_ctx *ctx, const char *acoustic_path, const vg_model *base,
                          vg_model **out);
int vg_residual_step(vg_stream *stream, const float *device_base_hidden,
                     const float *device_embed, int fsq_applied);
int vg_residual_step_host(vg_stream *stream, const float *base_hidden, const float *embed,
                          int fsq_applied);
int vg_residual_state(const vg_stream *stream, int which, const float **device_buffer);
/* Host copy of n <= H floats of one of those buffers, after the stream's work. */
int vg_residual_copy_state(vg_stream *stream, int which, float *host, size_t n);
/* prefill_tokens (src/baselm.rs:823-839): the n tokens at positions
 * position..position+n-1, then position += n; logits of the last position
 * only when want_logits_last is set. Results are those of n decode_token
 * steps. With the persistent step kernel, runs of up to 16 positions go
 * through the batched step kernel, one weight pass per run (the reference
 * records 16 or 32 positions per command buffer, src/runtime.rs:490-522,
 * and still reads the weights once per position); the LM head then runs once,
 * on the last position. Every token and the cache room are checked before
 * anything is enqueued. */
int vg_prefill_tokens(vg_stream *stream, const uint32_t *tokens, uint32_t n,
                      int want_logits_last);

/* Device pointer of the final normalised hidden state fp32[H]
 * (output_buffer, src/baselm.rs:610-612). Valid until the stream is destroyed. */
int vg_stream_output(const vg_stream *stream, const float **device_hidden);
/* Device pointer of the logits fp32[vocab] of the last step with logits. */
int vg_stream_logits(const vg_stream *stream, const float **device_logits);
/* Waits for the stream's work (bounded) and copies n floats to host memory. */
int vg_copy_output(vg_stream *stream, float *host, size_t n);
/* The final hidden states of n streams after a batched step, stream i's first
 * n_each floats into host[i * n_each ..]: every device-to-host copy is enqueued
 * before the first wait, so a caller stepping many streams (vg_decode_batch)
 * pays one round trip instead of n. Each stream's device error flag comes back
 * with its copy and is cleared; VG_EDEVICE names the first stream that had one
 * (the other streams' outputs are still copied). No counterpart in the
 * reference, which reads each engine's result separately
 * (BaseLmEngine::collect_result, src/baselm.rs:1204-1231). */
int vg_copy_outputs(vg_stream *const *streams, int n, float *host, size_t n_each);
int vg_copy_logits(vg_stream *stream, float *host, size_t n);
/* Bounded wait for all enqueued work: VG_ETIMEDOUT after timeout_ns, and
 * VG_EDEVICE when a kernel raised the device error flag (which is cleared). */
int vg_stream_sync(vg_stream *stream, uint64_t timeout_ns);
/* collect_result (src/baselm.rs:1204-1231, top_k_logits :1295-1309): fp64
 * checksum and L2 of the output, and the top_k finite logits in descending
 * order (top may be NULL when top_k == 0). */
int vg_step_result_get(vg_stream *stream, uint32_t top_k, vg_step_result *res,
                       vg_top_logit *top);
/* BaseLmEngine::benchmark (src/baselm.rs:841-880): reset, warmup and timed
 * decode_token steps (without logits when want_logits is 0), timed with CUDA
 * events on the stream. */
int vg_benchmark(vg_stream *stream, uint32_t token, uint32_t warmup,
                 uint32_t iterations, int want_logits, vg_benchmark_result *res);

/* Per-kernel GPU timing of one decode step, the counterpart of the reference's
 * timestamp-query profiler (gpu_profile_begin/end, src/vulkan.rs:573-689, span
 * names baselm.* in src/baselm.rs:1060-1191). Runs one token step (it advances
 * the position like vg_decode_token) with every kernel launched separately and
 * bracketed by CUDA events on the stream, without graph replay or programmatic
 * overlap, and reports each launch's duration and algorithmic HBM bytes. */
typedef struct vg_kernel_time {
  char name[24];      /* embedding, qkv, attention, o_proj, gate_up, down, final_norm, logits */
  uint32_t layer;
  float ms;
  uint64_t bytes;     /* algorithmic bytes: weights + norms + KV rows read/written */
} vg_kernel_time;
int vg_stream_profile_step(vg_stream *stream, uint32_t token, int want_logits,
                           vg_kernel_time *out, uint32_t capacity, uint32_t *n_out);

/* ---- multi-stream step --------------------------------------------------- */
/* One decode step (decode_token_gpu_only semantics, no logits) for n distinct
 * streams of the same model: tokens[i] feeds streams[i] and each stream
 * advances by one position. n <= 16. Every argument is checked before any
 * stream is advanced. With n >= 2 streams on the persistent step kernel, the
 * step is one launch of the batched step kernel, which reads every weight byte
 * once for all n streams (each stream attends over its own cache, at its own
 * position); it is ordered after the work already enqueued on every stream and
 * before their later work, and runs on a CUDA stream of the model (launches
 * of one model are serialised). Otherwise each stream takes its own step on
 * its own CUDA stream. Asynchronous, like vg_decode_token. The reference
 * serialises independent engines behind a Mutex (src/runtime.rs:177). */
int vg_decode_batch(vg_stream *const *streams, int n, const uint32_t *tokens);
/* 16 when vg_decode_batch and vg_prefill_tokens can use the batched step
 * kernel for this model (one weight format for every projection, cooperative
 * launch, head_dim 32, 64 or 128, at most 8 KV heads, query width = hidden width,
 * VOXGEN_BATCH_KERNEL not 0), else 0 with the reason in vg_last_error. The
 * first call plans the kernel and allocates its workspace (about 70 MB at the
 * BaseLM backbone's shape with a 32768-position context). */
int vg_model_batch_columns(vg_model *model, uint32_t *max_columns);

/* ---- kernel-level entry points (parity tests and integration) ----------- */
/* These run one kernel on raw device pointers on the given cudaStream_t
 * (NULL = legacy default stream) and return after the launch. */

/* y[r] = alpha * sum_c W[r][c] * x[c] over a GGUF-layout matrix given as its
 * raw GGUF bytes already on the device (dtype VG_FORMAT_Q8_0 or F16, rows x
 * cols, Q8_0 blocks of 34 bytes): matvec.comp:32-62 (dispatch_matvec,
 * src/baselm.rs:1115-1153). The matrix is repacked on the device into
 * `packed` (size from vg_k_packed_bytes) before the product. */
int vg_k_packed_bytes(int dtype, uint32_t rows, uint32_t cols, uint64_t *bytes);
int vg_k_repack(int dtype, const void *gguf_bytes, uint32_t rows, uint32_t cols,
                void *packed, void *cuda_stream);
int vg_k_matvec(int dtype, const void *packed, uint32_t rows, uint32_t cols,
                const float *x, float *y, float alpha, void *cuda_stream);
/* Dequantises row `row` of a packed matrix times alpha (embedding.comp:28-47). */
int vg_k_embedding(int dtype, const void *packed, uint32_t rows, uint32_t cols,
                   uint32_t row, float alpha, float *out, void *cuda_stream);
/* hidden[i] += scale*branch[i]; y = hidden*inv_rms*w (residual_rmsnorm.comp:
 * 23-42); with branch == NULL it is rmsnorm.comp:21-42 and hidden is not
 * written. */
int vg_k_residual_rmsnorm(float *hidden, const float *branch, const float *w,
                          uint32_t n, float eps, float scale, float *y,
                          void *cuda_stream);
/* Split-K flash-decoding GQA attention over a head-major fp16 cache
 * [kv_heads][ctx][head_dim] of one layer: attn_scores.comp:27-44 +
 * softmax.comp:15-47 + attn_values.comp:25-37 over positions 0..position. */
int vg_k_attention(const float *q, const uint16_t *k_cache,
                   const uint16_t *v_cache, uint32_t heads, uint32_t kv_heads,
                   uint32_t head_dim, uint32_t ctx, uint32_t position,
                   float *out, void *cuda_stream);

/* The same attention with its scratch in a fixed device buffer that lives in
 * the library (no reference counterpart: the reference records attention into
 * a command buffer whose scratch belongs to the session). It makes no device
 * allocation and frees nothing, for callers that must not allocate: a
 * streaming thread that may not wait on the allocator (cudaMallocAsync can
 * grow and map its pool with unbounded latency), or a process that has handed
 * all free HBM to weights and KV caches, where vg_k_attention's temporary
 * allocation could fail with VG_ENOMEM in the middle of a stream.
 *
 * Scratch: VG_K_ATTENTION_NOALLOC_TICKET_BYTES of merge counters, cleared on
 * every call with cudaMemsetAsync, plus at most
 * VG_K_ATTENTION_NOALLOC_PARTIAL_BYTES of per-cluster partial results, i.e.
 *   kv_heads * ceil(ceil(ctx / 64) / 8) * (heads / kv_heads) * (head_dim + 2) * 4
 * bytes (16 heads of 128 fit a context of 64,512 positions). A larger shape,
 * or more than 1024 heads, returns VG_ERANGE before anything is enqueued.
 * The first call on a device looks the buffer's address up with
 * cudaGetSymbolAddress, which may load the library's device code: make that
 * first call outside any stream capture. The address is kept for the life of
 * the library; cudaDeviceReset on that device unloads the device code and with
 * it the buffer, so a caller that resets a device must unload and reload this
 * library before calling this entry point on that device again. There is one buffer per device, so
 * calls on one device must not overlap: calls on different streams or host
 * threads that can run at the same time race on the scratch and give wrong
 * results. Order them on one stream or synchronise between them. */
#define VG_K_ATTENTION_NOALLOC_TICKET_BYTES 4096u
#define VG_K_ATTENTION_NOALLOC_PARTIAL_BYTES (1u << 20)
int vg_k_attention_noalloc(const float *q, const uint16_t *k_cache,
                           const uint16_t *v_cache, uint32_t heads,
                           uint32_t kv_heads, uint32_t head_dim, uint32_t ctx,
                           uint32_t position, float *out, void *cuda_stream);

/* ---- failure-detection test hooks (no reference counterpart) -------------- */
/* One token step (like vg_decode_token without logits) in which every grid-
 * barrier target is one arrival beyond what the grid provides, so the first
 * barrier wait runs out after the stream's wait limit (vg_stream_set_wait_limit)
 * and the kernel leaves with kErrGridWait (0x20) in its device error flag: the
 * next vg_stream_sync returns VG_EDEVICE. The position advances, the row it
 * writes holds garbage, and the stream stays usable (the barrier counter is
 * left aligned). Nothing traps, faults or hangs. Persistent step kernel only. */
int vg_test_stalled_step(vg_stream *stream, uint32_t token);
/* Host-side fake of a failing driver call: while `status` is nonzero, every
 * bounded host wait of the library (vg_stream_sync, output copies, staging
 * waits) sees cudaEventQuery return `status` (e.g. 702, cudaErrorLaunchTimeout:
 * "kernel timed out") and fails with VG_ECUDA; 0 restores real queries. The
 * GPU work itself is not affected. Process-wide. */
int vg_test_fake_event_status(int status);

#ifdef __cplusplus
}
#endif
#endif /* VOXGEN_CUDA_H */

/*
 * mfcuda.h -- C ABI of the B200 (sm_100a) backend for the Minifield LFM2
 * runtime.
 *
 * Two tiers:
 *
 *  1. `mf_*`  The InferenceOps mirror (crates/engine-api/src/inference.rs:33-425).
 *     The backend owns every buffer; handles carry backend identity,
 *     generation, dtype, shape and allocation class.  Each call validates every
 *     operand before it enqueues any work (so a failing call never mutates an
 *     output), then enqueues on the backend's CUDA stream.  Completions are
 *     polled, never waited on by the contract (resources.rs:89-99).
 *     This is the surface a Rust `crates/backend-cuda` binds with `extern "C"`.
 *
 *  2. `mfk_*` Raw-pointer kernel entry points (device pointers, sizes, a
 *     cudaStream_t passed as void*).  No allocation, no handle checks beyond
 *     argument validation; for callers that manage device memory themselves.
 *
 * Every function returns an int32 status (mf_status; 0 = Ok).  The numbering
 * follows ExecutorError's declaration order (crates/engine-api/src/error.rs:10-28)
 * offset by one.  mf_last_error() returns the static message of the most recent
 * failure on the calling thread.
 *
 * Threading: one backend per host thread, as the reference's `!Send` backends
 * (crates/engine-api/src/backend.rs:31-34).  Multi-GPU = one backend (and one
 * process or thread) per device ordinal.
 */
#ifndef MFCUDA_H
#define MFCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MF_ABI_VERSION 1

/* crates/engine-api/src/error.rs:10-28 (+1), plus MF_PENDING for polls. */
typedef enum mf_status {
    MF_OK = 0,
    MF_INVALID_ARGUMENT = 1,
    MF_INVALID_SHAPE = 2,
    MF_INVALID_LAYOUT = 3,
    MF_INVALID_DTYPE = 4,
    MF_OVERFLOW = 5,
    MF_OUT_OF_BOUNDS = 6,
    MF_UNSUPPORTED = 7,
    MF_RESOURCE_LIMIT = 8,
    MF_WRONG_BACKEND = 9,
    MF_STALE_BUFFER = 10,
    MF_DUPLICATE_NAME = 11,
    MF_MISSING_REQUIRED_TENSOR = 12,
    MF_UNEXPECTED_TENSOR = 13,
    MF_INVALID_TIE = 14,
    MF_CANCELLED = 15,
    MF_COMPLETION_CONSUMED = 16,
    MF_BACKEND_FAILURE = 17,
    MF_PENDING = 100
} mf_status;

/* crates/engine-api/src/tensor.rs:8 (the subset this backend stores). */
typedef enum mf_dtype { MF_DTYPE_F32 = 0, MF_DTYPE_U8 = 1 } mf_dtype;

/* crates/engine-api/src/resources.rs:19-24. */
typedef enum mf_alloc_class {
    MF_CLASS_WEIGHT = 0,
    MF_CLASS_CACHE = 1,
    MF_CLASS_SCRATCH = 2,
    MF_CLASS_BRANCH = 3
} mf_alloc_class;

/* Packed formats (crates/kernels-simd/src/lib.rs:86-96). */
typedef enum mf_format { MF_TERNARY = 0, MF_NF4 = 1, MF_INT8 = 2 } mf_format;

#define MF_MAX_RANK 4

typedef struct mf_backend mf_backend;
typedef struct mf_buffer mf_buffer;
typedef struct mf_fence mf_fence;
typedef struct mf_readback mf_readback;

/* crates/engine-api/src/resources.rs:6-11. */
typedef struct mf_limits {
    uint64_t max_allocation_bytes;
    uint64_t max_total_bytes;
    uint32_t max_pending_operations;
} mf_limits;

/* crates/engine-api/src/backend.rs:18-24; kind 2 = Cuda (backend.rs:9-15). */
typedef struct mf_identity {
    uint32_t kind;
    uint32_t ordinal;
    uint64_t owner;
    uint64_t generation;
} mf_identity;

/* crates/engine-api/src/resources.rs:45-53. */
typedef struct mf_resource_report {
    uint64_t resident_weight_bytes;
    uint64_t cache_bytes;
    uint64_t scratch_bytes;
    uint64_t staged_branch_bytes;
    uint64_t pending_operation_bytes;
    uint32_t pending_operations;
} mf_resource_report;

/* crates/engine-api/src/backend.rs:384-393.  `operations` uses the
 * OperationKind bit numbering of backend.rs:75-99. */
typedef struct mf_capabilities {
    uint32_t dtypes;  /* bit 0 = F32, bit 1 = U8 */
    uint64_t operations;
    uint32_t max_rank;
    uint64_t max_elements;
    uint64_t max_allocation_bytes;
    int32_t supports_nonblocking_completion;
} mf_capabilities;

/* crates/engine-api/src/backend.rs:133-140. */
typedef struct mf_rect_copy_2d {
    uint64_t source_row, source_column, destination_row, destination_column, rows, columns;
} mf_rect_copy_2d;

/* Launch accounting (the reference's `dispatch_counts`,
 * crates/backend-wgpu/src/lib.rs:229). */
typedef struct mf_dispatch_counts {
    uint64_t kernels;
    uint64_t copies;
    uint64_t fences;
    uint64_t readbacks;
} mf_dispatch_counts;

/* ------------------------------------------------------------------ */
/* Lifecycle, identity, accounting                                     */
/* ------------------------------------------------------------------ */

int32_t mf_abi_version(void);
const char *mf_last_error(void);
/* Programmatic dependent launch (on by default): consecutive kernels on a
 * stream overlap their launch and weight streaming with the previous
 * kernel's tail.  Off makes every launch wait for the previous kernel to
 * finish (for comparison runs).  Process-wide. */
int32_t mf_set_pdl(int32_t enabled);

/* Many-token packed matmuls (48 tokens and up) run on the tcgen05 tensor
 * cores by default: BF16 hi/lo split operands, F32 accumulators in TMEM.
 * 0 selects the CUDA-core F32 GEMM instead (for comparison runs).  Calls of
 * the raw-pointer tier always use the CUDA-core GEMM (no scratch).
 * Process-wide.  No counterpart in the reference. */
int32_t mf_set_gemm_tc(int32_t enabled);
/* Ternary and INT8 tensor-core GEMMs.  0 (default) and 2 run the
 * group-scaled kernel - the levels, exact in BF16, against the hi/lo split
 * activation, two MMA passes, each 128-wide K group's dot folded in as
 * sum += scale * dot; 3 runs the scale-folded kernel (hi/lo split weights
 * too, three passes), for comparison runs.  NF4 always runs the three-pass
 * kernel.  Process-wide.  No counterpart in the reference. */
int32_t mf_set_gemm_passes(int32_t passes);
/* Causal GQA of 64 tokens and more with head dimension 64 and a query group
 * dividing 128 runs on the tcgen05 tensor cores by default (scores and the
 * weighted sum as BF16 hi/lo split MMAs, three per product, with F32
 * accumulators; softmax in F32); 0 selects the F32 CUDA-core kernel
 * instead (for comparison runs).  Process-wide.  No counterpart in the
 * reference. */
int32_t mf_set_attention_tc(int32_t enabled);

/* Reads and clears the device fault words into *flags (bit 0: a tensor-core
 * GEMM or attention pipeline wait exceeded its time limit, the tiles or
 * query rows it affected were written as NaN; bit 1: a wait of the persistent decode step exceeded its
 * time limit, the step stopped and every later step returns at once until
 * this call clears the word; the states it ran on must then be recreated).
 * Synchronizes the device.  No counterpart in the reference. */
int32_t mf_device_faults(uint32_t *flags);

/* One backend per device ordinal and host thread.  `limits` may be NULL (no
 * caps beyond device memory).  crates/backend-cpu/src/storage.rs:145 analogue. */
int32_t mf_backend_create(int32_t ordinal, uint64_t owner, const mf_limits *limits,
                          mf_backend **out);
/* Waits for queued work, then frees everything the backend owns. */
int32_t mf_backend_destroy(mf_backend *backend);
int32_t mf_identity_get(const mf_backend *backend, mf_identity *out);
int32_t mf_capabilities_get(const mf_backend *backend, mf_capabilities *out);
int32_t mf_resource_report_get(const mf_backend *backend, mf_resource_report *out);
/* inference.rs:50-56. */
int32_t mf_peak_accounted_bytes(const mf_backend *backend, uint64_t *out);
/* inference.rs:57: buffers of earlier generations become StaleBuffer. */
int32_t mf_advance_generation(mf_backend *backend);
int32_t mf_dispatch_counts_get(const mf_backend *backend, mf_dispatch_counts *out);
/* The backend's CUDA stream (cudaStream_t) for interop. */
void *mf_backend_stream(const mf_backend *backend);
/* Test hook mirroring the reference's DeferredBackend::inject_copy_failure
 * (crates/executor-core/tests/model_executor.rs:369): kind 1 fails the next
 * fence, 2 the next allocation, 3 the next readback, with BackendFailure. */
int32_t mf_inject_failure(mf_backend *backend, int32_t kind);

/* ------------------------------------------------------------------ */
/* Buffers (inference.rs:59-104)                                        */
/* ------------------------------------------------------------------ */

/* Zero-initialised unless `uninit` (inference.rs:89-99). */
int32_t mf_allocate_f32(mf_backend *backend, const uint64_t *shape, uint32_t rank,
                        int32_t alloc_class, int32_t uninit, mf_buffer **out);
int32_t mf_upload_f32(mf_backend *backend, const uint64_t *shape, uint32_t rank,
                      const float *values, int32_t alloc_class, mf_buffer **out);
int32_t mf_upload_u8(mf_backend *backend, const uint64_t *shape, uint32_t rank,
                     const uint8_t *bytes, int32_t alloc_class, mf_buffer **out);
/* Storage is returned in stream order, after work already queued on it. */
int32_t mf_buffer_release(mf_backend *backend, mf_buffer *buffer);
int32_t mf_buffer_info(const mf_buffer *buffer, int32_t *dtype, uint32_t *rank,
                       uint64_t *shape, int32_t *alloc_class);
/* Device address (for interop and the mfk_* tier). */
void *mf_buffer_device_ptr(const mf_buffer *buffer);

/* ------------------------------------------------------------------ */
/* Completions (inference.rs:106-111)                                   */
/* ------------------------------------------------------------------ */

int32_t mf_fence_submit(mf_backend *backend, mf_fence **out);
/* MF_OK when complete, MF_PENDING while queued, else the failure. */
int32_t mf_fence_poll(mf_fence *fence);
int32_t mf_fence_release(mf_fence *fence);
/* inference.rs:41-42 and crates/engine-api/src/backend.rs:25-62
 * (BackendLease): the backend's identity plus an actual-instance token.
 * Tokens are unique within the process and never reused, so two backends
 * whose identity fields collide still differ (same_actual_instance = equal
 * tokens). */
typedef struct mf_lease {
    mf_identity identity;
    uint64_t instance;
} mf_lease;
int32_t mf_lease_get(const mf_backend *backend, mf_lease *out);
/* inference.rs:43-46 and crates/engine-api/src/resources.rs:143-185
 * (FenceRetirement): the backend is its own retirement queue.
 * mf_fence_retire admits an unresolved fence and every buffer its
 * submission still references.  The fence and each buffer must belong to
 * this backend and not be retired already; otherwise the call fails
 * (MF_WRONG_BACKEND for another backend's fence or buffer) before anything
 * changes and the caller keeps the whole payload (RetirementRejection).  On
 * success the backend owns them: mf_fence_release / mf_buffer_release refuse
 * them, and mf_poll_retired_fences releases them once the fence is terminal
 * (success or failure).  mf_poll_retired_fences is one nonblocking pass
 * (cudaEventQuery), poll_retired_fences / poll_retired.
 * mf_retired_fences_unresolved counts the retired fences not yet seen
 * terminal (has_unresolved = count > 0). */
int32_t mf_fence_retire(mf_backend *backend, mf_fence *fence, mf_buffer *const *retained,
                        uint64_t n_retained);
int32_t mf_poll_retired_fences(mf_backend *backend);
int32_t mf_retired_fences_unresolved(const mf_backend *backend, uint64_t *count);
int32_t mf_read_f32_async(mf_backend *backend, const mf_buffer *buffer, mf_readback **out);
/* Copies the values once ready (MF_PENDING before); a second successful poll
 * returns MF_COMPLETION_CONSUMED. */
int32_t mf_readback_poll(mf_readback *readback, float *out, uint64_t capacity,
                         uint64_t *length);
int32_t mf_readback_release(mf_readback *readback);

/* ------------------------------------------------------------------ */
/* Operations (inference.rs:113-425).  Token ids: either host ids     */
/* (`host_ids`, `n_ids`) or a device f32 [T] buffer (`device_ids`).    */
/* ------------------------------------------------------------------ */

int32_t mf_copy(mf_backend *b, mf_buffer *output, const mf_buffer *input);
int32_t mf_copy_rect_2d(mf_backend *b, mf_buffer *output, const mf_buffer *input,
                        const mf_rect_copy_2d *rect);
int32_t mf_argmax(mf_backend *b, mf_buffer *output, const mf_buffer *input);
int32_t mf_argmax_masked(mf_backend *b, mf_buffer *output, const mf_buffer *input,
                         const uint64_t *mask, uint64_t mask_words);
int32_t mf_gather_rows(mf_backend *b, mf_buffer *output, const mf_buffer *table,
                       const uint32_t *host_ids, uint64_t n_ids, const mf_buffer *device_ids);
int32_t mf_gather_columns(mf_backend *b, mf_buffer *output, const mf_buffer *input,
                          const uint32_t *columns, uint64_t n_columns);
int32_t mf_packed_gather_rows(mf_backend *b, mf_buffer *output, const mf_buffer *codes,
                              const mf_buffer *scales, const uint32_t *host_ids, uint64_t n_ids,
                              const mf_buffer *device_ids);
/* inference.rs:194-200. */
int32_t mf_packed_linear(mf_backend *b, mf_buffer *output, const mf_buffer *input,
                         const mf_buffer *codes, const mf_buffer *scales);
/* inference.rs:209-218. */
int32_t mf_packed_linear_pair(mf_backend *b, mf_buffer *out_a, mf_buffer *out_b,
                              const mf_buffer *input, const mf_buffer *codes_a,
                              const mf_buffer *scales_a, const mf_buffer *codes_b,
                              const mf_buffer *scales_b);
/* inference.rs:226-233. */
int32_t mf_packed_swiglu_linear(mf_backend *b, mf_buffer *output, const mf_buffer *gate,
                                const mf_buffer *up, const mf_buffer *codes,
                                const mf_buffer *scales);
/* inference.rs:244-252. */
int32_t mf_packed_swiglu_pair(mf_backend *b, mf_buffer *output, const mf_buffer *input,
                              const mf_buffer *codes_a, const mf_buffer *scales_a,
                              const mf_buffer *codes_b, const mf_buffer *scales_b);
/* inference.rs:253-311 (supports_ternary_lut2, repack_ternary_lut2,
 * packed_linear_lut2, packed_swiglu_pair_lut2).  Returns 1: this backend has
 * a LUT2 layout of its own, a lossless rearrangement of the ternary bytes
 * (same byte count): for each 16-row tile and 128-weight group, the 16 bytes
 * one lane of the decode GEMV's integer MMA reads (its 8 code bytes of rows
 * g and g + 8) are contiguous, so a warp reads one 512-byte block per group
 * with one 16-byte load per lane.  The repack allocates the result in the
 * source's allocation class; rows not a multiple of 16 (or a row that is not
 * whole 128-weight groups) fail with MF_RESOURCE_LIMIT, which a loader
 * answers by keeping the raw stream for that role, as the reference's does.
 * Repacked buffers are flagged: only the *_lut2 ops accept them, and the
 * *_lut2 ops accept nothing else.  Results equal the raw-stream ops bit for
 * bit. */
int32_t mf_supports_ternary_lut2(const mf_backend *b);
int32_t mf_repack_ternary_lut2(mf_backend *b, const mf_buffer *codes, mf_buffer **out);
int32_t mf_packed_linear_lut2(mf_backend *b, mf_buffer *output, const mf_buffer *input,
                              const mf_buffer *codes, const mf_buffer *scales);
int32_t mf_packed_swiglu_pair_lut2(mf_backend *b, mf_buffer *output, const mf_buffer *input,
                                   const mf_buffer *codes_a, const mf_buffer *scales_a,
                                   const mf_buffer *codes_b, const mf_buffer *scales_b);
int32_t mf_add_row_rms_norm(mf_backend *b, mf_buffer *sum, mf_buffer *normed,
                            const mf_buffer *left, const mf_buffer *right,
                            const mf_buffer *weight, float epsilon);
int32_t mf_qk_norm_rope(mf_backend *b, mf_buffer *query_out, mf_buffer *key_out,
                        const mf_buffer *query, const mf_buffer *key,
                        const mf_buffer *query_weight, const mf_buffer *key_weight,
                        const uint64_t *positions, uint64_t n_positions, uint32_t query_heads,
                        uint32_t head_dim, float theta, uint32_t key_value_heads, float epsilon);
int32_t mf_add(mf_backend *b, mf_buffer *output, const mf_buffer *left, const mf_buffer *right);
int32_t mf_multiply(mf_backend *b, mf_buffer *output, const mf_buffer *left,
                    const mf_buffer *right);
int32_t mf_linear(mf_backend *b, mf_buffer *output, const mf_buffer *input,
                  const mf_buffer *weight);
int32_t mf_row_rms_norm(mf_backend *b, mf_buffer *output, const mf_buffer *input,
                        const mf_buffer *weight, float epsilon);
int32_t mf_head_rms_norm(mf_backend *b, mf_buffer *output, const mf_buffer *input,
                         const mf_buffer *weight, uint32_t heads, uint32_t head_dim,
                         float epsilon);
int32_t mf_split_half_rotary(mf_backend *b, mf_buffer *output, const mf_buffer *input,
                             const uint64_t *positions, uint64_t n_positions, uint32_t heads,
                             uint32_t head_dim, float theta);
/* inference.rs:394-404; *cache_len advances only on success. */
int32_t mf_causal_gqa(mf_backend *b, mf_buffer *output, const mf_buffer *query,
                      const mf_buffer *key, const mf_buffer *value, mf_buffer *key_cache,
                      mf_buffer *value_cache, uint64_t *cache_len, uint32_t query_heads,
                      uint32_t key_value_heads, uint32_t head_dim);
/* inference.rs:409-416. */
int32_t mf_gated_short_convolution(mf_backend *b, mf_buffer *output,
                                   const mf_buffer *projection, const mf_buffer *kernel,
                                   mf_buffer *history, uint32_t hidden, uint32_t width);
int32_t mf_swiglu(mf_backend *b, mf_buffer *output, const mf_buffer *gate, const mf_buffer *up);

/* EncoderOps (crates/engine-api/src/encoder.rs:80-103; CPU equations
 * crates/backend-cpu/src/encoder.rs).  `segment_ids` (host, n_segments =
 * tokens) are EncoderSegments labels: every nonzero label on one contiguous
 * run (else MF_INVALID_ARGUMENT, encoder.rs:16-45), 0 = padding, whose output
 * rows are zero.  Nothing outside a token's run enters its output. */
/* encoder.rs:82-92: noncausal GQA within each token's segment; query/output
 * [tokens, query_heads * head_dim], key/value [tokens, key_value_heads *
 * head_dim]. */
int32_t mf_bidirectional_gqa(mf_backend *b, mf_buffer *output, const mf_buffer *query,
                             const mf_buffer *key, const mf_buffer *value,
                             const uint32_t *segment_ids, uint64_t n_segments,
                             uint32_t query_heads, uint32_t key_value_heads, uint32_t head_dim);
/* encoder.rs:94-102: out[t] = C[t] * sum_j kernel[j] * (B * V)[t + j - width / 2]
 * within the segment; projection [tokens, 3 * hidden], kernel [hidden, width],
 * output [tokens, hidden]. */
int32_t mf_centered_gated_convolution(mf_backend *b, mf_buffer *output,
                                      const mf_buffer *projection, const mf_buffer *kernel,
                                      const uint32_t *segment_ids, uint64_t n_segments,
                                      uint32_t hidden, uint32_t width);

/* ------------------------------------------------------------------ */
/* LFM2 executor (crates/executor-core/src/lfm2/executor/execution.rs) */
/* ------------------------------------------------------------------ */

typedef struct mf_lfm2 mf_lfm2;
typedef struct mf_lfm2_state mf_lfm2_state;

enum { MF_LAYER_CONV = 0, MF_LAYER_ATTENTION = 1 };

/* crates/executor-core/src/lfm2/config.rs:33-51 (the fields the pass reads). */
typedef struct mf_lfm2_config {
    uint32_t hidden, intermediate, q_heads, kv_heads, head_dim, conv_width, vocab;
    uint32_t n_layers;
    const int32_t *layer_kinds;
    float rope_theta, block_eps, norm_eps;
    uint64_t max_tokens;
} mf_lfm2_config;

/* A projection role: dense F32 [rows, cols] (`dense`) or packed (`codes`,
 * `scales`), as resolved by crates/executor-core/src/lfm2/weights.rs:1154-1171. */
typedef struct mf_lfm2_weight {
    const mf_buffer *dense;
    const mf_buffer *codes;
    const mf_buffer *scales;
} mf_lfm2_weight;

typedef struct mf_lfm2_layer {
    mf_lfm2_weight in_proj, out_proj;
    const mf_buffer *conv_kernel;
    mf_lfm2_weight q, k, v, o;
    const mf_buffer *q_norm, *k_norm;
    mf_lfm2_weight w1, w2, w3;
    const mf_buffer *ffn_norm, *operator_norm;
} mf_lfm2_layer;

/* Weight buffers stay owned by the caller and must outlive the model. */
int32_t mf_lfm2_create(mf_backend *b, const mf_lfm2_config *config,
                       const mf_lfm2_weight *embedding, const mf_buffer *embedding_norm,
                       const mf_lfm2_layer *layers, mf_lfm2 **out);
int32_t mf_lfm2_destroy(mf_lfm2 *model);
/* Empty prefix state (caches sized for config.max_tokens). */
int32_t mf_lfm2_state_create(mf_lfm2 *model, mf_lfm2_state **out);
/* Device-side deep copy (crates/executor-core/src/lfm2/executor/storage.rs:104-160). */
int32_t mf_lfm2_state_fork(mf_lfm2 *model, const mf_lfm2_state *source, mf_lfm2_state **out);
int32_t mf_lfm2_state_destroy(mf_lfm2_state *state);
uint64_t mf_lfm2_state_length(const mf_lfm2_state *state);
/* append_tokens (execution.rs:35-585): `n` host tokens; when `want_logits`
 * the last row's logits stay on device (mf_lfm2_state_logits). */
int32_t mf_lfm2_append(mf_lfm2 *model, mf_lfm2_state *state, const uint32_t *tokens, uint64_t n,
                       int32_t want_logits);
/* append_token + sample_epilogue (execution.rs:591-627).  The token comes
 * from the host (`token`) or, when `token_from_sample` is set, from the
 * state's device-resident sampled id.  The greedy id stays on device. */
int32_t mf_lfm2_append_argmax(mf_lfm2 *model, mf_lfm2_state *state, uint32_t token,
                              int32_t token_from_sample);
/* Device buffers owned by the state: logits [1, vocab] and sampled id [1]. */
const mf_buffer *mf_lfm2_state_logits(const mf_lfm2_state *state);
const mf_buffer *mf_lfm2_state_sampled(const mf_lfm2_state *state);
/* Blocking read of the sampled id (NaN = poisoned logits). */
int32_t mf_lfm2_read_sampled(mf_lfm2_state *state, float *out);
/* Decode-step replay: capture one append_argmax step (device-resident token
 * and positions) into a CUDA graph on first use, then replay it; `steps`
 * greedy tokens are appended.  Results are identical to calling
 * mf_lfm2_append_argmax(token_from_sample = 1) `steps` times. */
int32_t mf_lfm2_decode_graph(mf_lfm2 *model, mf_lfm2_state *state, uint64_t steps);
/* Single-token greedy steps (mf_lfm2_append_argmax, the decode graph,
 * mf_lfm2_decode_host) run fused by default: each RMSNorm in the prologue of
 * the projection that consumes it, q/k/v in one launch, the greedy argmax
 * and position advance in the LM head's epilogue.  Off runs the op-by-op
 * pass of mf_lfm2_append (for comparison).  Models whose projections are not
 * all packed always run op by op.  A state's decode graph captures the
 * setting in force when the graph is first built. */
int32_t mf_lfm2_set_fused(mf_lfm2 *model, int32_t enabled);
/* Single-token greedy steps of a fused model can run as ONE persistent
 * launch (off by default): one CTA per SM streams every stage's weights through a ring
 * of shared-memory slots while the stages' vectors pass between CTAs through
 * tagged global words.  Used where the model qualifies (every projection
 * packed, head_dim 64, at most 8 query heads per KV head, hidden <= 4096);
 * else the fused projections run as separate launches.  0 (the default)
 * selects the separate launches.  A state's decode graphs capture
 * the setting in force when they are first built.  No counterpart in the
 * reference. */
int32_t mf_lfm2_set_persistent(mf_lfm2 *model, int32_t enabled);
/* 1 when the state's single-token steps run the persistent launch. */
int32_t mf_lfm2_persistent_active(const mf_lfm2_state *state);
/* The reference executor's LUT2 routing (crates/executor-core/src/lfm2/
 * executor/construction.rs:404-470, Lfm2Lut2Mode and max_lut2_bytes of
 * executor.rs:27-51): mode 1 (Auto) repacks, per layer in order, the
 * ternary down projection and then the ternary gate/up pair into this
 * backend's LUT2 layout while the byte budget lasts; mode 2 (DownOnly) the
 * down projections only; mode 0 (Off) returns every role to its raw stream.
 * The model owns the repacks (weight allocation class); decode, prefill and
 * batched passes then run those roles on the LUT2 kernels, with results
 * equal bit for bit.  Captured graphs are recaptured on their next use.
 * `repacked_bytes` (may be null) receives the bytes repacked. */
int32_t mf_lfm2_set_lut2(mf_lfm2 *model, int32_t mode, uint64_t max_bytes, uint64_t *repacked_bytes);
/* The optional LM-head output-row split over NCCL for one sequence across
 * GPUs.  mf_nccl_unique_id writes a 128-byte NCCL id (rank 0 makes it, the
 * host hands it to the other ranks).  mf_lfm2_set_head_split is a
 * collective: every rank, each with its own backend, device and full model
 * replica, calls it with the same id and world size.  Each rank then scores
 * rows [r * S, min((r + 1) * S, vocab)) of the head (S = ceil(vocab / world)
 * rounded up to 16) in its greedy steps, the ranks all-gather their
 * (max, index, poisoned) candidates (12 bytes each) over NCCL, and every
 * rank takes the same first strict maximum (NaN if any shard saw a
 * non-finite logit), as one argmax over the whole row.  Ranks must run the
 * same steps on the same tokens.  After a split step a state's logits hold
 * only this rank's rows.  Prefill logits, batches and the persistent step
 * keep the whole head; the generation loop runs in its host form.  INT8,
 * ternary and dense F32 heads; world 1 turns the split off.  NCCL is loaded
 * on first use (libnccl.so.2); without it these return MF_UNSUPPORTED. */
int32_t mf_nccl_unique_id(uint8_t *out, uint64_t capacity);
/* One greedy step of `state` (it advances by one token, from its device
 * sample) with a CUDA event after every launch: us[i] = launch i's span
 * from the previous event, names[i] = its op label (ffn_gate_up, ffn_down,
 * conv_in_proj, conv_out_proj, attn_qkv, attention, attn_o, lm_head) or
 * kernel name, static strings.  The events stop launches from overlapping,
 * so the spans are per-launch times, not the step's overlapped total.  *n =
 * launches (entries past `capacity` are dropped).  No counterpart in the
 * reference: the bench's per-kernel roofline. */
int32_t mf_lfm2_time_step(mf_lfm2 *model, mf_lfm2_state *state, const char **names, float *us,
                          uint64_t capacity, uint64_t *n);
int32_t mf_lfm2_set_head_split(mf_lfm2 *model, const uint8_t *unique_id, int32_t rank, int32_t world);
/* Number of kernels one decode step launches (for launch accounting). */
uint64_t mf_lfm2_decode_kernels_per_step(const mf_lfm2 *model);
/* One greedy decode step with host I/O, the loop of
 * crates/text-generation/src/lib.rs:375-445 (sampled_token, then
 * append_argmax): when `token` is non-NULL it is copied to the device as the
 * step's input (else the device-resident sampled id is used), the captured
 * decode step runs, and the new greedy id is copied back to *sampled_out
 * (NaN = poisoned logits).  Blocks until the id is on the host. */
int32_t mf_lfm2_decode_host(mf_lfm2 *model, mf_lfm2_state *state, const uint32_t *token,
                            float *sampled_out);
/* The greedy loop of crates/text-generation/src/lib.rs:360-445 on the host
 * side of the C ABI: each iteration reads the state's current sample to the
 * host (sampled_token), returns at a stop id (*stopped = 1, the stop id not
 * recorded, crates/text-generation/src/lib.rs:391-399), records it, returns
 * after `max_tokens` ids, and otherwise appends it from the device-resident
 * sample (append_argmax) with the captured decode step.  When `first_token`
 * is non-NULL it replaces the current sample first.  ids_out[*n_out] gets the
 * ids; a sample that is not a valid id (poisoned logits) fails with
 * MF_BACKEND_FAILURE, as the reference's missing-sample error, and running out
 * of context fails with MF_RESOURCE_LIMIT after the ids produced so far.
 * With at most 64 stop ids the loop runs on the device: the first call on a
 * state builds a graph whose WHILE conditional node runs one decode step and
 * then a one-thread check of the same rules, so a call is one upload, one
 * graph launch and one read-back (call it outside stream capture); where the
 * driver does not build that graph, or with more stop ids, the loop runs on
 * the host with one read-back per token. */
int32_t mf_lfm2_generate(mf_lfm2 *model, mf_lfm2_state *state, const uint32_t *first_token,
                         uint64_t max_tokens, const uint32_t *stop_ids, uint64_t n_stop, float *ids_out,
                         uint64_t *n_out, int32_t *stopped);
/* Overwrites `dst` with `src` (conv histories, K/V rows up to the populated
 * length, position, logits, sampled id) without allocating: the branch copy
 * of crates/executor-core/src/lfm2/executor/storage.rs:236-300. */
int32_t mf_lfm2_state_copy(mf_lfm2 *model, mf_lfm2_state *dst, const mf_lfm2_state *src);

/* Batches of independent sequences (no counterpart in the reference, whose
 * executor holds one sequence per state): `sequences` sequences advance
 * together, each with its own caches, conv history, position and greedy id,
 * and every step is one pass over all of them (matmuls at `sequences` rows).
 * Per sequence the arithmetic is that of the single-state pass. */
/* Loads an LFM2 bundle directory written by the reference's converters
 * (tools/converters/src/minifield_converters/bundle.py): config.json and
 * model.safetensors (packed roles as `<name>.codes` U8 + `<name>.scales`
 * F16, dense roles F32/BF16/F16), following the reference loader
 * (crates/executor-core/src/loader.rs, src/lfm2/config.rs, weights.rs).
 * The model owns the uploaded weights; its caches hold max_tokens rows. */
int32_t mf_lfm2_load_bundle(mf_backend *backend, const char *directory, uint64_t max_tokens, mf_lfm2 **out);
/* A bundle's configuration (max_tokens 0, layer_kinds NULL in *out), its
 * layer kinds (if layer_kinds is not NULL; max_layers entries) and the
 * weight format marker (if format is not NULL), without a device. */
int32_t mf_bundle_config(const char *directory, mf_lfm2_config *out, int32_t *layer_kinds, uint32_t max_layers,
                         char *format, uint64_t format_len);

typedef struct mf_lfm2_batch mf_lfm2_batch;
int32_t mf_lfm2_batch_create(mf_lfm2 *model, uint32_t sequences, mf_lfm2_batch **out);
int32_t mf_lfm2_batch_destroy(mf_lfm2_batch *batch);
/* Every sequence becomes a copy of `prefix` (caches, histories, position,
 * greedy id). */
int32_t mf_lfm2_batch_fork(mf_lfm2_batch *batch, const mf_lfm2_state *prefix);
/* Appends n tokens to every sequence (tokens[s * n + t], host) and sets each
 * sequence's greedy id to the argmax of its last row's logits. */
int32_t mf_lfm2_batch_append_argmax(mf_lfm2_batch *batch, const uint32_t *tokens, uint64_t n);
/* `steps` greedy steps for every sequence (one captured pass per step, fed
 * by the device greedy ids).  With ids_out (steps x sequences f32, row per
 * step) the ids are copied out, synchronizing. */
int32_t mf_lfm2_batch_decode(mf_lfm2_batch *batch, uint64_t steps, float *ids_out);
/* Copies the greedy ids [sequences] and/or the last logits [sequences, vocab]
 * to the host (either may be NULL); synchronizes. */
int32_t mf_lfm2_batch_read(mf_lfm2_batch *batch, float *sampled_out, float *logits_out);
uint64_t mf_lfm2_batch_kernels_per_step(const mf_lfm2_batch *batch);

/* Op classes of the per-op decode profile. */
enum {
    MF_OP_PACKED_MATMUL = 0,
    MF_OP_DENSE_MATMUL = 1,
    MF_OP_ATTENTION = 2,
    MF_OP_CONV = 3,
    MF_OP_NORM_ROPE = 4,
    MF_OP_GATHER = 5,
    MF_OP_ARGMAX = 6,
    MF_OP_OTHER = 7,
    MF_OP_CLASSES = 8
};
typedef struct mf_op_profile {
    uint64_t launches; /* kernels launched by ops of this class */
    uint64_t bytes;    /* algorithmic bytes (each operand read or written once) */
    double ms;         /* summed CUDA-event durations of the class's ops */
    uint64_t ops;      /* number of ops */
} mf_op_profile;
/* Runs one append_argmax step (device-resident token, no graph) with CUDA
 * events recorded on the backend stream around every op, and sums per op
 * class into out[0..MF_OP_CLASSES).  Advances the state by one token, like
 * mf_lfm2_append_argmax(token_from_sample = 1).  The backend's own
 * diagnostics (crates/backend-wgpu/src/device.rs:183-190 counts dispatches;
 * this adds device time). */
int32_t mf_lfm2_profile_step(mf_lfm2 *model, mf_lfm2_state *state, mf_op_profile *out,
                             uint32_t n_classes);

/* ------------------------------------------------------------------ */
/* Raw-pointer kernel tier                                             */
/* ------------------------------------------------------------------ */

/* out[t, r] = sum_g scale[r, g] * sum_{j in g} w(code[r, j]) * x[t, j];
 * x F32 [t, k], codes U8 [n, k*bits/8], scales F32 [n, k/128], out F32 [t, n].
 * crates/backend-cpu/src/packed.rs:96-170. */
int32_t mfk_packed_linear(float *out, const float *x, uint64_t t, const uint8_t *codes,
                          const float *scales, uint64_t n, uint64_t k, int32_t format,
                          void *stream);
/* The LUT2 repack of mf_repack_ternary_lut2 on device pointers: codes U8
 * [rows, row_bytes] (ternary, row_bytes = k/4) -> out, same size, distinct,
 * 16-byte aligned.  The LUT2 matmuls need the backend's scratch and are
 * handle-tier only. */
int32_t mfk_repack_ternary_lut2(uint8_t *out, const uint8_t *codes, uint64_t rows, uint64_t row_bytes,
                                void *stream);
int32_t mfk_packed_linear_pair(float *out_a, float *out_b, const float *x, uint64_t t,
                               const uint8_t *codes_a, const float *scales_a,
                               const uint8_t *codes_b, const float *scales_b, uint64_t n,
                               uint64_t k, int32_t format, void *stream);
int32_t mfk_packed_swiglu_pair(float *out, const float *x, uint64_t t, const uint8_t *codes_a,
                               const float *scales_a, const uint8_t *codes_b,
                               const float *scales_b, uint64_t n, uint64_t k, int32_t format,
                               void *stream);
int32_t mfk_packed_swiglu_linear(float *out, const float *gate, const float *up, uint64_t t,
                                 const uint8_t *codes, const float *scales, uint64_t n,
                                 uint64_t k, int32_t format, void *stream);
/* ids: device f32 [n_ids] (argmax output convention); invalid ids -> NaN row. */
int32_t mfk_packed_gather_rows(float *out, const uint8_t *codes, const float *scales,
                               uint64_t rows, uint64_t k, int32_t format, const float *ids,
                               uint64_t n_ids, void *stream);
/* argmax over [rows, width]; first strict max; NaN if any non-finite. */
int32_t mfk_argmax(float *out, const float *logits, uint64_t rows, uint64_t width,
                   void *stream);
/* Host: validates EncoderSegments labels [tokens] (encoder.rs:16-45) and
 * writes ranges[2 * tokens] (host): the [start, end) run of each token's
 * segment, start == end for label 0.  Upload them for the two calls below. */
int32_t mfk_encoder_segment_ranges(const uint32_t *segment_ids, uint64_t tokens,
                                   uint32_t *ranges);
/* mf_bidirectional_gqa / mf_centered_gated_convolution on device pointers;
 * `ranges` is the device copy of mfk_encoder_segment_ranges' output.  F32
 * operands 16-byte aligned. */
int32_t mfk_bidirectional_gqa(float *out, const float *q, const float *k, const float *v,
                              const uint32_t *ranges, uint64_t tokens, uint32_t q_heads,
                              uint32_t kv_heads, uint32_t head_dim, void *stream);
int32_t mfk_centered_gated_convolution(float *out, const float *projection, const float *kernel,
                                       const uint32_t *ranges, uint64_t tokens, uint32_t hidden,
                                       uint32_t width, void *stream);

/* Causal GQA that allocates nothing.  It has no counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc, such as a
 * host whose own memory manager has already reserved the device's memory
 * into its pool (a cudaMalloc would fail, or escape the pool's accounting),
 * or a latency-bound decode loop that must not make a call that may
 * synchronize the whole device while other streams have work in flight.
 * Same arithmetic as mf_causal_gqa: appends `tokens` K/V rows at
 * `cache_len` and attends over rows [0, cache_len + t] for token t; q/out
 * [tokens, q_heads*head_dim], k/v [tokens, kv_heads*head_dim], caches
 * [capacity, kv_heads*head_dim], all F32 and 16-byte aligned.  The
 * split-key partials go to one 4 MiB static device array that every GPU
 * loading the library holds until exit; a call whose partials would exceed
 * it fails with MF_RESOURCE_LIMIT (single-token decode with 32 heads of 64
 * fits up to ~31k visible rows; 17+ tokens at head_dim 64 with a query group
 * dividing 64 need no partials at all).  The first call on a device looks
 * the array's device address up (cudaGetSymbolAddress), so make that first
 * call before any stream capture.  Under lazy module loading (the CUDA 12
 * default) that first call is also what loads this library's kernels on the
 * device, and loading them reserves the array: a host that cannot allocate
 * later must make one call during its initialisation, before its own pool
 * takes the device's memory.  The address is kept per device ordinal for the
 * life of the process; after cudaDeviceReset on a device, do not call this
 * entry point there again.  All calls share the array and it keeps the last
 * call's contents (nothing in it needs to start at zero): calls that can
 * overlap on the GPU, e.g. on two streams, race on it. */
int32_t mfk_causal_gqa_noalloc(float *out, const float *q, const float *k, const float *v,
                               float *key_cache, float *value_cache, uint64_t capacity,
                               uint64_t cache_len, uint64_t tokens, uint32_t q_heads,
                               uint32_t kv_heads, uint32_t head_dim, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* MFCUDA_H */

/*
 * mf_oracle.h -- CPU oracle for the Minifield packed-matmul path and the
 * LFM2 layer around it.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the
 * reference's scalar CPU backend (crates/backend-cpu + crates/kernels-simd,
 * x86 scalar summation order) and of the LFM2 op order in
 * crates/executor-core/src/lfm2/executor/execution.rs.  Only the test suite,
 * the smoke check and the bench's CPU-baseline leg may load it; the product
 * library never links or calls it.
 *
 * Arithmetic contract: compiled with -O2 -ffp-contract=off and no fast-math,
 * so every `a += b * c` below is a rounded multiply followed by a rounded
 * add, exactly as Rust evaluates the same expression.  Transcendentals go to
 * glibc (expf, pow, sin, cos), which is what Rust std calls on Linux.
 *
 * Threading: optional OpenMP parallelism is only ever over independent
 * outputs (rows, heads), never across a reduction, so results are
 * bit-identical for any thread count.
 *
 * Status codes match ExecutorError (crates/engine-api/src/error.rs:10-28)
 * in declaration order, offset by one so that 0 means Ok.
 */
#ifndef MF_ORACLE_H
#define MF_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum mfo_status {
    MFO_OK = 0,
    MFO_INVALID_ARGUMENT = 1,
    MFO_INVALID_SHAPE = 2,
    MFO_INVALID_LAYOUT = 3,
    MFO_INVALID_DTYPE = 4,
    MFO_OVERFLOW = 5,
    MFO_OUT_OF_BOUNDS = 6,
    MFO_UNSUPPORTED = 7,
    MFO_RESOURCE_LIMIT = 8,
    MFO_WRONG_BACKEND = 9,
    MFO_STALE_BUFFER = 10,
    MFO_BACKEND_FAILURE = 17
};

/* Packed formats (crates/kernels-simd/src/lib.rs:86-96). */
enum mfo_format { MFO_TERNARY = 0, MFO_NF4 = 1, MFO_INT8 = 2 };

/* NF4 codebook (crates/kernels-simd/src/lib.rs:113-130). */
extern const float MFO_NF4_LEVELS[16];

/* Format inference from stream widths (crates/backend-cpu/src/packed.rs:177-220).
 * Returns MFO_OK and fills *format / *inner, or the reference's error. */
int mfo_infer_format(uint64_t code_cols, uint64_t scale_cols, int *format, uint64_t *inner);

/* Row dots, exact reference order (crates/kernels-simd/src/lib.rs:31-81,145-208). */
float mfo_ternary_row_dot(const uint8_t *codes, const float *scales, const float *x, uint64_t k);
float mfo_nf4_row_dot(const uint8_t *codes, const float *scales, const float *x, uint64_t k);
float mfo_int8_row_dot(const uint8_t *codes, const float *scales, const float *x, uint64_t k);

/* Packed ops (crates/backend-cpu/src/packed.rs).  `threads` <= 1 runs serial. */
int mfo_packed_linear(float *out, const float *x, uint64_t t, const uint8_t *codes,
                      const float *scales, uint64_t n, uint64_t k, int format, int threads);
int mfo_packed_linear_pair(float *out_a, float *out_b, const float *x, uint64_t t,
                           const uint8_t *codes_a, const float *scales_a,
                           const uint8_t *codes_b, const float *scales_b,
                           uint64_t n, uint64_t k, int format, int threads);
int mfo_packed_swiglu_pair(float *out, const float *x, uint64_t t,
                           const uint8_t *codes_a, const float *scales_a,
                           const uint8_t *codes_b, const float *scales_b,
                           uint64_t n, uint64_t k, int format, int threads);
int mfo_packed_swiglu_linear(float *out, const float *gate, const float *up, uint64_t t,
                             const uint8_t *codes, const float *scales,
                             uint64_t n, uint64_t k, int format, int threads);
/* ids[i] < 0 marks an invalid device id and yields a NaN row
 * (crates/backend-cpu/src/dense.rs:24-53, packed.rs:33-38). */
int mfo_packed_gather_rows(float *out, const uint8_t *codes, const float *scales,
                           uint64_t rows, uint64_t k, int format,
                           const int64_t *ids, uint64_t n_ids);
/* Device-id resolution rule of dense.rs:35-50: finite, >= 0, integral, < 2^24. */
int64_t mfo_resolve_device_id(float value);

/* Dense ops (crates/backend-cpu/src/dense.rs). */
int mfo_linear(float *out, const float *x, uint64_t t, const float *w, uint64_t n, uint64_t k,
               int threads);
int mfo_argmax(float *out, const float *logits, uint64_t rows, uint64_t width);
int mfo_argmax_masked(float *out, const float *logits, uint64_t rows, uint64_t width,
                      const uint64_t *mask, uint64_t mask_words);
int mfo_gather_rows(float *out, const float *table, uint64_t rows, uint64_t cols,
                    const int64_t *ids, uint64_t n_ids);
int mfo_swiglu(float *out, const float *gate, const float *up, uint64_t n);
int mfo_add(float *out, const float *a, const float *b, uint64_t n);
int mfo_multiply(float *out, const float *a, const float *b, uint64_t n);

/* Normalisation and rotary (crates/backend-cpu/src/normalization_rotary.rs). */
int mfo_row_rms_norm(float *out, const float *x, uint64_t rows, uint64_t width,
                     const float *weight, float eps);
int mfo_add_row_rms_norm(float *sum, float *normed, const float *a, const float *b,
                         uint64_t rows, uint64_t width, const float *weight, float eps);
int mfo_head_rms_norm(float *out, const float *x, uint64_t tokens, uint32_t heads,
                      uint32_t head_dim, const float *weight, float eps);
int mfo_split_half_rotary(float *out, const float *x, uint64_t tokens, uint32_t heads,
                          uint32_t head_dim, const uint64_t *positions, float theta);
int mfo_qk_norm_rope(float *q_out, float *k_out, const float *q, const float *k,
                     uint64_t tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                     const float *q_weight, const float *k_weight,
                     const uint64_t *positions, float theta, float eps);

/* Attention and convolution (crates/backend-cpu/src/attention_convolution.rs). */
int mfo_causal_gqa(float *out, const float *q, const float *k, const float *v,
                   uint64_t tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                   float *key_cache, float *value_cache, uint64_t capacity,
                   uint64_t *cache_len, int threads);
int mfo_gated_short_conv(float *out, const float *projection, uint64_t tokens,
                         uint32_t hidden, const float *kernel, uint32_t width,
                         float *history);

/* Complete-sequence encoder ops (crates/backend-cpu/src/encoder.rs).
 * `segment_ids` [tokens]: nonzero labels each on one contiguous run, 0 =
 * padding (crates/engine-api/src/encoder.rs:16-45); tokens of label 0 get
 * zero output rows. */
int mfo_encoder_segments_check(const uint32_t *segment_ids, uint64_t tokens);
int mfo_bidirectional_gqa(float *out, const float *q, const float *k, const float *v,
                          const uint32_t *segment_ids, uint64_t tokens, uint32_t q_heads,
                          uint32_t kv_heads, uint32_t head_dim, int threads);
int mfo_centered_gated_conv(float *out, const float *projection, const float *kernel,
                            const uint32_t *segment_ids, uint64_t tokens, uint32_t hidden,
                            uint32_t width);

/* ---------------------------------------------------------------------
 * LFM2 model (crates/executor-core/src/lfm2/executor/execution.rs:35-627).
 * Weights are borrowed: the caller owns every array for the model's life.
 * ------------------------------------------------------------------- */
enum mfo_layer_kind { MFO_LAYER_CONV = 0, MFO_LAYER_ATTENTION = 1 };

/* A projection role: dense F32 [rows, cols] or packed codes + F32 scales. */
typedef struct mfo_weight {
    int packed;            /* 0 = dense f32, 1 = packed */
    int format;            /* mfo_format when packed */
    uint64_t rows, cols;   /* logical [rows, cols] */
    const float *dense;
    const uint8_t *codes;
    const float *scales;
} mfo_weight;

typedef struct mfo_lfm2_config {
    uint32_t hidden, intermediate, q_heads, kv_heads, head_dim, conv_width, vocab;
    uint32_t n_layers;
    const int32_t *layer_kinds;  /* n_layers entries of mfo_layer_kind */
    float rope_theta, block_eps, norm_eps;
    uint64_t max_tokens;         /* KV-cache capacity */
} mfo_lfm2_config;

typedef struct mfo_lfm2_layer_weights {
    mfo_weight in_proj, out_proj;          /* conv layers */
    const float *conv_kernel;              /* [hidden, width] */
    mfo_weight q, k, v, o;                 /* attention layers */
    const float *q_norm, *k_norm;          /* [head_dim] */
    mfo_weight w1, w2, w3;
    const float *ffn_norm, *operator_norm; /* [hidden] */
} mfo_lfm2_layer_weights;

typedef struct mfo_lfm2_weights {
    mfo_weight embedding;        /* [vocab, hidden], tied with the LM head */
    const float *embedding_norm; /* [hidden] */
    const mfo_lfm2_layer_weights *layers;
} mfo_lfm2_weights;

typedef struct mfo_lfm2 mfo_lfm2;

int mfo_lfm2_create(const mfo_lfm2_config *config, const mfo_lfm2_weights *weights,
                    int threads, mfo_lfm2 **out);
void mfo_lfm2_destroy(mfo_lfm2 *model);
/* Deep copy of every layer cache (crates/executor-core/src/lfm2/executor/storage.rs:104-160). */
int mfo_lfm2_fork(const mfo_lfm2 *model, mfo_lfm2 **out);
uint64_t mfo_lfm2_length(const mfo_lfm2 *model);
/* append_tokens: run `n` tokens; if want_logits, write [vocab] logits of the last row. */
int mfo_lfm2_append(mfo_lfm2 *model, const uint32_t *tokens, uint64_t n, float *logits);
/* append_token + sample_epilogue: one token, then greedy argmax (NaN = poisoned). */
int mfo_lfm2_append_argmax(mfo_lfm2 *model, uint32_t token, float *sampled, float *logits);

#ifdef __cplusplus
}
#endif
#endif

// Internal launcher declarations shared by the C-ABI layer and the executor.
#pragma once

#include <vector>

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace mf {

// Packed matmul modes.
enum PackedMode { kPackedSingle = 0, kPackedPairRows = 1, kPackedSwigluPair = 2 };

// Token count at or above which the tiled GEMM replaces the GEMV path.
constexpr uint64_t kGemmMinTokens = 48;
// NF4 has no integer-MMA GEMV beyond 2 tokens; from 16 tokens its tcgen05
// GEMM (one 256-token tile) beats the general F32 GEMV.
constexpr uint64_t kNf4GemmMinTokens = 16;
inline uint64_t gemm_min_tokens(int format) { return format == MF_NF4 ? kNf4GemmMinTokens : kGemmMinTokens; }

// Tensor-core GEMM for many-token matmuls on (1, default) or off.
extern std::atomic<int> g_gemm_tc;

// Split-K scratch of the decode GEMV: per-chunk partial sums (no
// initialisation needed) and per-row-block arrival counters (zero before
// the first launch; every launch leaves them zero again).
struct SplitScratch {
    float *partial = nullptr;
    size_t partial_floats = 0;
    unsigned *counters = nullptr;
    size_t n_counters = 0;
};

// Decode GEMV on the integer tensor cores (ternary, INT8; up to 47 tokens)
// and the FP32 NF4 path (up to 2 tokens).
bool packed_gemv_tc_supports(int format, uint64_t t);
size_t packed_gemv_tc_scratch_floats(uint64_t t, uint64_t n, uint64_t k);
size_t packed_gemv_tc_counters(uint64_t t, uint64_t n);
int32_t packed_gemv_tc(int mode, bool swiglu_input, float *out_a, float *out_b, const float *x, const float *gate,
                       const float *up, uint64_t t, const uint8_t *codes_a, const float *scales_a,
                       const uint8_t *codes_b, const float *scales_b, uint64_t n, uint64_t k, int format,
                       const SplitScratch &ss, cudaStream_t stream, bool lanetiled = false);

// The lane-tiled ternary layout (the backend's LUT2 layout; same bytes):
// for 16-row tile t, 128-weight group G and lane L = 4g + q (g < 8, q < 4)
// the 16 bytes at ((t * groups + G) * 32 + L) * 16 are row 16t + g's code
// bytes 8q .. 8q + 7 of group G followed by row 16t + g + 8's.  rows must be
// a multiple of 16 and row_bytes of 32.
int32_t ternary_repack_lanetiled(uint8_t *out, const uint8_t *codes, uint64_t rows, uint64_t row_bytes,
                                 cudaStream_t stream);

int32_t packed_gemv(int mode, bool swiglu_input, float *out_a, float *out_b, const float *x,
                    const float *gate, const float *up, uint64_t t, const uint8_t *codes_a,
                    const float *scales_a, const uint8_t *codes_b, const float *scales_b,
                    uint64_t n, uint64_t k, int format, cudaStream_t stream);

int32_t packed_gemm(int mode, bool swiglu_input, float *out_a, float *out_b, const float *x,
                    const float *gate, const float *up, uint64_t t, const uint8_t *codes_a,
                    const float *scales_a, const uint8_t *codes_b, const float *scales_b,
                    uint64_t n, uint64_t k, int format, cudaStream_t stream);

// Many-token packed matmul on the tcgen05 tensor cores (BF16 hi/lo split
// operands, F32 TMEM accumulators).  `ss.partial` holds the two BF16
// activation planes and, when the grid has too few tiles for the SMs, the
// split-K partials: at least packed_gemm_tc_scratch_floats(t, n, k) floats
// for an [n, k] weight (any mode).
size_t packed_gemm_tc_scratch_floats(uint64_t t, uint64_t n, uint64_t k);
int32_t packed_gemm_tc(int mode, bool swiglu_input, float *out_a, float *out_b, const float *x, const float *gate,
                       const float *up, uint64_t t, const uint8_t *codes_a, const float *scales_a,
                       const uint8_t *codes_b, const float *scales_b, uint64_t n, uint64_t k, int format,
                       const SplitScratch &ss, cudaStream_t stream, bool lanetiled = false);
// Ternary / INT8 tensor-core GEMMs: 0 (default) and 2 run the group-scaled
// two-pass kernel, 3 the scale-folded three-pass one.
void set_gemm_passes(int passes);
// Reads and clears the tensor-core GEMM fault word (bit 0: a pipeline wait
// timed out; the affected tiles were written as NaN).  Synchronizes.
int32_t packed_gemm_tc_faults(uint32_t *flags);

// One-token packed projection for the fused decode step.  Input: `x`, or
// (x null) the normalizing prologue: rmsnorm(na + nb) * nw, or of the
// embedding row of the device id *eid when na is null (ecodes/escales in
// `eformat`, or edense); the sum is written to nres.  With x null and nw
// null the prologue stages na (+ nb) unnormalized: each CTA splits the row
// itself, with no separate limb pass.  Modes: 0 single,
// 1 pair rows (equal shapes), 2 SwiGLU pair, 3 triple (A: n rows, B and C:
// n2 rows).  With `sampled`, mode 0 also writes the greedy id of its output
// row and advances *pos (scratch: CTA partials in ss.partial, after the
// activation limbs when the input is plain; ss.counters[0]).  Every matrix
// is [rows, k] in one packed format.
struct DecodeGemv {
    int mode = 0;
    int format = 0;
    const uint8_t *codes[3] = {nullptr, nullptr, nullptr};
    const float *scales[3] = {nullptr, nullptr, nullptr};
    float *out[3] = {nullptr, nullptr, nullptr};
    uint64_t n = 0, n2 = 0, k = 0;
    const float *x = nullptr;
    const float *na = nullptr, *nb = nullptr, *nw = nullptr;
    float *nres = nullptr;
    float eps = 0.0f;
    const uint8_t *ecodes = nullptr;
    const float *escales = nullptr, *edense = nullptr, *eid = nullptr;
    int eformat = 0;
    uint64_t erows = 0;
    float *sampled = nullptr;
    uint64_t *pos = nullptr;
    // Row shard of a split LM head (codes, scales and out already offset to
    // its first row `row0`): the argmax epilogue writes the shard's
    // candidate (value, global index, poisoned) to `cand` instead of
    // `sampled` and does not advance `pos`.
    float *cand = nullptr;
    uint64_t row0 = 0;
    // One-token FFN chaining (integer formats): a SwiGLU pair with the
    // normalizing prologue writes its outputs as the limbs of a plain-input
    // consumer of format `limbs_for` (-1: none) into the scratch, each
    // 64-value half group with its own exponent; that consumer, called with
    // `limbs_ready`, reads them instead of running the limb pass.
    int limbs_for = -1;
    bool limbs_ready = false;
    // Mode 4 (NF4, one token): the rows are the in_proj's B, C and x
    // projections of n channels (weight [3n, k]); out[0] gets the gated
    // short convolution of them (taps conv_kernel [n][conv_width]) and
    // conv_hist ([conv_width - 1][n]) moves on by one token.
    const float *conv_kernel = nullptr;
    float *conv_hist = nullptr;
    uint32_t conv_width = 0;
    // Ternary codes in the lane-tiled (LUT2) layout (rows in whole 16-row tiles).
    bool lanetiled = false;
};
bool decode_gemv_supports(const DecodeGemv &d);
bool decode_gemv_limbs_supported(const DecodeGemv &d);
bool decode_gemv_conv_supported(const DecodeGemv &d);
int32_t decode_gemv(const DecodeGemv &d, const SplitScratch &ss, cudaStream_t stream);

// Complete-sequence encoder ops (encoder_kernels.cu).  `ranges` is a device
// array of 2 * tokens u32: the [start, end) run of each token's segment,
// start == end for padding (label 0), built on the host by
// encoder_segment_ranges from the labels (which it validates).
int32_t encoder_segment_ranges(const uint32_t *ids, uint64_t tokens, uint32_t *ranges);
int32_t bidirectional_gqa(float *out, const float *q, const float *k, const float *v, const uint32_t *ranges,
                          uint64_t tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                          cudaStream_t stream);
int32_t centered_gated_conv(float *out, const float *projection, const float *kernel, const uint32_t *ranges,
                            uint64_t tokens, uint32_t hidden, uint32_t width, cudaStream_t stream);

// Chooses the tensor-core decode GEMV, the general GEMV or the GEMM by
// token count and format.  `ss` (may be null) is split-K scratch; without
// enough of it the decode GEMV is not used.  Lane-tiled ternary codes run
// only on the tensor-core paths (they need `ss`).
int32_t packed_matmul(int mode, bool swiglu_input, float *out_a, float *out_b, const float *x,
                      const float *gate, const float *up, uint64_t t, const uint8_t *codes_a,
                      const float *scales_a, const uint8_t *codes_b, const float *scales_b,
                      uint64_t n, uint64_t k, int format, const SplitScratch *ss, cudaStream_t stream,
                      bool lanetiled = false);

// One-token dense F32 LM head with the greedy argmax, position advance
// fused (k a power of two times 128, up to 2048); `parts` holds
// dense_head_parts_floats(), `count` one zeroed counter (left zero).
bool dense_head_argmax_supported(uint64_t n, uint64_t k);
size_t dense_head_parts_floats();
// With `cand`, a row shard starting at global row `row0`: the merge writes the
// shard's (value, global index, poisoned) there instead of the greedy id.
int32_t dense_head_argmax(float *logits, const float *x, const float *w, uint64_t n, uint64_t k, float *parts,
                          size_t parts_floats, unsigned *count, float *sampled, uint64_t *pos, cudaStream_t stream,
                          float *cand = nullptr, uint64_t row0 = 0);
// Greedy id from the row shards' candidates [world][3] (ascending row
// ranges): the first strict maximum, NaN if any shard saw a non-finite
// logit; advances the position.
int32_t head_shard_pick(const float *cand, int world, float *sampled, uint64_t *pos, cudaStream_t stream);

// Dense F32 linear: out[t, n] = sum_k x[t, k] * w[n, k].
int32_t dense_linear(float *out, const float *x, uint64_t t, const float *w, uint64_t n,
                     uint64_t k, cudaStream_t stream);

// Gathers.  Device ids are f32 (argmax convention); host ids are uploaded
// by the caller as u32 device arrays (`ids_u32`).  Exactly one of ids_f32 /
// ids_u32 is non-null.  Invalid or out-of-range device ids give NaN rows.
int32_t packed_gather_rows(float *out, const uint8_t *codes, const float *scales, uint64_t rows,
                           uint64_t k, int format, const float *ids_f32, const uint32_t *ids_u32,
                           uint64_t n_ids, cudaStream_t stream);
int32_t gather_rows(float *out, const float *table, uint64_t rows, uint64_t cols,
                    const float *ids_f32, const uint32_t *ids_u32, uint64_t n_ids,
                    cudaStream_t stream);
int32_t gather_columns(float *out, const float *in, uint64_t rows, uint64_t width,
                       const uint32_t *columns, uint64_t n_columns, cudaStream_t stream);

// Argmax over [rows, width] -> f32 index or NaN.  `mask` (device, may be null)
// is the LSB-first u64 candidate mask of the masked variant.  With scratch
// (argmax_scratch_floats partials, `rows` counters) a row is split over many
// CTAs; without it one CTA reduces each row.
size_t argmax_scratch_floats(uint64_t rows, uint64_t width);
int32_t argmax(float *out, const float *logits, uint64_t rows, uint64_t width,
               const uint64_t *mask, const SplitScratch *ss, cudaStream_t stream);

// Elementwise.  op: 0 add, 1 multiply, 2 swiglu.
int32_t elementwise(int op, float *out, const float *a, const float *b, uint64_t n,
                    cudaStream_t stream);

// out = rms_norm(x) * weight over rows of `width`; if `sum_out`, x = a + b is
// formed first and written to sum_out (add_row_rms_norm).
int32_t row_rms_norm(float *sum_out, float *out, const float *a, const float *b, uint64_t rows,
                     uint64_t width, const float *weight, float eps, cudaStream_t stream);

// Per-(token, head) RMS over head_dim (optional, weight may be null to skip)
// followed by split-half RoPE (positions: device u64 array, or null with
// `pos_base` giving position = *pos_base + token).  rope=false skips rotation.
int32_t head_norm_rope(float *out, const float *in, uint64_t tokens, uint32_t heads,
                       uint32_t head_dim, const float *weight, float eps, bool rope,
                       const uint64_t *positions, const uint64_t *pos_base, float theta,
                       cudaStream_t stream);

// Causal GQA over [cache rows, then new rows]; appends k/v to the caches after
// computing.  `cache_len_dev` (device u64, may be null) overrides `cache_len`
// and is advanced by `tokens` on device when `advance_len` is set.
// RoPE rotation table for positions [0, positions): (sin, cos) per pair,
// by the formula of head_norm_rope (normalization_rotary.rs:346-350).
int32_t rope_table(float2 *table, uint64_t positions, uint32_t head_dim, float theta, cudaStream_t stream);

// One-token decode attention for the fused step: raw q/k rows in, the head
// RMSNorm (q_norm / k_norm, eps) and RoPE (rotation table `rope`, position
// = *len_dev) applied inside, new rows appended at *len_dev, chunk merge by
// the last CTA (counters[0 .. kv_heads) zero before, left zero).
bool gqa_decode_fused_supported(uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim, uint64_t capacity);
int32_t gqa_decode_fused(float *out, const float *q_raw, const float *k_raw, const float *v_new,
                         const float *q_norm, const float *k_norm, float eps, const float2 *rope, float *key_cache,
                         float *value_cache, uint64_t capacity, const uint64_t *len_dev, uint32_t q_heads,
                         uint32_t kv_heads, uint32_t head_dim, float *scratch, size_t scratch_bytes,
                         unsigned *counters, size_t n_counters, cudaStream_t stream, uint32_t seqs = 1);

// Batched forms over `seqs` sequences with rows sequence-major (sequence b's
// seq_tokens rows follow b-1's).  Caches are [seqs][capacity][kv_heads *
// head_dim] per layer, histories [seqs][width-1][hidden], lengths lens[seqs]
// (positions of each sequence's first new row).  The fused decode attention
// takes seqs too (one row per sequence; counters kv_heads * seqs, scratch
// seqs times the one-sequence size).
int32_t causal_gqa_batch(float *out, const float *q, const float *k, const float *v, float *key_cache,
                         float *value_cache, uint64_t capacity, const uint64_t *lens_dev, uint32_t seqs,
                         uint64_t seq_tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                         cudaStream_t stream);
int32_t gated_short_conv_batch(float *out, const float *projection, uint32_t seqs, uint64_t tokens, uint32_t hidden,
                               const float *kernel, uint32_t width, float *history, cudaStream_t stream);
int32_t head_norm_rope_batch(float *out, const float *in, uint32_t seqs, uint64_t seq_tokens, uint32_t heads,
                             uint32_t head_dim, const float *weight, float eps, const uint64_t *pos_base, float theta,
                             cudaStream_t stream);
int32_t advance_positions(uint64_t *pos, uint64_t n, uint32_t seqs, cudaStream_t stream);

int32_t causal_gqa(float *out, const float *q, const float *k, const float *v, float *key_cache,
                   float *value_cache, uint64_t capacity, uint64_t cache_len,
                   uint64_t *cache_len_dev, bool advance_len, uint64_t tokens, uint32_t q_heads,
                   uint32_t kv_heads, uint32_t head_dim, float *scratch, size_t scratch_bytes,
                   cudaStream_t stream);
size_t causal_gqa_scratch_bytes(uint64_t tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                                uint64_t max_visible);
// Many-token causal GQA on the tensor cores (attention_tc.cu): head
// dimension 64 and a query group dividing 128; `seqs` sequences on
// blockIdx.z with caches cache_stride floats apart.
bool gqa_prefill_tc_fits(uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim);
int32_t gqa_prefill_tc(float *out, const float *q, const float *key_cache, const float *value_cache, uint64_t len,
                       const uint64_t *len_dev, uint64_t tokens, uint32_t q_heads, uint32_t kv_heads,
                       uint64_t cache_stride, uint32_t seqs, cudaStream_t stream);
// Token count from which many-token attention takes the tensor-core kernel.
constexpr uint64_t kAttnTcMinTokens = 64;
void set_attention_tc(bool on);
bool attention_tc_enabled();
// Reads and clears the tensor-core attention fault word.  Synchronizes.
int32_t attention_tc_faults(uint32_t *flags);

int32_t gated_short_conv(float *out, const float *projection, uint64_t tokens, uint32_t hidden,
                         const float *kernel, uint32_t width, float *history, cudaStream_t stream);

int32_t copy_rect_2d(float *dst, uint64_t dst_width, const float *src, uint64_t src_width,
                     uint64_t src_row, uint64_t src_col, uint64_t dst_row, uint64_t dst_col,
                     uint64_t rows, uint64_t cols, cudaStream_t stream);

// Persistent single-token decode step (decode_persistent.cu): one launch of
// one CTA per SM runs every stage of a greedy step.  The descriptors name the
// model's weights and one state's caches; the plan holds the stage program
// (uploaded into the state's workspace) and the launch geometry.
struct PersistMat {
    const uint8_t *codes = nullptr;
    const float *scales = nullptr;
    const float *dense = nullptr;
    int format = 0;
    uint32_t rows = 0;
};
struct PersistLayerDesc {
    int kind = 0;
    PersistMat in_proj, out_proj, q, k, v, o, w1, w2, w3;
    const float *conv_kernel = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    const float *ffn_norm = nullptr, *operator_norm = nullptr;
};
struct PersistModelDesc {
    uint32_t hidden = 0, intermediate = 0, q_heads = 0, kv_heads = 0, head_dim = 0, conv_width = 0, vocab = 0;
    float block_eps = 0.f, norm_eps = 0.f;
    uint64_t max_tokens = 0;
    PersistMat emb;
    const float *emb_norm = nullptr;
    const float2 *rope = nullptr;
    std::vector<PersistLayerDesc> layers;
};
struct PersistStateDesc {
    uint64_t *pos = nullptr;
    float *sampled = nullptr, *logits = nullptr;
    std::vector<float *> history, kcache, vcache;
};
struct PersistPlan;
bool persistent_geometry_ok(const PersistModelDesc &d);
size_t persistent_ws_bytes(const PersistModelDesc &d, int sms);
int32_t persistent_plan(const PersistModelDesc &d, const PersistStateDesc &s, int sms, void *ws, PersistPlan **out);
int32_t persistent_init(PersistPlan *pl, void *ws, size_t ws_bytes, cudaStream_t stream);
int32_t persistent_launch(const PersistPlan *pl, int sms, cudaStream_t stream);
void persistent_free(PersistPlan *pl);
int persistent_slots(const PersistPlan *pl);
// Reads and clears the persistent step's fault word (bit 0: a wait expired).
int32_t persistent_faults(uint32_t *flags);

}  // namespace mf

// LFM2 forward pass over the backend's kernels
// (crates/executor-core/src/lfm2/executor/execution.rs:35-627).
//
// The op order is the reference's: embedding gather, layer-0 operator norm,
// then per layer the conv or attention mixer, the fused residual add + FFN
// norm, the FFN (pair + SwiGLU-linear below 96 rows, SwiGLU-pair + linear at
// 96 rows and above, the final layer on its last row only), and the fused
// residual add + next norm; logits from the last row; greedy argmax.
//
// B200 specifics: the sequence position lives on the device (one u64 per
// state) and every kernel that needs it reads it there, so one decode step
// (embedding of the device-resident sampled id -> argmax -> position advance)
// is a fixed launch sequence that is captured once into a CUDA graph and
// replayed per token.
#include <cuda_runtime.h>
#include <string.h>

#include <algorithm>
#include <new>
#include <vector>

#include "backend_internal.h"
#include "mf_common.cuh"
#include "packed_kernels.h"

using namespace mf;

namespace {

struct Weight {
    bool present = false;
    bool packed = false;
    int format = 0;
    uint64_t rows = 0, cols = 0;
    const float *dense = nullptr;
    const uint8_t *codes = nullptr;
    const float *scales = nullptr;
    // Ternary codes in use are the model's LUT2 repack of raw_codes.
    bool lanetiled = false;
    const uint8_t *raw_codes = nullptr;
};

struct Layer {
    int kind = MF_LAYER_CONV;
    Weight in_proj, out_proj, q, k, v, o, w1, w2, w3;
    const float *conv_kernel = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    const float *ffn_norm = nullptr, *operator_norm = nullptr;
};

__global__ void advance_position_kernel(uint64_t *pos, uint64_t n) {
    pdl_wait();
    pdl_trigger(); *pos += n; }

// Per-op event bracketing of one pass (mf_lfm2_profile_step).  Each entry
// holds the op class, its algorithmic bytes, its kernel launches and the two
// events recorded on the backend stream around it.
struct OpRecord {
    int cls;
    uint64_t bytes;
    uint64_t kernels;
    cudaEvent_t start, stop;
};

struct Profiler {
    std::vector<cudaEvent_t> pool;
    size_t used = 0;
    std::vector<OpRecord> ops;
    cudaEvent_t next() {
        if (used == pool.size()) {
            cudaEvent_t e = nullptr;
            if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
            pool.push_back(e);
        }
        return pool[used++];
    }
    // Inside stream capture a plain cudaEventRecord only orders work; the
    // external flag makes it an event-record node that takes a timestamp.
    static void record(cudaEvent_t e, cudaStream_t s) { cudaEventRecordWithFlags(e, s, cudaEventRecordExternal); }
    ~Profiler() {
        for (cudaEvent_t e : pool) cudaEventDestroy(e);
    }
};

// Algorithmic bytes of one packed or dense projection over t rows: the
// weight streams (codes + F32 group scales, or dense F32) are read once,
// the input rows (x, or gate and up) are read once, outputs written once.
uint64_t matmul_bytes(const Weight &w, uint64_t t, uint64_t inputs, uint64_t outputs) {
    uint64_t wb;
    if (w.packed)
        wb = w.rows * w.cols / (uint64_t)weights_per_byte(w.format) + w.rows * (w.cols / 128) * 4;
    else
        wb = w.rows * w.cols * 4;
    return wb + inputs * t * w.cols * 4 + outputs * t * w.rows * 4;
}

}  // namespace

struct mf_lfm2 {
    mf_backend *b;
    mf_lfm2_config cfg;
    std::vector<int32_t> kinds;
    Weight emb;
    const float *emb_norm;
    std::vector<Layer> layers;
    uint64_t kernels_per_step;
    bool fused;  // one-token greedy steps through the fused projections (default on)
    // One-token greedy steps as one persistent launch where the model's
    // geometry allows it (off by default; mf_lfm2_set_persistent).
    bool persistent = false;
    bool persistent_ok = false;
    PersistModelDesc pdesc;
    mf_buffer *rope_buf = nullptr;   // RoPE (sin, cos) per position and pair
    const float2 *rope = nullptr;
    std::vector<mf_buffer *> owned;  // weights uploaded by the bundle loader
    std::vector<mf_buffer *> lut2;   // LUT2 repacks of FFN roles (mf_lfm2_set_lut2)
    // LM-head row split over GPUs (mf_lfm2_set_head_split): this rank's rows
    // [head_row0, head_row0 + head_rows), its candidate (3 floats) and every
    // rank's after the all-gather (3 * head_world floats).
    void *head_comm = nullptr;
    int head_rank = 0, head_world = 1;
    uint64_t head_row0 = 0, head_rows = 0;
    mf_buffer *head_buf = nullptr;
    float *head_cand = nullptr, *head_cands = nullptr;
    // Bumped whenever the weights' layout changes: captured graphs of an
    // older epoch are recaptured.
    uint64_t epoch = 0;
};

struct mf_lfm2_state {
    mf_lfm2 *model;
    uint64_t length;
    std::vector<mf_buffer *> owned;
    std::vector<float *> history, kcache, vcache;
    uint64_t *pos_dev;
    mf_buffer *pos_buf;
    mf_buffer *logits;
    mf_buffer *sampled;
    // workspace
    mf_buffer *ws_buf;
    uint64_t ws_rows;
    uint64_t ws_epoch;
    float *x, *u, *op, *proj, *conv, *q, *k, *v, *qr, *kr, *att, *residual, *ffn_in, *gate, *up, *down,
        *hidden_buf;
    uint32_t *ids;
    float *gqa_scratch;
    size_t gqa_scratch_bytes;
    SplitScratch split;           // decode-GEMV split-K partials + counters
    mf_buffer *split_counters_buf;
    // decode graph
    cudaGraphExec_t graph;
    uint64_t graph_epoch;
    // kMultiSteps consecutive greedy steps in one graph (the steps chain by
    // programmatic dependent launch instead of a graph boundary each).
    cudaGraphExec_t graph_multi = nullptr;
    uint64_t graph_multi_epoch = 0;
    // Persistent decode step: stage program + workspace (built on first use,
    // outside stream capture); pers_state -1 = this state cannot use it.
    PersistPlan *pplan = nullptr;
    mf_buffer *pers_buf = nullptr;
    int pers_state = 0;
    // set only inside mf_lfm2_profile_step
    Profiler *prof;
    // host staging of mf_lfm2_append_argmax's token (outlives the async copy)
    float host_token;
    // mf_lfm2_decode_host's [token in, greedy id out] in pinned host memory
    // (allocated on its first call): both copies are plain DMA, no staging;
    // the host waits on io_done (busy-wait event: the next token's launch
    // follows the result without a scheduler wake-up).
    float *io_pinned = nullptr;
    cudaEvent_t io_done = nullptr;
    // mf_lfm2_generate's device-side loop (built on its first call): one
    // graph whose WHILE node runs a greedy step, then the loop's check, until
    // the check ends it; the control block and ids live on the device, with
    // pinned host copies for the one upload and the one read-back per call.
    cudaGraphExec_t graph_gen = nullptr;
    uint64_t graph_gen_epoch = 0;
    uint64_t graph_model_epoch = 0, graph_gen_model_epoch = 0;
    bool gen_unsupported = false;
    struct GenCtl *gen_ctl = nullptr, *gen_ctl_host = nullptr;
    float *gen_ids = nullptr, *gen_ids_host = nullptr;
    uint64_t gen_ids_cap = 0;
};

namespace {

int32_t resolve_weight(const mf_backend *b, const mf_lfm2_weight &src, uint64_t rows, uint64_t cols, Weight *out) {
    out->present = true;
    if (src.dense) {
        int32_t st = check_buffer(b, src.dense);
        if (st) return st;
        if (src.dense->dtype != MF_DTYPE_F32 || src.dense->rank != 2 || src.dense->shape[0] != rows ||
            src.dense->shape[1] != cols)
            return fail(MF_INVALID_SHAPE, "LFM2 dense weight has the wrong shape");
        out->packed = false;
        out->rows = rows;
        out->cols = cols;
        out->dense = static_cast<const float *>(src.dense->ptr);
        return MF_OK;
    }
    if (!src.codes || !src.scales) return fail(MF_MISSING_REQUIRED_TENSOR, "required tensor is missing");
    int32_t st = check_buffer(b, src.codes);
    if (!st) st = check_buffer(b, src.scales);
    if (st) return st;
    if (src.codes->dtype != MF_DTYPE_U8 || src.scales->dtype != MF_DTYPE_F32 || src.codes->rank != 2 ||
        src.scales->rank != 2)
        return fail(MF_INVALID_SHAPE, "packed weight streams must be rank two");
    if (src.codes->shape[0] != rows || src.scales->shape[0] != rows || src.scales->shape[1] * 128 != cols)
        return fail(MF_INVALID_SHAPE, "LFM2 packed weight has the wrong shape");
    const uint64_t cw = src.codes->shape[1];
    int format;
    if (cw == cols / 4) format = MF_TERNARY;
    else if (cw == cols / 2) format = MF_NF4;
    else if (cw == cols) format = MF_INT8;
    else return fail(MF_INVALID_SHAPE, "packed code width must be inner/4 (ternary), inner/2 (nf4), or inner (int8)");
    if (format == MF_INT8 && src.codes->has_int8_reserved) return fail(MF_INVALID_ARGUMENT, "INT8 -128 code is reserved");
    if (src.codes->lut2) return fail(MF_INVALID_ARGUMENT, "LFM2 weights take raw code streams");
    out->packed = true;
    out->format = format;
    out->rows = rows;
    out->cols = cols;
    out->codes = static_cast<const uint8_t *>(src.codes->ptr);
    out->scales = static_cast<const float *>(src.scales->ptr);
    return MF_OK;
}

int32_t resolve_vector(const mf_backend *b, const mf_buffer *buf, uint64_t n, const float **out) {
    if (!buf) return fail(MF_MISSING_REQUIRED_TENSOR, "required tensor is missing");
    int32_t st = check_buffer(b, buf);
    if (st) return st;
    if (buf->dtype != MF_DTYPE_F32 || buf->elements != n) return fail(MF_INVALID_SHAPE, "LFM2 vector weight has the wrong shape");
    *out = static_cast<const float *>(buf->ptr);
    return MF_OK;
}

// execution.rs:12-25: dense `linear` or packed_linear by the role's storage.
int32_t weight_linear(float *out, const float *x, uint64_t t, const Weight &w, const SplitScratch *ss,
                      cudaStream_t s) {
    if (w.packed)
        return packed_matmul(kPackedSingle, false, out, nullptr, x, nullptr, nullptr, t, w.codes, w.scales, nullptr,
                             nullptr, w.rows, w.cols, w.format, ss, s, w.lanetiled);
    return dense_linear(out, x, t, w.dense, w.rows, w.cols, s);
}

int32_t alloc_dev(mf_backend *b, mf_lfm2_state *s, uint64_t elements, int32_t cls, float **out, mf_buffer **handle = nullptr) {
    mf_buffer *buf = nullptr;
    uint64_t shape[1] = {elements};
    int32_t st = mf_allocate_f32(b, shape, 1, cls, 0, &buf);
    if (st) return st;
    s->owned.push_back(buf);
    *out = static_cast<float *>(buf->ptr);
    if (handle) *handle = buf;
    return MF_OK;
}

// Tensor-core GEMM scratch (activation planes + split-K partials) for
// passes of `rows` rows: the largest over this model's projection shapes.
size_t gemm_scratch_floats(const mf_lfm2_config &c, uint64_t rows) {
    const uint64_t h = c.hidden, f = c.intermediate, kvw = (uint64_t)c.kv_heads * c.head_dim;
    const uint64_t shapes[][2] = {{3 * h, h}, {h, h}, {kvw, h}, {f, h}, {h, f}, {c.vocab, h}};
    size_t best = 0;
    for (const auto &sh : shapes) best = std::max(best, packed_gemm_tc_scratch_floats(rows, sh[0], sh[1]));
    return best;
}

int32_t ensure_workspace(mf_lfm2_state *s, uint64_t rows) {
    if (s->ws_buf && s->ws_rows >= rows) return MF_OK;
    mf_lfm2 *m = s->model;
    mf_backend *b = m->b;
    const mf_lfm2_config &c = m->cfg;
    const uint64_t h = c.hidden, f = c.intermediate, kvw = (uint64_t)c.kv_heads * c.head_dim;
    const uint64_t cap = std::max<uint64_t>(rows, s->ws_rows * 2);
    // Attention keeps split-key partials for decode-sized passes (up to 16
    // tokens) and, above that, while tokens x heads < 2048: the buffer is the
    // larger of the two regimes' largest cases.
    const uint64_t split_rows = std::min<uint64_t>(cap, 2047 / c.q_heads);
    const size_t gqa = std::max(causal_gqa_scratch_bytes(std::min<uint64_t>(cap, 16), c.q_heads, c.kv_heads, c.head_dim, c.max_tokens),
                                split_rows ? causal_gqa_scratch_bytes(split_rows, c.q_heads, c.kv_heads, c.head_dim, c.max_tokens)
                                           : (size_t)0);
    // Per-row float counts of each activation buffer, 64-float aligned.
    auto al = [](uint64_t v) { return (v + 63) & ~63ull; };
    const uint64_t sizes[] = {h, h, h, 3 * h, h, h, kvw, kvw, h, kvw, h, h, h, f, f, h, f};
    uint64_t total = 0;
    for (uint64_t sz : sizes) total += al(cap * sz);
    total += al((cap + 16) / 1);              // ids (u32, same byte size as floats)
    total += al(gqa / sizeof(float) + 1);
    if (s->ws_buf) {
        s->owned.erase(std::remove(s->owned.begin(), s->owned.end(), s->ws_buf), s->owned.end());
        mf_buffer_release(b, s->ws_buf);
        s->ws_buf = nullptr;
    }
    // Decode-GEMV split-K partials: the largest need over this model's
    // projection shapes at up to `cap` rows (the GEMV path takes < 48).
    const uint64_t tg = std::min<uint64_t>(cap, kGemmMinTokens - 1);
    const uint64_t shapes[][2] = {{3 * h, h}, {h, h}, {kvw, h}, {f, h}, {h, f}};
    size_t split_floats = std::max(packed_gemv_tc_scratch_floats(1, c.vocab, h), argmax_scratch_floats(1, c.vocab));
    split_floats = std::max<size_t>(split_floats, packed_gemv_tc_scratch_floats(1, c.vocab, h) +
                                                      3 * ((c.vocab + 15) / 16) + 64);  // fused head's CTA partials
    size_t split_counters = std::max<size_t>(64, packed_gemv_tc_counters(1, c.vocab));  // argmax uses 1
    for (const auto &sh : shapes) {
        split_floats = std::max(split_floats, packed_gemv_tc_scratch_floats(tg, sh[0], sh[1]));
        split_counters = std::max(split_counters, packed_gemv_tc_counters(tg, sh[0]));
    }
    // The tensor-core GEMM's BF16 activation planes for many-token passes
    // (widest input: the FFN down projection, k = intermediate).
    if (cap >= kNf4GemmMinTokens)
        split_floats = std::max(split_floats, gemm_scratch_floats(c, cap));
    total += al(split_floats);
    uint64_t shape[1] = {total};
    int32_t st = mf_allocate_f32(b, shape, 1, MF_CLASS_SCRATCH, 1, &s->ws_buf);
    if (st) return st;
    float *p = static_cast<float *>(s->ws_buf->ptr);
    float **dst[] = {&s->x, &s->u, &s->op, &s->proj, &s->conv, &s->q, &s->k, &s->v, &s->qr, &s->kr,
                     &s->att, &s->residual, &s->ffn_in, &s->gate, &s->up, &s->down, &s->hidden_buf};
    for (size_t i = 0; i < sizeof(sizes) / sizeof(sizes[0]); ++i) {
        *dst[i] = p;
        p += al(cap * sizes[i]);
    }
    s->ids = reinterpret_cast<uint32_t *>(p);
    p += al(cap + 16);
    s->gqa_scratch = p;
    s->gqa_scratch_bytes = gqa;
    p += al(gqa / sizeof(float) + 1);
    s->split.partial = p;
    s->split.partial_floats = split_floats;
    // Counters start at zero (zero-initialised allocation) and every launch
    // leaves them at zero, so they survive workspace growth only if large
    // enough; they are reallocated (zeroed) when the model needs more.
    if (!s->split_counters_buf || s->split.n_counters < split_counters) {
        if (s->split_counters_buf) {
            s->owned.erase(std::remove(s->owned.begin(), s->owned.end(), s->split_counters_buf), s->owned.end());
            mf_buffer_release(b, s->split_counters_buf);
            s->split_counters_buf = nullptr;
        }
        uint64_t cshape[1] = {split_counters};
        st = mf_allocate_f32(b, cshape, 1, MF_CLASS_SCRATCH, 0, &s->split_counters_buf);
        if (st) return st;
        s->owned.push_back(s->split_counters_buf);
        s->split.counters = static_cast<unsigned *>(s->split_counters_buf->ptr);
        s->split.n_counters = split_counters;
    }
    s->ws_rows = cap;
    s->ws_epoch++;
    return MF_OK;
}

// One append_tokens pass (execution.rs:35-585).  Token ids come from
// `ids_u32` (staged host ids) or `ids_f32` (device sampled id).
int32_t run_pass(mf_lfm2 *m, mf_lfm2_state *s, uint64_t n, const uint32_t *ids_u32, const float *ids_f32,
                 bool want_logits) {
    const mf_lfm2_config &c = m->cfg;
    cudaStream_t st_ = m->b->stream;
    const uint64_t h = c.hidden, f = c.intermediate, kvw = (uint64_t)c.kv_heads * c.head_dim;
    int32_t st;
    Profiler *prof = s->prof;
    // TRY(cls, bytes, expr): run one op; under the profiler, bracket it with
    // events and record its class, algorithmic bytes and launches.
#define TRY(cls, bytes, expr)                                                        \
    do {                                                                             \
        cudaEvent_t e0_ = nullptr;                                                   \
        uint64_t k0_ = 0;                                                            \
        if (prof) {                                                                  \
            e0_ = prof->next();                                                      \
            k0_ = launches();                                                        \
            if (e0_) Profiler::record(e0_, st_);                                     \
        }                                                                            \
        if ((st = (expr))) return st;                                                \
        if (prof && e0_) {                                                           \
            cudaEvent_t e1_ = prof->next();                                          \
            if (e1_) {                                                               \
                Profiler::record(e1_, st_);                                          \
                prof->ops.push_back({(cls), (uint64_t)(bytes), launches() - k0_, e0_, e1_}); \
            }                                                                        \
        }                                                                            \
    } while (0)
    const uint64_t ctx = s->length;  // cache rows before this pass (host view)
    auto wl = [&](const Weight &w, uint64_t t) { return matmul_bytes(w, t, 1, 1); };
    auto mcls = [](const Weight &w) { return w.packed ? MF_OP_PACKED_MATMUL : MF_OP_DENSE_MATMUL; };
    // execution.rs:69-77
    if (m->emb.packed)
        TRY(MF_OP_GATHER, n * (h * 4 + h / weights_per_byte(m->emb.format) + h / 128 * 4),
            packed_gather_rows(s->x, m->emb.codes, m->emb.scales, m->emb.rows, m->emb.cols, m->emb.format, ids_f32,
                               ids_u32, n, st_));
    else
        TRY(MF_OP_GATHER, n * h * 8, gather_rows(s->x, m->emb.dense, m->emb.rows, m->emb.cols, ids_f32, ids_u32, n, st_));
    // execution.rs:86-94
    if (c.n_layers)
        TRY(MF_OP_NORM_ROPE, n * h * 8 + h * 4,
            row_rms_norm(nullptr, s->u, s->x, nullptr, n, h, m->layers[0].operator_norm, c.block_eps, st_));
    uint64_t rows = n;
    for (uint32_t li = 0; li < c.n_layers; ++li) {
        const Layer &L = m->layers[li];
        if (L.kind == MF_LAYER_CONV) {
            TRY(mcls(L.in_proj), wl(L.in_proj, n), weight_linear(s->proj, s->u, n, L.in_proj, &s->split, st_));
            TRY(MF_OP_CONV, n * 4 * h * 4 + 2 * (uint64_t)(c.conv_width - 1) * h * 4 + h * c.conv_width * 4,
                gated_short_conv(s->conv, s->proj, n, c.hidden, L.conv_kernel, c.conv_width, s->history[li], st_));
            TRY(mcls(L.out_proj), wl(L.out_proj, n), weight_linear(s->op, s->conv, n, L.out_proj, &s->split, st_));
        } else {
            TRY(mcls(L.q), wl(L.q, n), weight_linear(s->q, s->u, n, L.q, &s->split, st_));
            if (L.k.packed && L.v.packed && L.k.format == L.v.format) {
                TRY(MF_OP_PACKED_MATMUL, wl(L.k, n) + wl(L.v, n) - n * h * 4,
                    packed_matmul(kPackedPairRows, false, s->k, s->v, s->u, nullptr, nullptr, n, L.k.codes, L.k.scales,
                                  L.v.codes, L.v.scales, L.k.rows, L.k.cols, L.k.format, &s->split, st_));
            } else {
                TRY(mcls(L.k), wl(L.k, n), weight_linear(s->k, s->u, n, L.k, &s->split, st_));
                TRY(mcls(L.v), wl(L.v, n), weight_linear(s->v, s->u, n, L.v, &s->split, st_));
            }
            TRY(MF_OP_NORM_ROPE, n * h * 8 + c.head_dim * 4,
                head_norm_rope(s->qr, s->q, n, c.q_heads, c.head_dim, L.q_norm, c.block_eps, true, nullptr, s->pos_dev,
                               c.rope_theta, st_));
            TRY(MF_OP_NORM_ROPE, n * kvw * 8 + c.head_dim * 4,
                head_norm_rope(s->kr, s->k, n, c.kv_heads, c.head_dim, L.k_norm, c.block_eps, true, nullptr, s->pos_dev,
                               c.rope_theta, st_));
            // K/V rows read (cache + new), new rows appended, q read, out written.
            TRY(MF_OP_ATTENTION, 2 * (ctx + n) * kvw * 4 + 2 * n * kvw * 4 + 2 * n * h * 4,
                causal_gqa(s->att, s->qr, s->kr, s->v, s->kcache[li], s->vcache[li], c.max_tokens, 0, s->pos_dev, false,
                           n, c.q_heads, c.kv_heads, c.head_dim, s->gqa_scratch, s->gqa_scratch_bytes, st_));
            TRY(mcls(L.o), wl(L.o, n), weight_linear(s->op, s->att, n, L.o, &s->split, st_));
        }
        // execution.rs:265-276
        TRY(MF_OP_NORM_ROPE, n * h * 16 + h * 4,
            row_rms_norm(s->residual, s->ffn_in, s->x, s->op, n, h, L.ffn_norm, c.block_eps, st_));
        // execution.rs:277-299: the final layer's FFN runs on the last row.
        const bool last = li + 1 == c.n_layers;
        const uint64_t ffn_rows = last ? 1 : n;
        const float *fin = last ? s->ffn_in + (n - 1) * h : s->ffn_in;
        const float *res = last ? s->residual + (n - 1) * h : s->residual;
        const bool packed_ffn = L.w1.packed && L.w3.packed && L.w1.format == L.w3.format;
        if (packed_ffn && L.w2.packed) {
            // execution.rs:307-405 fuses SwiGLU into the gate/up epilogue at
            // 96 rows and above, and below that runs the pair, then
            // packed_swiglu_linear.  Both form silu(gate) * up from the same
            // gate/up values with the same rounding (inference.rs:235-243
            // specifies the fused op as equal to pair + swiglu), so the
            // fused form is used at every row count: the activation is
            // formed once per element instead of once per consuming CTA.
            TRY(MF_OP_PACKED_MATMUL, wl(L.w1, ffn_rows) + wl(L.w3, ffn_rows) - ffn_rows * (h + f) * 4,
                packed_matmul(kPackedSwigluPair, false, s->hidden_buf, nullptr, fin, nullptr, nullptr, ffn_rows,
                              L.w1.codes, L.w1.scales, L.w3.codes, L.w3.scales, L.w1.rows, L.w1.cols, L.w1.format, &s->split, st_,
                              L.w1.lanetiled));
            TRY(mcls(L.w2), wl(L.w2, ffn_rows), weight_linear(s->down, s->hidden_buf, ffn_rows, L.w2, &s->split, st_));
        } else {
            if (packed_ffn) {
                TRY(MF_OP_PACKED_MATMUL, wl(L.w1, ffn_rows) + wl(L.w3, ffn_rows) - ffn_rows * h * 4,
                    packed_matmul(kPackedPairRows, false, s->gate, s->up, fin, nullptr, nullptr, ffn_rows, L.w1.codes,
                                  L.w1.scales, L.w3.codes, L.w3.scales, L.w1.rows, L.w1.cols, L.w1.format, &s->split, st_,
                                  L.w1.lanetiled));
            } else {
                TRY(mcls(L.w1), wl(L.w1, ffn_rows), weight_linear(s->gate, fin, ffn_rows, L.w1, &s->split, st_));
                TRY(mcls(L.w3), wl(L.w3, ffn_rows), weight_linear(s->up, fin, ffn_rows, L.w3, &s->split, st_));
            }
            if (L.w2.packed) {
                TRY(MF_OP_PACKED_MATMUL, matmul_bytes(L.w2, ffn_rows, 2, 1),
                    packed_matmul(kPackedSingle, true, s->down, nullptr, nullptr, s->gate, s->up, ffn_rows, L.w2.codes,
                                  L.w2.scales, nullptr, nullptr, L.w2.rows, L.w2.cols, L.w2.format, &s->split, st_,
                                  L.w2.lanetiled));
            } else {
                TRY(MF_OP_OTHER, ffn_rows * f * 12, elementwise(2, s->hidden_buf, s->gate, s->up, ffn_rows * f, st_));
                TRY(mcls(L.w2), wl(L.w2, ffn_rows), weight_linear(s->down, s->hidden_buf, ffn_rows, L.w2, &s->split, st_));
            }
        }
        // execution.rs:499-517: next operator norm or the final embedding norm.
        const float *norm_w = last ? m->emb_norm : m->layers[li + 1].operator_norm;
        const float eps = last ? c.norm_eps : c.block_eps;
        TRY(MF_OP_NORM_ROPE, ffn_rows * h * 16 + h * 4, row_rms_norm(s->x, s->u, res, s->down, ffn_rows, h, norm_w, eps, st_));
        rows = ffn_rows;
    }
    if (c.n_layers == 0)
        TRY(MF_OP_NORM_ROPE, n * h * 8 + h * 4, row_rms_norm(nullptr, s->u, s->x, nullptr, n, h, m->emb_norm, c.norm_eps, st_));
    if (want_logits) {
        // execution.rs:540-572
        float *logits = static_cast<float *>(s->logits->ptr);
        TRY(mcls(m->emb), wl(m->emb, 1), weight_linear(logits, s->u + (rows - 1) * h, 1, m->emb, &s->split, st_));
    }
    if (int32_t e_ = ::mf::launch(advance_position_kernel, dim3(1), dim3(1), 0, st_, "advance_position_kernel", s->pos_dev, n)) return e_;
#undef TRY
    return MF_OK;
}

// Whether a one-token step can run through the fused projections: every
// projection packed, q/k/v in one format (one three-matrix launch), w1/w3
// in one format (one SwiGLU-pair launch), widths the shared-memory staging
// of the normalizing prologue takes.
bool fused_step_ok(const mf_lfm2 *m) {
    const mf_lfm2_config &c = m->cfg;
    if (c.n_layers == 0 || c.hidden > 8192 || c.hidden % 128 || c.intermediate % 128) return false;
    for (const Layer &L : m->layers) {
        if (L.kind == MF_LAYER_CONV) {
            if (!L.in_proj.packed || !L.out_proj.packed) return false;
        } else {
            if (!L.q.packed || !L.k.packed || !L.v.packed || !L.o.packed) return false;
            if (L.q.format != L.k.format || L.k.format != L.v.format) return false;
        }
        if (!L.w1.packed || !L.w2.packed || !L.w3.packed || L.w1.format != L.w3.format) return false;
        if (L.w2.format == MF_NF4 && c.intermediate > 8192) return false;
    }
    return true;
}

// A projection of the plain row `x`: the integer-MMA formats stage the row
// and split it into limbs inside each CTA (no separate limb pass) when the
// row fits the staged prologue; NF4 reads its x slices directly.
DecodeGemv plain(DecodeGemv d, const float *x) {
    d.x = x;
    if (d.format == MF_NF4) return d;
    // Every CTA re-reads and re-splits the whole row: worth it only for
    // short rows (a long row pays more than the separate limb pass).
    if (d.k > 2048) return d;
    DecodeGemv staged = d;
    staged.x = nullptr;
    staged.na = x;
    return decode_gemv_supports(staged) ? staged : d;
}

DecodeGemv proj(const Weight &w, float *out) {
    DecodeGemv d;
    d.format = w.format;
    d.codes[0] = w.codes;
    d.scales[0] = w.scales;
    d.out[0] = out;
    d.n = w.rows;
    d.k = w.cols;
    d.lanetiled = w.lanetiled;
    return d;
}

// One greedy step (the op order of execution.rs:35-627 for one row, then
// sample_epilogue :591-614), with every RMSNorm moved into the prologue of
// the projection that consumes it and the argmax and position advance into
// the LM head's epilogue.  The token id is the device f32 in s->sampled;
// the greedy id replaces it.  Same values as run_pass + argmax: the norms,
// SwiGLU and residual adds round exactly as there; only the order of the
// reductions inside the norms and the projections differs.
int32_t run_decode_fused(mf_lfm2 *m, mf_lfm2_state *s) {
    const mf_lfm2_config &c = m->cfg;
    cudaStream_t st_ = m->b->stream;
    const uint64_t h = c.hidden;
    const float *sampled = static_cast<const float *>(s->sampled->ptr);
    int32_t st;
    // Labels for mf_lfm2_time_step (no effect unless a recorder is set).
    LaunchRecorder *rec = launch_recorder();
    auto label = [&](const char *l) {
        if (rec) rec->label = l;
    };
    for (uint32_t li = 0; li < c.n_layers; ++li) {
        const Layer &L = m->layers[li];
        // Layer input residual: the embedding row (layer 0) or the previous
        // layer's residual + FFN output; normalized by this layer's operator norm.
        auto with_norm = [&](DecodeGemv d) {
            d.x = nullptr;
            d.nw = L.operator_norm;
            d.eps = c.block_eps;
            d.nres = s->x;
            if (li == 0) {
                d.eid = sampled;
                d.erows = m->emb.rows;
                if (m->emb.packed) {
                    d.ecodes = m->emb.codes;
                    d.escales = m->emb.scales;
                    d.eformat = m->emb.format;
                } else {
                    d.edense = m->emb.dense;
                }
            } else {
                d.na = s->residual;
                d.nb = s->down;
            }
            return d;
        };
        if (L.kind == MF_LAYER_CONV) {
            // An NF4 in_proj computes the convolution in its epilogue (each CTA
            // owns the B, C and x rows of its channels and their history).
            label("conv_in_proj");
            DecodeGemv ip = with_norm(proj(L.in_proj, s->conv));
            ip.mode = 4;
            ip.n = c.hidden;
            ip.conv_kernel = L.conv_kernel;
            ip.conv_hist = s->history[li];
            ip.conv_width = c.conv_width;
            if (decode_gemv_conv_supported(ip)) {
                if ((st = decode_gemv(ip, s->split, st_))) return st;
            } else {
                if ((st = decode_gemv(with_norm(proj(L.in_proj, s->proj)), s->split, st_))) return st;
                if ((st = gated_short_conv(s->conv, s->proj, 1, c.hidden, L.conv_kernel, c.conv_width, s->history[li],
                                           st_)))
                    return st;
            }
            label("conv_out_proj");
            if ((st = decode_gemv(plain(proj(L.out_proj, s->op), s->conv), s->split, st_))) return st;
        } else {
            label("attn_qkv");
            DecodeGemv qkv = proj(L.q, s->q);
            qkv.mode = 3;
            qkv.codes[1] = L.k.codes;
            qkv.scales[1] = L.k.scales;
            qkv.out[1] = s->k;
            qkv.codes[2] = L.v.codes;
            qkv.scales[2] = L.v.scales;
            qkv.out[2] = s->v;
            qkv.n2 = L.k.rows;
            if ((st = decode_gemv(with_norm(qkv), s->split, st_))) return st;
            label("attention");
            if (m->rope && gqa_decode_fused_supported(c.q_heads, c.kv_heads, c.head_dim, c.max_tokens)) {
                if ((st = gqa_decode_fused(s->att, s->q, s->k, s->v, L.q_norm, L.k_norm, c.block_eps, m->rope,
                                           s->kcache[li], s->vcache[li], c.max_tokens, s->pos_dev, c.q_heads,
                                           c.kv_heads, c.head_dim, s->gqa_scratch, s->gqa_scratch_bytes,
                                           s->split.counters, s->split.n_counters, st_)))
                    return st;
            } else {
                if ((st = head_norm_rope(s->qr, s->q, 1, c.q_heads, c.head_dim, L.q_norm, c.block_eps, true, nullptr,
                                         s->pos_dev, c.rope_theta, st_)))
                    return st;
                if ((st = head_norm_rope(s->kr, s->k, 1, c.kv_heads, c.head_dim, L.k_norm, c.block_eps, true, nullptr,
                                         s->pos_dev, c.rope_theta, st_)))
                    return st;
                if ((st = causal_gqa(s->att, s->qr, s->kr, s->v, s->kcache[li], s->vcache[li], c.max_tokens, 0,
                                     s->pos_dev, false, 1, c.q_heads, c.kv_heads, c.head_dim, s->gqa_scratch,
                                     s->gqa_scratch_bytes, st_)))
                    return st;
            }
            label("attn_o");
            if ((st = decode_gemv(plain(proj(L.o, s->op), s->att), s->split, st_))) return st;
        }
        // FFN: residual + mixer output, FFN norm, gate/up with SwiGLU, down.
        label("ffn_gate_up");
        DecodeGemv ff = proj(L.w1, s->hidden_buf);
        ff.mode = 2;
        ff.codes[1] = L.w3.codes;
        ff.scales[1] = L.w3.scales;
        ff.x = nullptr;
        ff.na = s->x;
        ff.nb = s->op;
        ff.nw = L.ffn_norm;
        ff.eps = c.block_eps;
        ff.nres = s->residual;
        // An integer-MMA w2 takes its input limbs from the pair's epilogue.
        DecodeGemv down = proj(L.w2, s->down);
        ff.limbs_for = L.w2.format;
        if (L.w2.format != MF_NF4 && decode_gemv_limbs_supported(ff)) {
            down.x = s->hidden_buf;
            down.limbs_ready = true;
        } else {
            ff.limbs_for = -1;
            down = plain(down, s->hidden_buf);
        }
        if ((st = decode_gemv(ff, s->split, st_))) return st;
        label("ffn_down");
        if ((st = decode_gemv(down, s->split, st_))) return st;
    }
    label("lm_head");
    float *logits = static_cast<float *>(s->logits->ptr);
    float *sampled_out = static_cast<float *>(s->sampled->ptr);
    const float *res = s->residual, *dlt = s->down;
    if (m->head_world > 1) {
        // Row-split head (every rank runs the same layers on the same token,
        // so each holds the same normed row): this rank's rows and their
        // candidate, the all-gather of the ranks' candidates, then the pick.
        const Weight &e = m->emb;
        const uint64_t r0 = m->head_row0, nr = m->head_rows;
        if ((st = row_rms_norm(s->x, s->u, res, dlt, 1, h, m->emb_norm, c.norm_eps, st_))) return st;
        if (e.packed) {
            DecodeGemv hd = proj(e, logits + r0);
            const uint64_t row_bytes = e.cols / (e.format == MF_TERNARY ? 4 : 1);
            hd.codes[0] = e.codes + r0 * row_bytes;
            hd.scales[0] = e.scales + r0 * (e.cols / kGroup);
            hd.n = nr;
            hd.x = s->u;
            hd.cand = m->head_cand;
            hd.row0 = r0;
            st = decode_gemv(hd, s->split, st_);
        } else {
            st = dense_head_argmax(logits + r0, s->u, e.dense + r0 * e.cols, nr, e.cols, s->split.partial,
                                   s->split.partial_floats, s->split.counters, nullptr, nullptr, st_, m->head_cand, r0);
        }
        if (st) return st;
        if ((st = nccl_all_gather_f32(m->head_cand, m->head_cands, 3, m->head_comm, st_))) return st;
        return head_shard_pick(m->head_cands, m->head_world, sampled_out, s->pos_dev, st_);
    }
    if (m->emb.packed && m->emb.format != MF_NF4) {
        // execution.rs:499-572 + :591-614: final norm, LM head, greedy id.
        // A head of many row tiles runs in several waves, so its norm is one
        // small kernel rather than a prologue repeated by every CTA.
        DecodeGemv hd = proj(m->emb, logits);
        hd.sampled = sampled_out;
        hd.pos = s->pos_dev;
        if (m->emb.rows > 16384) {
            if ((st = row_rms_norm(s->x, s->u, res, dlt, 1, h, m->emb_norm, c.norm_eps, st_))) return st;
            hd.x = s->u;
        } else {
            hd.x = nullptr;
            hd.na = res;
            hd.nb = dlt;
            hd.nw = m->emb_norm;
            hd.eps = c.norm_eps;
            hd.nres = s->x;
        }
        return decode_gemv(hd, s->split, st_);
    }
    // Dense F32 head: the norm, then one streaming head kernel with the
    // greedy argmax and the position advance fused.
    if (!m->emb.packed && dense_head_argmax_supported(m->emb.rows, m->emb.cols) &&
        s->split.partial_floats >= dense_head_parts_floats() && s->split.n_counters >= 1) {
        if ((st = row_rms_norm(s->x, s->u, res, dlt, 1, h, m->emb_norm, c.norm_eps, st_))) return st;
        return dense_head_argmax(logits, s->u, m->emb.dense, m->emb.rows, m->emb.cols, s->split.partial,
                                 s->split.partial_floats, s->split.counters, sampled_out, s->pos_dev, st_);
    }
    // NF4 head: separate norm, head and argmax, then the position.
    if ((st = row_rms_norm(s->x, s->u, res, dlt, 1, h, m->emb_norm, c.norm_eps, st_))) return st;
    if ((st = weight_linear(logits, s->u, 1, m->emb, &s->split, st_))) return st;
    if ((st = argmax(sampled_out, logits, 1, c.vocab, nullptr, &s->split, st_))) return st;
    if (int32_t e_ = ::mf::launch(advance_position_kernel, dim3(1), dim3(1), 0, st_, "advance_position_kernel",
                                  s->pos_dev, (uint64_t)1))
        return e_;
    return MF_OK;
}

// Builds the state's persistent-step program on first use.  Must run
// outside stream capture (it allocates and uploads); a state whose model or
// device cannot take the persistent step keeps the fused path.
int32_t ensure_persistent(mf_lfm2 *m, mf_lfm2_state *s) {
    if (!m->fused || !m->persistent || !m->persistent_ok || s->pplan || s->pers_state < 0 || m->head_world > 1)
        return MF_OK;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(m->b->stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return MF_OK;
    const int sms = sm_count();
    PersistStateDesc sd;
    sd.pos = s->pos_dev;
    sd.sampled = static_cast<float *>(s->sampled->ptr);
    sd.logits = static_cast<float *>(s->logits->ptr);
    sd.history = s->history;
    sd.kcache = s->kcache;
    sd.vcache = s->vcache;
    const size_t bytes = persistent_ws_bytes(m->pdesc, sms);
    float *ws = nullptr;
    int32_t st = alloc_dev(m->b, s, (bytes + 3) / 4, MF_CLASS_SCRATCH, &ws, &s->pers_buf);
    if (st) return st;
    PersistPlan *pl = nullptr;
    st = persistent_plan(m->pdesc, sd, sms, ws, &pl);
    if (st == MF_UNSUPPORTED) {
        s->pers_state = -1;
        return MF_OK;
    }
    if (!st) st = persistent_init(pl, ws, bytes, m->b->stream);
    if (st) {
        if (pl) persistent_free(pl);
        return st;
    }
    s->pplan = pl;
    s->pers_state = 1;
    return MF_OK;
}

// One greedy step on the device-resident id in s->sampled: the persistent
// step, else the fused step when the model allows it, else the op-by-op
// pass and a separate argmax.
int32_t greedy_step(mf_lfm2 *m, mf_lfm2_state *s) {
    if (m->fused && m->persistent && s->pplan) return persistent_launch(s->pplan, sm_count(), m->b->stream);
    if (m->fused && fused_step_ok(m)) return run_decode_fused(m, s);
    int32_t st = run_pass(m, s, 1, nullptr, static_cast<const float *>(s->sampled->ptr), true);
    if (!st)
        st = argmax(static_cast<float *>(s->sampled->ptr), static_cast<float *>(s->logits->ptr), 1, m->cfg.vocab,
                    nullptr, &s->split, m->b->stream);
    return st;
}

uint64_t count_step_kernels(const mf_lfm2 *m) {
    // gather + norm + per layer (mixer + 2 norms + ffn) + head + argmax + advance,
    // counted by running the accounting once (set at model creation).
    return m->kernels_per_step;
}

}  // namespace

extern "C" {

int32_t mf_lfm2_create(mf_backend *b, const mf_lfm2_config *config, const mf_lfm2_weight *embedding,
                       const mf_buffer *embedding_norm, const mf_lfm2_layer *layers, mf_lfm2 **out) {
    if (!b || !config || !embedding || !out || (config->n_layers && (!layers || !config->layer_kinds)))
        return fail(MF_INVALID_ARGUMENT, "null argument");
    const mf_lfm2_config &c = *config;
    if (!c.hidden || !c.q_heads || !c.kv_heads || c.q_heads % c.kv_heads || !c.head_dim ||
        (uint64_t)c.q_heads * c.head_dim != c.hidden || !c.conv_width || !c.vocab || c.head_dim % 2)
        return fail(MF_INVALID_SHAPE, "LFM2 configuration geometry is inconsistent");
    if (c.vocab > (1u << 24)) return fail(MF_UNSUPPORTED, "vocabulary exceeds exact f32 token ids");
    mf_lfm2 *m = new (std::nothrow) mf_lfm2();
    if (!m) return fail(MF_RESOURCE_LIMIT, "host allocation failed");
    m->b = b;
    m->cfg = c;
    m->kinds.assign(c.layer_kinds, c.layer_kinds + c.n_layers);
    m->cfg.layer_kinds = m->kinds.data();
    const uint64_t h = c.hidden, f = c.intermediate, kvw = (uint64_t)c.kv_heads * c.head_dim;
    int32_t st = resolve_weight(b, *embedding, c.vocab, h, &m->emb);
    if (!st) st = resolve_vector(b, embedding_norm, h, &m->emb_norm);
    m->layers.resize(c.n_layers);
    for (uint32_t i = 0; !st && i < c.n_layers; ++i) {
        const mf_lfm2_layer &src = layers[i];
        Layer &L = m->layers[i];
        L.kind = c.layer_kinds[i];
        if (L.kind == MF_LAYER_CONV) {
            st = resolve_weight(b, src.in_proj, 3 * h, h, &L.in_proj);
            if (!st) st = resolve_weight(b, src.out_proj, h, h, &L.out_proj);
            if (!st) st = resolve_vector(b, src.conv_kernel, h * c.conv_width, &L.conv_kernel);
        } else if (L.kind == MF_LAYER_ATTENTION) {
            st = resolve_weight(b, src.q, h, h, &L.q);
            if (!st) st = resolve_weight(b, src.k, kvw, h, &L.k);
            if (!st) st = resolve_weight(b, src.v, kvw, h, &L.v);
            if (!st) st = resolve_weight(b, src.o, h, h, &L.o);
            if (!st) st = resolve_vector(b, src.q_norm, c.head_dim, &L.q_norm);
            if (!st) st = resolve_vector(b, src.k_norm, c.head_dim, &L.k_norm);
        } else {
            st = fail(MF_INVALID_ARGUMENT, "unknown layer kind");
        }
        if (!st) st = resolve_weight(b, src.w1, f, h, &L.w1);
        if (!st) st = resolve_weight(b, src.w3, f, h, &L.w3);
        if (!st) st = resolve_weight(b, src.w2, h, f, &L.w2);
        if (!st) st = resolve_vector(b, src.ffn_norm, h, &L.ffn_norm);
        if (!st) st = resolve_vector(b, src.operator_norm, h, &L.operator_norm);
    }
    if (st) {
        delete m;
        return st;
    }
    if (std::count(m->kinds.begin(), m->kinds.end(), (int32_t)MF_LAYER_ATTENTION)) {
        // (sin, cos) for every position the caches can hold.
        uint64_t shape[1] = {2 * c.max_tokens * (c.head_dim / 2)};
        st = mf_allocate_f32(b, shape, 1, MF_CLASS_WEIGHT, 1, &m->rope_buf);
        if (!st) {
            m->rope = static_cast<const float2 *>(m->rope_buf->ptr);
            st = rope_table(static_cast<float2 *>(m->rope_buf->ptr), c.max_tokens, c.head_dim, c.rope_theta, b->stream);
        }
        if (st) {
            mf_lfm2_destroy(m);
            return st;
        }
    }
    m->kernels_per_step = 0;
    m->fused = true;
    {
        PersistModelDesc &d = m->pdesc;
        auto pm = [](const Weight &w) {
            PersistMat r;
            r.codes = w.packed ? w.codes : nullptr;
            r.scales = w.packed ? w.scales : nullptr;
            r.dense = w.packed ? nullptr : w.dense;
            r.format = w.format;
            r.rows = (uint32_t)w.rows;
            return r;
        };
        d.hidden = c.hidden;
        d.intermediate = c.intermediate;
        d.q_heads = c.q_heads;
        d.kv_heads = c.kv_heads;
        d.head_dim = c.head_dim;
        d.conv_width = c.conv_width;
        d.vocab = c.vocab;
        d.block_eps = c.block_eps;
        d.norm_eps = c.norm_eps;
        d.max_tokens = c.max_tokens;
        d.emb = pm(m->emb);
        d.emb_norm = m->emb_norm;
        d.rope = m->rope;
        for (const Layer &L : m->layers) {
            PersistLayerDesc pl;
            pl.kind = L.kind;
            pl.in_proj = pm(L.in_proj);
            pl.out_proj = pm(L.out_proj);
            pl.q = pm(L.q);
            pl.k = pm(L.k);
            pl.v = pm(L.v);
            pl.o = pm(L.o);
            pl.w1 = pm(L.w1);
            pl.w2 = pm(L.w2);
            pl.w3 = pm(L.w3);
            pl.conv_kernel = L.conv_kernel;
            pl.q_norm = L.q_norm;
            pl.k_norm = L.k_norm;
            pl.ffn_norm = L.ffn_norm;
            pl.operator_norm = L.operator_norm;
            d.layers.push_back(pl);
        }
        m->persistent_ok = c.n_layers > 0 && persistent_geometry_ok(d);
    }
    *out = m;
    return MF_OK;
}

int32_t mf_lfm2_destroy(mf_lfm2 *m) {
    if (m && m->rope_buf) mf_buffer_release(m->b, m->rope_buf);
    if (m) {
        for (mf_buffer *buf : m->owned) mf_buffer_release(m->b, buf);
        for (mf_buffer *buf : m->lut2) mf_buffer_release(m->b, buf);
        if (m->head_buf) mf_buffer_release(m->b, m->head_buf);
        if (m->head_comm) {
            cudaStreamSynchronize(m->b->stream);
            nccl_comm_destroy(m->head_comm);
        }
    }
    delete m;
    return MF_OK;
}

int32_t mf_lfm2_state_create(mf_lfm2 *m, mf_lfm2_state **out) {
    if (!m || !out) return fail(MF_INVALID_ARGUMENT, "null argument");
    mf_lfm2_state *s = new (std::nothrow) mf_lfm2_state();
    if (!s) return fail(MF_RESOURCE_LIMIT, "host allocation failed");
    s->model = m;
    const mf_lfm2_config &c = m->cfg;
    const uint64_t h = c.hidden, kvw = (uint64_t)c.kv_heads * c.head_dim;
    s->history.assign(c.n_layers, nullptr);
    s->kcache.assign(c.n_layers, nullptr);
    s->vcache.assign(c.n_layers, nullptr);
    int32_t st = MF_OK;
    for (uint32_t i = 0; !st && i < c.n_layers; ++i) {
        if (m->layers[i].kind == MF_LAYER_CONV) {
            st = alloc_dev(m->b, s, (uint64_t)(c.conv_width - 1) * h + 1, MF_CLASS_CACHE, &s->history[i]);
        } else {
            st = alloc_dev(m->b, s, c.max_tokens * kvw + 1, MF_CLASS_CACHE, &s->kcache[i]);
            if (!st) st = alloc_dev(m->b, s, c.max_tokens * kvw + 1, MF_CLASS_CACHE, &s->vcache[i]);
        }
    }
    float *tmp = nullptr;
    if (!st) st = alloc_dev(m->b, s, 2, MF_CLASS_CACHE, &tmp, &s->pos_buf);
    s->pos_dev = reinterpret_cast<uint64_t *>(tmp);
    if (!st) {
        uint64_t shape[2] = {1, c.vocab};
        st = mf_allocate_f32(m->b, shape, 2, MF_CLASS_CACHE, 0, &s->logits);
        if (!st) s->owned.push_back(s->logits);
    }
    if (!st) {
        uint64_t shape[1] = {1};
        st = mf_allocate_f32(m->b, shape, 1, MF_CLASS_CACHE, 0, &s->sampled);
        if (!st) s->owned.push_back(s->sampled);
    }
    if (!st) st = ensure_workspace(s, 1);
    if (st) {
        mf_lfm2_state_destroy(s);
        return st;
    }
    *out = s;
    return MF_OK;
}

int32_t mf_lfm2_state_destroy(mf_lfm2_state *s) {
    if (!s) return MF_OK;
    if (s->pplan) persistent_free(s->pplan);
    if (s->graph) cudaGraphExecDestroy(s->graph);
    if (s->graph_multi) cudaGraphExecDestroy(s->graph_multi);
    if (s->graph_gen) cudaGraphExecDestroy(s->graph_gen);
    if (s->gen_ctl_host) cudaFreeHost(s->gen_ctl_host);
    if (s->gen_ids_host) cudaFreeHost(s->gen_ids_host);
    if (s->io_pinned) cudaFreeHost(s->io_pinned);
    if (s->io_done) cudaEventDestroy(s->io_done);
    for (mf_buffer *buf : s->owned) mf_buffer_release(s->model->b, buf);
    delete s;
    return MF_OK;
}

int32_t mf_lfm2_state_fork(mf_lfm2 *m, const mf_lfm2_state *src, mf_lfm2_state **out) {
    if (!m || !src || !out || src->model != m) return fail(MF_INVALID_ARGUMENT, "state belongs to another model");
    mf_lfm2_state *s = nullptr;
    int32_t st = mf_lfm2_state_create(m, &s);
    if (st) return st;
    const mf_lfm2_config &c = m->cfg;
    const uint64_t h = c.hidden, kvw = (uint64_t)c.kv_heads * c.head_dim;
    cudaStream_t stream = m->b->stream;
    for (uint32_t i = 0; i < c.n_layers; ++i) {
        if (m->layers[i].kind == MF_LAYER_CONV) {
            MF_CUDA_TRY(cudaMemcpyAsync(s->history[i], src->history[i], (c.conv_width - 1) * h * sizeof(float),
                                        cudaMemcpyDeviceToDevice, stream));
        } else if (src->length) {
            MF_CUDA_TRY(cudaMemcpyAsync(s->kcache[i], src->kcache[i], src->length * kvw * sizeof(float),
                                        cudaMemcpyDeviceToDevice, stream));
            MF_CUDA_TRY(cudaMemcpyAsync(s->vcache[i], src->vcache[i], src->length * kvw * sizeof(float),
                                        cudaMemcpyDeviceToDevice, stream));
        }
    }
    MF_CUDA_TRY(cudaMemcpyAsync(s->pos_dev, src->pos_dev, sizeof(uint64_t), cudaMemcpyDeviceToDevice, stream));
    MF_CUDA_TRY(cudaMemcpyAsync(s->logits->ptr, src->logits->ptr, src->logits->bytes, cudaMemcpyDeviceToDevice, stream));
    MF_CUDA_TRY(cudaMemcpyAsync(s->sampled->ptr, src->sampled->ptr, sizeof(float), cudaMemcpyDeviceToDevice, stream));
    s->length = src->length;
    *out = s;
    return MF_OK;
}

uint64_t mf_lfm2_state_length(const mf_lfm2_state *s) { return s ? s->length : 0; }
const mf_buffer *mf_lfm2_state_logits(const mf_lfm2_state *s) { return s ? s->logits : nullptr; }
const mf_buffer *mf_lfm2_state_sampled(const mf_lfm2_state *s) { return s ? s->sampled : nullptr; }

int32_t mf_lfm2_append(mf_lfm2 *m, mf_lfm2_state *s, const uint32_t *tokens, uint64_t n, int32_t want_logits) {
    if (!m || !s || s->model != m) return fail(MF_INVALID_ARGUMENT, "state belongs to another model");
    if (n == 0) return fail(MF_INVALID_ARGUMENT, "token pass requires at least one token");
    if (!tokens) return fail(MF_INVALID_ARGUMENT, "null tokens");
    for (uint64_t i = 0; i < n; ++i)
        if (tokens[i] >= m->cfg.vocab) return fail(MF_OUT_OF_BOUNDS, "valid token ID exceeds loaded model vocabulary");
    if (s->length > m->cfg.max_tokens || n > m->cfg.max_tokens - s->length)
        return fail(MF_RESOURCE_LIMIT, "token pass exceeds the configured context capacity");
    int32_t st = ensure_workspace(s, n);
    if (st) return st;
    MF_CUDA_TRY(cudaMemcpyAsync(s->ids, tokens, n * sizeof(uint32_t), cudaMemcpyHostToDevice, m->b->stream));
    st = run_pass(m, s, n, s->ids, nullptr, want_logits != 0);
    if (st) return st;
    s->length += n;
    return MF_OK;
}

int32_t mf_lfm2_append_argmax(mf_lfm2 *m, mf_lfm2_state *s, uint32_t token, int32_t token_from_sample) {
    if (!m || !s || s->model != m) return fail(MF_INVALID_ARGUMENT, "state belongs to another model");
    if (!token_from_sample && token >= m->cfg.vocab)
        return fail(MF_OUT_OF_BOUNDS, "valid token ID exceeds loaded model vocabulary");
    if (s->length >= m->cfg.max_tokens) return fail(MF_RESOURCE_LIMIT, "token pass exceeds the configured context capacity");
    int32_t st = ensure_workspace(s, 1);
    if (st) return st;
    const uint64_t before = launches();
    if (!token_from_sample) {
        // The step embeds the id held in the sampled slot (f32, exact below 2^24).
        s->host_token = (float)token;
        MF_CUDA_TRY(cudaMemcpyAsync(s->sampled->ptr, &s->host_token, sizeof(float), cudaMemcpyHostToDevice,
                                    m->b->stream));
    }
    if ((st = ensure_persistent(m, s))) return st;
    st = greedy_step(m, s);
    if (st) return st;
    m->kernels_per_step = launches() - before;
    s->length += 1;
    return MF_OK;
}

int32_t mf_lfm2_read_sampled(mf_lfm2_state *s, float *out) {
    if (!s || !out) return fail(MF_INVALID_ARGUMENT, "null argument");
    MF_CUDA_TRY(cudaMemcpyAsync(out, s->sampled->ptr, sizeof(float), cudaMemcpyDeviceToHost, s->model->b->stream));
    MF_CUDA_TRY(cudaStreamSynchronize(s->model->b->stream));
    return MF_OK;
}

}  // extern "C"

namespace {

// Captures one decode step (device-resident token and position) into the
// state's graph if it has none, or if the workspace moved since capture.
int32_t ensure_decode_graph(mf_lfm2 *m, mf_lfm2_state *s) {
    int32_t st = ensure_workspace(s, 1);
    if (st) return st;
    if ((st = ensure_persistent(m, s))) return st;
    if (s->graph && s->graph_epoch == s->ws_epoch && s->graph_model_epoch == m->epoch) return MF_OK;
    cudaStream_t stream = m->b->stream;
    if (s->graph) {
        cudaGraphExecDestroy(s->graph);
        s->graph = nullptr;
    }
    const uint64_t before = launches();
    MF_CUDA_TRY(cudaStreamBeginCapture(stream, cudaStreamCaptureModeRelaxed));
    st = greedy_step(m, s);
    cudaGraph_t graph = nullptr;
    cudaError_t err = cudaStreamEndCapture(stream, &graph);
    if (st) {
        if (graph) cudaGraphDestroy(graph);
        return st;
    }
    if (err != cudaSuccess) return cuda_fail(err, "cudaStreamEndCapture");
    m->kernels_per_step = launches() - before;
    // Captured launches did not run; back them out of the launch count.
    count_launch(-(int64_t)m->kernels_per_step);
    err = cudaGraphInstantiate(&s->graph, graph, 0);
    cudaGraphDestroy(graph);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGraphInstantiate");
    s->graph_epoch = s->ws_epoch;
    s->graph_model_epoch = m->epoch;
    return MF_OK;
}

constexpr uint64_t kMultiSteps = 8;

// The kMultiSteps-step graph (after ensure_decode_graph sized the workspace).
int32_t ensure_multi_graph(mf_lfm2 *m, mf_lfm2_state *s) {
    if (s->graph_multi && s->graph_multi_epoch == s->ws_epoch) return MF_OK;
    cudaStream_t stream = m->b->stream;
    if (s->graph_multi) {
        cudaGraphExecDestroy(s->graph_multi);
        s->graph_multi = nullptr;
    }
    const uint64_t before = launches();
    MF_CUDA_TRY(cudaStreamBeginCapture(stream, cudaStreamCaptureModeRelaxed));
    int32_t st = MF_OK;
    for (uint64_t i = 0; i < kMultiSteps && !st; ++i) st = greedy_step(m, s);
    cudaGraph_t graph = nullptr;
    cudaError_t err = cudaStreamEndCapture(stream, &graph);
    count_launch(-(int64_t)(launches() - before));   // captured, not run
    if (st) {
        if (graph) cudaGraphDestroy(graph);
        return st;
    }
    if (err != cudaSuccess) return cuda_fail(err, "cudaStreamEndCapture");
    err = cudaGraphInstantiate(&s->graph_multi, graph, 0);
    cudaGraphDestroy(graph);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGraphInstantiate");
    s->graph_multi_epoch = s->ws_epoch;
    return MF_OK;
}

constexpr uint32_t kGenMaxStop = 64;

}  // namespace

// Control block of the device-side generation loop.
struct GenCtl {
    uint64_t max_tokens;   // ids to produce at most
    uint64_t n_out;        // ids produced
    uint64_t steps;        // greedy steps run
    uint64_t cap_left;     // context positions left when the call started
    uint64_t ids_cap;      // capacity of the device id buffer
    uint32_t n_stop, vocab;
    int32_t stopped;
    int32_t error;         // 1: the step published no valid sample; 2: context capacity
    uint32_t stop_ids[kGenMaxStop];
};

namespace {

// One check of the generation loop, on one thread: the body of the host
// loop of crates/text-generation/src/lib.rs:304-460 as mf_lfm2_generate's
// fallback runs it (read the greedy sample; a stop id ends the call; else
// append it; the token budget, then the context capacity, bound the next
// step), its verdict written to the WHILE node's condition.
__global__ void gen_check_kernel(GenCtl *c, const float *sampled, float *ids, cudaGraphConditionalHandle h) {
    unsigned go = 0;
    const float id = *sampled;
    if (!(id >= 0.0f) || id >= (float)c->vocab) {
        c->error = 1;
    } else {
        const uint32_t tok = (uint32_t)id;
        bool stop = false;
        for (uint32_t i = 0; i < c->n_stop && i < kGenMaxStop; ++i) stop |= c->stop_ids[i] == tok;
        if (stop) {
            c->stopped = 1;
        } else if (c->n_out >= c->ids_cap) {
            c->error = 2;
        } else {
            ids[c->n_out++] = id;
            if (c->n_out < c->max_tokens) {
                if (c->steps >= c->cap_left) {
                    c->error = 2;
                } else {
                    c->steps++;
                    go = 1;
                }
            }
        }
    }
    cudaGraphSetConditional(h, go);
}

// The generation graph: check -> WHILE(check said go) { greedy step; check }.
// Every iteration that continues appends one id, and the ids are bounded by
// max_tokens and by the context capacity, so the loop ends.  Returns
// MF_UNSUPPORTED (and remembers it) where the driver does not build it.
int32_t ensure_gen_graph(mf_lfm2 *m, mf_lfm2_state *s) {
    if (s->gen_unsupported) return MF_UNSUPPORTED;
    // A split head's all-gather stays out of the conditional graph: the
    // host form of the loop runs instead.
    if (m->head_world > 1) return MF_UNSUPPORTED;
    if (int32_t pst = ensure_persistent(m, s)) return pst;
    if (s->graph_gen && s->graph_gen_epoch == s->ws_epoch && s->graph_gen_model_epoch == m->epoch) return MF_OK;
    const mf_lfm2_config &c = m->cfg;
    if (!s->gen_ctl) {
        const uint64_t ctl_words = (sizeof(GenCtl) + 3) / 4;
        float *ctl = nullptr;
        int32_t st = alloc_dev(m->b, s, ctl_words, MF_CLASS_SCRATCH, &ctl);
        if (!st) st = alloc_dev(m->b, s, (uint64_t)c.max_tokens + 1, MF_CLASS_SCRATCH, &s->gen_ids);
        if (st) return st;
        s->gen_ctl = reinterpret_cast<GenCtl *>(ctl);
        s->gen_ids_cap = (uint64_t)c.max_tokens + 1;
    }
    if (!s->gen_ctl_host)
        MF_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void **>(&s->gen_ctl_host), sizeof(GenCtl), cudaHostAllocDefault));
    if (!s->gen_ids_host)
        MF_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void **>(&s->gen_ids_host), s->gen_ids_cap * sizeof(float),
                                  cudaHostAllocDefault));
    if (s->graph_gen) {
        cudaGraphExecDestroy(s->graph_gen);
        s->graph_gen = nullptr;
    }
    cudaStream_t stream = m->b->stream;
    float *sampled = static_cast<float *>(s->sampled->ptr);
    cudaGraph_t g = nullptr;
    cudaGraphConditionalHandle h = 0;
    cudaGraphNode_t first = nullptr, loop = nullptr;
    size_t n_nodes = 1;
    int32_t st = MF_OK;
    bool ok = cudaGraphCreate(&g, 0) == cudaSuccess &&
              cudaGraphConditionalHandleCreate(&h, g, 0, cudaGraphCondAssignDefault) == cudaSuccess;
    if (ok && cudaStreamBeginCaptureToGraph(stream, g, nullptr, nullptr, 0, cudaStreamCaptureModeRelaxed) == cudaSuccess) {
        gen_check_kernel<<<1, 1, 0, stream>>>(s->gen_ctl, sampled, s->gen_ids, h);
        cudaGraph_t same = nullptr;
        ok = cudaStreamEndCapture(stream, &same) == cudaSuccess && same == g;
    } else {
        ok = false;
    }
    ok = ok && cudaGraphGetNodes(g, &first, &n_nodes) == cudaSuccess && n_nodes == 1;
    cudaGraphNodeParams cp = {};
    cp.type = cudaGraphNodeTypeConditional;
    cp.conditional.handle = h;
    cp.conditional.type = cudaGraphCondTypeWhile;
    cp.conditional.size = 1;
    ok = ok && cudaGraphAddNode(&loop, g, &first, 1, &cp) == cudaSuccess;
    if (ok && cudaStreamBeginCaptureToGraph(stream, cp.conditional.phGraph_out[0], nullptr, nullptr, 0,
                                            cudaStreamCaptureModeRelaxed) == cudaSuccess) {
        const uint64_t before = launches();
        st = greedy_step(m, s);
        if (!st) gen_check_kernel<<<1, 1, 0, stream>>>(s->gen_ctl, sampled, s->gen_ids, h);
        count_launch(-(int64_t)(launches() - before));   // captured, not run
        cudaGraph_t body = nullptr;
        ok = cudaStreamEndCapture(stream, &body) == cudaSuccess && !st;
    } else {
        ok = false;
    }
    ok = ok && cudaGraphInstantiate(&s->graph_gen, g, 0) == cudaSuccess;
    if (g) cudaGraphDestroy(g);
    if (st) return st;
    if (!ok) {
        // Not built here: the host loop serves every call on this state.
        cudaGetLastError();
        if (s->graph_gen) cudaGraphExecDestroy(s->graph_gen);
        s->graph_gen = nullptr;
        s->gen_unsupported = true;
        return MF_UNSUPPORTED;
    }
    s->graph_gen_epoch = s->ws_epoch;
    s->graph_gen_model_epoch = m->epoch;
    return MF_OK;
}

}  // namespace

extern "C" {

int32_t mf_lfm2_decode_graph(mf_lfm2 *m, mf_lfm2_state *s, uint64_t steps) {
    if (!m || !s || s->model != m) return fail(MF_INVALID_ARGUMENT, "state belongs to another model");
    if (s->length > m->cfg.max_tokens || steps > m->cfg.max_tokens - s->length)
        return fail(MF_RESOURCE_LIMIT, "token pass exceeds the configured context capacity");
    if (steps == 0) return MF_OK;
    int32_t st = ensure_decode_graph(m, s);
    if (st) return st;
    if (steps >= kMultiSteps && (st = ensure_multi_graph(m, s))) return st;
    cudaStream_t stream = m->b->stream;
    uint64_t i = 0;
    for (; i + kMultiSteps <= steps; i += kMultiSteps) {
        MF_CUDA_TRY(cudaGraphLaunch(s->graph_multi, stream));
        count_launch(m->kernels_per_step * kMultiSteps);
    }
    for (; i < steps; ++i) {
        MF_CUDA_TRY(cudaGraphLaunch(s->graph, stream));
        count_launch(m->kernels_per_step);
    }
    s->length += steps;
    return MF_OK;
}

int32_t mf_lfm2_decode_host(mf_lfm2 *m, mf_lfm2_state *s, const uint32_t *token, float *sampled_out) {
    if (!m || !s || s->model != m) return fail(MF_INVALID_ARGUMENT, "state belongs to another model");
    if (!sampled_out) return fail(MF_INVALID_ARGUMENT, "null sampled output");
    if (token && *token >= m->cfg.vocab) return fail(MF_OUT_OF_BOUNDS, "valid token ID exceeds loaded model vocabulary");
    if (s->length >= m->cfg.max_tokens) return fail(MF_RESOURCE_LIMIT, "token pass exceeds the configured context capacity");
    int32_t st = ensure_decode_graph(m, s);
    if (st) return st;
    if (!s->io_pinned) MF_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void **>(&s->io_pinned), 2 * sizeof(float),
                                                 cudaHostAllocDefault));
    if (!s->io_done) MF_CUDA_TRY(cudaEventCreateWithFlags(&s->io_done, cudaEventDisableTiming));
    cudaStream_t stream = m->b->stream;
    if (token) {
        // The graph embeds the id held in the sampled slot (f32, exact below 2^24).
        s->io_pinned[0] = (float)*token;
        MF_CUDA_TRY(cudaMemcpyAsync(s->sampled->ptr, s->io_pinned, sizeof(float), cudaMemcpyHostToDevice, stream));
    }
    MF_CUDA_TRY(cudaGraphLaunch(s->graph, stream));
    count_launch(m->kernels_per_step);
    s->length += 1;
    MF_CUDA_TRY(cudaMemcpyAsync(s->io_pinned + 1, s->sampled->ptr, sizeof(float), cudaMemcpyDeviceToHost, stream));
    MF_CUDA_TRY(cudaEventRecord(s->io_done, stream));
    MF_CUDA_TRY(cudaEventSynchronize(s->io_done));
    *sampled_out = s->io_pinned[1];
    return MF_OK;
}

int32_t mf_lfm2_generate(mf_lfm2 *m, mf_lfm2_state *s, const uint32_t *first_token, uint64_t max_tokens,
                         const uint32_t *stop_ids, uint64_t n_stop, float *ids_out, uint64_t *n_out,
                         int32_t *stopped) {
    if (!m || !s || s->model != m) return fail(MF_INVALID_ARGUMENT, "state belongs to another model");
    if (!n_out || (max_tokens && !ids_out) || (n_stop && !stop_ids)) return fail(MF_INVALID_ARGUMENT, "null argument");
    if (first_token && *first_token >= m->cfg.vocab)
        return fail(MF_OUT_OF_BOUNDS, "valid token ID exceeds loaded model vocabulary");
    *n_out = 0;
    if (stopped) *stopped = 0;
    int32_t st = ensure_decode_graph(m, s);
    if (st) return st;
    if (!s->io_pinned) MF_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void **>(&s->io_pinned), 2 * sizeof(float),
                                                 cudaHostAllocDefault));
    if (!s->io_done) MF_CUDA_TRY(cudaEventCreateWithFlags(&s->io_done, cudaEventDisableTiming));
    cudaStream_t stream = m->b->stream;
    if (first_token) {
        s->io_pinned[0] = (float)*first_token;
        MF_CUDA_TRY(cudaMemcpyAsync(s->sampled->ptr, s->io_pinned, sizeof(float), cudaMemcpyHostToDevice, stream));
    }
    if (max_tokens && n_stop <= kGenMaxStop && ensure_gen_graph(m, s) == MF_OK) {
        // The whole loop on the device: one upload, one graph, one read-back.
        GenCtl *c = s->gen_ctl_host;
        memset(c, 0, sizeof(GenCtl));
        c->max_tokens = max_tokens;
        c->cap_left = s->length < m->cfg.max_tokens ? m->cfg.max_tokens - s->length : 0;
        c->ids_cap = s->gen_ids_cap;
        c->n_stop = (uint32_t)n_stop;
        c->vocab = m->cfg.vocab;
        for (uint64_t i = 0; i < n_stop; ++i) c->stop_ids[i] = stop_ids[i];
        const uint64_t want = std::min<uint64_t>(max_tokens, s->gen_ids_cap);
        MF_CUDA_TRY(cudaMemcpyAsync(s->gen_ctl, c, sizeof(GenCtl), cudaMemcpyHostToDevice, stream));
        MF_CUDA_TRY(cudaGraphLaunch(s->graph_gen, stream));
        MF_CUDA_TRY(cudaMemcpyAsync(c, s->gen_ctl, sizeof(GenCtl), cudaMemcpyDeviceToHost, stream));
        MF_CUDA_TRY(cudaMemcpyAsync(s->gen_ids_host, s->gen_ids, want * sizeof(float), cudaMemcpyDeviceToHost, stream));
        MF_CUDA_TRY(cudaEventRecord(s->io_done, stream));
        MF_CUDA_TRY(cudaEventSynchronize(s->io_done));
        count_launch(c->steps * (m->kernels_per_step + 1) + 1);
        s->length += c->steps;
        const uint64_t got = std::min<uint64_t>(c->n_out, want);
        for (uint64_t i = 0; i < got; ++i) ids_out[i] = s->gen_ids_host[i];
        *n_out = got;
        if (c->error == 1) return fail(MF_BACKEND_FAILURE, "executor published no greedy next-token sample");
        if (c->error) return fail(MF_RESOURCE_LIMIT, "token pass exceeds the configured context capacity");
        if (c->stopped && stopped) *stopped = 1;
        return MF_OK;
    }
    while (*n_out < max_tokens) {
        // The current sample on the host (sampled_token), before any append.
        MF_CUDA_TRY(cudaMemcpyAsync(s->io_pinned + 1, s->sampled->ptr, sizeof(float), cudaMemcpyDeviceToHost, stream));
        MF_CUDA_TRY(cudaEventRecord(s->io_done, stream));
        MF_CUDA_TRY(cudaEventSynchronize(s->io_done));
        const float id = s->io_pinned[1];
        if (!(id >= 0.0f) || id >= (float)m->cfg.vocab)
            return fail(MF_BACKEND_FAILURE, "executor published no greedy next-token sample");
        const uint32_t tok = (uint32_t)id;
        bool stop = false;
        for (uint64_t i = 0; i < n_stop && !stop; ++i) stop = stop_ids[i] == tok;
        if (stop) {
            if (stopped) *stopped = 1;
            return MF_OK;
        }
        ids_out[(*n_out)++] = id;
        if (*n_out == max_tokens) break;
        if (s->length >= m->cfg.max_tokens)
            return fail(MF_RESOURCE_LIMIT, "token pass exceeds the configured context capacity");
        MF_CUDA_TRY(cudaGraphLaunch(s->graph, stream));
        count_launch(m->kernels_per_step);
        s->length += 1;
    }
    return MF_OK;
}

int32_t mf_lfm2_state_copy(mf_lfm2 *m, mf_lfm2_state *dst, const mf_lfm2_state *src) {
    if (!m || !dst || !src || dst->model != m || src->model != m)
        return fail(MF_INVALID_ARGUMENT, "state belongs to another model");
    if (dst == src) return MF_OK;
    const mf_lfm2_config &c = m->cfg;
    const uint64_t h = c.hidden, kvw = (uint64_t)c.kv_heads * c.head_dim;
    cudaStream_t stream = m->b->stream;
    for (uint32_t i = 0; i < c.n_layers; ++i) {
        if (m->layers[i].kind == MF_LAYER_CONV) {
            MF_CUDA_TRY(cudaMemcpyAsync(dst->history[i], src->history[i], (c.conv_width - 1) * h * sizeof(float),
                                        cudaMemcpyDeviceToDevice, stream));
        } else if (src->length) {
            MF_CUDA_TRY(cudaMemcpyAsync(dst->kcache[i], src->kcache[i], src->length * kvw * sizeof(float),
                                        cudaMemcpyDeviceToDevice, stream));
            MF_CUDA_TRY(cudaMemcpyAsync(dst->vcache[i], src->vcache[i], src->length * kvw * sizeof(float),
                                        cudaMemcpyDeviceToDevice, stream));
        }
    }
    MF_CUDA_TRY(cudaMemcpyAsync(dst->pos_dev, src->pos_dev, sizeof(uint64_t), cudaMemcpyDeviceToDevice, stream));
    MF_CUDA_TRY(cudaMemcpyAsync(dst->logits->ptr, src->logits->ptr, src->logits->bytes, cudaMemcpyDeviceToDevice, stream));
    MF_CUDA_TRY(cudaMemcpyAsync(dst->sampled->ptr, src->sampled->ptr, sizeof(float), cudaMemcpyDeviceToDevice, stream));
    dst->length = src->length;
    return MF_OK;
}

int32_t mf_lfm2_profile_step(mf_lfm2 *m, mf_lfm2_state *s, mf_op_profile *out, uint32_t n_classes) {
    if (!m || !s || s->model != m) return fail(MF_INVALID_ARGUMENT, "state belongs to another model");
    if (!out || n_classes < MF_OP_CLASSES) return fail(MF_INVALID_ARGUMENT, "profile needs one slot per op class");
    if (s->length >= m->cfg.max_tokens) return fail(MF_RESOURCE_LIMIT, "token pass exceeds the configured context capacity");
    int32_t st = ensure_workspace(s, 1);
    if (st) return st;
    // The step is captured into a graph with event-record nodes between the
    // ops, so the ops run back to back as in the decode graph and each event
    // pair brackets device time only (no host enqueue gaps).
    Profiler prof;
    cudaStream_t stream = m->b->stream;
    MF_CUDA_TRY(cudaStreamBeginCapture(stream, cudaStreamCaptureModeRelaxed));
    s->prof = &prof;
    st = run_pass(m, s, 1, nullptr, static_cast<const float *>(s->sampled->ptr), true);
    s->prof = nullptr;
    if (!st) {
        cudaEvent_t a = prof.next(), z = prof.next();
        const uint64_t k0 = launches();
        if (a) Profiler::record(a, stream);
        st = argmax(static_cast<float *>(s->sampled->ptr), static_cast<float *>(s->logits->ptr), 1, m->cfg.vocab,
                    nullptr, &s->split, stream);
        if (!st && a && z) {
            Profiler::record(z, stream);
            prof.ops.push_back({MF_OP_ARGMAX, (uint64_t)m->cfg.vocab * 4 + 4, launches() - k0, a, z});
        }
    }
    cudaGraph_t graph = nullptr;
    cudaError_t err = cudaStreamEndCapture(stream, &graph);
    if (st) {
        if (graph) cudaGraphDestroy(graph);
        return st;
    }
    if (err != cudaSuccess) return cuda_fail(err, "cudaStreamEndCapture");
    cudaGraphExec_t exec = nullptr;
    err = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGraphInstantiate");
    err = cudaGraphLaunch(exec, stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(stream);
    cudaGraphExecDestroy(exec);
    if (err != cudaSuccess) return cuda_fail(err, "profiled decode step");
    s->length += 1;
    for (uint32_t i = 0; i < n_classes; ++i) out[i] = mf_op_profile{0, 0, 0.0};
    for (const OpRecord &r : prof.ops) {
        float ms = 0.0f;
        MF_CUDA_TRY(cudaEventElapsedTime(&ms, r.start, r.stop));
        out[r.cls].launches += r.kernels;
        out[r.cls].bytes += r.bytes;
        out[r.cls].ms += ms;
        out[r.cls].ops += 1;
    }
    return MF_OK;
}

int32_t mf_lfm2_set_fused(mf_lfm2 *m, int32_t enabled) {
    if (!m) return fail(MF_INVALID_ARGUMENT, "null model");
    m->fused = enabled != 0;
    return MF_OK;
}

int32_t mf_lfm2_set_persistent(mf_lfm2 *m, int32_t enabled) {
    if (!m) return fail(MF_INVALID_ARGUMENT, "null model");
    m->persistent = enabled != 0;
    return MF_OK;
}

int32_t mf_lfm2_persistent_active(const mf_lfm2_state *s) { return s && s->pplan ? 1 : 0; }

// One greedy step of the state (as mf_lfm2_append_argmax from the device
// sample: the state advances by one token) with a CUDA event recorded after
// every launch: us[i] is launch i's time from the previous event, names[i]
// its op label (ffn_gate_up, ffn_down, conv_in_proj, conv_out_proj,
// attn_qkv, attention, attn_o, lm_head) or kernel name.  The events keep the
// launches from overlapping (programmatic dependent launch cannot start a
// kernel ahead of an event), so the times are per-launch spans, not the
// step's overlapped total.  *n receives the launch count (entries past
// `capacity` are not written).
int32_t mf_lfm2_time_step(mf_lfm2 *m, mf_lfm2_state *s, const char **names, float *us, uint64_t capacity,
                          uint64_t *n) {
    if (!m || !s || !n || (capacity && (!names || !us))) return fail(MF_INVALID_ARGUMENT, "null argument");
    if (s->model != m) return fail(MF_INVALID_ARGUMENT, "state belongs to another model");
    if (s->length >= m->cfg.max_tokens) return fail(MF_RESOURCE_LIMIT, "token pass exceeds the configured context capacity");
    int32_t st = ensure_workspace(s, 1);
    if (st) return st;
    cudaStream_t stream = m->b->stream;
    std::vector<cudaEvent_t> ev(capacity + 1, nullptr);
    for (auto &e : ev) MF_CUDA_TRY(cudaEventCreate(&e));
    std::vector<const char *> nm(capacity, nullptr);
    LaunchRecorder rec;
    rec.events = ev.data() + 1;
    rec.names = nm.data();
    rec.cap = capacity;
    MF_CUDA_TRY(cudaEventRecord(ev[0], stream));
    launch_recorder() = &rec;
    st = greedy_step(m, s);
    launch_recorder() = nullptr;
    cudaError_t err = cudaStreamSynchronize(stream);
    if (!st && err != cudaSuccess) st = cuda_fail(err, "mf_lfm2_time_step");
    if (!st) {
        s->length += 1;
        const size_t k = std::min<size_t>(rec.n, capacity);
        for (size_t i = 0; i < k; ++i) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
            us[i] = ms * 1e3f;
            names[i] = nm[i];
        }
        *n = rec.n;
    }
    for (auto &e : ev) cudaEventDestroy(e);
    return st;
}

int32_t mf_nccl_unique_id(uint8_t *out, uint64_t capacity) {
    if (!out) return fail(MF_INVALID_ARGUMENT, "null argument");
    return nccl_unique_id(out, capacity);
}

// The LM-head row split of a single sequence across GPUs: each rank holds a
// full replica and runs the same decode steps; the head's rows are split
// into contiguous shards (multiples of 16 rows), each rank scores its shard
// and its candidate (max, index, poisoned) is all-gathered over NCCL, and
// every rank picks the same greedy id.  A collective: all ranks call it with
// the same id and world size.  World 1 turns it off.
int32_t mf_lfm2_set_head_split(mf_lfm2 *m, const uint8_t *unique_id, int32_t rank, int32_t world) {
    if (!m) return fail(MF_INVALID_ARGUMENT, "null model");
    if (world < 1 || rank < 0 || rank >= world) return fail(MF_INVALID_ARGUMENT, "head split rank out of range");
    if (world > 1 && !unique_id) return fail(MF_INVALID_ARGUMENT, "head split needs the NCCL unique id");
    const Weight &e = m->emb;
    if (world > 1) {
        if (e.packed && e.format == MF_NF4) return fail(MF_UNSUPPORTED, "NF4 heads are not split");
        if (!e.packed && !dense_head_argmax_supported(e.rows, e.cols))
            return fail(MF_UNSUPPORTED, "dense head width is not a multiple of 128 up to 2048");
        const uint64_t chunk = ((e.rows + world - 1) / world + 15) / 16 * 16;
        if (chunk * (uint64_t)(world - 1) >= e.rows) return fail(MF_UNSUPPORTED, "head has too few rows for this split");
    }
    // Tear down any previous split (after the stream's queued steps).
    MF_CUDA_TRY(cudaStreamSynchronize(m->b->stream));
    if (m->head_comm) nccl_comm_destroy(m->head_comm);
    m->head_comm = nullptr;
    if (m->head_buf) mf_buffer_release(m->b, m->head_buf);
    m->head_buf = nullptr;
    m->head_cand = m->head_cands = nullptr;
    m->head_world = 1;
    m->head_rank = 0;
    m->epoch++;
    if (world == 1) return MF_OK;
    const uint64_t chunk = ((e.rows + world - 1) / world + 15) / 16 * 16;
    const uint64_t shape[1] = {4 + 3 * (uint64_t)world};
    int32_t st = mf_allocate_f32(m->b, shape, 1, MF_CLASS_SCRATCH, 0, &m->head_buf);
    if (st) return st;
    int dev = 0;
    MF_CUDA_TRY(cudaGetDevice(&dev));
    if (dev != m->b->ordinal) MF_CUDA_TRY(cudaSetDevice(m->b->ordinal));
    st = nccl_comm_init(&m->head_comm, unique_id, rank, world);
    if (dev != m->b->ordinal) cudaSetDevice(dev);
    if (st) {
        mf_buffer_release(m->b, m->head_buf);
        m->head_buf = nullptr;
        m->head_comm = nullptr;
        return st;
    }
    m->head_cand = static_cast<float *>(m->head_buf->ptr);
    m->head_cands = m->head_cand + 4;
    m->head_world = world;
    m->head_rank = rank;
    m->head_row0 = chunk * (uint64_t)rank;
    m->head_rows = std::min(chunk, e.rows - m->head_row0);
    return MF_OK;
}

// The reference executor's LUT2 routing (crates/executor-core/src/lfm2/
// executor/construction.rs:404-470, execution.rs:343-400): per layer in
// order, the ternary down projection first, then the ternary gate/up pair,
// each repacked while the byte budget lasts; a role the layout cannot take
// stays raw.  Mode 0 restores every role's raw stream, 1 repacks down and
// gate/up (Auto), 2 the down projections only (DownOnly).  The model owns
// the repacks; the caller's raw buffers stay in use by nothing else.
int32_t mf_lfm2_set_lut2(mf_lfm2 *m, int32_t mode, uint64_t max_bytes, uint64_t *repacked_bytes) {
    if (!m) return fail(MF_INVALID_ARGUMENT, "null model");
    if (mode < 0 || mode > 2) return fail(MF_INVALID_ARGUMENT, "LUT2 mode must be 0 (off), 1 (auto) or 2 (down only)");
    // Back to the raw streams first.
    for (Layer &L : m->layers)
        for (Weight *w : {&L.w1, &L.w2, &L.w3})
            if (w->lanetiled) {
                w->codes = w->raw_codes;
                w->lanetiled = false;
            }
    for (mf_buffer *buf : m->lut2) mf_buffer_release(m->b, buf);
    m->lut2.clear();
    m->epoch++;
    uint64_t used = 0;
    auto fits = [&](const Weight &w) {
        return w.packed && w.format == MF_TERNARY && w.rows % 16 == 0 && w.cols % kGroup == 0;
    };
    auto repack = [&](Weight &w) -> int32_t {
        const uint64_t shape[2] = {w.rows, w.cols / 4};
        mf_buffer *buf = nullptr;
        int32_t st = backend_alloc_buffer(m->b, MF_DTYPE_U8, shape, 2, MF_CLASS_WEIGHT, &buf);
        if (st) return st;
        buf->lut2 = true;
        st = ternary_repack_lanetiled(static_cast<uint8_t *>(buf->ptr), w.codes, w.rows, w.cols / 4, m->b->stream);
        if (st) {
            mf_buffer_release(m->b, buf);
            return st;
        }
        m->lut2.push_back(buf);
        w.raw_codes = w.codes;
        w.codes = static_cast<const uint8_t *>(buf->ptr);
        w.lanetiled = true;
        return MF_OK;
    };
    if (mode != 0) {
        for (Layer &L : m->layers) {
            const uint64_t down_bytes = L.w2.rows * L.w2.cols / 4;
            if (fits(L.w2) && used + down_bytes <= max_bytes) {
                if (int32_t st = repack(L.w2)) return st;
                used += down_bytes;
            }
            const uint64_t pair_bytes = 2 * L.w1.rows * L.w1.cols / 4;
            if (mode == 1 && fits(L.w1) && fits(L.w3) && used + pair_bytes <= max_bytes) {
                if (int32_t st = repack(L.w1)) return st;
                if (int32_t st = repack(L.w3)) return st;
                used += pair_bytes;
            }
        }
    }
    if (repacked_bytes) *repacked_bytes = used;
    return MF_OK;
}

uint64_t mf_lfm2_decode_kernels_per_step(const mf_lfm2 *m) { return m ? count_step_kernels(m) : 0; }

}  // extern "C"

// ---------------------------------------------------------------------
// Batches of independent sequences: S sequences that advance together,
// each with its own KV caches, conv histories, position and greedy id, one
// pass over all of them per step (every matmul at S rows, so each weight
// byte is read once per step for all sequences).  The reference's executor
// holds one sequence per state and has no batch API; per sequence the
// arithmetic is that of run_pass (execution.rs:35-627), so each sequence's
// logits and greedy stream match a single-sequence run within the matmul
// tolerance.
// ---------------------------------------------------------------------
struct mf_lfm2_batch {
    mf_lfm2 *model = nullptr;
    uint32_t seqs = 0;
    uint64_t length = 0;   // common length of every sequence (host view)
    std::vector<mf_buffer *> owned;
    std::vector<float *> history, kcache, vcache;   // per layer: [seqs][...]
    uint64_t *pos = nullptr;                        // [seqs] positions (device)
    float *sampled = nullptr;                       // [seqs] greedy ids (device f32)
    float *logits = nullptr;                        // [seqs][vocab]
    mf_buffer *ws_buf = nullptr;
    uint64_t ws_rows = 0, ws_group = 0, ws_epoch = 0;
    float *x = nullptr, *u = nullptr, *op = nullptr, *proj = nullptr, *conv = nullptr, *q = nullptr, *k = nullptr,
          *v = nullptr, *qr = nullptr, *kr = nullptr, *att = nullptr, *residual = nullptr, *ffn_in = nullptr,
          *gate = nullptr, *up = nullptr, *down = nullptr, *hidden_buf = nullptr, *last = nullptr;
    uint32_t *ids = nullptr;
    float *gqa_scratch = nullptr;
    size_t gqa_scratch_bytes = 0;
    SplitScratch split;
    mf_buffer *counters_buf = nullptr;
    float *id_log = nullptr;   // [id_log_steps][seqs] greedy ids of a decode call
    uint64_t id_log_steps = 0;
    mf_buffer *id_log_buf = nullptr;
    cudaGraphExec_t graph = nullptr;
    uint64_t graph_epoch = 0, graph_model_epoch = 0;
    uint64_t kernels_per_step = 0;
};

namespace {

// Rows per batched pass when sequences append many tokens at once: the
// sequences are processed in groups of at most this many rows.
constexpr uint64_t kBatchPassRows = 4096;

// out[b][:] = in[(b * n + n - 1)][:] (the last row of each sequence).
__global__ void last_rows_kernel(float *out, const float *in, uint32_t seqs, uint64_t n, uint64_t width) {
    pdl_wait();
    pdl_trigger();
    const uint64_t total = (uint64_t)seqs * width;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t b = e / width, c = e - b * width;
        out[e] = in[(b * n + n - 1) * width + c];
    }
}

// dst + b * stride <- src[0 .. count) for every b < copies (32-bit words).
__global__ void replicate_kernel(uint32_t *dst, uint64_t stride, const uint32_t *src, uint64_t count,
                                 uint32_t copies) {
    pdl_wait();
    pdl_trigger();
    const uint64_t total = count * copies;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t b = e / count, i = e - b * count;
        dst[b * stride + i] = src[i];
    }
}

int32_t replicate(void *dst, uint64_t stride_words, const void *src, uint64_t words, uint32_t copies,
                  cudaStream_t stream) {
    if (!words || !copies) return MF_OK;
    const uint64_t total = words * copies;
    const unsigned blocks = (unsigned)std::min<uint64_t>((total + 255) / 256, 148 * 32);
    return ::mf::launch(replicate_kernel, dim3(blocks), dim3(256), 0, stream, "replicate_kernel",
                        static_cast<uint32_t *>(dst), stride_words, static_cast<const uint32_t *>(src), words, copies);
}

int32_t batch_alloc(mf_lfm2_batch *bt, uint64_t elements, int32_t cls, float **out, mf_buffer **handle = nullptr) {
    mf_buffer *buf = nullptr;
    uint64_t shape[1] = {std::max<uint64_t>(elements, 1)};
    int32_t st = mf_allocate_f32(bt->model->b, shape, 1, cls, 0, &buf);
    if (st) return st;
    bt->owned.push_back(buf);
    *out = static_cast<float *>(buf->ptr);
    if (handle) *handle = buf;
    return MF_OK;
}

void batch_release(mf_lfm2_batch *bt, mf_buffer **buf) {
    if (!*buf) return;
    bt->owned.erase(std::remove(bt->owned.begin(), bt->owned.end(), *buf), bt->owned.end());
    mf_buffer_release(bt->model->b, *buf);
    *buf = nullptr;
}

// Workspace for passes of up to `rows` rows over up to `group` sequences.
int32_t ensure_batch_workspace(mf_lfm2_batch *bt, uint64_t rows, uint64_t group) {
    if (bt->ws_buf && bt->ws_rows >= rows && bt->ws_group >= group) return MF_OK;
    mf_lfm2 *m = bt->model;
    const mf_lfm2_config &c = m->cfg;
    rows = std::max(rows, bt->ws_rows);
    group = std::max(group, bt->ws_group);
    const uint64_t h = c.hidden, f = c.intermediate, kvw = (uint64_t)c.kv_heads * c.head_dim;
    auto al = [](uint64_t v) { return (v + 63) & ~63ull; };
    const uint64_t sizes[] = {h, h, h, 3 * h, h, h, kvw, kvw, h, kvw, h, h, h, f, f, h, f, h};
    uint64_t total = 0;
    for (uint64_t sz : sizes) total += al(rows * sz);
    total += al(rows + 16);   // ids (u32)
    // Decode attention partials: one sequence's worth per sequence of a group.
    const size_t gqa = (size_t)group * causal_gqa_scratch_bytes(1, c.q_heads, c.kv_heads, c.head_dim, c.max_tokens);
    total += al(gqa / sizeof(float) + 1);
    const uint64_t tg = std::min<uint64_t>(rows, kGemmMinTokens - 1);
    const uint64_t shapes[][2] = {{3 * h, h}, {h, h}, {kvw, h}, {f, h}, {h, f}, {c.vocab, h}};
    size_t split_floats = argmax_scratch_floats(group, c.vocab);
    size_t counters = std::max<size_t>(64, (size_t)c.kv_heads * group);
    counters = std::max<size_t>(counters, group);
    for (const auto &sh : shapes) {
        split_floats = std::max(split_floats, packed_gemv_tc_scratch_floats(tg, sh[0], sh[1]));
        counters = std::max(counters, packed_gemv_tc_counters(tg, sh[0]));
    }
    if (rows >= kNf4GemmMinTokens)
        split_floats = std::max(split_floats, gemm_scratch_floats(c, rows));
    total += al(split_floats);
    batch_release(bt, &bt->ws_buf);
    float *p = nullptr;
    int32_t st = batch_alloc(bt, total, MF_CLASS_SCRATCH, &p, &bt->ws_buf);
    if (st) return st;
    float **dst[] = {&bt->x, &bt->u, &bt->op, &bt->proj, &bt->conv, &bt->q, &bt->k, &bt->v, &bt->qr, &bt->kr,
                     &bt->att, &bt->residual, &bt->ffn_in, &bt->gate, &bt->up, &bt->down, &bt->hidden_buf, &bt->last};
    for (size_t i = 0; i < sizeof(sizes) / sizeof(sizes[0]); ++i) {
        *dst[i] = p;
        p += al(rows * sizes[i]);
    }
    bt->ids = reinterpret_cast<uint32_t *>(p);
    p += al(rows + 16);
    bt->gqa_scratch = p;
    bt->gqa_scratch_bytes = gqa;
    p += al(gqa / sizeof(float) + 1);
    bt->split.partial = p;
    bt->split.partial_floats = split_floats;
    if (!bt->counters_buf || bt->split.n_counters < counters) {
        batch_release(bt, &bt->counters_buf);
        float *cp = nullptr;
        st = batch_alloc(bt, counters, MF_CLASS_SCRATCH, &cp, &bt->counters_buf);   // zero-initialised
        if (st) return st;
        bt->split.counters = reinterpret_cast<unsigned *>(cp);
        bt->split.n_counters = counters;
    }
    bt->ws_rows = rows;
    bt->ws_group = group;
    bt->ws_epoch++;
    return MF_OK;
}

// One pass over sequences [s0, s0 + ns), n new rows each (rows sequence-major),
// ids from `ids_u32` (staged host ids, ns * n) or `ids_f32` (the sequences'
// device greedy ids, n = 1).  Ends with each sequence's greedy id and n more
// rows of position.
int32_t run_batch_pass(mf_lfm2 *m, mf_lfm2_batch *bt, uint32_t s0, uint32_t ns, uint64_t n, const uint32_t *ids_u32,
                       const float *ids_f32) {
    const mf_lfm2_config &c = m->cfg;
    cudaStream_t st_ = m->b->stream;
    const uint64_t h = c.hidden, f = c.intermediate, kvw = (uint64_t)c.kv_heads * c.head_dim;
    const uint64_t R = (uint64_t)ns * n, cap = c.max_tokens;
    uint64_t *pos = bt->pos + s0;
    const SplitScratch *ss = &bt->split;
    int32_t st;
#define BTRY(expr)                    \
    do {                              \
        if ((st = (expr))) return st; \
    } while (0)
    if (m->emb.packed)
        BTRY(packed_gather_rows(bt->x, m->emb.codes, m->emb.scales, m->emb.rows, m->emb.cols, m->emb.format, ids_f32,
                                ids_u32, R, st_));
    else
        BTRY(gather_rows(bt->x, m->emb.dense, m->emb.rows, m->emb.cols, ids_f32, ids_u32, R, st_));
    const float *first_norm = c.n_layers ? m->layers[0].operator_norm : m->emb_norm;
    BTRY(row_rms_norm(nullptr, bt->u, bt->x, nullptr, R, h, first_norm, c.n_layers ? c.block_eps : c.norm_eps, st_));
    for (uint32_t li = 0; li < c.n_layers; ++li) {
        const Layer &L = m->layers[li];
        if (L.kind == MF_LAYER_CONV) {
            BTRY(weight_linear(bt->proj, bt->u, R, L.in_proj, ss, st_));
            BTRY(gated_short_conv_batch(bt->conv, bt->proj, ns, n, c.hidden, L.conv_kernel, c.conv_width,
                                        bt->history[li] + (uint64_t)s0 * (c.conv_width - 1) * h, st_));
            BTRY(weight_linear(bt->op, bt->conv, R, L.out_proj, ss, st_));
        } else {
            BTRY(weight_linear(bt->q, bt->u, R, L.q, ss, st_));
            if (L.k.packed && L.v.packed && L.k.format == L.v.format) {
                BTRY(packed_matmul(kPackedPairRows, false, bt->k, bt->v, bt->u, nullptr, nullptr, R, L.k.codes,
                                   L.k.scales, L.v.codes, L.v.scales, L.k.rows, L.k.cols, L.k.format, ss, st_));
            } else {
                BTRY(weight_linear(bt->k, bt->u, R, L.k, ss, st_));
                BTRY(weight_linear(bt->v, bt->u, R, L.v, ss, st_));
            }
            float *kc = bt->kcache[li] + (uint64_t)s0 * cap * kvw, *vc = bt->vcache[li] + (uint64_t)s0 * cap * kvw;
            if (n == 1 && m->rope && gqa_decode_fused_supported(c.q_heads, c.kv_heads, c.head_dim, cap)) {
                BTRY(gqa_decode_fused(bt->att, bt->q, bt->k, bt->v, L.q_norm, L.k_norm, c.block_eps, m->rope, kc, vc,
                                      cap, pos, c.q_heads, c.kv_heads, c.head_dim, bt->gqa_scratch,
                                      bt->gqa_scratch_bytes, bt->split.counters, bt->split.n_counters, st_, ns));
            } else {
                BTRY(head_norm_rope_batch(bt->qr, bt->q, ns, n, c.q_heads, c.head_dim, L.q_norm, c.block_eps, pos,
                                          c.rope_theta, st_));
                BTRY(head_norm_rope_batch(bt->kr, bt->k, ns, n, c.kv_heads, c.head_dim, L.k_norm, c.block_eps, pos,
                                          c.rope_theta, st_));
                BTRY(causal_gqa_batch(bt->att, bt->qr, bt->kr, bt->v, kc, vc, cap, pos, ns, n, c.q_heads, c.kv_heads,
                                      c.head_dim, st_));
            }
            BTRY(weight_linear(bt->op, bt->att, R, L.o, ss, st_));
        }
        BTRY(row_rms_norm(bt->residual, bt->ffn_in, bt->x, bt->op, R, h, L.ffn_norm, c.block_eps, st_));
        // The reference runs the final layer's FFN on the last row only
        // (execution.rs:277-299); rows are independent, so running it on
        // every row gives each sequence's last row the same values.
        const bool packed_ffn = L.w1.packed && L.w3.packed && L.w1.format == L.w3.format;
        if (packed_ffn && L.w2.packed) {
            BTRY(packed_matmul(kPackedSwigluPair, false, bt->hidden_buf, nullptr, bt->ffn_in, nullptr, nullptr, R,
                               L.w1.codes, L.w1.scales, L.w3.codes, L.w3.scales, L.w1.rows, L.w1.cols, L.w1.format, ss,
                               st_, L.w1.lanetiled));
            BTRY(weight_linear(bt->down, bt->hidden_buf, R, L.w2, ss, st_));
        } else {
            if (packed_ffn) {
                BTRY(packed_matmul(kPackedPairRows, false, bt->gate, bt->up, bt->ffn_in, nullptr, nullptr, R,
                                   L.w1.codes, L.w1.scales, L.w3.codes, L.w3.scales, L.w1.rows, L.w1.cols,
                                   L.w1.format, ss, st_, L.w1.lanetiled));
            } else {
                BTRY(weight_linear(bt->gate, bt->ffn_in, R, L.w1, ss, st_));
                BTRY(weight_linear(bt->up, bt->ffn_in, R, L.w3, ss, st_));
            }
            if (L.w2.packed) {
                BTRY(packed_matmul(kPackedSingle, true, bt->down, nullptr, nullptr, bt->gate, bt->up, R, L.w2.codes,
                                   L.w2.scales, nullptr, nullptr, L.w2.rows, L.w2.cols, L.w2.format, ss, st_,
                                   L.w2.lanetiled));
            } else {
                BTRY(elementwise(2, bt->hidden_buf, bt->gate, bt->up, R * f, st_));
                BTRY(weight_linear(bt->down, bt->hidden_buf, R, L.w2, ss, st_));
            }
        }
        const bool last = li + 1 == c.n_layers;
        const float *norm_w = last ? m->emb_norm : m->layers[li + 1].operator_norm;
        BTRY(row_rms_norm(bt->x, bt->u, bt->residual, bt->down, R, h, norm_w, last ? c.norm_eps : c.block_eps, st_));
    }
    const float *head_in = bt->u;
    if (n > 1) {
        BTRY(::mf::launch(last_rows_kernel, dim3((unsigned)std::min<uint64_t>((ns * h + 255) / 256, 148 * 32)),
                          dim3(256), 0, st_, "last_rows_kernel", bt->last, (const float *)bt->u, ns, n, h));
        head_in = bt->last;
    }
    float *logits = bt->logits + (uint64_t)s0 * c.vocab;
    BTRY(weight_linear(logits, head_in, ns, m->emb, ss, st_));
    BTRY(argmax(bt->sampled + s0, logits, ns, c.vocab, nullptr, ss, st_));
    BTRY(advance_positions(pos, n, ns, st_));
#undef BTRY
    return MF_OK;
}

int32_t ensure_batch_graph(mf_lfm2 *m, mf_lfm2_batch *bt) {
    int32_t st = ensure_batch_workspace(bt, bt->seqs, bt->seqs);
    if (st) return st;
    if (bt->graph && bt->graph_epoch == bt->ws_epoch && bt->graph_model_epoch == bt->model->epoch) return MF_OK;
    cudaStream_t stream = m->b->stream;
    if (bt->graph) {
        cudaGraphExecDestroy(bt->graph);
        bt->graph = nullptr;
    }
    const uint64_t before = launches();
    MF_CUDA_TRY(cudaStreamBeginCapture(stream, cudaStreamCaptureModeRelaxed));
    st = run_batch_pass(m, bt, 0, bt->seqs, 1, nullptr, bt->sampled);
    cudaGraph_t graph = nullptr;
    cudaError_t err = cudaStreamEndCapture(stream, &graph);
    if (st) {
        if (graph) cudaGraphDestroy(graph);
        return st;
    }
    if (err != cudaSuccess) return cuda_fail(err, "cudaStreamEndCapture");
    bt->kernels_per_step = launches() - before;
    count_launch(-(int64_t)bt->kernels_per_step);
    err = cudaGraphInstantiate(&bt->graph, graph, 0);
    cudaGraphDestroy(graph);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGraphInstantiate");
    bt->graph_epoch = bt->ws_epoch;
    bt->graph_model_epoch = bt->model->epoch;
    return MF_OK;
}

}  // namespace

extern "C" {

int32_t mf_lfm2_batch_create(mf_lfm2 *m, uint32_t sequences, mf_lfm2_batch **out) {
    if (!m || !out) return fail(MF_INVALID_ARGUMENT, "null argument");
    if (sequences == 0) return fail(MF_INVALID_ARGUMENT, "a batch needs at least one sequence");
    if (sequences > 65535) return fail(MF_UNSUPPORTED, "batch sequence count exceeds grid limit");
    mf_lfm2_batch *bt = new (std::nothrow) mf_lfm2_batch();
    if (!bt) return fail(MF_RESOURCE_LIMIT, "host allocation failed");
    bt->model = m;
    bt->seqs = sequences;
    const mf_lfm2_config &c = m->cfg;
    const uint64_t h = c.hidden, kvw = (uint64_t)c.kv_heads * c.head_dim, S = sequences;
    bt->history.assign(c.n_layers, nullptr);
    bt->kcache.assign(c.n_layers, nullptr);
    bt->vcache.assign(c.n_layers, nullptr);
    int32_t st = MF_OK;
    for (uint32_t i = 0; !st && i < c.n_layers; ++i) {
        if (m->layers[i].kind == MF_LAYER_CONV) {
            st = batch_alloc(bt, S * (c.conv_width - 1) * h, MF_CLASS_CACHE, &bt->history[i]);
        } else {
            st = batch_alloc(bt, S * c.max_tokens * kvw, MF_CLASS_CACHE, &bt->kcache[i]);
            if (!st) st = batch_alloc(bt, S * c.max_tokens * kvw, MF_CLASS_CACHE, &bt->vcache[i]);
        }
    }
    float *tmp = nullptr;
    if (!st) st = batch_alloc(bt, 2 * S, MF_CLASS_CACHE, &tmp);
    bt->pos = reinterpret_cast<uint64_t *>(tmp);
    if (!st) st = batch_alloc(bt, S, MF_CLASS_CACHE, &bt->sampled);
    if (!st) st = batch_alloc(bt, S * c.vocab, MF_CLASS_CACHE, &bt->logits);
    if (!st) st = ensure_batch_workspace(bt, S, S);
    if (st) {
        mf_lfm2_batch_destroy(bt);
        return st;
    }
    *out = bt;
    return MF_OK;
}

int32_t mf_lfm2_batch_destroy(mf_lfm2_batch *bt) {
    if (!bt) return MF_OK;
    if (bt->graph) cudaGraphExecDestroy(bt->graph);
    for (mf_buffer *buf : bt->owned) mf_buffer_release(bt->model->b, buf);
    delete bt;
    return MF_OK;
}

int32_t mf_lfm2_batch_fork(mf_lfm2_batch *bt, const mf_lfm2_state *prefix) {
    if (!bt || !prefix || prefix->model != bt->model) return fail(MF_INVALID_ARGUMENT, "state belongs to another model");
    mf_lfm2 *m = bt->model;
    const mf_lfm2_config &c = m->cfg;
    cudaStream_t stream = m->b->stream;
    const uint64_t h = c.hidden, kvw = (uint64_t)c.kv_heads * c.head_dim, len = prefix->length;
    int32_t st;
    for (uint32_t i = 0; i < c.n_layers; ++i) {
        if (m->layers[i].kind == MF_LAYER_CONV) {
            const uint64_t words = (uint64_t)(c.conv_width - 1) * h;
            if ((st = replicate(bt->history[i], words, prefix->history[i], words, bt->seqs, stream))) return st;
        } else {
            const uint64_t stride = c.max_tokens * kvw;
            if ((st = replicate(bt->kcache[i], stride, prefix->kcache[i], len * kvw, bt->seqs, stream))) return st;
            if ((st = replicate(bt->vcache[i], stride, prefix->vcache[i], len * kvw, bt->seqs, stream))) return st;
        }
    }
    if ((st = replicate(bt->pos, 2, prefix->pos_dev, 2, bt->seqs, stream))) return st;
    if ((st = replicate(bt->sampled, 1, prefix->sampled->ptr, 1, bt->seqs, stream))) return st;
    bt->length = len;
    return MF_OK;
}

int32_t mf_lfm2_batch_append_argmax(mf_lfm2_batch *bt, const uint32_t *tokens, uint64_t n) {
    if (!bt || !tokens) return fail(MF_INVALID_ARGUMENT, "null argument");
    mf_lfm2 *m = bt->model;
    if (n == 0) return fail(MF_INVALID_ARGUMENT, "token pass requires at least one token");
    if (bt->length > m->cfg.max_tokens || n > m->cfg.max_tokens - bt->length)
        return fail(MF_RESOURCE_LIMIT, "token pass exceeds the configured context capacity");
    const uint64_t total = (uint64_t)bt->seqs * n;
    for (uint64_t i = 0; i < total; ++i)
        if (tokens[i] >= m->cfg.vocab) return fail(MF_OUT_OF_BOUNDS, "valid token ID exceeds loaded model vocabulary");
    const uint32_t group = (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(bt->seqs, kBatchPassRows / n));
    int32_t st = ensure_batch_workspace(bt, (uint64_t)group * n, group);
    if (st) return st;
    for (uint32_t s0 = 0; s0 < bt->seqs; s0 += group) {
        const uint32_t ns = std::min(group, bt->seqs - s0);
        MF_CUDA_TRY(cudaMemcpyAsync(bt->ids, tokens + (uint64_t)s0 * n, (uint64_t)ns * n * sizeof(uint32_t),
                                    cudaMemcpyHostToDevice, m->b->stream));
        if ((st = run_batch_pass(m, bt, s0, ns, n, bt->ids, nullptr))) return st;
    }
    bt->length += n;
    return MF_OK;
}

int32_t mf_lfm2_batch_decode(mf_lfm2_batch *bt, uint64_t steps, float *ids_out) {
    if (!bt) return fail(MF_INVALID_ARGUMENT, "null batch");
    mf_lfm2 *m = bt->model;
    if (bt->length > m->cfg.max_tokens || steps > m->cfg.max_tokens - bt->length)
        return fail(MF_RESOURCE_LIMIT, "token pass exceeds the configured context capacity");
    if (steps == 0) return MF_OK;
    int32_t st = ensure_batch_graph(m, bt);
    if (st) return st;
    cudaStream_t stream = m->b->stream;
    if (ids_out && bt->id_log_steps < steps) {
        batch_release(bt, &bt->id_log_buf);
        bt->id_log_steps = 0;
        if ((st = batch_alloc(bt, steps * bt->seqs, MF_CLASS_SCRATCH, &bt->id_log, &bt->id_log_buf))) return st;
        bt->id_log_steps = steps;
    }
    for (uint64_t i = 0; i < steps; ++i) {
        MF_CUDA_TRY(cudaGraphLaunch(bt->graph, stream));
        count_launch((int64_t)bt->kernels_per_step);
        bt->length += 1;
        if (ids_out)
            MF_CUDA_TRY(cudaMemcpyAsync(bt->id_log + i * bt->seqs, bt->sampled, bt->seqs * sizeof(float),
                                        cudaMemcpyDeviceToDevice, stream));
    }
    if (ids_out) {
        MF_CUDA_TRY(cudaMemcpyAsync(ids_out, bt->id_log, steps * bt->seqs * sizeof(float), cudaMemcpyDeviceToHost,
                                    stream));
        MF_CUDA_TRY(cudaStreamSynchronize(stream));
    }
    return MF_OK;
}

int32_t mf_lfm2_batch_read(mf_lfm2_batch *bt, float *sampled_out, float *logits_out) {
    if (!bt) return fail(MF_INVALID_ARGUMENT, "null batch");
    cudaStream_t stream = bt->model->b->stream;
    if (sampled_out)
        MF_CUDA_TRY(cudaMemcpyAsync(sampled_out, bt->sampled, bt->seqs * sizeof(float), cudaMemcpyDeviceToHost, stream));
    if (logits_out)
        MF_CUDA_TRY(cudaMemcpyAsync(logits_out, bt->logits, (uint64_t)bt->seqs * bt->model->cfg.vocab * sizeof(float),
                                    cudaMemcpyDeviceToHost, stream));
    MF_CUDA_TRY(cudaStreamSynchronize(stream));
    return MF_OK;
}

uint64_t mf_lfm2_batch_kernels_per_step(const mf_lfm2_batch *bt) { return bt ? bt->kernels_per_step : 0; }

}  // extern "C"

namespace mf {
void lfm2_adopt_buffers(mf_lfm2 *m, const std::vector<mf_buffer *> &bufs) {
    m->owned.insert(m->owned.end(), bufs.begin(), bufs.end());
}
}  // namespace mf

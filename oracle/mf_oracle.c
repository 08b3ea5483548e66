/*
 * mf_oracle.c -- CPU oracle (test infrastructure, not product code).
 *
 * A plain-C restatement of the reference's scalar CPU backend for the packed
 * matmul path and the LFM2 layer ops, in the reference's exact summation
 * order.  Every function names the reference file:line it follows.  Build
 * with -O2 -ffp-contract=off (see oracle/Makefile): no FMA contraction, no
 * fast-math, glibc transcendentals.
 */
#include "mf_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>

/* Static-partition parallel for over independent items: item ranges are
 * disjoint and every item is computed exactly as in the serial loop, so the
 * thread count never changes a result bit. */
typedef void (*range_fn)(void *ctx, int64_t begin, int64_t end, int *bad);

typedef struct {
    range_fn fn;
    void *ctx;
    int64_t begin, end;
    int bad;
} range_job;

static void *range_worker(void *arg) {
    range_job *job = (range_job *)arg;
    job->fn(job->ctx, job->begin, job->end, &job->bad);
    return NULL;
}

static int parallel_for(int64_t n, int threads, range_fn fn, void *ctx) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if ((int64_t)threads > n) threads = n > 0 ? (int)n : 1;
    range_job jobs[256];
    pthread_t tids[256];
    int started[256];
    for (int i = 0; i < threads; ++i) {
        jobs[i].fn = fn;
        jobs[i].ctx = ctx;
        jobs[i].begin = n * i / threads;
        jobs[i].end = n * (i + 1) / threads;
        jobs[i].bad = 0;
        started[i] = 0;
    }
    for (int i = 1; i < threads; ++i)
        started[i] = pthread_create(&tids[i], NULL, range_worker, &jobs[i]) == 0;
    range_worker(&jobs[0]);
    int bad = jobs[0].bad;
    for (int i = 1; i < threads; ++i) {
        if (started[i]) pthread_join(tids[i], NULL);
        else range_worker(&jobs[i]);
        bad |= jobs[i].bad;
    }
    return bad;
}

/* crates/kernels-simd/src/lib.rs:113-130; equal bit-for-bit to the NF4 table in
 * tools/converters/src/minifield_converters/quantization.py:22-42. */
const float MFO_NF4_LEVELS[16] = {
    -0x1.000000p+0f, -0x1.647362p-1f, -0x1.0cd660p-1f, -0x1.946540p-2f,
    -0x1.23449ap-2f, -0x1.7a6a7ep-3f, -0x1.74f0e2p-4f, 0.0f,
    0x1.45f5fep-4f,  0x1.4995c6p-3f,  0x1.f809bap-3f,  0x1.5a0674p-2f,
    0x1.c34970p-2f,  0x1.200f56p-1f,  0x1.722766p-1f,  0x1.000000p+0f,
};

static int finite_f(float v) { return isfinite(v) != 0; }

/* crates/backend-cpu/src/packed.rs:177-220 (width inference only; the INT8
 * reserved-code scan needs the bytes and is done by int8_codes_ok). */
int mfo_infer_format(uint64_t code_cols, uint64_t scale_cols, int *format, uint64_t *inner) {
    if (scale_cols > UINT64_MAX / 128) return MFO_OVERFLOW;
    uint64_t k = scale_cols * 128;
    if (code_cols == k / 4) *format = MFO_TERNARY;
    else if (code_cols == k / 2) *format = MFO_NF4;
    else if (code_cols == k) *format = MFO_INT8;
    else return MFO_INVALID_SHAPE;
    *inner = k;
    return MFO_OK;
}

/* packed.rs:205-207: INT8 byte 0x80 (-128) is reserved. */
static int int8_codes_ok(const uint8_t *codes, uint64_t bytes) {
    for (uint64_t i = 0; i < bytes; ++i)
        if (codes[i] == 128) return 0;
    return 1;
}

/* crates/kernels-simd/src/lib.rs:31-57 (row) and :74-81 (scalar group dot). */
float mfo_ternary_row_dot(const uint8_t *codes, const float *scales, const float *x, uint64_t k) {
    float row = 0.0f;
    for (uint64_t g = 0; g < k / 128; ++g) {
        const uint8_t *c = codes + g * 32;
        const float *xg = x + g * 128;
        float acc = 0.0f;
        for (int j = 0; j < 128; ++j) {
            unsigned code = (c[j / 4] >> (2 * (j % 4))) & 0x3u;
            acc += ((float)code - 1.0f) * xg[j];
        }
        row += scales[g] * acc;
    }
    return row;
}

/* crates/kernels-simd/src/lib.rs:145-183: two interleaved accumulators per group. */
float mfo_nf4_row_dot(const uint8_t *codes, const float *scales, const float *x, uint64_t k) {
    float row = 0.0f;
    for (uint64_t g = 0; g < k / 128; ++g) {
        const uint8_t *c = codes + g * 64;
        const float *xg = x + g * 128;
        float lo = 0.0f, hi = 0.0f;
        for (int i = 0; i < 64; ++i) {
            lo += MFO_NF4_LEVELS[c[i] & 0x0F] * xg[2 * i];
            hi += MFO_NF4_LEVELS[c[i] >> 4] * xg[2 * i + 1];
        }
        row += scales[g] * (lo + hi);
    }
    return row;
}

/* crates/kernels-simd/src/lib.rs:191-208: `total += dot * scale`. */
float mfo_int8_row_dot(const uint8_t *codes, const float *scales, const float *x, uint64_t k) {
    float total = 0.0f;
    for (uint64_t g = 0; g < k / 128; ++g) {
        float dot = 0.0f;
        for (int j = 0; j < 128; ++j)
            dot += (float)(int8_t)codes[g * 128 + j] * x[g * 128 + j];
        total += dot * scales[g];
    }
    return total;
}

typedef float (*row_dot_fn)(const uint8_t *, const float *, const float *, uint64_t);

static row_dot_fn row_dot_for(int format) {
    switch (format) {
    case MFO_TERNARY: return mfo_ternary_row_dot;
    case MFO_NF4: return mfo_nf4_row_dot;
    case MFO_INT8: return mfo_int8_row_dot;
    default: return NULL;
    }
}

static uint64_t code_width(int format, uint64_t k) {
    return format == MFO_TERNARY ? k / 4 : format == MFO_NF4 ? k / 2 : k;
}

static int check_packed(const uint8_t *codes, uint64_t n, uint64_t k, int format) {
    if (k % 128 != 0) return MFO_INVALID_SHAPE;
    if (!row_dot_for(format)) return MFO_INVALID_ARGUMENT;
    if (format == MFO_INT8 && !int8_codes_ok(codes, n * k)) return MFO_INVALID_ARGUMENT;
    return MFO_OK;
}

typedef struct {
    float *out;
    const float *x;
    const float *w; /* dense weight (mfo_linear) */
    const uint8_t *codes_a;
    const float *scales_a;
    const uint8_t *codes_b;
    const float *scales_b;
    uint64_t n, k;
    int format, swiglu;
} linear_job;

static void packed_linear_range(void *ctx, int64_t begin, int64_t end, int *bad) {
    const linear_job *j = (const linear_job *)ctx;
    row_dot_fn dot = row_dot_for(j->format);
    const uint64_t cw = code_width(j->format, j->k), groups = j->k / 128;
    for (int64_t idx = begin; idx < end; ++idx) {
        uint64_t row = (uint64_t)idx / j->n, col = (uint64_t)idx % j->n;
        const float *xr = j->x + row * j->k;
        float value = dot(j->codes_a + col * cw, j->scales_a + col * groups, xr, j->k);
        if (j->swiglu) {
            /* packed.rs:351-362 */
            float up = dot(j->codes_b + col * cw, j->scales_b + col * groups, xr, j->k);
            float sigmoid = 1.0f / (1.0f + expf(-value));
            value = (value * sigmoid) * up;
        }
        if (!finite_f(value)) *bad = 1;
        j->out[row * j->n + col] = value;
    }
}

/* crates/backend-cpu/src/packed.rs:96-170: loop rows (tokens) then columns. */
int mfo_packed_linear(float *out, const float *x, uint64_t t, const uint8_t *codes,
                      const float *scales, uint64_t n, uint64_t k, int format, int threads) {
    int st = check_packed(codes, n, k, format);
    if (st) return st;
    linear_job job = {out, x, NULL, codes, scales, NULL, NULL, n, k, format, 0};
    return parallel_for((int64_t)(t * n), threads, packed_linear_range, &job) ? MFO_BACKEND_FAILURE
                                                                               : MFO_OK;
}

/* packed.rs:222-272: admission of both weight sets, then two sequential passes. */
int mfo_packed_linear_pair(float *out_a, float *out_b, const float *x, uint64_t t,
                           const uint8_t *codes_a, const float *scales_a,
                           const uint8_t *codes_b, const float *scales_b,
                           uint64_t n, uint64_t k, int format, int threads) {
    int st = check_packed(codes_a, n, k, format);
    if (!st) st = check_packed(codes_b, n, k, format);
    if (st) return st;
    st = mfo_packed_linear(out_a, x, t, codes_a, scales_a, n, k, format, threads);
    if (st) return st;
    return mfo_packed_linear(out_b, x, t, codes_b, scales_b, n, k, format, threads);
}

/* packed.rs:278-372: out = (a * sigmoid(a)) * b with sigmoid = 1 / (1 + exp(-a)). */
int mfo_packed_swiglu_pair(float *out, const float *x, uint64_t t,
                           const uint8_t *codes_a, const float *scales_a,
                           const uint8_t *codes_b, const float *scales_b,
                           uint64_t n, uint64_t k, int format, int threads) {
    int st = check_packed(codes_a, n, k, format);
    if (!st) st = check_packed(codes_b, n, k, format);
    if (st) return st;
    linear_job job = {out, x, NULL, codes_a, scales_a, codes_b, scales_b, n, k, format, 1};
    return parallel_for((int64_t)(t * n), threads, packed_linear_range, &job) ? MFO_BACKEND_FAILURE
                                                                               : MFO_OK;
}

/* packed.rs:377-465: stage silu(gate) * up per token row, then row dots. */
int mfo_packed_swiglu_linear(float *out, const float *gate, const float *up, uint64_t t,
                             const uint8_t *codes, const float *scales,
                             uint64_t n, uint64_t k, int format, int threads) {
    int st = check_packed(codes, n, k, format);
    if (st) return st;
    float *act = (float *)malloc(sizeof(float) * (t * k + 1));
    if (!act) return MFO_RESOURCE_LIMIT;
    for (uint64_t i = 0; i < t * k; ++i) {
        float g = gate[i];
        float sigmoid = 1.0f / (1.0f + expf(-g));
        float value = (g * sigmoid) * up[i];
        if (!finite_f(value)) {
            free(act);
            return MFO_BACKEND_FAILURE;
        }
        act[i] = value;
    }
    st = mfo_packed_linear(out, act, t, codes, scales, n, k, format, threads);
    free(act);
    return st;
}

/* crates/backend-cpu/src/dense.rs:35-50. */
int64_t mfo_resolve_device_id(float value) {
    if (finite_f(value) && value >= 0.0f && floorf(value) == value && value < 16777216.0f)
        return (int64_t)value;
    return -1;
}

/* crates/backend-cpu/src/packed.rs:11-91: out = level(code) * scale, one multiply. */
int mfo_packed_gather_rows(float *out, const uint8_t *codes, const float *scales,
                           uint64_t rows, uint64_t k, int format,
                           const int64_t *ids, uint64_t n_ids) {
    int st = check_packed(codes, rows, k, format);
    if (st) return st;
    const uint64_t cw = code_width(format, k), groups = k / 128;
    for (uint64_t i = 0; i < n_ids; ++i)
        if (ids[i] >= 0 && (uint64_t)ids[i] >= rows) return MFO_OUT_OF_BOUNDS;
    for (uint64_t i = 0; i < n_ids; ++i) {
        float *dst = out + i * k;
        if (ids[i] < 0) {
            for (uint64_t j = 0; j < k; ++j) dst[j] = NAN;
            continue;
        }
        const uint8_t *c = codes + (uint64_t)ids[i] * cw;
        const float *s = scales + (uint64_t)ids[i] * groups;
        for (uint64_t j = 0; j < k; ++j) {
            uint64_t g = j / 128, w = j % 128;
            float level;
            if (format == MFO_TERNARY) {
                unsigned code = (c[g * 32 + w / 4] >> (2 * (w % 4))) & 0x3u;
                level = (float)code - 1.0f;
            } else if (format == MFO_INT8) {
                level = (float)(int8_t)c[j];
            } else {
                uint8_t b = c[g * 64 + w / 2];
                level = MFO_NF4_LEVELS[(w % 2 == 0) ? (b & 0x0F) : (b >> 4)];
            }
            dst[j] = level * s[g];
        }
    }
    return MFO_OK;
}

/* crates/backend-cpu/src/dense.rs:200-270: sequential increasing-k accumulation. */
static void linear_range(void *ctx, int64_t begin, int64_t end, int *bad) {
    const linear_job *j = (const linear_job *)ctx;
    for (int64_t idx = begin; idx < end; ++idx) {
        uint64_t row = (uint64_t)idx / j->n, col = (uint64_t)idx % j->n;
        const float *xr = j->x + row * j->k, *wr = j->w + col * j->k;
        float acc = 0.0f;
        for (uint64_t i = 0; i < j->k; ++i) acc += xr[i] * wr[i];
        if (!finite_f(acc)) *bad = 1;
        j->out[row * j->n + col] = acc;
    }
}

int mfo_linear(float *out, const float *x, uint64_t t, const float *w, uint64_t n, uint64_t k,
               int threads) {
    linear_job job = {out, x, w, NULL, NULL, NULL, NULL, n, k, 0, 0};
    return parallel_for((int64_t)(t * n), threads, linear_range, &job) ? MFO_BACKEND_FAILURE
                                                                        : MFO_OK;
}

/* crates/backend-cpu/src/dense.rs:369-411: first strict maximum, NaN if poisoned. */
int mfo_argmax(float *out, const float *logits, uint64_t rows, uint64_t width) {
    if (width == 0 || width > (1ull << 24)) return MFO_UNSUPPORTED;
    for (uint64_t r = 0; r < rows; ++r) {
        const float *row = logits + r * width;
        float best = -INFINITY;
        uint64_t best_index = 0;
        int poisoned = 0;
        for (uint64_t i = 0; i < width; ++i) {
            if (!finite_f(row[i])) poisoned = 1;
            else if (row[i] > best) {
                best = row[i];
                best_index = i;
            }
        }
        out[r] = poisoned ? NAN : (float)best_index;
    }
    return MFO_OK;
}

/* crates/backend-cpu/src/dense.rs:413-473. */
int mfo_argmax_masked(float *out, const float *logits, uint64_t rows, uint64_t width,
                      const uint64_t *mask, uint64_t mask_words) {
    if (width == 0 || width > (1ull << 24)) return MFO_UNSUPPORTED;
    if (mask_words != (width + 63) / 64) return MFO_INVALID_ARGUMENT;
    for (uint64_t r = 0; r < rows; ++r) {
        const float *row = logits + r * width;
        float best = -INFINITY;
        uint64_t best_index = UINT64_MAX;
        int poisoned = 0;
        for (uint64_t i = 0; i < width; ++i) {
            if (!(mask[i / 64] & (1ull << (i % 64)))) continue;
            if (!finite_f(row[i])) poisoned = 1;
            else if (row[i] > best || (row[i] == best && i < best_index)) {
                best = row[i];
                best_index = i;
            }
        }
        out[r] = (poisoned || best_index == UINT64_MAX) ? NAN : (float)best_index;
    }
    return MFO_OK;
}

/* crates/backend-cpu/src/dense.rs:55-109. */
int mfo_gather_rows(float *out, const float *table, uint64_t rows, uint64_t cols,
                    const int64_t *ids, uint64_t n_ids) {
    for (uint64_t i = 0; i < n_ids; ++i)
        if (ids[i] >= 0 && (uint64_t)ids[i] >= rows) return MFO_OUT_OF_BOUNDS;
    for (uint64_t i = 0; i < n_ids; ++i) {
        if (ids[i] < 0) {
            for (uint64_t j = 0; j < cols; ++j) out[i * cols + j] = NAN;
        } else {
            memcpy(out + i * cols, table + (uint64_t)ids[i] * cols, sizeof(float) * cols);
        }
    }
    return MFO_OK;
}

/* crates/backend-cpu/src/dense.rs:343-367. */
int mfo_swiglu(float *out, const float *gate, const float *up, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        float sigmoid = 1.0f / (1.0f + expf(-gate[i]));
        float r = (gate[i] * sigmoid) * up[i];
        if (!finite_f(r)) return MFO_BACKEND_FAILURE;
        out[i] = r;
    }
    return MFO_OK;
}

/* crates/backend-cpu/src/dense.rs:153-198. */
int mfo_add(float *out, const float *a, const float *b, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        float r = a[i] + b[i];
        if (!finite_f(r)) return MFO_BACKEND_FAILURE;
        out[i] = r;
    }
    return MFO_OK;
}

int mfo_multiply(float *out, const float *a, const float *b, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        float r = a[i] * b[i];
        if (!finite_f(r)) return MFO_BACKEND_FAILURE;
        out[i] = r;
    }
    return MFO_OK;
}

/* Shared RMS step of normalization_rotary.rs:55-79 / :124-150 / :332-344:
 * sequential sum of squares, then 1 / sqrt(sum / width + eps). */
static int rms_reciprocal(const float *x, uint64_t width, float eps, float *out) {
    float sq = 0.0f;
    for (uint64_t i = 0; i < width; ++i) sq += x[i] * x[i];
    float r = 1.0f / sqrtf(sq / (float)width + eps);
    if (!finite_f(r)) return MFO_BACKEND_FAILURE;
    *out = r;
    return MFO_OK;
}

/* crates/backend-cpu/src/normalization_rotary.rs:11-81. */
int mfo_row_rms_norm(float *out, const float *x, uint64_t rows, uint64_t width,
                     const float *weight, float eps) {
    if (!finite_f(eps) || eps <= 0.0f) return MFO_INVALID_ARGUMENT;
    if (width == 0) return MFO_OK;
    if (width > (1ull << 24)) return MFO_UNSUPPORTED;
    for (uint64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * width;
        float rec;
        int st = rms_reciprocal(xr, width, eps, &rec);
        if (st) return st;
        for (uint64_t c = 0; c < width; ++c) {
            float normalized = xr[c] * rec;
            float v = normalized * weight[c];
            if (!finite_f(v)) return MFO_BACKEND_FAILURE;
            out[r * width + c] = v;
        }
    }
    return MFO_OK;
}

/* normalization_rotary.rs:221-235: add, then row_rms_norm over the sum. */
int mfo_add_row_rms_norm(float *sum, float *normed, const float *a, const float *b,
                         uint64_t rows, uint64_t width, const float *weight, float eps) {
    int st = mfo_add(sum, a, b, rows * width);
    if (st) return st;
    return mfo_row_rms_norm(normed, sum, rows, width, weight, eps);
}

/* normalization_rotary.rs:83-153. */
int mfo_head_rms_norm(float *out, const float *x, uint64_t tokens, uint32_t heads,
                      uint32_t head_dim, const float *weight, float eps) {
    if (!finite_f(eps) || eps <= 0.0f) return MFO_INVALID_ARGUMENT;
    for (uint64_t t = 0; t < tokens; ++t)
        for (uint32_t h = 0; h < heads; ++h) {
            uint64_t start = t * (uint64_t)heads * head_dim + (uint64_t)h * head_dim;
            float rec;
            int st = rms_reciprocal(x + start, head_dim, eps, &rec);
            if (st) return st;
            for (uint32_t c = 0; c < head_dim; ++c) {
                float v = (x[start + c] * rec) * weight[c];
                if (!finite_f(v)) return MFO_BACKEND_FAILURE;
                out[start + c] = v;
            }
        }
    return MFO_OK;
}

/* normalization_rotary.rs:196-201 / :346-350: f64 pow and trig, cast to f32 at
 * the documented boundaries; the angle is an f32 product. */
static void rope_cos_sin(uint64_t position, uint32_t column, uint32_t head_dim, float theta,
                         float *cosine, float *sine) {
    double exponent = -2.0 * (double)column / (double)head_dim;
    float frequency = (float)pow((double)theta, exponent);
    float angle = (float)position * frequency;
    *sine = (float)sin((double)angle);
    *cosine = (float)cos((double)angle);
}

/* normalization_rotary.rs:155-219. */
int mfo_split_half_rotary(float *out, const float *x, uint64_t tokens, uint32_t heads,
                          uint32_t head_dim, const uint64_t *positions, float theta) {
    uint32_t half = head_dim / 2;
    for (uint64_t t = 0; t < tokens; ++t)
        for (uint32_t h = 0; h < heads; ++h) {
            uint64_t start = t * (uint64_t)heads * head_dim + (uint64_t)h * head_dim;
            for (uint32_t c = 0; c < half; ++c) {
                float cosine, sine;
                rope_cos_sin(positions[t], c, head_dim, theta, &cosine, &sine);
                float first = x[start + c], second = x[start + half + c];
                float rf = first * cosine - second * sine;
                float rs = second * cosine + first * sine;
                if (!finite_f(rf) || !finite_f(rs)) return MFO_BACKEND_FAILURE;
                out[start + c] = rf;
                out[start + half + c] = rs;
            }
        }
    return MFO_OK;
}

/* normalization_rotary.rs:246-369: per-head RMS then split-half RoPE. */
static int norm_rope_one(float *out, const float *x, uint64_t tokens, uint32_t heads,
                         uint32_t head_dim, const float *weight, const uint64_t *positions,
                         float theta, float eps, float *normed) {
    uint32_t half = head_dim / 2;
    for (uint64_t t = 0; t < tokens; ++t)
        for (uint32_t h = 0; h < heads; ++h) {
            uint64_t start = t * (uint64_t)heads * head_dim + (uint64_t)h * head_dim;
            float rec;
            int st = rms_reciprocal(x + start, head_dim, eps, &rec);
            if (st) return st;
            for (uint32_t i = 0; i < head_dim; ++i) normed[i] = x[start + i] * rec * weight[i];
            for (uint32_t c = 0; c < half; ++c) {
                float cosine, sine;
                rope_cos_sin(positions[t], c, head_dim, theta, &cosine, &sine);
                float first = normed[c], second = normed[half + c];
                float rf = first * cosine - second * sine;
                float rs = second * cosine + first * sine;
                if (!finite_f(rf) || !finite_f(rs)) return MFO_BACKEND_FAILURE;
                out[start + c] = rf;
                out[start + half + c] = rs;
            }
        }
    return MFO_OK;
}

int mfo_qk_norm_rope(float *q_out, float *k_out, const float *q, const float *k,
                     uint64_t tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                     const float *q_weight, const float *k_weight,
                     const uint64_t *positions, float theta, float eps) {
    if (!finite_f(eps) || eps <= 0.0f) return MFO_INVALID_ARGUMENT;
    float *normed = (float *)malloc(sizeof(float) * (head_dim ? head_dim : 1));
    if (!normed) return MFO_RESOURCE_LIMIT;
    int st = norm_rope_one(q_out, q, tokens, q_heads, head_dim, q_weight, positions, theta, eps,
                           normed);
    if (!st)
        st = norm_rope_one(k_out, k, tokens, kv_heads, head_dim, k_weight, positions, theta, eps,
                           normed);
    free(normed);
    return st;
}

/* crates/backend-cpu/src/attention_convolution.rs:11-216.  The reference
 * recomputes each score in every pass; the recomputation is deterministic, so
 * computing each score (and each probability) once gives identical bits. */
typedef struct {
    float *staged;
    const float *q, *k, *v, *key_cache, *value_cache;
    uint64_t initial;
    uint32_t q_heads, group, head_dim;
    uint64_t qw, kvw;
    float scale;
} gqa_job;

static void gqa_range(void *ctx, int64_t begin, int64_t end, int *bad) {
    const gqa_job *j = (const gqa_job *)ctx;
    if (begin >= end) return;
    uint64_t last_t = (uint64_t)(end - 1) / j->q_heads;
    float *scores = (float *)malloc(sizeof(float) * (j->initial + last_t + 1));
    if (!scores) {
        *bad = 1;
        return;
    }
    const uint32_t hd = j->head_dim;
    for (int64_t item = begin; item < end; ++item) {
        uint64_t t = (uint64_t)item / j->q_heads;
        uint32_t qh = (uint32_t)((uint64_t)item % j->q_heads), kvh = qh / j->group;
        uint64_t visible = j->initial + t + 1;
        const float *qr = j->q + t * j->qw + (uint64_t)qh * hd;
        float maximum = -INFINITY;
        for (uint64_t key = 0; key < visible; ++key) {
            const float *kr = key < j->initial
                                  ? j->key_cache + key * j->kvw + (uint64_t)kvh * hd
                                  : j->k + (key - j->initial) * j->kvw + (uint64_t)kvh * hd;
            float dot = 0.0f;
            for (uint32_t d = 0; d < hd; ++d) dot += qr[d] * kr[d];
            float s = dot * j->scale;
            if (!finite_f(s)) *bad = 1;
            scores[key] = s;
            maximum = fmaxf(maximum, s);
        }
        float denominator = 0.0f;
        for (uint64_t key = 0; key < visible; ++key) denominator += expf(scores[key] - maximum);
        if (!finite_f(denominator) || denominator <= 0.0f) *bad = 1;
        for (uint64_t key = 0; key < visible; ++key)
            scores[key] = expf(scores[key] - maximum) / denominator;
        for (uint32_t d = 0; d < hd; ++d) {
            float weighted = 0.0f;
            for (uint64_t key = 0; key < visible; ++key) {
                const float *vr = key < j->initial
                                      ? j->value_cache + key * j->kvw + (uint64_t)kvh * hd
                                      : j->v + (key - j->initial) * j->kvw + (uint64_t)kvh * hd;
                weighted += scores[key] * vr[d];
            }
            if (!finite_f(weighted)) *bad = 1;
            j->staged[t * j->qw + (uint64_t)qh * hd + d] = weighted;
        }
    }
    free(scores);
}

int mfo_causal_gqa(float *out, const float *q, const float *k, const float *v,
                   uint64_t tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                   float *key_cache, float *value_cache, uint64_t capacity,
                   uint64_t *cache_len, int threads) {
    if (kv_heads == 0 || q_heads == 0 || q_heads % kv_heads) return MFO_INVALID_SHAPE;
    uint64_t initial = *cache_len;
    if (initial > capacity || initial + tokens > capacity) return MFO_OUT_OF_BOUNDS;
    const uint64_t qw = (uint64_t)q_heads * head_dim, kvw = (uint64_t)kv_heads * head_dim;
    float *staged = (float *)malloc(sizeof(float) * (tokens * qw + 1));
    if (!staged) return MFO_RESOURCE_LIMIT;
    gqa_job job = {staged, q, k, v, key_cache, value_cache, initial, q_heads,
                   q_heads / kv_heads, head_dim, qw, kvw, 1.0f / sqrtf((float)head_dim)};
    if (parallel_for((int64_t)(tokens * q_heads), threads, gqa_range, &job)) {
        free(staged);
        return MFO_BACKEND_FAILURE;
    }
    memcpy(key_cache + initial * kvw, k, sizeof(float) * tokens * kvw);
    memcpy(value_cache + initial * kvw, v, sizeof(float) * tokens * kvw);
    memcpy(out, staged, sizeof(float) * tokens * qw);
    free(staged);
    *cache_len = initial + tokens;
    return MFO_OK;
}

/* crates/backend-cpu/src/attention_convolution.rs:218-340.  `history` is the
 * [width - 1, hidden] rolling U buffer, oldest row first. */
int mfo_gated_short_conv(float *out, const float *projection, uint64_t tokens,
                         uint32_t hidden, const float *kernel, uint32_t width,
                         float *history) {
    if (hidden == 0 || width == 0) return MFO_INVALID_ARGUMENT;
    const uint64_t h = hidden, pw = 3 * h, hist_rows = width - 1;
    float *u = (float *)malloc(sizeof(float) * (2 * tokens * h + 1));
    if (!u) return MFO_RESOURCE_LIMIT;
    float *produced = u + tokens * h;
    for (uint64_t i = 0; i < tokens * h; ++i) {
        uint64_t t = i / h, c = i % h, base = t * pw + c;
        float gate = projection[base] * projection[base + 2 * h];
        if (!finite_f(gate)) {
            free(u);
            return MFO_BACKEND_FAILURE;
        }
        u[i] = gate;
    }
    for (uint64_t t = 0; t < tokens; ++t)
        for (uint64_t c = 0; c < h; ++c) {
            float total = 0.0f;
            for (uint64_t tap = 0; tap < width; ++tap) {
                int64_t rel = (int64_t)t + (int64_t)tap - (int64_t)hist_rows;
                float uv = rel < 0 ? history[(uint64_t)(rel + (int64_t)hist_rows) * h + c]
                                   : u[(uint64_t)rel * h + c];
                total += kernel[c * width + tap] * uv;
            }
            float r = total * projection[t * pw + h + c];
            if (!finite_f(r)) {
                free(u);
                return MFO_BACKEND_FAILURE;
            }
            produced[t * h + c] = r;
        }
    if (hist_rows > 0) {
        if (tokens >= hist_rows) {
            memcpy(history, u + (tokens - hist_rows) * h, sizeof(float) * hist_rows * h);
        } else {
            uint64_t keep = hist_rows - tokens;
            memmove(history, history + (hist_rows - keep) * h, sizeof(float) * keep * h);
            memcpy(history + keep * h, u, sizeof(float) * tokens * h);
        }
    }
    memcpy(out, produced, sizeof(float) * tokens * h);
    free(u);
    return MFO_OK;
}

/* ------------------------------------------------------------------------
 * Encoder ops: crates/backend-cpu/src/encoder.rs.
 * --------------------------------------------------------------------- */
static int cmp_u32(const void *a, const void *b) {
    uint32_t x = *(const uint32_t *)a, y = *(const uint32_t *)b;
    return x < y ? -1 : x > y;
}

/* crates/engine-api/src/encoder.rs:16-45: every nonzero label occupies one
 * contiguous run. */
int mfo_encoder_segments_check(const uint32_t *segment_ids, uint64_t tokens) {
    uint32_t *runs = (uint32_t *)malloc(sizeof(uint32_t) * (tokens + 1));
    if (!runs) return MFO_RESOURCE_LIMIT;
    uint64_t n = 0;
    uint32_t previous = 0;
    for (uint64_t i = 0; i < tokens; ++i) {
        if (segment_ids[i] != previous && segment_ids[i] != 0) runs[n++] = segment_ids[i];
        previous = segment_ids[i];
    }
    qsort(runs, n, sizeof(uint32_t), cmp_u32);
    int st = MFO_OK;
    for (uint64_t i = 1; i < n; ++i)
        if (runs[i] == runs[i - 1]) st = MFO_INVALID_ARGUMENT;
    free(runs);
    return st;
}

typedef struct {
    float *staged;
    const float *q, *k, *v;
    const uint32_t *ids;
    uint64_t tokens;
    uint32_t heads, group, dim;
    uint64_t qw, kvw;
    float scale;
} enc_gqa_job;

/* crates/backend-cpu/src/encoder.rs:62-118 for items (token, head). */
static void enc_gqa_range(void *ctx, int64_t begin, int64_t end, int *bad) {
    const enc_gqa_job *j = (const enc_gqa_job *)ctx;
    float *scores = (float *)malloc(sizeof(float) * (j->tokens + 1));
    if (!scores) {
        *bad = 1;
        return;
    }
    for (int64_t item = begin; item < end && !*bad; ++item) {
        const uint64_t token = (uint64_t)item / j->heads, head = (uint64_t)item % j->heads;
        const uint32_t segment = j->ids[token];
        if (segment == 0) continue;
        const uint64_t q_off = token * j->qw + head * j->dim, kv_head = head / j->group;
        float maximum = -INFINITY;
        for (uint64_t other = 0; other < j->tokens; ++other) {
            scores[other] = -INFINITY;
            if (j->ids[other] != segment) continue;
            const float *kr = j->k + other * j->kvw + kv_head * j->dim;
            float dot = 0.0f;
            for (uint32_t c = 0; c < j->dim; ++c) dot += j->q[q_off + c] * kr[c];
            scores[other] = dot * j->scale;
            if (!finite_f(scores[other])) {
                *bad = 1;
                break;
            }
            maximum = fmaxf(maximum, scores[other]);
        }
        if (*bad) break;
        float denominator = 0.0f;
        for (uint64_t other = 0; other < j->tokens; ++other) {
            scores[other] = j->ids[other] == segment ? expf(scores[other] - maximum) : 0.0f;
            denominator += scores[other];
        }
        if (!finite_f(denominator) || denominator <= 0.0f) {
            *bad = 1;
            break;
        }
        for (uint32_t c = 0; c < j->dim; ++c) {
            float weighted = 0.0f;
            for (uint64_t other = 0; other < j->tokens; ++other)
                if (j->ids[other] == segment)
                    weighted += (scores[other] / denominator) * j->v[other * j->kvw + kv_head * j->dim + c];
            if (!finite_f(weighted)) {
                *bad = 1;
                break;
            }
            j->staged[q_off + c] = weighted;
        }
    }
    free(scores);
}

int mfo_bidirectional_gqa(float *out, const float *q, const float *k, const float *v,
                          const uint32_t *segment_ids, uint64_t tokens, uint32_t q_heads,
                          uint32_t kv_heads, uint32_t head_dim, int threads) {
    if (kv_heads == 0 || q_heads == 0 || q_heads % kv_heads) return MFO_INVALID_SHAPE;
    int st = mfo_encoder_segments_check(segment_ids, tokens);
    if (st) return st;
    const uint64_t qw = (uint64_t)q_heads * head_dim, kvw = (uint64_t)kv_heads * head_dim;
    float *staged = (float *)calloc(tokens * qw + 1, sizeof(float));
    if (!staged) return MFO_RESOURCE_LIMIT;
    enc_gqa_job job = {staged, q, k, v, segment_ids, tokens, q_heads, q_heads / kv_heads, head_dim, qw, kvw,
                       1.0f / sqrtf((float)head_dim)};
    if (parallel_for((int64_t)(tokens * q_heads), threads, enc_gqa_range, &job)) {
        free(staged);
        return MFO_BACKEND_FAILURE;
    }
    memcpy(out, staged, sizeof(float) * tokens * qw);
    free(staged);
    return MFO_OK;
}

/* crates/backend-cpu/src/encoder.rs:126-189. */
int mfo_centered_gated_conv(float *out, const float *projection, const float *kernel,
                            const uint32_t *segment_ids, uint64_t tokens, uint32_t hidden,
                            uint32_t width) {
    if (hidden == 0 || width == 0) return MFO_INVALID_ARGUMENT;
    int st = mfo_encoder_segments_check(segment_ids, tokens);
    if (st) return st;
    const uint64_t h = hidden;
    float *staged = (float *)calloc(tokens * h + 1, sizeof(float));
    if (!staged) return MFO_RESOURCE_LIMIT;
    for (uint64_t token = 0; token < tokens; ++token) {
        const uint32_t segment = segment_ids[token];
        if (segment == 0) continue;
        for (uint64_t c = 0; c < h; ++c) {
            float total = 0.0f;
            for (uint32_t tap = 0; tap < width; ++tap) {
                if (token + tap < width / 2) continue;
                const uint64_t other = token + tap - width / 2;
                if (other < tokens && segment_ids[other] == segment) {
                    const uint64_t base = other * 3 * h + c;
                    total += kernel[c * width + tap] * (projection[base] * projection[base + 2 * h]);
                }
            }
            const float value = projection[token * 3 * h + h + c] * total;
            if (!finite_f(value)) {
                free(staged);
                return MFO_BACKEND_FAILURE;
            }
            staged[token * h + c] = value;
        }
    }
    memcpy(out, staged, sizeof(float) * tokens * h);
    free(staged);
    return MFO_OK;
}

/* ------------------------------------------------------------------------
 * LFM2 model: crates/executor-core/src/lfm2/executor/execution.rs:35-627.
 * --------------------------------------------------------------------- */
struct mfo_lfm2 {
    mfo_lfm2_config config;
    int32_t *kinds;
    mfo_lfm2_weights weights;
    int threads;
    uint64_t length;
    float **conv_history; /* per layer, [width - 1, hidden] or NULL */
    float **key_cache, **value_cache;
    uint64_t *cache_len;
};

static int weight_ok(const mfo_weight *w, uint64_t rows, uint64_t cols) {
    if (w->rows != rows || w->cols != cols) return MFO_INVALID_SHAPE;
    if (w->packed) {
        if (cols % 128) return MFO_INVALID_SHAPE;
        if (w->format == MFO_INT8 && !int8_codes_ok(w->codes, rows * cols))
            return MFO_INVALID_ARGUMENT;
    }
    return MFO_OK;
}

/* execution.rs:12-25: dense `linear` or `packed_linear` by the role's storage. */
static int weight_linear(const mfo_lfm2 *m, float *out, const float *x, uint64_t t,
                         const mfo_weight *w) {
    if (w->packed)
        return mfo_packed_linear(out, x, t, w->codes, w->scales, w->rows, w->cols, w->format,
                                 m->threads);
    return mfo_linear(out, x, t, w->dense, w->rows, w->cols, m->threads);
}

int mfo_lfm2_create(const mfo_lfm2_config *config, const mfo_lfm2_weights *weights,
                    int threads, mfo_lfm2 **out) {
    const mfo_lfm2_config *c = config;
    if (!c->hidden || !c->q_heads || !c->kv_heads || c->q_heads % c->kv_heads ||
        c->q_heads * c->head_dim != c->hidden || !c->conv_width)
        return MFO_INVALID_SHAPE;
    int st = weight_ok(&weights->embedding, c->vocab, c->hidden);
    if (st) return st;
    const uint64_t h = c->hidden, f = c->intermediate, kvw = (uint64_t)c->kv_heads * c->head_dim;
    for (uint32_t i = 0; i < c->n_layers; ++i) {
        const mfo_lfm2_layer_weights *L = &weights->layers[i];
        if (c->layer_kinds[i] == MFO_LAYER_CONV) {
            if ((st = weight_ok(&L->in_proj, 3 * h, h)) || (st = weight_ok(&L->out_proj, h, h)))
                return st;
        } else {
            if ((st = weight_ok(&L->q, h, h)) || (st = weight_ok(&L->k, kvw, h)) ||
                (st = weight_ok(&L->v, kvw, h)) || (st = weight_ok(&L->o, h, h)))
                return st;
        }
        if ((st = weight_ok(&L->w1, f, h)) || (st = weight_ok(&L->w3, f, h)) ||
            (st = weight_ok(&L->w2, h, f)))
            return st;
    }
    mfo_lfm2 *m = (mfo_lfm2 *)calloc(1, sizeof(*m));
    if (!m) return MFO_RESOURCE_LIMIT;
    m->config = *c;
    m->kinds = (int32_t *)malloc(sizeof(int32_t) * (c->n_layers + 1));
    memcpy(m->kinds, c->layer_kinds, sizeof(int32_t) * c->n_layers);
    m->config.layer_kinds = m->kinds;
    m->weights = *weights;
    m->threads = threads;
    m->conv_history = (float **)calloc(c->n_layers + 1, sizeof(float *));
    m->key_cache = (float **)calloc(c->n_layers + 1, sizeof(float *));
    m->value_cache = (float **)calloc(c->n_layers + 1, sizeof(float *));
    m->cache_len = (uint64_t *)calloc(c->n_layers + 1, sizeof(uint64_t));
    for (uint32_t i = 0; i < c->n_layers; ++i) {
        if (c->layer_kinds[i] == MFO_LAYER_CONV) {
            m->conv_history[i] = (float *)calloc((c->conv_width - 1) * h + 1, sizeof(float));
        } else {
            m->key_cache[i] = (float *)calloc(c->max_tokens * kvw + 1, sizeof(float));
            m->value_cache[i] = (float *)calloc(c->max_tokens * kvw + 1, sizeof(float));
        }
    }
    *out = m;
    return MFO_OK;
}

void mfo_lfm2_destroy(mfo_lfm2 *m) {
    if (!m) return;
    for (uint32_t i = 0; i < m->config.n_layers; ++i) {
        free(m->conv_history[i]);
        free(m->key_cache[i]);
        free(m->value_cache[i]);
    }
    free(m->conv_history);
    free(m->key_cache);
    free(m->value_cache);
    free(m->cache_len);
    free(m->kinds);
    free(m);
}

int mfo_lfm2_fork(const mfo_lfm2 *src, mfo_lfm2 **out) {
    mfo_lfm2 *m = NULL;
    int st = mfo_lfm2_create(&src->config, &src->weights, src->threads, &m);
    if (st) return st;
    const uint64_t h = src->config.hidden,
                   kvw = (uint64_t)src->config.kv_heads * src->config.head_dim;
    for (uint32_t i = 0; i < src->config.n_layers; ++i) {
        if (src->kinds[i] == MFO_LAYER_CONV) {
            memcpy(m->conv_history[i], src->conv_history[i],
                   sizeof(float) * (src->config.conv_width - 1) * h);
        } else {
            memcpy(m->key_cache[i], src->key_cache[i],
                   sizeof(float) * src->config.max_tokens * kvw);
            memcpy(m->value_cache[i], src->value_cache[i],
                   sizeof(float) * src->config.max_tokens * kvw);
        }
        m->cache_len[i] = src->cache_len[i];
    }
    m->length = src->length;
    *out = m;
    return MFO_OK;
}

uint64_t mfo_lfm2_length(const mfo_lfm2 *m) { return m->length; }

#define TRY(expr)             \
    do {                      \
        st = (expr);          \
        if (st) goto cleanup; \
    } while (0)

int mfo_lfm2_append(mfo_lfm2 *m, const uint32_t *tokens, uint64_t n, float *logits) {
    const mfo_lfm2_config *c = &m->config;
    if (n == 0) return MFO_INVALID_ARGUMENT;
    for (uint64_t i = 0; i < n; ++i)
        if (tokens[i] >= c->vocab) return MFO_OUT_OF_BOUNDS;
    if (m->length + n > c->max_tokens) return MFO_RESOURCE_LIMIT;
    const uint64_t h = c->hidden, f = c->intermediate, kvw = (uint64_t)c->kv_heads * c->head_dim;
    int st = MFO_OK;
    uint64_t *positions = (uint64_t *)malloc(sizeof(uint64_t) * n);
    int64_t *ids = (int64_t *)malloc(sizeof(int64_t) * n);
    float *x = (float *)malloc(sizeof(float) * n * h);
    float *u = (float *)malloc(sizeof(float) * n * h);
    float *op = (float *)malloc(sizeof(float) * n * h);
    float *proj = (float *)malloc(sizeof(float) * n * 3 * h);
    float *conv = (float *)malloc(sizeof(float) * n * h);
    float *q = (float *)malloc(sizeof(float) * n * h);
    float *k = (float *)malloc(sizeof(float) * n * kvw);
    float *v = (float *)malloc(sizeof(float) * n * kvw);
    float *qr = (float *)malloc(sizeof(float) * n * h);
    float *kr = (float *)malloc(sizeof(float) * n * kvw);
    float *att = (float *)malloc(sizeof(float) * n * h);
    float *residual = (float *)malloc(sizeof(float) * n * h);
    float *ffn_in = (float *)malloc(sizeof(float) * n * h);
    float *gate = (float *)malloc(sizeof(float) * n * f);
    float *up = (float *)malloc(sizeof(float) * n * f);
    float *down = (float *)malloc(sizeof(float) * n * h);
    for (uint64_t i = 0; i < n; ++i) {
        positions[i] = m->length + i;
        ids[i] = tokens[i];
    }
    /* execution.rs:69-77: embedding gather. */
    const mfo_weight *emb = &m->weights.embedding;
    if (emb->packed)
        TRY(mfo_packed_gather_rows(x, emb->codes, emb->scales, emb->rows, emb->cols, emb->format,
                                   ids, n));
    else
        TRY(mfo_gather_rows(x, emb->dense, emb->rows, emb->cols, ids, n));
    /* execution.rs:86-94: layer-0 operator norm. */
    if (c->n_layers)
        TRY(mfo_row_rms_norm(u, x, n, h, m->weights.layers[0].operator_norm, c->block_eps));
    uint64_t rows = n;
    for (uint32_t li = 0; li < c->n_layers; ++li) {
        const mfo_lfm2_layer_weights *L = &m->weights.layers[li];
        if (m->kinds[li] == MFO_LAYER_CONV) {
            /* execution.rs:98-139. */
            TRY(weight_linear(m, proj, u, n, &L->in_proj));
            TRY(mfo_gated_short_conv(conv, proj, n, c->hidden, L->conv_kernel, c->conv_width,
                                     m->conv_history[li]));
            TRY(weight_linear(m, op, conv, n, &L->out_proj));
        } else {
            /* execution.rs:141-262 (the K/V pair is two packed_linear passes). */
            TRY(weight_linear(m, q, u, n, &L->q));
            TRY(weight_linear(m, k, u, n, &L->k));
            TRY(weight_linear(m, v, u, n, &L->v));
            TRY(mfo_qk_norm_rope(qr, kr, q, k, n, c->q_heads, c->kv_heads, c->head_dim, L->q_norm,
                                 L->k_norm, positions, c->rope_theta, c->block_eps));
            TRY(mfo_causal_gqa(att, qr, kr, v, n, c->q_heads, c->kv_heads, c->head_dim,
                               m->key_cache[li], m->value_cache[li], c->max_tokens,
                               &m->cache_len[li], m->threads));
            TRY(weight_linear(m, op, att, n, &L->o));
        }
        /* execution.rs:265-276. */
        TRY(mfo_add_row_rms_norm(residual, ffn_in, x, op, n, h, L->ffn_norm, c->block_eps));
        /* execution.rs:277-299: the final layer's FFN runs on the last row only. */
        const int last = li + 1 == c->n_layers;
        uint64_t ffn_rows = last ? 1 : n;
        const float *fin = ffn_in, *res = residual;
        if (ffn_rows != n) {
            fin = ffn_in + (n - 1) * h;
            res = residual + (n - 1) * h;
        }
        /* execution.rs:300-498: both FFN routes compute identical arithmetic. */
        TRY(weight_linear(m, gate, fin, ffn_rows, &L->w1));
        TRY(weight_linear(m, up, fin, ffn_rows, &L->w3));
        if (L->w2.packed) {
            TRY(mfo_packed_swiglu_linear(down, gate, up, ffn_rows, L->w2.codes, L->w2.scales,
                                         L->w2.rows, L->w2.cols, L->w2.format, m->threads));
        } else {
            TRY(mfo_swiglu(gate, gate, up, ffn_rows * f));
            TRY(weight_linear(m, down, gate, ffn_rows, &L->w2));
        }
        /* execution.rs:499-517: next operator norm or the final embedding norm. */
        const float *norm_w = last ? m->weights.embedding_norm : m->weights.layers[li + 1].operator_norm;
        float eps = last ? c->norm_eps : c->block_eps;
        TRY(mfo_add_row_rms_norm(x, u, res, down, ffn_rows, h, norm_w, eps));
        rows = ffn_rows;
    }
    if (c->n_layers == 0) TRY(mfo_row_rms_norm(u, x, n, h, m->weights.embedding_norm, c->norm_eps));
    if (logits) {
        /* execution.rs:540-572: logits from the last row. */
        const float *last_row = u + (rows - 1) * h;
        TRY(weight_linear(m, logits, last_row, 1, emb));
    }
    m->length += n;
cleanup:
    free(positions); free(ids); free(x); free(u); free(op); free(proj); free(conv);
    free(q); free(k); free(v); free(qr); free(kr); free(att); free(residual); free(ffn_in);
    free(gate); free(up); free(down);
    return st;
}

/* execution.rs:591-627: append one token, then argmax into the sampled id. */
int mfo_lfm2_append_argmax(mfo_lfm2 *m, uint32_t token, float *sampled, float *logits) {
    float *buf = logits ? logits : (float *)malloc(sizeof(float) * m->config.vocab);
    int st = mfo_lfm2_append(m, &token, 1, buf);
    if (!st) st = mfo_argmax(sampled, buf, 1, m->config.vocab);
    if (!logits) free(buf);
    return st;
}

// LFM2 layer kernels around the packed matmuls, for sm_100a.
//
// Arithmetic follows the reference CPU backend where the order is cheap to
// keep (elementwise ops, RoPE combination, the conv tap sum, the RMS
// reciprocal and scaling use explicitly rounded IEEE ops, so they match the
// CPU bit-for-bit given equal inputs); reductions (RMS sum of squares,
// attention, dense dots) are parallel and agree within F32 reorder error.
#include <algorithm>
#include <cfloat>
#include <atomic>
#include <mutex>

#include "mf_common.cuh"
#include "packed_kernels.h"

namespace mf {

// Many-token matmuls use the tcgen05 GEMM when enabled (default) and the
// caller supplies activation scratch; otherwise the CUDA-core GEMM.
std::atomic<int> g_gemm_tc{1};

int32_t packed_matmul(int mode, bool swiglu_input, float *out_a, float *out_b, const float *x,
                      const float *gate, const float *up, uint64_t t, const uint8_t *codes_a,
                      const float *scales_a, const uint8_t *codes_b, const float *scales_b,
                      uint64_t n, uint64_t k, int format, const SplitScratch *ss, cudaStream_t stream,
                      bool lanetiled) {
    if (lanetiled && (format != MF_TERNARY || n % 16 || k % kGroup))
        return fail(MF_INVALID_ARGUMENT, "LUT2 codes are ternary with rows in multiples of 16");
    if (t >= gemm_min_tokens(format) && k > 0 && k % kGroup == 0 && g_gemm_tc.load(std::memory_order_relaxed) && ss &&
        ss->partial && ss->partial_floats >= packed_gemm_tc_scratch_floats(t, n, k))
        return packed_gemm_tc(mode, swiglu_input, out_a, out_b, x, gate, up, t, codes_a, scales_a, codes_b,
                              scales_b, n, k, format, *ss, stream, lanetiled);
    if (k > 0 && k % kGroup == 0 && t < kGemmMinTokens && packed_gemv_tc_supports(format, t) && ss && ss->partial &&
        ss->partial_floats >= packed_gemv_tc_scratch_floats(t, n, k) && (format != MF_NF4 || k <= 8192))
        return packed_gemv_tc(mode, swiglu_input, out_a, out_b, x, gate, up, t, codes_a, scales_a, codes_b,
                              scales_b, n, k, format, *ss, stream, lanetiled);
    if (lanetiled) return fail(MF_UNSUPPORTED, "LUT2 codes run on the tensor-core matmuls only");
    if (t >= kGemmMinTokens && k > 0)
        return packed_gemm(mode, swiglu_input, out_a, out_b, x, gate, up, t, codes_a, scales_a,
                           codes_b, scales_b, n, k, format, stream);
    return packed_gemv(mode, swiglu_input, out_a, out_b, x, gate, up, t, codes_a, scales_a,
                       codes_b, scales_b, n, k, format, stream);
}

namespace {

__device__ __constant__ float kLevels[16] = {
    -0x1.000000p+0f, -0x1.647362p-1f, -0x1.0cd660p-1f, -0x1.946540p-2f,
    -0x1.23449ap-2f, -0x1.7a6a7ep-3f, -0x1.74f0e2p-4f, 0.0f,
    0x1.45f5fep-4f,  0x1.4995c6p-3f,  0x1.f809bap-3f,  0x1.5a0674p-2f,
    0x1.c34970p-2f,  0x1.200f56p-1f,  0x1.722766p-1f,  0x1.000000p+0f,
};

inline unsigned blocks_for(uint64_t n, unsigned threads) {
    uint64_t b = (n + threads - 1) / threads;
    return (unsigned)std::min<uint64_t>(b, 1u << 20);
}

// crates/backend-cpu/src/dense.rs:35-50: finite, >= 0, integral, < 2^24.
__device__ __forceinline__ long long resolve_id(float v, uint64_t rows) {
    if (isfinite(v) && v >= 0.0f && floorf(v) == v && v < 16777216.0f) {
        const long long id = (long long)v;
        return (uint64_t)id < rows ? id : -1;
    }
    return -1;
}

// ---------------------------------------------------------------------
// Dense F32 linear (the F32 tied LM head of the 350M configuration):
// one warp per output row, 128-bit loads along K, x staged per CTA.
// ---------------------------------------------------------------------
constexpr int kDenseTT = 4;

__global__ void __launch_bounds__(256) dense_linear_kernel(float *out, const float *x, int T,
                                                           const float *w, int N, int K) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) float xs[];  // kDenseTT * K
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int t0 = 0; t0 < T; t0 += kDenseTT) {
        const int tn = min(kDenseTT, T - t0);
        __syncthreads();
        for (int e = threadIdx.x; e < kDenseTT * K; e += blockDim.x) {
            const int t = e / K;
            xs[e] = t < tn ? x[(size_t)(t0 + t) * K + (e - t * K)] : 0.0f;
        }
        __syncthreads();
        for (int row = blockIdx.x * 8 + warp; row < N; row += gridDim.x * 8) {
            const float *wr = w + (size_t)row * K;
            float acc[kDenseTT] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int k = lane * 4; k < K; k += 128) {
                float4 wv;
                if (((K & 3) == 0)) {
                    wv = *reinterpret_cast<const float4 *>(wr + k);
                } else {
                    wv.x = wr[k];
                    wv.y = k + 1 < K ? wr[k + 1] : 0.0f;
                    wv.z = k + 2 < K ? wr[k + 2] : 0.0f;
                    wv.w = k + 3 < K ? wr[k + 3] : 0.0f;
                }
#pragma unroll
                for (int t = 0; t < kDenseTT; ++t) {
                    const float *xr = xs + t * K + k;
                    float a = acc[t];
                    a = fmaf(wv.x, xr[0], a);
                    if (k + 1 < K) a = fmaf(wv.y, xr[1], a);
                    if (k + 2 < K) a = fmaf(wv.z, xr[2], a);
                    if (k + 3 < K) a = fmaf(wv.w, xr[3], a);
                    acc[t] = a;
                }
            }
#pragma unroll
            for (int t = 0; t < kDenseTT; ++t) {
                const float v = warp_sum(acc[t]);
                if (lane == 0 && t < tn) out[(size_t)(t0 + t) * N + row] = v;
            }
        }
    }
}

// ---------------------------------------------------------------------
// Dense F32 LM head with the greedy argmax fused (one token): the tied
// [vocab, K] F32 embedding of the 350M configuration is 268 MB, read once
// per token, so the kernel is a pure weight stream.  Persistent CTAs (two
// per SM) stride over rows, a warp per row; each lane holds its K/128 float4
// of x in registers and streams its slice of two rows at a time with 16-byte
// evict-first loads (the first rows are issued before the dependency wait:
// weights are constants).  Every row's logit is written; each warp carries
// the first strict maximum (and a non-finite flag) across its rows, the
// CTA's candidate goes to `parts`, and the last CTA to arrive merges them in
// the rule of crates/backend-cpu/src/dense.rs:369-411, writes the greedy id
// (NaN when any logit is non-finite), advances the position and clears the
// counter.  The dot order is lane-parallel (a reordering of the sequential
// sum of dense.rs:202-270).
// ---------------------------------------------------------------------
constexpr int kHeadWarps = 8;
constexpr int kHeadMaxK4 = 16;   // K <= 2048 (K / 128 float4 per lane)

__device__ __forceinline__ void head_merge(float &bv, int &bi, int &bp, float ov, int oi, int op) {
    bp |= op;
    if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
        bv = ov;
        bi = oi;
    }
}

template <int K4>
__global__ void __launch_bounds__(kHeadWarps * 32) dense_head_argmax_kernel(float *logits, const float *x, const float *w,
                                                                           int N, float *parts, unsigned *count,
                                                                           float *sampled, uint64_t *pos, float *cand,
                                                                           int row0) {
    __shared__ float s_v[kHeadWarps];
    __shared__ int s_i[kHeadWarps], s_p[kHeadWarps];
    __shared__ bool s_last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int K = K4 * 128;
    const int stride = gridDim.x * kHeadWarps;
    int row = blockIdx.x * kHeadWarps + warp;
    // Two rows in flight: the current one and the next.
    float4 wa[K4], wb[K4];
    auto load_row = [&](float4 (&dst)[K4], int r) {
#pragma unroll
        for (int j = 0; j < K4; ++j) {
            if (r < N) {
                const uint4 u = ld_stream_u4(w + (size_t)r * K + 4 * lane + 128 * j);
                dst[j] = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w));
            }
        }
    };
    load_row(wa, row);
    load_row(wb, row + stride);
    pdl_wait();
    pdl_trigger();
    float4 xv[K4];
#pragma unroll
    for (int j = 0; j < K4; ++j) xv[j] = *reinterpret_cast<const float4 *>(x + 4 * lane + 128 * j);
    float bv = -INFINITY;
    int bi = -1, bp = 0;
    auto dot = [&](const float4 (&wr)[K4]) {
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int j = 0; j < K4; ++j) {
            a0 = fmaf(wr[j].x, xv[j].x, a0);
            a1 = fmaf(wr[j].y, xv[j].y, a1);
            a2 = fmaf(wr[j].z, xv[j].z, a2);
            a3 = fmaf(wr[j].w, xv[j].w, a3);
        }
        return warp_sum((a0 + a1) + (a2 + a3));
    };
    for (; row < N; row += 2 * stride) {
        const float va = dot(wa);
        const int rb = row + stride;
        float vb = 0.0f;
        if (rb < N) vb = dot(wb);
        load_row(wa, row + 2 * stride);
        load_row(wb, row + 3 * stride);
        if (lane == 0) {
            logits[row] = va;
            if (rb < N) logits[rb] = vb;
        }
        head_merge(bv, bi, bp, va, row, isfinite(va) ? 0 : 1);
        if (rb < N) head_merge(bv, bi, bp, vb, rb, isfinite(vb) ? 0 : 1);
    }
    if (lane == 0) {
        s_v[warp] = bv;
        s_i[warp] = bi;
        s_p[warp] = bp;
    }
    if (!parts) return;   // plain one-token linear: logits only
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int wv = 1; wv < kHeadWarps; ++wv) head_merge(bv, bi, bp, s_v[wv], s_i[wv], s_p[wv]);
        float *mine = parts + (size_t)blockIdx.x * 3;
        mine[0] = bv;
        mine[1] = __int_as_float(bi);
        mine[2] = __int_as_float(bp);
        __threadfence();
        s_last = atomicAdd(count, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    bv = -INFINITY;
    bi = -1;
    bp = 0;
    for (int c = threadIdx.x; c < (int)gridDim.x; c += blockDim.x) {
        const float *pc = parts + (size_t)c * 3;
        head_merge(bv, bi, bp, __ldcg(pc), __float_as_int(__ldcg(pc + 1)), __float_as_int(__ldcg(pc + 2)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        head_merge(bv, bi, bp, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o),
                   __shfl_xor_sync(0xffffffffu, bp, o));
    __syncthreads();
    if (lane == 0) {
        s_v[warp] = bv;
        s_i[warp] = bi;
        s_p[warp] = bp;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int wv = 1; wv < kHeadWarps; ++wv) head_merge(bv, bi, bp, s_v[wv], s_i[wv], s_p[wv]);
        if (cand) {
            cand[0] = bv;
            cand[1] = bi < 0 ? -1.0f : (float)(bi + row0);
            cand[2] = (bp || bi < 0) ? 1.0f : 0.0f;
        } else {
            *sampled = (bp || bi < 0) ? __int_as_float(0x7fc00000) : (float)bi;
            if (pos) *pos += 1;
        }
        *count = 0u;
    }
}

// ---------------------------------------------------------------------
// Gathers
// ---------------------------------------------------------------------
__global__ void packed_gather_kernel(float *out, const uint8_t *codes, const float *scales,
                                     uint64_t rows, uint64_t k, int format, const float *ids_f32,
                                     const uint32_t *ids_u32, uint64_t n_ids) {
    pdl_wait();
    pdl_trigger();
    const uint64_t total = n_ids * k;
    const uint64_t groups = k / 128;
    const uint64_t cw = format == MF_TERNARY ? k / 4 : format == MF_NF4 ? k / 2 : k;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t i = e / k, j = e - i * k;
        long long id = ids_f32 ? resolve_id(ids_f32[i], rows) : (long long)ids_u32[i];
        if (id < 0) {
            out[e] = __int_as_float(0x7fc00000);
            continue;
        }
        const uint8_t *c = codes + (uint64_t)id * cw;
        const uint64_t g = j / 128, w = j % 128;
        float level;
        if (format == MF_TERNARY) {
            const unsigned code = (c[g * 32 + w / 4] >> (2 * (w % 4))) & 3u;
            level = (float)code - 1.0f;
        } else if (format == MF_INT8) {
            level = (float)(int8_t)c[j];
        } else {
            const uint8_t b = c[g * 64 + w / 2];
            level = kLevels[(w & 1) ? (b >> 4) : (b & 15)];
        }
        out[e] = __fmul_rn(level, scales[(uint64_t)id * groups + g]);
    }
}

__global__ void gather_rows_kernel(float *out, const float *table, uint64_t rows, uint64_t cols,
                                   const float *ids_f32, const uint32_t *ids_u32, uint64_t n_ids) {
    pdl_wait();
    pdl_trigger();
    const uint64_t total = n_ids * cols;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t i = e / cols, j = e - i * cols;
        long long id = ids_f32 ? resolve_id(ids_f32[i], rows) : (long long)ids_u32[i];
        out[e] = id < 0 ? __int_as_float(0x7fc00000) : table[(uint64_t)id * cols + j];
    }
}

__global__ void gather_columns_kernel(float *out, const float *in, uint64_t rows, uint64_t width,
                                      const uint32_t *columns, uint64_t n_columns) {
    pdl_wait();
    pdl_trigger();
    const uint64_t total = rows * n_columns;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = e / n_columns, c = e - r * n_columns;
        out[e] = in[r * width + columns[c]];
    }
}

// ---------------------------------------------------------------------
// Argmax: first strict maximum; NaN if any (allowed) element is non-finite
// or no element is allowed (crates/backend-cpu/src/dense.rs:369-473).
// ---------------------------------------------------------------------
struct ArgBest {
    float v;
    unsigned idx;
    int poisoned;
};

__device__ __forceinline__ ArgBest arg_merge(ArgBest a, ArgBest b) {
    ArgBest r;
    r.poisoned = a.poisoned | b.poisoned;
    if (b.idx != 0xffffffffu && (a.idx == 0xffffffffu || b.v > a.v || (b.v == a.v && b.idx < a.idx))) {
        r.v = b.v;
        r.idx = b.idx;
    } else {
        r.v = a.v;
        r.idx = a.idx;
    }
    return r;
}

__global__ void __launch_bounds__(1024) argmax_kernel(float *out, const float *logits,
                                                      uint64_t width, const uint64_t *mask) {
    pdl_wait();
    pdl_trigger();
    const float *row = logits + blockIdx.x * width;
    ArgBest best{-INFINITY, 0xffffffffu, 0};
    for (uint64_t i = threadIdx.x; i < width; i += blockDim.x) {
        if (mask && !((mask[i >> 6] >> (i & 63)) & 1ull)) continue;
        const float v = row[i];
        if (!isfinite(v)) {
            best.poisoned = 1;
        } else if (best.idx == 0xffffffffu || v > best.v) {
            best.v = v;
            best.idx = (unsigned)i;
        }
    }
    // warp then block reduction
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgBest other;
        other.v = __shfl_xor_sync(0xffffffffu, best.v, o);
        other.idx = __shfl_xor_sync(0xffffffffu, best.idx, o);
        other.poisoned = __shfl_xor_sync(0xffffffffu, best.poisoned, o);
        best = arg_merge(best, other);
    }
    __shared__ ArgBest part[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) part[warp] = best;
    __syncthreads();
    if (warp == 0) {
        const int nw = (blockDim.x + 31) / 32;
        best = lane < nw ? part[lane] : ArgBest{-INFINITY, 0xffffffffu, 0};
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            ArgBest other;
            other.v = __shfl_xor_sync(0xffffffffu, best.v, o);
            other.idx = __shfl_xor_sync(0xffffffffu, best.idx, o);
            other.poisoned = __shfl_xor_sync(0xffffffffu, best.poisoned, o);
            best = arg_merge(best, other);
        }
        if (lane == 0)
            out[blockIdx.x] = (best.poisoned || best.idx == 0xffffffffu) ? __int_as_float(0x7fc00000)
                                                                         : (float)best.idx;
    }
}

// Multi-CTA argmax: each CTA reduces 4096 elements of a row (16 coalesced
// loads per thread, all in flight) to its first strict maximum; with several
// CTAs per row each writes its (value, index, poisoned) triple and the last
// CTA to arrive (atomic counter) merges the triples in block order, writes
// the row's result and resets the counter.
constexpr int kArgThreads = 256;
constexpr int kArgPerThread = 16;
constexpr int kArgSpan = kArgThreads * kArgPerThread;

__device__ __forceinline__ ArgBest block_arg_reduce(ArgBest best) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgBest other;
        other.v = __shfl_xor_sync(0xffffffffu, best.v, o);
        other.idx = __shfl_xor_sync(0xffffffffu, best.idx, o);
        other.poisoned = __shfl_xor_sync(0xffffffffu, best.poisoned, o);
        best = arg_merge(best, other);
    }
    __shared__ ArgBest part[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) part[warp] = best;
    __syncthreads();
    if (warp == 0) {
        const int nw = (blockDim.x + 31) / 32;
        best = lane < nw ? part[lane] : ArgBest{-INFINITY, 0xffffffffu, 0};
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            ArgBest other;
            other.v = __shfl_xor_sync(0xffffffffu, best.v, o);
            other.idx = __shfl_xor_sync(0xffffffffu, best.idx, o);
            other.poisoned = __shfl_xor_sync(0xffffffffu, best.poisoned, o);
            best = arg_merge(best, other);
        }
    }
    return best;  // valid in thread 0
}

__global__ void __launch_bounds__(kArgThreads) argmax_split_kernel(float *out, const float *logits, uint64_t width,
                                                                   const uint64_t *mask, int nblk, float *parts,
                                                                   unsigned *counters) {
    pdl_wait();
    pdl_trigger();
    const uint64_t row = blockIdx.y;
    const int blk = blockIdx.x, tid = threadIdx.x;
    const float *rp = logits + row * width;
    const uint64_t base = (uint64_t)blk * kArgSpan;
    float v[kArgPerThread];
#pragma unroll
    for (int u = 0; u < kArgPerThread; ++u) {
        const uint64_t i = base + (uint64_t)u * kArgThreads + tid;
        v[u] = i < width ? rp[i] : 0.0f;
    }
    ArgBest best{-INFINITY, 0xffffffffu, 0};
#pragma unroll
    for (int u = 0; u < kArgPerThread; ++u) {
        const uint64_t i = base + (uint64_t)u * kArgThreads + tid;
        if (i >= width) continue;
        if (mask && !((mask[i >> 6] >> (i & 63)) & 1ull)) continue;
        if (!isfinite(v[u])) best.poisoned = 1;
        else if (best.idx == 0xffffffffu || v[u] > best.v) {
            best.v = v[u];
            best.idx = (unsigned)i;
        }
    }
    best = block_arg_reduce(best);
    if (tid != 0) return;
    auto result = [](const ArgBest &b) {
        return (b.poisoned || b.idx == 0xffffffffu) ? __int_as_float(0x7fc00000) : (float)b.idx;
    };
    if (nblk == 1) {
        out[row] = result(best);
        return;
    }
    float *mine = parts + (row * nblk + blk) * 3;
    mine[0] = best.v;
    mine[1] = __uint_as_float(best.idx);
    mine[2] = __int_as_float(best.poisoned);
    __threadfence();
    if (atomicAdd(&counters[row], 1u) != (unsigned)(nblk - 1)) return;
    __threadfence();
    ArgBest acc{-INFINITY, 0xffffffffu, 0};
    for (int b = 0; b < nblk; ++b) {
        const float *pb = parts + (row * nblk + b) * 3;
        ArgBest o{__ldcg(pb), __float_as_uint(__ldcg(pb + 1)), __float_as_int(__ldcg(pb + 2))};
        acc = arg_merge(acc, o);
    }
    out[row] = result(acc);
    counters[row] = 0u;
}

// ---------------------------------------------------------------------
// Elementwise (dense.rs:153-198, :343-367)
// ---------------------------------------------------------------------
__global__ void elementwise_kernel(int op, float *out, const float *a, const float *b, uint64_t n) {
    pdl_wait();
    pdl_trigger();
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const float x = a[i], y = b[i];
        out[i] = op == 0 ? __fadd_rn(x, y) : op == 1 ? __fmul_rn(x, y) : silu_mul(x, y);
    }
}

// ---------------------------------------------------------------------
// Row RMS norm (normalization_rotary.rs:11-81, :221-235): one CTA per row.
// Each thread loads its VPT float4 slices of the row (and of `b`) up front,
// keeps them in registers for the scaling pass, and the CTA reduces the sum
// of squares through shared memory.  The sum (a + b), the reciprocal and the
// two scaling products are rounded as the reference rounds them.
// ---------------------------------------------------------------------
template <int VPT>
__global__ void __launch_bounds__(256) rms_norm_vec_kernel(float *sum_out, float *out, const float *a,
                                                           const float *b, uint32_t width,
                                                           const float *weight, float eps) {
    pdl_wait();
    pdl_trigger();
    const uint64_t base = blockIdx.x * (uint64_t)width;
    const uint32_t nvec = width >> 2;
    float4 v[VPT];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const uint32_t e = threadIdx.x + i * blockDim.x;
        v[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (e < nvec) {
            v[i] = *reinterpret_cast<const float4 *>(a + base + 4 * (uint64_t)e);
            if (b) {
                const float4 w = *reinterpret_cast<const float4 *>(b + base + 4 * (uint64_t)e);
                v[i].x = __fadd_rn(v[i].x, w.x);
                v[i].y = __fadd_rn(v[i].y, w.y);
                v[i].z = __fadd_rn(v[i].z, w.z);
                v[i].w = __fadd_rn(v[i].w, w.w);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const uint32_t e = threadIdx.x + i * blockDim.x;
        if (e < nvec) {
            if (b) *reinterpret_cast<float4 *>(sum_out + base + 4 * (uint64_t)e) = v[i];
            ss = fmaf(v[i].x, v[i].x, ss);
            ss = fmaf(v[i].y, v[i].y, ss);
            ss = fmaf(v[i].z, v[i].z, ss);
            ss = fmaf(v[i].w, v[i].w, ss);
        }
    }
    ss = warp_sum(ss);
    __shared__ float red[32];
    __shared__ float rec_s;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
        float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) rec_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)width), eps)));
    }
    __syncthreads();
    const float rec = rec_s;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const uint32_t e = threadIdx.x + i * blockDim.x;
        if (e < nvec) {
            const float4 w = *reinterpret_cast<const float4 *>(weight + 4 * (uint64_t)e);
            float4 r;
            r.x = __fmul_rn(__fmul_rn(v[i].x, rec), w.x);
            r.y = __fmul_rn(__fmul_rn(v[i].y, rec), w.y);
            r.z = __fmul_rn(__fmul_rn(v[i].z, rec), w.z);
            r.w = __fmul_rn(__fmul_rn(v[i].w, rec), w.w);
            *reinterpret_cast<float4 *>(out + base + 4 * (uint64_t)e) = r;
        }
    }
}

// General widths (any alignment): strided scalar loop.
__global__ void __launch_bounds__(256) rms_norm_kernel(float *sum_out, float *out, const float *a,
                                                       const float *b, uint64_t width,
                                                       const float *weight, float eps) {
    pdl_wait();
    pdl_trigger();
    const uint64_t base = blockIdx.x * width;
    float ss = 0.0f;
    for (uint64_t i = threadIdx.x; i < width; i += blockDim.x) {
        float v = a[base + i];
        if (b) {
            v = __fadd_rn(v, b[base + i]);
            sum_out[base + i] = v;
        }
        ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    __shared__ float red[32];
    __shared__ float rec_s;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
        float v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
        v = warp_sum(v);
        if (lane == 0)
            rec_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, (float)width), eps)));
    }
    __syncthreads();
    const float rec = rec_s;
    for (uint64_t i = threadIdx.x; i < width; i += blockDim.x) {
        const float v = b ? sum_out[base + i] : a[base + i];
        out[base + i] = __fmul_rn(__fmul_rn(v, rec), weight[i]);
    }
}

// ---------------------------------------------------------------------
// Per-head RMS + split-half RoPE (normalization_rotary.rs:83-219, :246-369).
// One warp per (token, head); head_dim <= 256.
// ---------------------------------------------------------------------
__global__ void head_norm_rope_kernel(float *out, const float *in, uint64_t tokens, uint32_t heads,
                                      uint32_t head_dim, const float *weight, float eps, int rope,
                                      const uint64_t *positions, const uint64_t *pos_base,
                                      float theta, uint64_t seq_tokens) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const uint64_t item = blockIdx.x * (uint64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= tokens * heads) return;
    const uint64_t token = item / heads;
    const float *x = in + item * head_dim;
    float *y = out + item * head_dim;
    float v[8];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t d = lane + 32 * i;
        v[i] = d < head_dim ? x[d] : 0.0f;
        ss = fmaf(v[i], v[i], ss);
    }
    if (weight) {
        ss = warp_sum(ss);
        const float rec =
            __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)head_dim), eps)));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t d = lane + 32 * i;
            if (d < head_dim) v[i] = __fmul_rn(__fmul_rn(v[i], rec), weight[d]);
        }
    }
    if (!rope) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t d = lane + 32 * i;
            if (d < head_dim) y[d] = v[i];
        }
        return;
    }
    // Stage the normed row so each lane can read its rotation partner.
    __shared__ float rowbuf[8][256];
    float *rb = rowbuf[threadIdx.x >> 5];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t d = lane + 32 * i;
        if (d < head_dim) rb[d] = v[i];
    }
    __syncwarp();
    // Batched rows: sequence token / seq_tokens starts at pos_base[sequence].
    const uint64_t position = positions    ? positions[token]
                              : seq_tokens ? pos_base[token / seq_tokens] + token % seq_tokens
                                           : (*pos_base + token);
    const float pos_f = (float)position;
    const uint32_t half = head_dim / 2;
    for (uint32_t c = lane; c < half; c += 32) {
        const double exponent = -2.0 * (double)c / (double)head_dim;
        const float frequency = (float)pow((double)theta, exponent);
        const float angle = __fmul_rn(pos_f, frequency);
        const float sine = (float)sin((double)angle);
        const float cosine = (float)cos((double)angle);
        const float first = rb[c], second = rb[half + c];
        y[c] = __fsub_rn(__fmul_rn(first, cosine), __fmul_rn(second, sine));
        y[half + c] = __fadd_rn(__fmul_rn(second, cosine), __fmul_rn(first, sine));
    }
    if ((head_dim & 1) && lane == 0) y[head_dim - 1] = rb[head_dim - 1];
}

// ---------------------------------------------------------------------
// Causal GQA (attention_convolution.rs:11-216), split over key chunks.
// Pass 1: per (token, q head, key chunk) a warp computes the chunk's running
// max m, sum l = sum exp(s - m), and o = sum exp(s - m) v over its keys
// (online softmax over 32-key blocks; lane j owns key j of a block for the
// scores, lane d owns output dims d, d+32, ... for the weighted sum).
// Pass 2 merges the chunks.  Keys [0, len + t] are visible to token t; the
// new rows are appended to the caches before pass 1.
// ---------------------------------------------------------------------
constexpr int kKeyChunk = 256;
constexpr int kMaxHeadDim = 256;

__global__ void kv_append_kernel(float *key_cache, float *value_cache, const float *k,
                                 const float *v, uint64_t len, const uint64_t *len_dev,
                                 uint64_t tokens, uint64_t kvw) {
    pdl_wait();
    pdl_trigger();
    const uint64_t base = (len_dev ? *len_dev : len) * kvw;
    const uint64_t total = tokens * kvw;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
         i += (uint64_t)gridDim.x * blockDim.x) {
        key_cache[base + i] = k[i];
        value_cache[base + i] = v[i];
    }
}

// Batched append: row t of sequence b goes to row lens[b] + t of cache b
// (caches `stride` floats apart).
__global__ void kv_append_batch_kernel(float *key_cache, float *value_cache, const float *k, const float *v,
                                       const uint64_t *lens, uint64_t seq_tokens, uint64_t kvw, uint64_t stride,
                                       uint64_t seqs) {
    pdl_wait();
    pdl_trigger();
    const uint64_t per_seq = seq_tokens * kvw;
    const uint64_t total = seqs * per_seq;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t b = i / per_seq, r = i - b * per_seq;
        const uint64_t dst = b * stride + lens[b] * kvw + r;
        key_cache[dst] = k[i];
        value_cache[dst] = v[i];
    }
}

__global__ void __launch_bounds__(128) gqa_chunk_kernel(
    float *out, float *partial, const float *q, const float *key_cache, const float *value_cache,
    uint64_t len, const uint64_t *len_dev, uint64_t tokens, uint32_t q_heads, uint32_t kv_heads,
    uint32_t head_dim, int nchunks, int chunk_keys) {
    pdl_wait();
    pdl_trigger();
    __shared__ __align__(16) float qs[4][kMaxHeadDim];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t group = q_heads / kv_heads;
    const uint32_t kvh = blockIdx.y;
    const uint64_t token = blockIdx.z;
    const int chunk = blockIdx.x;
    const uint64_t base_len = len_dev ? *len_dev : len;
    const uint64_t visible = base_len + token + 1;
    const uint64_t key0 = (uint64_t)chunk * chunk_keys;
    const uint64_t key1 = min(visible, key0 + (uint64_t)chunk_keys);
    const uint64_t kvw = (uint64_t)kv_heads * head_dim;
    const uint64_t qw = (uint64_t)q_heads * head_dim;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)head_dim));
    const int dpl = (head_dim + 31) / 32;  // dims per lane

    for (uint32_t gh = warp; gh < group; gh += 4) {
        const uint32_t qh = kvh * group + gh;
        const float *qr = q + token * qw + (uint64_t)qh * head_dim;
        for (uint32_t d = lane; d < head_dim; d += 32) qs[warp][d] = qr[d];
        __syncwarp();
        float m = -INFINITY, l = 0.0f;
        float o[kMaxHeadDim / 32];
#pragma unroll
        for (int i = 0; i < kMaxHeadDim / 32; ++i) o[i] = 0.0f;
        for (uint64_t kb = key0; kb < key1; kb += 32) {
            const uint64_t key = kb + lane;
            float s = -INFINITY;
            if (key < key1) {
                const float *kr = key_cache + key * kvw + (uint64_t)kvh * head_dim;
                float dot = 0.0f;
                if ((head_dim & 3) == 0) {
                    for (uint32_t d = 0; d < head_dim; d += 4) {
                        const float4 kv4 = *reinterpret_cast<const float4 *>(kr + d);
                        const float4 q4 = *reinterpret_cast<const float4 *>(&qs[warp][d]);
                        dot = fmaf(q4.x, kv4.x, dot);
                        dot = fmaf(q4.y, kv4.y, dot);
                        dot = fmaf(q4.z, kv4.z, dot);
                        dot = fmaf(q4.w, kv4.w, dot);
                    }
                } else {
                    for (uint32_t d = 0; d < head_dim; ++d) dot = fmaf(qs[warp][d], kr[d], dot);
                }
                s = __fmul_rn(dot, scale);
            }
            const float bmax = warp_max(s);
            const float m_new = fmaxf(m, bmax);
            const float corr = m == -INFINITY ? 0.0f : expf(m - m_new);
            const float pj = key < key1 ? expf(s - m_new) : 0.0f;
            l = l * corr + warp_sum(pj);
#pragma unroll
            for (int i = 0; i < kMaxHeadDim / 32; ++i) o[i] *= corr;
            const int nk = (int)min((uint64_t)32, key1 - kb);
            for (int j = 0; j < nk; ++j) {
                const float p = __shfl_sync(0xffffffffu, pj, j);
                const float *vr = value_cache + (kb + j) * kvw + (uint64_t)kvh * head_dim;
#pragma unroll
                for (int i = 0; i < kMaxHeadDim / 32; ++i) {
                    const uint32_t d = lane + 32 * i;
                    if (i < dpl && d < head_dim) o[i] = fmaf(p, vr[d], o[i]);
                }
            }
            m = m_new;
        }
        const uint64_t row = token * q_heads + qh;
        if (nchunks == 1) {
            float *dst = out + token * qw + (uint64_t)qh * head_dim;
#pragma unroll
            for (int i = 0; i < kMaxHeadDim / 32; ++i) {
                const uint32_t d = lane + 32 * i;
                if (i < dpl && d < head_dim) dst[d] = o[i] / l;
            }
        } else {
            float *dst = partial + (row * nchunks + chunk) * (uint64_t)(head_dim + 2);
            if (lane == 0) {
                dst[0] = m;
                dst[1] = l;
            }
#pragma unroll
            for (int i = 0; i < kMaxHeadDim / 32; ++i) {
                const uint32_t d = lane + 32 * i;
                if (i < dpl && d < head_dim) dst[2 + d] = o[i];
            }
        }
        __syncwarp();
    }
}

// Many-token causal GQA with head dimension 64 (prefill): one CTA per
// (block of 64 / group tokens, kv head) owns 64 query rows (each token's
// `group` query heads that share the kv head) and walks the key range in
// 64-key tiles staged in shared memory, so every K and V row is read once
// per 64 query rows instead of once per row.  Thread (rg, cg) of 256 owns
// the 4 x 4 score tile rows 4rg.., keys 4cg.. and the 4 x 4 output tile
// rows 4rg.., dims 4cg..; the 16 threads of a row group sit in one
// half-warp and combine the online-softmax max and sum by shuffles.  Scores
// are dot(q, k) * (1 / sqrt(64)) with causal masking (key <= the token's
// position), softmax with expf, output = sum p v / sum p, as in
// crates/backend-cpu/src/attention_convolution.rs:11-187 up to F32 reorder.
constexpr int kPfRows = 64, kPfKeys = 64, kPfDim = 64, kPfPitch = 68;

size_t gqa_prefill_smem_bytes() {
    return (size_t)(3 * kPfDim * 64 + kPfRows * kPfPitch) * sizeof(float);
}

__global__ void __launch_bounds__(256) gqa_prefill_kernel(float *out, const float *q, const float *key_cache,
                                                          const float *value_cache, uint64_t len,
                                                          const uint64_t *len_dev, uint64_t tokens,
                                                          uint32_t q_heads, uint32_t kv_heads,
                                                          uint64_t cache_stride) {
    pdl_wait();
    pdl_trigger();
    // blockIdx.z: sequence of a batch (tokens rows each, caches cache_stride
    // floats apart, its own length).
    {
        const uint64_t b = blockIdx.z;
        const uint64_t qw_ = (uint64_t)q_heads * kPfDim;
        q += b * tokens * qw_;
        out += b * tokens * qw_;
        key_cache += b * cache_stride;
        value_cache += b * cache_stride;
        if (len_dev) len_dev += b;
    }
    extern __shared__ __align__(16) float pf_smem[];
    float *qt = pf_smem;                       // [dim][row]  (Q transposed)
    float *kt = qt + kPfDim * kPfRows;         // [dim][key]  (K transposed)
    float *vs = kt + kPfDim * kPfKeys;         // [key][dim]
    float *ps = vs + kPfKeys * kPfDim;         // [row][key], pitch kPfPitch
    const int tid = threadIdx.x;
    const int rg = tid >> 4, cg = tid & 15;
    const uint32_t group = q_heads / kv_heads;
    const int tpc = kPfRows / (int)group;      // tokens per CTA
    const uint32_t kvh = blockIdx.y;
    const uint64_t tb = (uint64_t)(gridDim.x - 1 - blockIdx.x) * tpc;   // longest blocks first
    const uint64_t base_len = len_dev ? *len_dev : len;
    const uint64_t kvw = (uint64_t)kv_heads * kPfDim, qw = (uint64_t)q_heads * kPfDim;
    const uint64_t t_last = min(tb + tpc, tokens) - 1;   // last valid token of the block
    const uint64_t kend = base_len + t_last + 1;         // keys any row of the block sees
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)kPfDim));

    for (int e = tid; e < kPfRows * (kPfDim / 4); e += 256) {
        const int r = e & (kPfRows - 1), d4 = e / kPfRows;
        const uint64_t t = tb + r / group;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < tokens)
            v = *reinterpret_cast<const float4 *>(q + t * qw + (uint64_t)(kvh * group + r % group) * kPfDim + 4 * d4);
        qt[(4 * d4 + 0) * kPfRows + r] = v.x;
        qt[(4 * d4 + 1) * kPfRows + r] = v.y;
        qt[(4 * d4 + 2) * kPfRows + r] = v.z;
        qt[(4 * d4 + 3) * kPfRows + r] = v.w;
    }
    uint64_t lim[4];   // keys below lim[i] are visible to row 4rg+i
#pragma unroll
    for (int i = 0; i < 4; ++i) lim[i] = base_len + min(tb + (uint64_t)((4 * rg + i) / group), t_last) + 1;
    float m[4], l[4], o[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) o[i][j] = 0.0f;
    }
    for (uint64_t k0 = 0; k0 < kend; k0 += kPfKeys) {
        __syncthreads();   // the previous tile's readers are done
        for (int e = tid; e < kPfKeys * (kPfDim / 4); e += 256) {
            const int key = e & (kPfKeys - 1), d4 = e / kPfKeys;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k0 + key < kend)
                v = *reinterpret_cast<const float4 *>(key_cache + (k0 + key) * kvw + (uint64_t)kvh * kPfDim + 4 * d4);
            kt[(4 * d4 + 0) * kPfKeys + key] = v.x;
            kt[(4 * d4 + 1) * kPfKeys + key] = v.y;
            kt[(4 * d4 + 2) * kPfKeys + key] = v.z;
            kt[(4 * d4 + 3) * kPfKeys + key] = v.w;
        }
        for (int e = tid; e < kPfKeys * (kPfDim / 4); e += 256) {
            const int d4 = e & 15, key = e >> 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k0 + key < kend)
                v = *reinterpret_cast<const float4 *>(value_cache + (k0 + key) * kvw + (uint64_t)kvh * kPfDim + 4 * d4);
            *reinterpret_cast<float4 *>(vs + key * kPfDim + 4 * d4) = v;
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll 8
        for (int d = 0; d < kPfDim; ++d) {
            const float4 a = *reinterpret_cast<const float4 *>(qt + d * kPfRows + 4 * rg);
            const float4 b = *reinterpret_cast<const float4 *>(kt + d * kPfKeys + 4 * cg);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[i][j] = fmaf(av[i], bv[j], s[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float tmax = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint64_t key = k0 + 4 * cg + j;
                s[i][j] = key < lim[i] ? __fmul_rn(s[i][j], scale) : -INFINITY;
                tmax = fmaxf(tmax, s[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float m_new = fmaxf(m[i], tmax);   // finite: key 0 is visible to every row
            const float corr = m[i] == -INFINITY ? 0.0f : expf(m[i] - m_new);
            float p[4], psum = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                p[j] = s[i][j] == -INFINITY ? 0.0f : expf(s[i][j] - m_new);
                psum += p[j];
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
            l[i] = l[i] * corr + psum;
            m[i] = m_new;
#pragma unroll
            for (int j = 0; j < 4; ++j) o[i][j] *= corr;
            *reinterpret_cast<float4 *>(ps + (4 * rg + i) * kPfPitch + 4 * cg) = make_float4(p[0], p[1], p[2], p[3]);
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < kPfKeys; ++k) {
            const float4 vv = *reinterpret_cast<const float4 *>(vs + k * kPfDim + 4 * cg);
            const float vd[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float pk = ps[(4 * rg + i) * kPfPitch + k];
#pragma unroll
                for (int j = 0; j < 4; ++j) o[i][j] = fmaf(pk, vd[j], o[i][j]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = 4 * rg + i;
        const uint64_t t = tb + r / group;
        if (t < tokens) {
            float *dst = out + t * qw + (uint64_t)(kvh * group + r % group) * kPfDim + 4 * cg;
            *reinterpret_cast<float4 *>(dst) = make_float4(o[i][0] / l[i], o[i][1] / l[i], o[i][2] / l[i], o[i][3] / l[i]);
        }
    }
}

// Decode-shaped GQA (few tokens): one CTA per (key chunk of kDecKeys rows,
// kv head, token).  The chunk's K and V rows and the group's query rows are
// staged in shared memory with coalesced loads (rows at or past the cache
// length come straight from this call's new k/v input, so the append needs
// no separate pass; the chunk-0 CTA of each (kv head, token) writes the new
// row into the caches, and no CTA reads the caches at those rows).  After
// one barrier, warp w serves query heads w, w+4, ... of the kv head's group:
// lane j scores keys j and j+32, the warp forms the chunk's max, sum and
// weighted V sum, and writes them as one partial row for the combine pass.
constexpr int kDecKeys = 64;
constexpr int kDecWarps = 4;
constexpr uint32_t kDecMaxGroup = 32;

size_t gqa_decode_smem_bytes(uint32_t group, uint32_t head_dim) {
    return ((size_t)kDecKeys * (head_dim + 1) + (size_t)kDecKeys * head_dim + (size_t)group * head_dim) *
           sizeof(float);
}

__global__ void __launch_bounds__(kDecWarps * 32) gqa_decode_chunk_kernel(
    float *partial, const float *q, const float *k_new, const float *v_new, float *key_cache,
    float *value_cache, uint64_t len, const uint64_t *len_dev, uint32_t q_heads, uint32_t kv_heads,
    uint32_t head_dim, int nchunks) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) float sm_dec[];
    const uint32_t D = head_dim;
    const uint32_t KP = D + 1;  // padded K row: lane-per-key reads hit distinct banks
    const uint32_t group = q_heads / kv_heads;
    float *ks = sm_dec;                     // [kDecKeys][D + 1]
    float *vs = ks + kDecKeys * KP;         // [kDecKeys][D]
    float *qs = vs + kDecKeys * D;          // [group][D]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int chunk = blockIdx.x;
    const uint32_t kvh = blockIdx.y;
    const uint64_t token = blockIdx.z;
    const uint64_t base_len = len_dev ? *len_dev : len;
    const uint64_t visible = base_len + token + 1;
    const uint64_t key0 = (uint64_t)chunk * kDecKeys;
    const uint64_t kvw = (uint64_t)kv_heads * D;
    const uint64_t qw = (uint64_t)q_heads * D;
    const uint64_t col = (uint64_t)kvh * D;
    if (chunk == 0) {
        const uint64_t row = base_len + token;
        for (uint32_t d = tid; d < D; d += blockDim.x) {
            key_cache[row * kvw + col + d] = k_new[token * kvw + col + d];
            value_cache[row * kvw + col + d] = v_new[token * kvw + col + d];
        }
    }
    if (key0 >= visible) {
        // Past the visible rows (whole CTA takes this branch): empty partials.
        for (uint32_t gh = warp; gh < group; gh += kDecWarps) {
            const uint64_t row = token * q_heads + (uint64_t)kvh * group + gh;
            if (lane == 0) {
                float *dst = partial + (row * nchunks + chunk) * (uint64_t)(D + 2);
                dst[0] = -INFINITY;
                dst[1] = 0.0f;
            }
        }
        return;
    }
    const int nkeys = (int)min((uint64_t)kDecKeys, visible - key0);
    const uint32_t vec = (D & 3) == 0 ? 4 : 1;
    const uint32_t per_row = D / vec;
    const uint32_t total = (uint32_t)nkeys * per_row;
    // Stage K and V rows [key0, key0 + nkeys): kStageUnroll independent
    // loads per thread are issued before any is stored.
    constexpr int kStageUnroll = 8;
    for (uint32_t e0 = tid; e0 < total; e0 += kStageUnroll * blockDim.x) {
        float4 kv4[kStageUnroll], vv4[kStageUnroll];
#pragma unroll
        for (int u = 0; u < kStageUnroll; ++u) {
            const uint32_t e = e0 + u * blockDim.x;
            if (e >= total) continue;
            const uint32_t r = e / per_row, c = (e - r * per_row) * vec;
            const uint64_t key = key0 + r;
            const float *kr, *vr;
            if (key < base_len) {
                kr = key_cache + key * kvw + col + c;
                vr = value_cache + key * kvw + col + c;
            } else {
                kr = k_new + (key - base_len) * kvw + col + c;
                vr = v_new + (key - base_len) * kvw + col + c;
            }
            if (vec == 4) {
                kv4[u] = *reinterpret_cast<const float4 *>(kr);
                vv4[u] = *reinterpret_cast<const float4 *>(vr);
            } else {
                kv4[u].x = *kr;
                vv4[u].x = *vr;
            }
        }
#pragma unroll
        for (int u = 0; u < kStageUnroll; ++u) {
            const uint32_t e = e0 + u * blockDim.x;
            if (e >= total) continue;
            const uint32_t r = e / per_row, c = (e - r * per_row) * vec;
            if (vec == 4) {
                float *kd = ks + r * KP + c;
                kd[0] = kv4[u].x;
                kd[1] = kv4[u].y;
                kd[2] = kv4[u].z;
                kd[3] = kv4[u].w;
                *reinterpret_cast<float4 *>(vs + r * D + c) = vv4[u];
            } else {
                ks[r * KP + c] = kv4[u].x;
                vs[r * D + c] = vv4[u].x;
            }
        }
    }
    const float *qg = q + token * qw + (uint64_t)kvh * group * D;
    for (uint32_t e = tid; e < group * D; e += blockDim.x) qs[e] = qg[e];
    __syncthreads();

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
    for (uint32_t gh = warp; gh < group; gh += kDecWarps) {
        const float *qr = qs + gh * D;
        float s0 = -INFINITY, s1 = -INFINITY;
        if (lane < nkeys) {
            float dot = 0.0f;
            const float *kr = ks + lane * KP;
            for (uint32_t d = 0; d < D; ++d) dot = fmaf(qr[d], kr[d], dot);
            s0 = __fmul_rn(dot, scale);
        }
        if (lane + 32 < nkeys) {
            float dot = 0.0f;
            const float *kr = ks + (lane + 32) * KP;
            for (uint32_t d = 0; d < D; ++d) dot = fmaf(qr[d], kr[d], dot);
            s1 = __fmul_rn(dot, scale);
        }
        const float m = warp_max(fmaxf(s0, s1));
        const float p0 = lane < nkeys ? expf(s0 - m) : 0.0f;
        const float p1 = lane + 32 < nkeys ? expf(s1 - m) : 0.0f;
        const float l = warp_sum(p0 + p1);
        float o[kMaxHeadDim / 32];
#pragma unroll
        for (int i = 0; i < kMaxHeadDim / 32; ++i) o[i] = 0.0f;
        for (int j = 0; j < nkeys; ++j) {
            const float pj = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
            const float *vr = vs + j * D;
#pragma unroll
            for (int i = 0; i < kMaxHeadDim / 32; ++i) {
                const uint32_t d = lane + 32 * i;
                if (d < D) o[i] = fmaf(pj, vr[d], o[i]);
            }
        }
        const uint64_t row = token * q_heads + (uint64_t)kvh * group + gh;
        float *dst = partial + (row * nchunks + chunk) * (uint64_t)(D + 2);
        if (lane == 0) {
            dst[0] = m;
            dst[1] = l;
        }
#pragma unroll
        for (int i = 0; i < kMaxHeadDim / 32; ++i) {
            const uint32_t d = lane + 32 * i;
            if (d < D) dst[2 + d] = o[i];
        }
    }
}

// One-token decode attention of the fused step, with the per-head RMSNorm
// and RoPE of the query group and of the new key row folded in
// (normalization_rotary.rs:246-369 with the arithmetic of
// head_norm_rope_kernel, the rotation read from a per-position table built
// by the same formula, so the values are the same), and the chunk merge
// done by the last CTA to finish for each kv head (an arrival counter, left
// at zero).  Grid (chunks, kv heads).  Each CTA first issues the loads of
// its cached K and V rows, then normalizes and rotates its queries (and the
// new key when it appends it, chunk 0, or holds it, the last chunk); the
// last CTA copies every partial of its query group into shared memory with
// independent loads before merging.
constexpr int kFdWarps = 8;
constexpr uint32_t kFdMaxDim = 128;
constexpr int kFdItems = 4;   // (head, dim) items per thread: group * head_dim <= 1024

// K tile (padded rows), V tile, queries, new key, scores/weights
// [group][64], per-head rescale and running (m, l); rounded to 16 bytes.
// Pitch of a staged key row (head_dim % 4 == 0 here).  The two-half CTAs of
// one sequence use head_dim + 4: rows stay 16-byte aligned for the scores'
// 128-bit loads, and a quarter warp's eight rows cover 32 distinct banks.
// The one-half CTAs (many sequences, two CTAs per SM) measured faster with
// head_dim + 1 and scalar loads.
__host__ __device__ inline uint32_t fd_key_pitch(uint32_t head_dim, int halves) {
    return halves == 2 ? head_dim + 4 : head_dim + 1;
}

__host__ __device__ inline uint32_t fd_stage_floats(uint32_t group, uint32_t head_dim, int halves) {
    return (kDecKeys * fd_key_pitch(head_dim, halves) + kDecKeys * head_dim + group * head_dim + head_dim +
            group * kDecKeys + 3 * group + 3) & ~3u;
}

size_t gqa_decode_fused_smem_bytes(uint32_t group, uint32_t head_dim, int nchunks, int halves = 1) {
    // halves == 2: two stage regions, then the halves' combine buffer.
    const size_t stage = (size_t)halves * fd_stage_floats(group, head_dim, halves) +
                         (halves == 2 ? (size_t)group * (head_dim + 2) : 0);
    const size_t merge = (size_t)group * nchunks * (head_dim + 3);
    return std::max(stage, merge) * sizeof(float);
}

// Warp-cooperative RMSNorm (weight w) + split-half RoPE (rot[c] = (sin, cos))
// of one head row x into dst (shared memory).
template <uint32_t DM>
__device__ __forceinline__ void fd_norm_rope_row(const float *x, const float *w, float eps, uint32_t D,
                                                 const float2 *rot, float *dst, int lane) {
    float v[DM / 32];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < (int)(DM / 32); ++i) {
        const uint32_t d = lane + 32 * i;
        v[i] = d < D ? x[d] : 0.0f;
        ss = fmaf(v[i], v[i], ss);
    }
    const uint32_t half = D / 2;
    float2 r[DM / 64];
#pragma unroll
    for (int i = 0; i < (int)(DM / 64); ++i) {
        const uint32_t c = lane + 32 * i;
        r[i] = c < half ? rot[c] : make_float2(0.f, 1.f);
    }
    if (w) {
        ss = warp_sum(ss);
        const float rec = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps)));
#pragma unroll
        for (int i = 0; i < (int)(DM / 32); ++i) {
            const uint32_t d = lane + 32 * i;
            if (d < D) v[i] = __fmul_rn(__fmul_rn(v[i], rec), w[d]);
        }
    }
    // Stage the normed row so each lane can read its rotation partner.
#pragma unroll
    for (int i = 0; i < (int)(DM / 32); ++i) {
        const uint32_t d = lane + 32 * i;
        if (d < D) dst[d] = v[i];
    }
    __syncwarp();
    float a[DM / 64], b[DM / 64];
#pragma unroll
    for (int i = 0; i < (int)(DM / 64); ++i) {
        const uint32_t c = lane + 32 * i;
        if (c < half) {
            a[i] = dst[c];
            b[i] = dst[half + c];
        }
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < (int)(DM / 64); ++i) {
        const uint32_t c = lane + 32 * i;
        if (c < half) {
            dst[c] = __fsub_rn(__fmul_rn(a[i], r[i].y), __fmul_rn(b[i], r[i].x));
            dst[half + c] = __fadd_rn(__fmul_rn(b[i], r[i].y), __fmul_rn(a[i], r[i].x));
        }
    }
    __syncwarp();
}

template <uint32_t DM, int HV>
__global__ void __launch_bounds__(kFdWarps * 32 * HV) gqa_decode_fused_kernel(
    float *out, float *partial, unsigned *counters, const float *q_raw, const float *k_raw, const float *v_new,
    const float *q_w, const float *k_w, float eps, const float2 *rope, float *key_cache, float *value_cache,
    const uint64_t *len_dev, uint32_t q_heads, uint32_t kv_heads, uint32_t D, int nchunks, int chunk_tiles,
    uint64_t cache_stride) {
    // No pdl_wait() yet: the cached K/V rows and the length were written by
    // kernels that completed before the previous kernel could start (a
    // kernel is launched only after its predecessor passed its own wait), so
    // the first tile's loads are issued before the wait; this call's new
    // q/k/v rows (the previous kernel's output) are read after it.
    // blockIdx.z: sequence of a batch (one row each, caches cache_stride
    // floats apart, its own length, counters and partials).
    {
        const uint64_t b = blockIdx.z;
        q_raw += b * q_heads * D;
        out += b * q_heads * D;
        k_raw += b * kv_heads * D;
        v_new += b * kv_heads * D;
        key_cache += b * cache_stride;
        value_cache += b * cache_stride;
        len_dev += b;
        counters += b * kv_heads;
        partial += b * q_heads * (uint64_t)nchunks * (D + 2);
    }
    extern __shared__ __align__(16) float sm_fd[];
    __shared__ unsigned s_last;
    const uint32_t KP = fd_key_pitch(D, HV), group = q_heads / kv_heads, half = D / 2;
    // HV == 2: the two 8-warp halves of the CTA each take one key sub-chunk
    // (their own stage region and barrier) and fold their sums together.
    const int hv = HV == 2 ? (int)(threadIdx.x >> 8) : 0;
    const uint32_t stage_f = fd_stage_floats(group, D, HV);
    auto hsync = [&] {
        if constexpr (HV == 1) __syncthreads();
        else asm volatile("bar.sync %0, %1;" ::"r"(1 + hv), "r"(kFdWarps * 32) : "memory");
    };
    float *ks = sm_fd + (size_t)hv * stage_f;   // [kDecKeys][KP]
    float *vs = ks + kDecKeys * KP;    // [kDecKeys][D]
    float *qs = vs + kDecKeys * D;     // [group][D] normed, rotated queries
    float *kn = qs + group * D;        // [D] normed, rotated new key
    const int tid = threadIdx.x & (kFdWarps * 32 - 1), lane = tid & 31, warp = tid >> 5;
    const int chunk = blockIdx.x;
    const int sub = chunk * HV + hv;   // this half's key sub-chunk
    const uint32_t kvh = blockIdx.y;
    const uint64_t base_len = *len_dev;
    const uint64_t visible = base_len + 1;
    const uint64_t key_begin = (uint64_t)sub * chunk_tiles * kDecKeys;
    const uint64_t key_end = min(visible, key_begin + (uint64_t)chunk_tiles * kDecKeys);
    const uint64_t kvw = (uint64_t)kv_heads * D, col = (uint64_t)kvh * D;
    const uint64_t S = D + 2;   // partial row: m, l, o[D]
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));

    float *sp = kn + D;                 // [group][64] scores, then weights
    float *mrun = sp + group * kDecKeys; // [group] running max
    float *lrun = mrun + group;          // [group] running sum
    float *crr = lrun + group;           // [group] this tile's rescale
    for (uint32_t gh = tid; gh < group; gh += (kFdWarps * 32)) {
        mrun[gh] = -INFINITY;
        lrun[gh] = 0.0f;
    }
    // Weighted V of (head, dim) items tid, tid + 256, ... (group * D <= 256 * kFdItems).
    float o_run[kFdItems];
#pragma unroll
    for (int i = 0; i < kFdItems; ++i) o_run[i] = 0.0f;

    if (key_begin >= visible) {
        pdl_wait();
        pdl_trigger();
    } else {
        // Cached K and V rows of a tile: 16-byte loads into registers (a
        // 64-row tile of head_dim <= 128 is at most 8 + 8 loads per thread),
        // issued one tile ahead so their latency overlaps the current tile's
        // arithmetic; stored to shared memory after the tile barrier.
        const uint32_t per_row = D / 4;
        constexpr int kU = (kDecKeys * DM / 4 + kFdWarps * 32 - 1) / (kFdWarps * 32);
        float4 kv4[kU], vv4[kU];
        auto cached_rows = [&](uint64_t key0) {
            const int nkeys = (int)min((uint64_t)kDecKeys, visible - key0);
            return base_len < key0 + kDecKeys ? nkeys - 1 : nkeys;
        };
        auto load_tile = [&](uint64_t key0) {
            const uint32_t total = (uint32_t)cached_rows(key0) * per_row;
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const uint32_t e = tid + u * (kFdWarps * 32);
                if (e >= total) continue;
                const uint32_t r = e / per_row, c = (e - r * per_row) * 4;
                kv4[u] = *reinterpret_cast<const float4 *>(key_cache + (key0 + r) * kvw + col + c);
                vv4[u] = *reinterpret_cast<const float4 *>(value_cache + (key0 + r) * kvw + col + c);
            }
        };
        auto store_tile = [&](uint64_t key0) {
            const uint32_t total = (uint32_t)cached_rows(key0) * per_row;
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const uint32_t e = tid + u * (kFdWarps * 32);
                if (e >= total) continue;
                const uint32_t r = e / per_row, c = (e - r * per_row) * 4;
                if constexpr (HV == 2) {
                    *reinterpret_cast<float4 *>(ks + r * KP + c) = kv4[u];
                } else {
                    float *kd = ks + r * KP + c;
                    kd[0] = kv4[u].x;
                    kd[1] = kv4[u].y;
                    kd[2] = kv4[u].z;
                    kd[3] = kv4[u].w;
                }
                *reinterpret_cast<float4 *>(vs + r * D + c) = vv4[u];
            }
        };
        load_tile(key_begin);
        pdl_wait();
        pdl_trigger();
        for (uint64_t key0 = key_begin; key0 < key_end; key0 += kDecKeys) {
            const bool first = key0 == key_begin;
            const bool has_new = base_len < key0 + kDecKeys;   // this tile holds the new row
            const int nkeys = (int)min((uint64_t)kDecKeys, visible - key0);
            if (!first) hsync();   // the previous tile's readers are done
            store_tile(key0);
            if (key0 + kDecKeys < key_end) load_tile(key0 + kDecKeys);   // next tile, in flight during this one
            if (first) {
                const float2 *rot = rope + base_len * half;
                const bool need_k = sub == 0 || base_len < key_end;
                const int items = (int)group + (need_k ? 1 : 0);
                for (int it = warp; it < items; it += kFdWarps) {
                    const bool isk = it == (int)group;
                    fd_norm_rope_row<DM>(isk ? k_raw + col : q_raw + (uint64_t)(kvh * group + it) * D, isk ? k_w : q_w,
                                     eps, D, rot, isk ? kn : qs + it * D, lane);
                }
                hsync();
                if (sub == 0) {
                    for (uint32_t d = tid; d < D; d += (kFdWarps * 32)) {
                        key_cache[base_len * kvw + col + d] = kn[d];
                        value_cache[base_len * kvw + col + d] = v_new[col + d];
                    }
                }
            }
            if (has_new) {
                const int r = nkeys - 1;   // the new row, last in this tile
                for (uint32_t d = tid; d < D; d += (kFdWarps * 32)) {
                    ks[r * KP + d] = kn[d];
                    vs[r * D + d] = v_new[col + d];
                }
            }
            // V rows past the tile's keys take weight 0 below; zero them so
            // stale shared memory cannot contribute 0 * NaN.
            for (uint32_t e = tid; e < (uint32_t)(kDecKeys - nkeys) * D; e += (kFdWarps * 32))
                vs[(uint32_t)nkeys * D + e] = 0.0f;
            hsync();
            // Scores: thread per (head, key), four partial dots.
            for (uint32_t idx = tid; idx < group * kDecKeys; idx += (kFdWarps * 32)) {
                const uint32_t gh = idx / kDecKeys, j = idx % kDecKeys;
                float sc = -INFINITY;
                if ((int)j < nkeys) {
                    const float *qr = qs + gh * D, *kr = ks + j * KP;
                    float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
                    // Four partial sums (elements d = 0, 1, 2, 3 mod 4); the
                    // two-half CTAs load q and k 128 bits at a time.
                    if constexpr (HV == 2) {
                        const float4 *q4 = reinterpret_cast<const float4 *>(qr);
                        const float4 *k4 = reinterpret_cast<const float4 *>(kr);
                        for (uint32_t d4 = 0; d4 < D / 4; ++d4) {
                            const float4 a = q4[d4], b = k4[d4];
                            d0 = fmaf(a.x, b.x, d0);
                            d1 = fmaf(a.y, b.y, d1);
                            d2 = fmaf(a.z, b.z, d2);
                            d3 = fmaf(a.w, b.w, d3);
                        }
                    } else {
                        for (uint32_t d = 0; d < D; d += 4) {
                            d0 = fmaf(qr[d], kr[d], d0);
                            d1 = fmaf(qr[d + 1], kr[d + 1], d1);
                            d2 = fmaf(qr[d + 2], kr[d + 2], d2);
                            d3 = fmaf(qr[d + 3], kr[d + 3], d3);
                        }
                    }
                    sc = __fmul_rn((d0 + d1) + (d2 + d3), scale);
                }
                sp[gh * kDecKeys + j] = sc;
            }
            hsync();
            // Online softmax: warp per head over the tile's 64 scores.
            for (uint32_t gh = warp; gh < group; gh += kFdWarps) {
                const float s0 = sp[gh * kDecKeys + lane], s1 = sp[gh * kDecKeys + 32 + lane];
                const float m_old = mrun[gh];
                const float m_new = fmaxf(m_old, warp_max(fmaxf(s0, s1)));   // finite: every tile has a visible key
                const float p0 = s0 == -INFINITY ? 0.0f : expf(s0 - m_new);
                const float p1 = s1 == -INFINITY ? 0.0f : expf(s1 - m_new);
                const float corr = m_old == -INFINITY ? 0.0f : expf(m_old - m_new);
                const float psum = warp_sum(p0 + p1);
                sp[gh * kDecKeys + lane] = p0;
                sp[gh * kDecKeys + 32 + lane] = p1;
                if (lane == 0) {
                    lrun[gh] = lrun[gh] * corr + psum;
                    mrun[gh] = m_new;
                    crr[gh] = corr;
                }
            }
            hsync();
            // Weighted V: thread per (head, dim), four partial sums over keys.
#pragma unroll
            for (int it = 0; it < kFdItems; ++it) {
                const uint32_t idx = tid + it * (kFdWarps * 32);
                if (idx >= group * D) break;
                const uint32_t gh = idx / D, d = idx % D;
                const float *pr = sp + gh * kDecKeys;
                float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
                for (int j = 0; j < kDecKeys; j += 4) {
                    a0 = fmaf(pr[j], vs[j * D + d], a0);
                    a1 = fmaf(pr[j + 1], vs[(j + 1) * D + d], a1);
                    a2 = fmaf(pr[j + 2], vs[(j + 2) * D + d], a2);
                    a3 = fmaf(pr[j + 3], vs[(j + 3) * D + d], a3);
                }
                o_run[it] = fmaf(o_run[it], crr[gh], (a0 + a1) + (a2 + a3));
            }
        }
    }
    hsync();   // running (m, l) of every head are final
    if constexpr (HV == 2) {
        // The second half publishes its running max, sum and weighted V; the
        // first folds them into its own (the rule of the chunk merge) and
        // carries on alone.
        float *cm = sm_fd + 2 * (size_t)stage_f, *cl = cm + group, *co = cl + group;   // [group] [group] [group][D]
        if (hv == 1) {
            for (uint32_t gh = tid; gh < group; gh += kFdWarps * 32) {
                cm[gh] = mrun[gh];
                cl[gh] = lrun[gh];
            }
#pragma unroll
            for (int it = 0; it < kFdItems; ++it) {
                const uint32_t idx = tid + it * (kFdWarps * 32);
                if (idx < group * D) co[idx] = o_run[it];
            }
        }
        __syncthreads();
        if (hv == 1) return;
        auto fold = [&](uint32_t gh, float &w0, float &w1) {
            const float m0 = mrun[gh], m1 = cm[gh], mm = fmaxf(m0, m1);
            w0 = m0 == -INFINITY ? 0.0f : expf(m0 - mm);
            w1 = m1 == -INFINITY ? 0.0f : expf(m1 - mm);
            return mm;
        };
#pragma unroll
        for (int it = 0; it < kFdItems; ++it) {
            const uint32_t idx = tid + it * (kFdWarps * 32);
            if (idx >= group * D) break;
            float w0, w1;
            fold(idx / D, w0, w1);
            o_run[it] = fmaf(o_run[it], w0, co[idx] * w1);
        }
        hsync();   // every item has read mrun
        for (uint32_t gh = tid; gh < group; gh += kFdWarps * 32) {
            float w0, w1;
            const float mm = fold(gh, w0, w1);
            lrun[gh] = fmaf(lrun[gh], w0, cl[gh] * w1);
            mrun[gh] = mm;
        }
        hsync();
    }
    if (nchunks == 1) {
        // One chunk holds every key: the running sums are the output.
#pragma unroll
        for (int it = 0; it < kFdItems; ++it) {
            const uint32_t idx = tid + it * (kFdWarps * 32);
            if (idx >= group * D) break;
            const uint32_t gh = idx / D, d = idx % D;
            out[((uint64_t)kvh * group + gh) * D + d] = o_run[it] / lrun[gh];
        }
        return;
    }
    for (uint32_t gh = tid; gh < group; gh += (kFdWarps * 32)) {
        float *dst = partial + ((uint64_t)(kvh * group + gh) * nchunks + chunk) * S;
        dst[0] = mrun[gh];   // -inf and 0 for a chunk past the visible rows (its o is never read)
        dst[1] = lrun[gh];
    }
#pragma unroll
    for (int it = 0; it < kFdItems; ++it) {
        const uint32_t idx = tid + it * (kFdWarps * 32);
        if (idx >= group * D) break;
        const uint32_t gh = idx / D, d = idx % D;
        if (lrun[gh] > 0.0f) partial[((uint64_t)(kvh * group + gh) * nchunks + chunk) * S + 2 + d] = o_run[it];
    }
    // The last CTA of this kv head merges the chunks of its query group.
    hsync();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(&counters[kvh], 1u) == (unsigned)nchunks - 1u;
    }
    hsync();
    if (!s_last) return;
    __threadfence();
    // The group's partials are contiguous: group x nchunks rows of S floats.
    const float *pg = partial + (uint64_t)kvh * group * nchunks * S;
    const uint32_t nflt = group * (uint32_t)nchunks * (uint32_t)S;
    float *ms = sm_fd;                 // [group * nchunks * S]
    float *ws = ms + nflt;             // [group * nchunks] chunk weights
    {
        // 8-byte pieces (S is even), 16 per thread in flight.
        const float2 *pg2 = reinterpret_cast<const float2 *>(pg);
        float2 *ms2 = reinterpret_cast<float2 *>(ms);
        const uint32_t n2 = nflt / 2;
        constexpr int kM = 16;
        for (uint32_t e0 = tid; e0 < n2; e0 += kM * (kFdWarps * 32)) {
            float2 t[kM];
#pragma unroll
            for (int u = 0; u < kM; ++u) {
                const uint32_t e = e0 + u * (kFdWarps * 32);
                t[u] = e < n2 ? __ldcg(pg2 + e) : make_float2(0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < kM; ++u) {
                const uint32_t e = e0 + u * (kFdWarps * 32);
                if (e < n2) ms2[e] = t[u];
            }
        }
    }
    hsync();
    for (uint32_t gh = warp; gh < group; gh += kFdWarps) {
        const float *pr = ms + (uint64_t)gh * nchunks * S;
        float M = -INFINITY;
        for (int c = lane; c < nchunks; c += 32)
            if (pr[c * S + 1] > 0.0f) M = fmaxf(M, pr[c * S]);
        M = warp_max(M);
        float L = 0.0f;
        for (int c = lane; c < nchunks; c += 32) {
            const float l = pr[c * S + 1];
            const float w = l > 0.0f ? expf(pr[c * S] - M) : 0.0f;
            ws[gh * nchunks + c] = w;
            L += l * w;
        }
        L = warp_sum(L);
        __syncwarp();
        float o[DM / 32];
#pragma unroll
        for (int i = 0; i < (int)(DM / 32); ++i) o[i] = 0.0f;
        for (int c = 0; c < nchunks; ++c) {
            const float w = ws[gh * nchunks + c];
            if (w > 0.0f) {
#pragma unroll
                for (int i = 0; i < (int)(DM / 32); ++i) {
                    const uint32_t d = lane + 32 * i;
                    if (d < D) o[i] = fmaf(pr[c * S + 2 + d], w, o[i]);
                }
            }
        }
        const uint64_t row = (uint64_t)kvh * group + gh;
#pragma unroll
        for (int i = 0; i < (int)(DM / 32); ++i) {
            const uint32_t d = lane + 32 * i;
            if (d < D) out[row * D + d] = o[i] / L;
        }
    }
    if (tid == 0) counters[kvh] = 0;
}

// ---------------------------------------------------------------------
// One-token attention of many sequences at once (batched decode), head_dim
// 64, query group G: one CTA of 4 warps per (kv head, sequence) over all of
// that sequence's keys, no split and no merge across CTAs.  The CTA first
// normalizes and rotates its G query rows and the new key (the fused
// kernel's prologue) and appends the new K/V row to the caches; then warp w
// takes the 32-key tiles w, w + 4, ... : lane j loads key j's 64-float K
// row (16-byte loads, straight into registers) and scores it against the G
// queries (broadcast shared-memory reads), the warp keeps a running max,
// sum and weighted V per query head (online softmax over its tiles), and
// for the weighted V lane d holds dims 2d, 2d + 1 and reads every key's V
// pair with one coalesced 8-byte load per key, the softmax weight coming
// from the key's lane by a shuffle.  Nothing is staged in shared memory, so
// each warp has its whole next tile's K and V (16 KB) in flight at once.
// The four warps' running sums are folded at the end by the chunk-merge
// rule.  Ordering of rounding: scores as four interleaved partial dots
// (d mod 4), then * 1/sqrt(64); the weighted V in key order per tile.
// ---------------------------------------------------------------------
constexpr int kBdWarps = 4;

// A 16-byte shared-memory read that stays inside the loop it is written in
// (the queries are loop-invariant; hoisting them would hold G * 64 floats in
// registers per thread instead of reading them, broadcast, per key tile).
__device__ __forceinline__ float4 lds4_volatile(const float *p) {
    float4 v;
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}

// KVH (kv heads) is a template argument so the cache row stride is a
// compile-time constant: the 32 V loads of a tile and the 16 K loads of a
// row then share one address register each, with immediate offsets.
template <int G, int KVH>
__global__ void __launch_bounds__(kBdWarps * 32, 3) gqa_decode_batch_kernel(
    float *out, const float *q_raw, const float *k_raw, const float *v_new, const float *q_w, const float *k_w,
    float eps, const float2 *rope, float *key_cache, float *value_cache, const uint64_t *len_dev,
    uint64_t cache_stride) {
    constexpr uint32_t D = 64, kv_heads = KVH;
    __shared__ __align__(16) float s_q[G][D];
    __shared__ __align__(16) float s_kn[D];
    __shared__ float s_m[kBdWarps][G], s_l[kBdWarps][G];
    __shared__ __align__(16) float s_o[kBdWarps][G][D];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t kvh = blockIdx.x;
    const uint64_t b = blockIdx.y;
    const uint32_t q_heads = kv_heads * G;
    q_raw += b * q_heads * D;
    out += b * q_heads * D;
    k_raw += b * kv_heads * D;
    v_new += b * kv_heads * D;
    key_cache += b * cache_stride;
    value_cache += b * cache_stride;
    const uint64_t base_len = len_dev[b];
    const uint64_t visible = base_len + 1;
    constexpr uint64_t kvw = (uint64_t)KVH * D;
    const uint64_t col = (uint64_t)kvh * D;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
    pdl_wait();
    pdl_trigger();
    {
        const float2 *rot = rope + base_len * (D / 2);
        for (int it = warp; it <= G; it += kBdWarps) {
            const bool isk = it == G;
            fd_norm_rope_row<D>(isk ? k_raw + col : q_raw + (uint64_t)(kvh * G + it) * D, isk ? k_w : q_w, eps, D, rot,
                                isk ? s_kn : s_q[it], lane);
        }
        __syncthreads();
        for (uint32_t d = tid; d < D; d += kBdWarps * 32) {
            key_cache[base_len * kvw + col + d] = s_kn[d];
            value_cache[base_len * kvw + col + d] = v_new[col + d];
        }
        __syncthreads();   // the new row is in the caches for every warp
    }
    float m_run[G], l_run[G], o0[G], o1[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        m_run[h] = -INFINITY;
        l_run[h] = 0.0f;
        o0[h] = o1[h] = 0.0f;
    }
    // A tile's K row (this lane's key) and V pairs (this lane's two dims of
    // every key) are all requested before any is used: 16 KB per warp in
    // flight.  (Requesting the next tile's K before this tile's weighted V
    // instead measured 3% slower on the 512-sequence step.)
#pragma unroll 1
    for (uint64_t key0 = (uint64_t)warp * 32; key0 < visible; key0 += kBdWarps * 32) {
        const uint64_t j = key0 + lane;
        const bool valid = j < visible;
        const int nk = (int)min((uint64_t)32, visible - key0);
        const float4 *kp = reinterpret_cast<const float4 *>(key_cache + (valid ? j : key0) * kvw + col);
        float4 kr[D / 4];
#pragma unroll
        for (int i = 0; i < (int)(D / 4); ++i) kr[i] = kp[i];
        const float *vp = value_cache + key0 * kvw + col + 2 * lane;
        float2 vr[32];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
            vr[jj] = jj < nk ? *reinterpret_cast<const float2 *>(vp + (uint64_t)jj * kvw) : make_float2(0.f, 0.f);
        float p[G];
#pragma unroll
        for (int h = 0; h < G; ++h) {
            // Four interleaved partial dots (d mod 4).
            float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
            for (int i = 0; i < (int)(D / 4); ++i) {
                const float4 a = lds4_volatile(s_q[h] + 4 * i);
                d0 = fmaf(a.x, kr[i].x, d0);
                d1 = fmaf(a.y, kr[i].y, d1);
                d2 = fmaf(a.z, kr[i].z, d2);
                d3 = fmaf(a.w, kr[i].w, d3);
            }
            const float sc = valid ? __fmul_rn((d0 + d1) + (d2 + d3), scale) : -INFINITY;
            const float m_new = fmaxf(m_run[h], warp_max(sc));   // finite: every tile has a visible key
            const float pj = valid ? expf(sc - m_new) : 0.0f;
            const float corr = m_run[h] == -INFINITY ? 0.0f : expf(m_run[h] - m_new);
            l_run[h] = fmaf(l_run[h], corr, warp_sum(pj));
            m_run[h] = m_new;
            o0[h] *= corr;
            o1[h] *= corr;
            p[h] = pj;
        }
        // Weighted V in key order, the key's weight from its lane.
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float pj = __shfl_sync(0xffffffffu, p[h], jj);
                o0[h] = fmaf(pj, vr[jj].x, o0[h]);
                o1[h] = fmaf(pj, vr[jj].y, o1[h]);
            }
        }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
        if (lane == 0) {
            s_m[warp][h] = m_run[h];
            s_l[warp][h] = l_run[h];
        }
        reinterpret_cast<float2 *>(s_o[warp][h])[lane] = make_float2(o0[h], o1[h]);
    }
    __syncthreads();
    for (uint32_t idx = tid; idx < G * D; idx += kBdWarps * 32) {
        const uint32_t h = idx / D, d = idx % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kBdWarps; ++w) M = fmaxf(M, s_m[w][h]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < kBdWarps; ++w) {
            const float e = s_m[w][h] == -INFINITY ? 0.0f : expf(s_m[w][h] - M);
            L = fmaf(s_l[w][h], e, L);
            O = fmaf(s_o[w][h][d], e, O);
        }
        out[((uint64_t)kvh * G + h) * D + d] = O / L;
    }
}

// RoPE rotation table: table[p * (D / 2) + c] = (sin, cos) of position p,
// pair c, by the formula of head_norm_rope_kernel.
__global__ void rope_table_kernel(float2 *table, uint64_t positions, uint32_t head_dim, float theta) {
    const uint32_t half = head_dim / 2;
    const uint64_t total = positions * half;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t p = e / half;
        const uint32_t c = (uint32_t)(e - p * half);
        const double exponent = -2.0 * (double)c / (double)head_dim;
        const float frequency = (float)pow((double)theta, exponent);
        const float angle = __fmul_rn((float)p, frequency);
        table[e] = make_float2((float)sin((double)angle), (float)cos((double)angle));
    }
}

// Merges the per-chunk partials of one (token, query head) row per CTA:
// warp 0 reduces the chunks' maxima and sums; then every thread owns one
// output dim for a quarter of the chunks (independent loads, unrolled), and
// the quarters are added in a fixed order.
constexpr int kCombineThreads = 256;

__global__ void __launch_bounds__(kCombineThreads) gqa_combine_kernel(float *out, const float *partial,
                                                                      uint64_t rows, uint32_t head_dim,
                                                                      int nchunks) {
    pdl_wait();
    pdl_trigger();
    __shared__ float s_w[1024];
    __shared__ float s_sum[4][kMaxHeadDim];
    __shared__ float s_L, s_M;
    const uint64_t row = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t stride = head_dim + 2;
    const float *pr = partial + row * nchunks * stride;
    const int nc = nchunks;
    if (warp == 0) {
        float M = -INFINITY;
        for (int c = lane; c < nc; c += 32)
            if (pr[c * stride + 1] > 0.0f) M = fmaxf(M, pr[c * stride]);
        M = warp_max(M);
        float L = 0.0f;
        for (int c = lane; c < nc; c += 32) {
            const float l = pr[c * stride + 1];
            const float w = l > 0.0f ? expf(pr[c * stride] - M) : 0.0f;
            if (c < 1024) s_w[c] = w;
            L += l * w;
        }
        L = warp_sum(L);
        if (lane == 0) {
            s_L = L;
            s_M = M;
        }
    }
    __syncthreads();
    const float M = s_M;
    // thread -> (quarter, dim); dims beyond head_dim idle.
    const int quarter = tid / (kCombineThreads / 4), d = tid % (kCombineThreads / 4);
    for (int d0 = d; d0 < (int)head_dim; d0 += kCombineThreads / 4) {
        float acc = 0.0f;
        constexpr int U = 8;
        for (int c0 = quarter; c0 < nc; c0 += 4 * U) {
            float v[U], w[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = c0 + 4 * u;
                w[u] = c >= nc ? 0.0f
                       : c < 1024 ? s_w[c]
                       : (pr[c * stride + 1] > 0.0f ? expf(pr[c * stride] - M) : 0.0f);
                v[u] = (c < nc && w[u] != 0.0f) ? pr[c * stride + 2 + d0] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < U; ++u) acc = fmaf(w[u], v[u], acc);
        }
        s_sum[quarter][d0] = acc;
    }
    __syncthreads();
    for (int d0 = tid; d0 < (int)head_dim; d0 += kCombineThreads)
        out[row * head_dim + d0] = (((s_sum[0][d0] + s_sum[1][d0]) + s_sum[2][d0]) + s_sum[3][d0]) / s_L;
}

// ---------------------------------------------------------------------
// Gated short convolution (attention_convolution.rs:218-340): one thread per
// channel walks the tokens in order with a rolling window; every product and
// sum is rounded as in the reference, so results match it bit-for-bit.
// ---------------------------------------------------------------------
constexpr int kMaxConvWidth = 16;

// One thread per (channel, chunk of kConvChunk tokens): the window of the
// previous width-1 gated inputs u = B * V is recomputed from the projection
// (or read from the rolling history before the first token), so chunks are
// independent.  The chunk-0 thread of a channel is the only reader of its
// history rows and writes the new history (the last width-1 entries of
// [history, u_0 .. u_{T-1}]) after its reads.  Per output the tap sum runs
// in tap order with explicitly rounded products and sums, as in
// crates/backend-cpu/src/attention_convolution.rs:220-340.
constexpr int kConvChunk = 16;
static_assert(kConvChunk >= kMaxConvWidth, "chunk 0 must hold every history reader");

// W > 0: the width is the compile-time constant W (the window stays in
// registers); W == 0: any width up to kMaxConvWidth.
template <int W>
__global__ void gated_conv_kernel(float *out, const float *proj, uint64_t tokens, uint32_t hidden,
                                  const float *kernel, uint32_t width_arg, float *history) {
    pdl_wait();
    pdl_trigger();
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= hidden) return;
    // blockIdx.z: sequence of a batch (tokens rows each, its own history).
    proj += (uint64_t)blockIdx.z * tokens * 3ull * hidden;
    out += (uint64_t)blockIdx.z * tokens * hidden;
    history += (uint64_t)blockIdx.z * ((W > 0 ? (uint32_t)W : width_arg) - 1) * hidden;
    const uint32_t width = W > 0 ? (uint32_t)W : width_arg;
    const uint32_t hist = width - 1;
    const uint64_t pw = 3ull * hidden;
    const int64_t t0 = (int64_t)blockIdx.y * kConvChunk;
    const int64_t t1 = min((int64_t)tokens, t0 + kConvChunk);
    auto u_at = [&](int64_t t) { return __fmul_rn(proj[t * pw + c], proj[t * pw + 2ull * hidden + c]); };
    constexpr int NW = W > 0 ? W : kMaxConvWidth;
    float kw[NW], win[NW], old[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i)
        if (i < (int)width) kw[i] = kernel[(uint64_t)c * width + i];
    if (blockIdx.y == 0) {
#pragma unroll
        for (int i = 0; i < NW - 1; ++i)
            if (i < (int)hist) old[i] = history[(uint64_t)i * hidden + c];
    }
#pragma unroll
    for (int i = 0; i < NW - 1; ++i) {
        if (i < (int)hist) {
            const int64_t pos = t0 - (int64_t)hist + i;
            // pos < 0 only in chunk 0 (t0 = 0): old[hist + pos] = old[i]
            win[i] = pos >= 0 ? u_at(pos) : old[i];
        }
    }
    for (int64_t t = t0; t < t1; ++t) {
        if (W > 0) win[NW - 1] = u_at(t);
        else win[hist] = u_at(t);
        float total = 0.0f;
#pragma unroll
        for (int tap = 0; tap < NW; ++tap)
            if (tap < (int)width) total = __fadd_rn(total, __fmul_rn(kw[tap], win[tap]));
        out[t * hidden + c] = __fmul_rn(total, proj[t * pw + hidden + c]);
#pragma unroll
        for (int i = 0; i < NW - 1; ++i)
            if (i < (int)hist) win[i] = win[i + 1];
    }
    if (blockIdx.y == 0) {
        // New history: the last `hist` entries of [old history, u_0 .. u_{T-1}].
        // Entry i is u at pos = T - hist + i, or old[i + T] when pos < 0.
#pragma unroll
        for (int i = 0; i < NW - 1; ++i) {
            if (i < (int)hist) {
                const int64_t pos = (int64_t)tokens - (int64_t)hist + i;
                float v = 0.0f;
                if (pos >= 0) {
                    v = u_at(pos);
                } else {
#pragma unroll
                    for (int jj = 0; jj < NW - 1; ++jj)
                        if (jj == i + (int)tokens) v = old[jj];
                }
                history[(uint64_t)i * hidden + c] = v;
            }
        }
    }
}

__global__ void copy_rect_kernel(float *dst, uint64_t dst_width, const float *src,
                                 uint64_t src_width, uint64_t src_row, uint64_t src_col,
                                 uint64_t dst_row, uint64_t dst_col, uint64_t rows, uint64_t cols) {
    pdl_wait();
    pdl_trigger();
    const uint64_t total = rows * cols;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = e / cols, c = e - r * cols;
        dst[(dst_row + r) * dst_width + dst_col + c] = src[(src_row + r) * src_width + src_col + c];
    }
}

}  // namespace

// The greedy id of a row-split LM head from its shards' candidates
// (value, global index, poisoned) in rank order, rank r holding rows below
// rank r + 1's: the first strict maximum over ranks keeps the lowest index
// on ties, as one argmax over the whole row would (dense.rs:369-411).
__global__ void head_shard_pick_kernel(const float *cand, int world, float *sampled, uint64_t *pos) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x != 0) return;
    float bv = -INFINITY, bi = -1.0f;
    bool poisoned = false;
    for (int r = 0; r < world; ++r) {
        const float v = cand[3 * r], i = cand[3 * r + 1];
        if (cand[3 * r + 2] != 0.0f) poisoned = true;
        else if (i >= 0.0f && (bi < 0.0f || v > bv)) {
            bv = v;
            bi = i;
        }
    }
    *sampled = (poisoned || bi < 0.0f) ? __int_as_float(0x7fc00000) : bi;
    if (pos) *pos += 1;
}

// ---------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------
int32_t dense_linear(float *out, const float *x, uint64_t t, const float *w, uint64_t n,
                     uint64_t k, cudaStream_t stream) {
    if (t == 0 || n == 0) return MF_OK;
    if (k == 0) {
        MF_CUDA_TRY(cudaMemsetAsync(out, 0, t * n * sizeof(float), stream));
        return MF_OK;
    }
    // One token through a matrix of many waves (an LM head): the streaming
    // head kernel without its argmax epilogue.
    if (t == 1 && n >= (uint64_t)kHeadWarps * 2 * sm_count() && dense_head_argmax_supported(n, k))
        return dense_head_argmax(out, x, w, n, k, nullptr, 0, nullptr, nullptr, nullptr, stream);
    const size_t smem = (size_t)kDenseTT * k * sizeof(float);
    if (smem > 200 * 1024) return fail(MF_UNSUPPORTED, "dense linear inner width too large");
    MF_CUDA_TRY(cudaFuncSetAttribute(dense_linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
    int per_sm = 0;
    MF_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dense_linear_kernel, 256, smem));
    const unsigned grid = (unsigned)std::min<uint64_t>((n + 7) / 8, (uint64_t)std::max(1, per_sm) * sm_count());
    if (int32_t e_ = ::mf::launch(dense_linear_kernel, dim3(grid), dim3(256), smem, stream, "dense_linear_kernel", out, x, (int)t, w, (int)n, (int)k)) return e_;
    return MF_OK;
}

bool dense_head_argmax_supported(uint64_t n, uint64_t k) {
    return n > 0 && n < (1u << 24) && k % 128 == 0 && k >= 128 && k / 128 <= (uint64_t)kHeadMaxK4;
}

size_t dense_head_parts_floats() { return (size_t)2 * sm_count() * 3; }

int32_t dense_head_argmax(float *logits, const float *x, const float *w, uint64_t n, uint64_t k, float *parts,
                          size_t parts_floats, unsigned *count, float *sampled, uint64_t *pos, cudaStream_t stream,
                          float *cand, uint64_t row0) {
    if (!dense_head_argmax_supported(n, k)) return fail(MF_UNSUPPORTED, "dense head width is not a multiple of 128 up to 2048");
    using Kern = void (*)(float *, const float *, const float *, int, float *, unsigned *, float *, uint64_t *, float *,
                          int);
    Kern kern = nullptr;
    switch (k / 128) {
    case 1: kern = dense_head_argmax_kernel<1>; break;
    case 2: kern = dense_head_argmax_kernel<2>; break;
    case 4: kern = dense_head_argmax_kernel<4>; break;
    case 8: kern = dense_head_argmax_kernel<8>; break;
    case 16: kern = dense_head_argmax_kernel<16>; break;
    default: return fail(MF_UNSUPPORTED, "dense head width must be 128, 256, 512, 1024 or 2048");
    }
    // Every CTA resident at once (one wave): as many per SM as fit, at most 2.
    int per_sm = 0;
    MF_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kHeadWarps * 32, 0));
    per_sm = std::max(1, std::min(per_sm, 2));
    const unsigned grid = (unsigned)std::min<uint64_t>((n + kHeadWarps - 1) / kHeadWarps, (uint64_t)per_sm * sm_count());
    if (parts && (parts_floats < (size_t)grid * 3 || !count)) return fail(MF_RESOURCE_LIMIT, "dense head needs argmax partials");
    if (row0 >= (1u << 24)) return fail(MF_UNSUPPORTED, "head shard offset exceeds f32 index range");
    return ::mf::launch(kern, dim3(grid), dim3(kHeadWarps * 32), 0, stream, "dense_head_argmax_kernel", logits, x, w, (int)n,
                        parts, count, sampled, pos, cand, (int)row0);
}

int32_t head_shard_pick(const float *cand, int world, float *sampled, uint64_t *pos, cudaStream_t stream) {
    if (world < 1) return fail(MF_INVALID_ARGUMENT, "head shard count must be positive");
    return ::mf::launch(head_shard_pick_kernel, dim3(1), dim3(32), 0, stream, "head_shard_pick_kernel", cand, world, sampled,
                        pos);
}

int32_t packed_gather_rows(float *out, const uint8_t *codes, const float *scales, uint64_t rows,
                           uint64_t k, int format, const float *ids_f32, const uint32_t *ids_u32,
                           uint64_t n_ids, cudaStream_t stream) {
    if (n_ids == 0 || k == 0) return MF_OK;
    if (int32_t e_ = ::mf::launch(packed_gather_kernel, dim3(blocks_for(n_ids * k, 256)), dim3(256), 0, stream, "packed_gather_kernel", out, codes, scales, rows, k,
                                                                         format, ids_f32, ids_u32, n_ids)) return e_;
    return MF_OK;
}

int32_t gather_rows(float *out, const float *table, uint64_t rows, uint64_t cols,
                    const float *ids_f32, const uint32_t *ids_u32, uint64_t n_ids,
                    cudaStream_t stream) {
    if (n_ids == 0 || cols == 0) return MF_OK;
    if (int32_t e_ = ::mf::launch(gather_rows_kernel, dim3(blocks_for(n_ids * cols, 256)), dim3(256), 0, stream, "gather_rows_kernel", out, table, rows, cols,
                                                                          ids_f32, ids_u32, n_ids)) return e_;
    return MF_OK;
}

int32_t gather_columns(float *out, const float *in, uint64_t rows, uint64_t width,
                       const uint32_t *columns, uint64_t n_columns, cudaStream_t stream) {
    if (rows == 0 || n_columns == 0) return MF_OK;
    if (int32_t e_ = ::mf::launch(gather_columns_kernel, dim3(blocks_for(rows * n_columns, 256)), dim3(256), 0, stream, "gather_columns_kernel", out, in, rows, width,
                                                                                 columns, n_columns)) return e_;
    return MF_OK;
}

size_t argmax_scratch_floats(uint64_t rows, uint64_t width) {
    const uint64_t nblk = (width + kArgSpan - 1) / kArgSpan;
    return nblk > 1 ? (size_t)(rows * nblk * 3) : 0;
}

int32_t argmax(float *out, const float *logits, uint64_t rows, uint64_t width,
               const uint64_t *mask, const SplitScratch *ss, cudaStream_t stream) {
    if (rows == 0) return MF_OK;
    if (rows > 0x7fffffffu) return fail(MF_UNSUPPORTED, "argmax row count exceeds grid limit");
    const uint64_t nblk = (width + kArgSpan - 1) / kArgSpan;
    const bool split_ok = nblk > 1 && rows <= 65535 && ss && ss->partial &&
                          ss->partial_floats >= argmax_scratch_floats(rows, width) && ss->counters &&
                          ss->n_counters >= rows;
    if (nblk <= 1 || split_ok) {
        dim3 grid((unsigned)std::max<uint64_t>(1, nblk), (unsigned)rows);
        if (int32_t e_ = ::mf::launch(argmax_split_kernel, dim3(grid), dim3(kArgThreads), 0, stream, "argmax_split_kernel", out, logits, width, mask, (int)std::max<uint64_t>(1, nblk),
                                                              split_ok ? ss->partial : nullptr,
                                                              split_ok ? ss->counters : nullptr)) return e_;
        return MF_OK;
    }
    if (int32_t e_ = ::mf::launch(argmax_kernel, dim3((unsigned)rows), dim3(1024), 0, stream, "argmax_kernel", out, logits, width, mask)) return e_;
    return MF_OK;
}

int32_t elementwise(int op, float *out, const float *a, const float *b, uint64_t n,
                    cudaStream_t stream) {
    if (n == 0) return MF_OK;
    if (int32_t e_ = ::mf::launch(elementwise_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, stream, "elementwise_kernel", op, out, a, b, n)) return e_;
    return MF_OK;
}

int32_t row_rms_norm(float *sum_out, float *out, const float *a, const float *b, uint64_t rows,
                     uint64_t width, const float *weight, float eps, cudaStream_t stream) {
    if (rows == 0 || width == 0) {
        if (b && rows && width == 0) return MF_OK;
        return MF_OK;
    }
    if (rows > 0x7fffffffu) return fail(MF_UNSUPPORTED, "RMS row count exceeds grid limit");
    const bool aligned = (width & 3) == 0 && !((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                                                 reinterpret_cast<uintptr_t>(sum_out) |
                                                 reinterpret_cast<uintptr_t>(out) |
                                                 reinterpret_cast<uintptr_t>(weight)) & 15u);
    if (aligned && width <= 4u * 256u * 8u) {
        const uint32_t nvec = (uint32_t)(width / 4);
        const unsigned threads = nvec >= 256 ? 256 : nvec >= 128 ? 128 : nvec >= 64 ? 64 : 32;
        const uint32_t vpt = (nvec + threads - 1) / threads;
        auto kernel = vpt <= 1 ? rms_norm_vec_kernel<1> : vpt <= 2 ? rms_norm_vec_kernel<2>
                    : vpt <= 4 ? rms_norm_vec_kernel<4> : rms_norm_vec_kernel<8>;
        if (int32_t e_ = ::mf::launch(kernel, dim3((unsigned)rows), dim3(threads), 0, stream, "rms_norm_vec_kernel", sum_out, out, a, b, (uint32_t)width, weight, eps)) return e_;
        return MF_OK;
    }
    const unsigned threads = width >= 1024 ? 256 : width >= 256 ? 128 : 64;
    if (int32_t e_ = ::mf::launch(rms_norm_kernel, dim3((unsigned)rows), dim3(threads), 0, stream, "rms_norm_kernel", sum_out, out, a, b, width, weight, eps)) return e_;
    return MF_OK;
}

int32_t head_norm_rope(float *out, const float *in, uint64_t tokens, uint32_t heads,
                       uint32_t head_dim, const float *weight, float eps, bool rope,
                       const uint64_t *positions, const uint64_t *pos_base, float theta,
                       cudaStream_t stream) {
    const uint64_t items = tokens * heads;
    if (items == 0) return MF_OK;
    if (head_dim > 256) return fail(MF_UNSUPPORTED, "head dimension above 256 is unsupported");
    if (int32_t e_ = ::mf::launch(head_norm_rope_kernel, dim3(blocks_for(items, 8)), dim3(256), 0, stream, "head_norm_rope_kernel", out, in, tokens, heads, head_dim, weight, eps, rope ? 1 : 0, positions, pos_base, theta, (uint64_t)0)) return e_;
    return MF_OK;
}

int32_t head_norm_rope_batch(float *out, const float *in, uint32_t seqs, uint64_t seq_tokens, uint32_t heads,
                             uint32_t head_dim, const float *weight, float eps, const uint64_t *pos_base, float theta,
                             cudaStream_t stream) {
    const uint64_t tokens = (uint64_t)seqs * seq_tokens;
    const uint64_t items = tokens * heads;
    if (items == 0) return MF_OK;
    if (head_dim > 256) return fail(MF_UNSUPPORTED, "head dimension above 256 is unsupported");
    return ::mf::launch(head_norm_rope_kernel, dim3(blocks_for(items, 8)), dim3(256), 0, stream, "head_norm_rope_kernel",
                        out, in, tokens, heads, head_dim, weight, eps, 1, (const uint64_t *)nullptr, pos_base, theta,
                        seq_tokens);
}

int32_t rope_table(float2 *table, uint64_t positions, uint32_t head_dim, float theta, cudaStream_t stream) {
    if (positions == 0 || head_dim < 2) return MF_OK;
    return ::mf::launch(rope_table_kernel, dim3(blocks_for(positions * (head_dim / 2), 256)), dim3(256), 0, stream,
                        "rope_table_kernel", table, positions, head_dim, theta);
}

bool gqa_decode_fused_supported(uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim, uint64_t capacity) {
    if (!kv_heads || q_heads % kv_heads || !head_dim || head_dim > kFdMaxDim || head_dim % 4) return false;
    if ((q_heads / kv_heads) * head_dim > (uint32_t)(kFdItems * kFdWarps * 32)) return false;
    const int nchunks = (int)((std::max<uint64_t>(1, capacity) + kDecKeys - 1) / kDecKeys);
    return std::max(gqa_decode_fused_smem_bytes(q_heads / kv_heads, head_dim, nchunks),
                    gqa_decode_fused_smem_bytes(q_heads / kv_heads, head_dim, (nchunks + 1) / 2, 2)) <= 200 * 1024;
}

int32_t gqa_decode_fused(float *out, const float *q_raw, const float *k_raw, const float *v_new,
                         const float *q_norm, const float *k_norm, float eps, const float2 *rope, float *key_cache,
                         float *value_cache, uint64_t capacity, const uint64_t *len_dev, uint32_t q_heads,
                         uint32_t kv_heads, uint32_t head_dim, float *scratch, size_t scratch_bytes,
                         unsigned *counters, size_t n_counters, cudaStream_t stream, uint32_t seqs) {
    if (seqs == 0) return MF_OK;
    if (seqs > 65535) return fail(MF_UNSUPPORTED, "attention sequence count exceeds grid limit");
    if (!gqa_decode_fused_supported(q_heads, kv_heads, head_dim, capacity))
        return fail(MF_UNSUPPORTED, "fused decode attention does not take this geometry");
    if (!counters || n_counters < (size_t)kv_heads * seqs)
        return fail(MF_RESOURCE_LIMIT, "fused decode attention needs counters");
    if (!rope) return fail(MF_INVALID_ARGUMENT, "fused decode attention needs the rotation table");
    // Key tiles per CTA: enough CTAs to fill the GPU a few times over, and
    // no more (a batch of sequences supplies the parallelism split keys
    // would; one chunk needs no merge).
    const uint64_t tiles = (std::max<uint64_t>(1, capacity) + kDecKeys - 1) / kDecKeys;
    const uint64_t want = (uint64_t)sm_count() * 12;
    const uint64_t per_seq = std::max<uint64_t>(1, (want + (uint64_t)seqs * kv_heads - 1) / ((uint64_t)seqs * kv_heads));
    const int chunk_tiles = (int)((tiles + std::min(per_seq, tiles) - 1) / std::min(per_seq, tiles));
    const int nchunks = (int)((tiles + chunk_tiles - 1) / chunk_tiles);
    const size_t seq_bytes = causal_gqa_scratch_bytes(1, q_heads, kv_heads, head_dim, capacity);
    const size_t need = seq_bytes > SIZE_MAX / seqs ? SIZE_MAX : (size_t)seqs * seq_bytes;
    if (nchunks > 1 && (!scratch || need > scratch_bytes)) return fail(MF_RESOURCE_LIMIT, "GQA scratch buffer too small");
    const uint32_t group = q_heads / kv_heads;
    // Many sequences, one chunk each: the batched kernel (no staging, no
    // merge), for head_dim 64 with 8 kv heads (every LFM2 preset).
    if (nchunks == 1 && head_dim == 64 && kv_heads == 8 && (group == 1 || group == 2 || group == 4 || group == 8)) {
        auto bk = group == 1 ? gqa_decode_batch_kernel<1, 8> : group == 2 ? gqa_decode_batch_kernel<2, 8>
                : group == 4 ? gqa_decode_batch_kernel<4, 8> : gqa_decode_batch_kernel<8, 8>;
        return ::mf::launch(bk, dim3(kv_heads, seqs), dim3(kBdWarps * 32), 0, stream, "gqa_decode_batch_kernel", out,
                            q_raw, k_raw, v_new, q_norm, k_norm, eps, rope, key_cache, value_cache, len_dev,
                            capacity * kv_heads * (uint64_t)head_dim);
    }
    // One sequence: CTAs of two halves, each half one key sub-chunk, so the
    // grid is half as many CTAs (about one per SM) with half as many partials
    // to merge.
    const int hv = (seqs == 1 && nchunks >= 2) ? 2 : 1;
    const int ctas = (nchunks + hv - 1) / hv;
    const size_t smem = gqa_decode_fused_smem_bytes(group, head_dim, ctas, hv);
    // Head dims up to 64 take the variant with half the prefetch registers.
    auto kernel = head_dim <= 64 ? (hv == 2 ? gqa_decode_fused_kernel<64, 2> : gqa_decode_fused_kernel<64, 1>)
                                 : (hv == 2 ? gqa_decode_fused_kernel<kFdMaxDim, 2> : gqa_decode_fused_kernel<kFdMaxDim, 1>);
    if (smem > 48 * 1024)
        MF_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    return ::mf::launch(kernel, dim3(ctas, kv_heads, seqs), dim3(kFdWarps * 32 * hv), smem, stream,
                        "gqa_decode_fused_kernel", out, scratch, counters, q_raw, k_raw, v_new, q_norm, k_norm, eps,
                        rope, key_cache, value_cache, len_dev, q_heads, kv_heads, head_dim, ctas, chunk_tiles,
                        capacity * kv_heads * (uint64_t)head_dim);
}

int32_t causal_gqa_batch(float *out, const float *q, const float *k, const float *v, float *key_cache,
                         float *value_cache, uint64_t capacity, const uint64_t *lens_dev, uint32_t seqs,
                         uint64_t seq_tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                         cudaStream_t stream) {
    if (seqs == 0 || seq_tokens == 0) return MF_OK;
    const uint32_t group = kv_heads ? q_heads / kv_heads : 0;
    if (head_dim != (uint32_t)kPfDim || !group || q_heads % kv_heads || kPfRows % group)
        return fail(MF_UNSUPPORTED, "batched attention needs head dimension 64 and a query group dividing 64");
    if (seqs > 65535) return fail(MF_UNSUPPORTED, "attention sequence count exceeds grid limit");
    const uint64_t kvw = (uint64_t)kv_heads * head_dim, stride = capacity * kvw;
    if (int32_t e_ = ::mf::launch(kv_append_batch_kernel, dim3(blocks_for((uint64_t)seqs * seq_tokens * kvw, 256)),
                                  dim3(256), 0, stream, "kv_append_batch_kernel", key_cache, value_cache, k, v, lens_dev,
                                  seq_tokens, kvw, stride, (uint64_t)seqs))
        return e_;
    if (seq_tokens >= kAttnTcMinTokens && attention_tc_enabled() && gqa_prefill_tc_fits(q_heads, kv_heads, head_dim))
        return gqa_prefill_tc(out, q, key_cache, value_cache, 0, lens_dev, seq_tokens, q_heads, kv_heads, stride,
                              seqs, stream);
    const size_t smem = gqa_prefill_smem_bytes();
    MF_CUDA_TRY(cudaFuncSetAttribute(gqa_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const uint64_t tpc = kPfRows / group;
    const dim3 grid((unsigned)((seq_tokens + tpc - 1) / tpc), kv_heads, seqs);
    return ::mf::launch(gqa_prefill_kernel, grid, dim3(256), smem, stream, "gqa_prefill_kernel", out, q,
                        (const float *)key_cache, (const float *)value_cache, (uint64_t)0, lens_dev, seq_tokens,
                        q_heads, kv_heads, stride);
}

__global__ void advance_positions_kernel(uint64_t *pos, uint64_t n, uint32_t seqs) {
    pdl_wait();
    pdl_trigger();
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < seqs) pos[i] += n;
}

int32_t advance_positions(uint64_t *pos, uint64_t n, uint32_t seqs, cudaStream_t stream) {
    if (seqs == 0) return MF_OK;
    return ::mf::launch(advance_positions_kernel, dim3((seqs + 255) / 256), dim3(256), 0, stream,
                        "advance_positions_kernel", pos, n, seqs);
}

static int gqa_chunks(uint64_t max_visible, uint64_t rows, int *chunk_keys) {
    // Split keys so that small-token (decode) calls fill the GPU; large-token
    // calls already have tokens x heads parallelism and run one chunk.
    if (rows >= 2048 || max_visible <= (uint64_t)kKeyChunk) {
        *chunk_keys = (int)std::max<uint64_t>(1, max_visible);
        return 1;
    }
    *chunk_keys = kKeyChunk;
    return (int)((max_visible + kKeyChunk - 1) / kKeyChunk);
}

// Token counts up to this use the decode-shaped kernel (64-key chunks).
constexpr uint64_t kDecodeMaxTokens = 16;

// Bytes of split-key partials causal_gqa writes for this call shape, 0 when
// the path it takes needs none (the tiled prefill kernel, or one key chunk).
// SIZE_MAX when the product overflows.
size_t causal_gqa_scratch_bytes(uint64_t tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                                uint64_t max_visible) {
    uint64_t nchunks = 1;
    if (tokens <= kDecodeMaxTokens) {
        nchunks = (std::max<uint64_t>(1, max_visible) + kDecKeys - 1) / kDecKeys;
    } else {
        const uint32_t group = kv_heads ? q_heads / kv_heads : 0;
        if (head_dim == (uint32_t)kPfDim && group && kPfRows % group == 0) return 0;  // gqa_prefill_kernel
        if (tokens >= kAttnTcMinTokens && gqa_prefill_tc_fits(q_heads, kv_heads, head_dim)) return 0;
        int ck = 0;
        nchunks = (uint64_t)gqa_chunks(max_visible, tokens * q_heads, &ck);
        if (nchunks == 1) return 0;
    }
    uint64_t n = 0;
    if (__builtin_mul_overflow(tokens, (uint64_t)q_heads, &n) || __builtin_mul_overflow(n, nchunks, &n) ||
        __builtin_mul_overflow(n, (uint64_t)head_dim + 2, &n) || __builtin_mul_overflow(n, (uint64_t)sizeof(float), &n) ||
        n > (uint64_t)SIZE_MAX)
        return SIZE_MAX;
    return (size_t)n;
}

int32_t causal_gqa(float *out, const float *q, const float *k, const float *v, float *key_cache,
                   float *value_cache, uint64_t capacity, uint64_t cache_len,
                   uint64_t *cache_len_dev, bool advance_len, uint64_t tokens, uint32_t q_heads,
                   uint32_t kv_heads, uint32_t head_dim, float *scratch, size_t scratch_bytes,
                   cudaStream_t stream) {
    (void)advance_len;
    if (tokens == 0) return MF_OK;
    if (head_dim > (uint32_t)kMaxHeadDim) return fail(MF_UNSUPPORTED, "head dimension above 256 is unsupported");
    if (tokens > 65535) return fail(MF_UNSUPPORTED, "GQA token count exceeds grid limit");
    const uint64_t kvw = (uint64_t)kv_heads * head_dim;
    // With a device-resident length the kernels size for the full capacity.
    const uint64_t max_visible = cache_len_dev ? capacity : cache_len + tokens;
    if (max_visible / kDecKeys >= (uint64_t)INT32_MAX) return fail(MF_UNSUPPORTED, "GQA key count exceeds grid limit");
    if (tokens <= kDecodeMaxTokens) {
        const uint32_t group = q_heads / kv_heads;
        const size_t smem = gqa_decode_smem_bytes(group, head_dim);
        if (smem > 200 * 1024) return fail(MF_UNSUPPORTED, "GQA query group too large for the decode kernel");
        const int nchunks = (int)((std::max<uint64_t>(1, max_visible) + kDecKeys - 1) / kDecKeys);
        const size_t need = causal_gqa_scratch_bytes(tokens, q_heads, kv_heads, head_dim, max_visible);
        if (need > scratch_bytes || !scratch) return fail(MF_RESOURCE_LIMIT, "GQA scratch buffer too small");
        MF_CUDA_TRY(cudaFuncSetAttribute(gqa_decode_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
        dim3 grid(nchunks, kv_heads, (unsigned)tokens);
        if (int32_t e_ = ::mf::launch(gqa_decode_chunk_kernel, dim3(grid), dim3(kDecWarps * 32), smem, stream, "gqa_decode_chunk_kernel", scratch, q, k, v, key_cache, value_cache,
                                                                         cache_len, cache_len_dev, q_heads,
                                                                         kv_heads, head_dim, nchunks)) return e_;
        const uint64_t rows = tokens * q_heads;
        if (int32_t e_ = ::mf::launch(gqa_combine_kernel, dim3((unsigned)rows), dim3(kCombineThreads), 0, stream, "gqa_combine_kernel", out, scratch, rows, head_dim, nchunks)) return e_;
        return MF_OK;
    }
    if (int32_t e_ = ::mf::launch(kv_append_kernel, dim3(blocks_for(tokens * kvw, 256)), dim3(256), 0, stream, "kv_append_kernel", key_cache, value_cache, k, v, cache_len, cache_len_dev, tokens, kvw)) return e_;
    const uint32_t group = kv_heads ? q_heads / kv_heads : 0;
    if (tokens >= kAttnTcMinTokens && attention_tc_enabled() && gqa_prefill_tc_fits(q_heads, kv_heads, head_dim))
        return gqa_prefill_tc(out, q, key_cache, value_cache, cache_len, cache_len_dev, tokens, q_heads, kv_heads, 0, 1,
                              stream);
    if (head_dim == (uint32_t)kPfDim && group && kPfRows % group == 0) {
        const size_t smem = gqa_prefill_smem_bytes();
        static std::once_flag once;
        static cudaError_t attr = cudaSuccess;
        std::call_once(once, [&] {
            attr = cudaFuncSetAttribute(gqa_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        });
        MF_CUDA_TRY(attr);
        const uint64_t tpc = kPfRows / group;
        const dim3 grid((unsigned)((tokens + tpc - 1) / tpc), kv_heads);
        return ::mf::launch(gqa_prefill_kernel, grid, dim3(256), smem, stream, "gqa_prefill_kernel", out, q,
                            (const float *)key_cache, (const float *)value_cache, cache_len,
                            (const uint64_t *)cache_len_dev, tokens, q_heads, kv_heads, (uint64_t)0);
    }
    int chunk_keys = 0;
    const int nchunks = gqa_chunks(max_visible, tokens * q_heads, &chunk_keys);
    const size_t need = nchunks > 1 ? (size_t)tokens * q_heads * nchunks * (head_dim + 2) * sizeof(float) : 0;
    if (need > scratch_bytes) return fail(MF_RESOURCE_LIMIT, "GQA scratch buffer too small");
    dim3 grid(nchunks, kv_heads, (unsigned)tokens);
    if (int32_t e_ = ::mf::launch(gqa_chunk_kernel, dim3(grid), dim3(128), 0, stream, "gqa_chunk_kernel", out, scratch, q, key_cache, value_cache, cache_len,
                                               cache_len_dev, tokens, q_heads, kv_heads, head_dim,
                                               nchunks, chunk_keys)) return e_;
    if (nchunks > 1) {
        const uint64_t rows = tokens * q_heads;
        if (int32_t e_ = ::mf::launch(gqa_combine_kernel, dim3((unsigned)rows), dim3(kCombineThreads), 0, stream, "gqa_combine_kernel", out, scratch, rows, head_dim, nchunks)) return e_;
    }
    return MF_OK;
}

int32_t gated_short_conv(float *out, const float *projection, uint64_t tokens, uint32_t hidden,
                         const float *kernel, uint32_t width, float *history, cudaStream_t stream) {
    return gated_short_conv_batch(out, projection, 1, tokens, hidden, kernel, width, history, stream);
}

int32_t gated_short_conv_batch(float *out, const float *projection, uint32_t seqs, uint64_t tokens, uint32_t hidden,
                               const float *kernel, uint32_t width, float *history, cudaStream_t stream) {
    if (seqs == 0) return MF_OK;
    if (seqs > 65535) return fail(MF_UNSUPPORTED, "conv sequence count exceeds grid limit");
    if (hidden == 0) return MF_OK;
    if (width > (uint32_t)kMaxConvWidth) return fail(MF_UNSUPPORTED, "conv width above 16 is unsupported");
    if (width == 0) return fail(MF_INVALID_ARGUMENT, "conv width must be positive");
    if (tokens > 65535ull * kConvChunk) return fail(MF_UNSUPPORTED, "conv token count exceeds grid limit");
    const dim3 grid((hidden + 127) / 128, (unsigned)std::max<uint64_t>(1, (tokens + kConvChunk - 1) / kConvChunk), seqs);
    auto conv = width == 3 ? gated_conv_kernel<3> : gated_conv_kernel<0>;
    if (int32_t e_ = ::mf::launch(conv, grid, dim3(128), 0, stream, "gated_conv_kernel", out, projection,
                                  tokens, hidden, kernel, width, history)) return e_;
    return MF_OK;
}

int32_t copy_rect_2d(float *dst, uint64_t dst_width, const float *src, uint64_t src_width,
                     uint64_t src_row, uint64_t src_col, uint64_t dst_row, uint64_t dst_col,
                     uint64_t rows, uint64_t cols, cudaStream_t stream) {
    if (rows == 0 || cols == 0) return MF_OK;
    if (int32_t e_ = ::mf::launch(copy_rect_kernel, dim3(blocks_for(rows * cols, 256)), dim3(256), 0, stream, "copy_rect_kernel", dst, dst_width, src, src_width, src_row, src_col, dst_row, dst_col, rows, cols)) return e_;
    return MF_OK;
}

}  // namespace mf

// ---------------------------------------------------------------------
// Non-allocating causal GQA (mfk_causal_gqa_noalloc).
//
// Some callers cannot call cudaMalloc: a host whose memory manager has
// already reserved the device's memory into its own pool (where a
// cudaMalloc either fails or escapes that pool's accounting), and a
// latency-bound decode loop that must not make a call that may synchronize
// the whole device while other streams have work in flight.
// For them the split-key partials live in one file-scope device array,
// allocated when the library's module is loaded on a device and held until
// the process exits.  In host code `g_gqa_static_scratch` names a host-side
// stand-in, not device memory: its device address is looked up once per
// device with cudaGetSymbolAddress and that address is what the kernels get.
// With lazy module loading (the CUDA 12 default) that first lookup is also
// what loads the module on the device, and loading it reserves the array:
// a host that cannot allocate later makes its first call while it still
// can (at initialisation).  The address is cached per device ordinal for the
// life of the process, so a cudaDeviceReset (or anything else that destroys
// the device's primary context) ends this entry point's use on that device.
// ---------------------------------------------------------------------
namespace {

constexpr size_t kGqaStaticScratchBytes = size_t(4) << 20;  // 4 MiB
constexpr int kMaxStaticDevices = 64;

__device__ __align__(256) unsigned char g_gqa_static_scratch[kGqaStaticScratchBytes];

std::mutex g_gqa_static_mu;
void *g_gqa_static_addr[kMaxStaticDevices];

// Device address of the static scratch on the current device (looked up on
// the first call per device, with that device current).
int32_t gqa_static_scratch(void **out) {
    int dev = 0;
    MF_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxStaticDevices)
        return mf::fail(MF_UNSUPPORTED, "device ordinal exceeds the static scratch table");
    std::lock_guard<std::mutex> lock(g_gqa_static_mu);
    if (!g_gqa_static_addr[dev]) {
        void *p = nullptr;
        MF_CUDA_TRY(cudaGetSymbolAddress(&p, g_gqa_static_scratch));
        if (!p) return mf::fail(MF_BACKEND_FAILURE, "static GQA scratch has no device address");
        g_gqa_static_addr[dev] = p;
    }
    *out = g_gqa_static_addr[dev];
    return MF_OK;
}

}  // namespace

extern "C" int32_t mfk_causal_gqa_noalloc(float *out, const float *q, const float *k, const float *v,
                                          float *key_cache, float *value_cache, uint64_t capacity,
                                          uint64_t cache_len, uint64_t tokens, uint32_t q_heads,
                                          uint32_t kv_heads, uint32_t head_dim, void *stream) {
    if (!out || !q || !k || !v || !key_cache || !value_cache)
        return mf::fail(MF_INVALID_ARGUMENT, "null device pointer");
    if (kv_heads == 0 || q_heads == 0 || q_heads % kv_heads)
        return mf::fail(MF_INVALID_SHAPE, "query heads must be a nonzero multiple of key/value heads");
    if (head_dim == 0) return mf::fail(MF_INVALID_SHAPE, "head dimension must be nonzero");
    if (key_cache == value_cache) return mf::fail(MF_INVALID_ARGUMENT, "key and value caches must have distinct storage");
    if (cache_len > capacity || tokens > capacity - cache_len)
        return mf::fail(MF_OUT_OF_BOUNDS, "GQA append exceeds cache capacity");
    for (const void *p : {(const void *)out, (const void *)q, (const void *)k, (const void *)v,
                          (const void *)key_cache, (const void *)value_cache})
        if (reinterpret_cast<uintptr_t>(p) & 15u) return mf::fail(MF_INVALID_LAYOUT, "device operands must be 16-byte aligned");
    // The bytes the path causal_gqa takes for this shape will write (0 for
    // the tiled prefill kernel and single-chunk calls; SIZE_MAX on overflow).
    const size_t need = mf::causal_gqa_scratch_bytes(tokens, q_heads, kv_heads, head_dim, cache_len + tokens);
    if (need > kGqaStaticScratchBytes)
        return mf::fail(MF_RESOURCE_LIMIT,
                        "GQA split-key partials exceed the 4 MiB static scratch of the non-allocating entry point");
    void *scratch = nullptr;
    if (need) {
        int32_t st = gqa_static_scratch(&scratch);
        if (st) return st;
    }
    return mf::causal_gqa(out, q, k, v, key_cache, value_cache, capacity, cache_len, nullptr, false, tokens,
                          q_heads, kv_heads, head_dim, static_cast<float *>(scratch), need,
                          static_cast<cudaStream_t>(stream));
}


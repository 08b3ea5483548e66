// Complete-sequence encoder operations (EncoderOps,
// crates/engine-api/src/encoder.rs:80-103; CPU equations in
// crates/backend-cpu/src/encoder.rs).
//
// A packed sequence carries one segment label per token; every nonzero label
// occupies one contiguous run and 0 marks padding.  The host turns the labels
// into per-token key ranges: token t of an active segment sees exactly the
// rows [start[t], end[t]) of its run, and a padding token has start == end
// and gets a zero output row.  Rows outside a token's run are never combined
// into its output, so non-finite values in other segments or in padding do
// not reach it.
//
// bidirectional_gqa: softmax(q k^T / sqrt(D)) v over the token's run, per
// query head, kv head = head / group.  Head dimension 64 with a group
// dividing 64 runs tiled: one CTA owns 64 query rows (the group's heads of
// 64 / group tokens) of one kv head and walks the union of their runs in
// 64-key tiles staged in shared memory, each row masked to its own run.
// Other shapes run one CTA per (token, head).  Scores and sums are F32 in
// a different order than the CPU loop and exp is CUDA's expf, so results
// agree within the reference's GPU tolerance (1e-4 + 1e-4 |x|,
// crates/backend-wgpu/tests/encoder.rs:19-28).
//
// centered_gated_conv: out[t, c] = C[t, c] * sum_tap kernel[c, tap] *
// (B * V)[t + tap - width / 2, c] over taps inside the token's run, with the
// CPU's rounding order (product B * V, product with the tap, sum in tap
// order, product with C, no fused multiply-add), so it is bit-identical.
#include <algorithm>
#include <climits>
#include <vector>

#include "mf_common.cuh"
#include "packed_kernels.h"

namespace mf {
namespace {

constexpr int kMaxHeadDim = 256;

unsigned blocks_for(uint64_t n, unsigned threads) { return (unsigned)((n + threads - 1) / threads); }

constexpr int kEnRows = 64, kEnKeys = 64, kEnDim = 64, kEnPitch = 68;

size_t encoder_gqa64_smem_bytes() {
    return (size_t)(3 * kEnDim * 64 + kEnRows * kEnPitch) * sizeof(float);
}

__global__ void __launch_bounds__(256) encoder_gqa64_kernel(float *out, const float *q, const float *k,
                                                            const float *v, const uint32_t *ranges,
                                                            uint64_t tokens, uint32_t q_heads, uint32_t kv_heads) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) float en_smem[];
    __shared__ uint32_t s_lo[kEnRows], s_hi[kEnRows];
    __shared__ uint32_t s_kb, s_ke;
    float *qt = en_smem;                       // [dim][row]  (Q transposed)
    float *kt = qt + kEnDim * kEnRows;         // [dim][key]  (K transposed)
    float *vs = kt + kEnDim * kEnKeys;         // [key][dim]
    float *ps = vs + kEnKeys * kEnDim;         // [row][key], pitch kEnPitch
    const int tid = threadIdx.x, lane = tid & 31;
    const int rg = tid >> 4, cg = tid & 15;
    const uint32_t group = q_heads / kv_heads;
    const int tpc = kEnRows / (int)group;      // tokens per CTA
    const uint32_t kvh = blockIdx.y;
    const uint64_t tb = (uint64_t)blockIdx.x * tpc;
    const uint64_t kvw = (uint64_t)kv_heads * kEnDim, qw = (uint64_t)q_heads * kEnDim;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)kEnDim));

    if (tid < kEnRows) {
        const uint64_t t = tb + tid / group;
        uint32_t lo = 0, hi = 0;
        if (t < tokens) {
            const uint64_t h64 = ranges[2 * t + 1];
            hi = (uint32_t)(h64 < tokens ? h64 : tokens);
            lo = ranges[2 * t] < hi ? ranges[2 * t] : hi;
        }
        s_lo[tid] = lo;
        s_hi[tid] = hi;
    }
    for (int e = tid; e < kEnRows * (kEnDim / 4); e += 256) {
        const int r = e & (kEnRows - 1), d4 = e / kEnRows;
        const uint64_t t = tb + r / group;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < tokens)
            x = *reinterpret_cast<const float4 *>(q + t * qw + (uint64_t)(kvh * group + r % group) * kEnDim + 4 * d4);
        qt[(4 * d4 + 0) * kEnRows + r] = x.x;
        qt[(4 * d4 + 1) * kEnRows + r] = x.y;
        qt[(4 * d4 + 2) * kEnRows + r] = x.z;
        qt[(4 * d4 + 3) * kEnRows + r] = x.w;
    }
    __syncthreads();
    if (tid < 32) {
        // Key span of the block: the union of its active rows' runs.
        uint32_t kb = UINT_MAX, ke = 0;
        for (int r = lane; r < kEnRows; r += 32)
            if (s_hi[r] > s_lo[r]) {
                kb = min(kb, s_lo[r]);
                ke = max(ke, s_hi[r]);
            }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            kb = min(kb, __shfl_xor_sync(0xffffffffu, kb, off));
            ke = max(ke, __shfl_xor_sync(0xffffffffu, ke, off));
        }
        if (lane == 0) {
            s_kb = kb < ke ? kb : 0;
            s_ke = kb < ke ? ke : 0;
        }
    }
    __syncthreads();
    const uint64_t kb = s_kb, ke = s_ke;
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo[i] = s_lo[4 * rg + i];
        hi[i] = s_hi[4 * rg + i];
    }
    float m[4], l[4], o[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) o[i][j] = 0.0f;
    }
    for (uint64_t k0 = kb; k0 < ke; k0 += kEnKeys) {
        __syncthreads();   // the previous tile's readers are done
        for (int e = tid; e < kEnKeys * (kEnDim / 4); e += 256) {
            const int key = e & (kEnKeys - 1), d4 = e / kEnKeys;
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k0 + key < ke) x = *reinterpret_cast<const float4 *>(k + (k0 + key) * kvw + (uint64_t)kvh * kEnDim + 4 * d4);
            kt[(4 * d4 + 0) * kEnKeys + key] = x.x;
            kt[(4 * d4 + 1) * kEnKeys + key] = x.y;
            kt[(4 * d4 + 2) * kEnKeys + key] = x.z;
            kt[(4 * d4 + 3) * kEnKeys + key] = x.w;
        }
        int dirty = 0;
        for (int e = tid; e < kEnKeys * (kEnDim / 4); e += 256) {
            const int d4 = e & 15, key = e >> 4;
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k0 + key < ke) x = *reinterpret_cast<const float4 *>(v + (k0 + key) * kvw + (uint64_t)kvh * kEnDim + 4 * d4);
            dirty |= !(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w));
            *reinterpret_cast<float4 *>(vs + key * kEnDim + 4 * d4) = x;
        }
        // A tile holding a non-finite value takes the guarded weighted sum
        // below (rows skip keys outside their run instead of adding 0 * inf).
        dirty = __syncthreads_or(dirty);
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll 8
        for (int d = 0; d < kEnDim; ++d) {
            const float4 a = *reinterpret_cast<const float4 *>(qt + d * kEnRows + 4 * rg);
            const float4 b = *reinterpret_cast<const float4 *>(kt + d * kEnKeys + 4 * cg);
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
                s[i][j] = (key >= lo[i] && key < hi[i]) ? __fmul_rn(s[i][j], scale) : -INFINITY;
                tmax = fmaxf(tmax, s[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            // m_new stays -inf while no key of the row's run has been seen.
            const float m_new = fmaxf(m[i], tmax);
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
            *reinterpret_cast<float4 *>(ps + (4 * rg + i) * kEnPitch + 4 * cg) = make_float4(p[0], p[1], p[2], p[3]);
        }
        __syncthreads();
        if (!dirty) {
#pragma unroll 8
            for (int kk = 0; kk < kEnKeys; ++kk) {
                const float4 vv = *reinterpret_cast<const float4 *>(vs + kk * kEnDim + 4 * cg);
                const float vd[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float pk = ps[(4 * rg + i) * kEnPitch + kk];
#pragma unroll
                    for (int j = 0; j < 4; ++j) o[i][j] = fmaf(pk, vd[j], o[i][j]);
                }
            }
        } else {
            for (int kk = 0; kk < kEnKeys; ++kk) {
                const uint64_t key = k0 + kk;
                const float4 vv = *reinterpret_cast<const float4 *>(vs + kk * kEnDim + 4 * cg);
                const float vd[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if (key < lo[i] || key >= hi[i]) continue;
                    const float pk = ps[(4 * rg + i) * kEnPitch + kk];
#pragma unroll
                    for (int j = 0; j < 4; ++j) o[i][j] = fmaf(pk, vd[j], o[i][j]);
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = 4 * rg + i;
        const uint64_t t = tb + r / group;
        if (t < tokens) {
            float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
            if (hi[i] > lo[i]) y = make_float4(o[i][0] / l[i], o[i][1] / l[i], o[i][2] / l[i], o[i][3] / l[i]);
            *reinterpret_cast<float4 *>(out + t * qw + (uint64_t)(kvh * group + r % group) * kEnDim + 4 * cg) = y;
        }
    }
}

// Any head dimension up to kMaxHeadDim and any group: one CTA per (token,
// query head) walks its run in chunks of 128 keys (thread per key score,
// block max and sum, thread per output dimension).
constexpr int kEgThreads = 128;

__device__ __forceinline__ float eg_block_max(float x, float *red) {
    x = warp_max(x);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = x;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int w = 1; w < kEgThreads / 32; ++w) r = fmaxf(r, red[w]);
    return r;
}

__device__ __forceinline__ float eg_block_sum(float x, float *red) {
    x = warp_sum(x);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = x;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int w = 1; w < kEgThreads / 32; ++w) r += red[w];
    return r;
}

__global__ void __launch_bounds__(kEgThreads) encoder_gqa_generic_kernel(float *out, const float *q, const float *k,
                                                                         const float *v, const uint32_t *ranges,
                                                                         uint32_t q_heads, uint32_t kv_heads,
                                                                         uint32_t D) {
    pdl_wait();
    pdl_trigger();
    __shared__ float qs[kMaxHeadDim];
    __shared__ float pw[kEgThreads];
    __shared__ float red[kEgThreads / 32];
    const uint64_t t = blockIdx.x;
    const uint32_t head = blockIdx.y, kvh = head / (q_heads / kv_heads);
    const int tid = threadIdx.x;
    const uint64_t qw = (uint64_t)q_heads * D, kvw = (uint64_t)kv_heads * D;
    float *dst = out + t * qw + (uint64_t)head * D;
    const uint64_t r_hi = ranges[2 * t + 1], r_lo = ranges[2 * t];
    const uint64_t hi = r_hi < gridDim.x ? r_hi : gridDim.x, lo = r_lo < hi ? r_lo : hi;
    if (hi <= lo) {
        for (uint32_t d = tid; d < D; d += kEgThreads) dst[d] = 0.0f;
        return;
    }
    for (uint32_t d = tid; d < D; d += kEgThreads) qs[d] = q[t * qw + (uint64_t)head * D + d];
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
    constexpr int kPer = kMaxHeadDim / kEgThreads;
    float acc[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) acc[i] = 0.0f;
    float m = -INFINITY, l = 0.0f;
    for (uint64_t c0 = lo; c0 < hi; c0 += kEgThreads) {
        const uint64_t key = c0 + tid;
        float s = -INFINITY;
        if (key < hi) {
            const float *kr = k + key * kvw + (uint64_t)kvh * D;
            float dot = 0.0f;
            for (uint32_t d = 0; d < D; ++d) dot = fmaf(qs[d], kr[d], dot);
            s = __fmul_rn(dot, scale);
        }
        const float m_new = fmaxf(m, eg_block_max(s, red));   // finite: the chunk holds a key of the run
        const float p = s == -INFINITY ? 0.0f : expf(s - m_new);
        const float corr = m == -INFINITY ? 0.0f : expf(m - m_new);
        const float psum = eg_block_sum(p, red);
        l = l * corr + psum;
        m = m_new;
        pw[tid] = p;
        __syncthreads();
        const int n = hi - c0 < (uint64_t)kEgThreads ? (int)(hi - c0) : kEgThreads;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const uint32_t d = tid + i * kEgThreads;
            if (d >= D) break;
            float a = acc[i] * corr;
            for (int j = 0; j < n; ++j) a = fmaf(pw[j], v[(c0 + j) * kvw + (uint64_t)kvh * D + d], a);
            acc[i] = a;
        }
        __syncthreads();   // pw is rewritten by the next chunk
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const uint32_t d = tid + i * kEgThreads;
        if (d < D) dst[d] = acc[i] / l;
    }
}

__global__ void centered_conv_kernel(float *out, const float *projection, const float *kernel,
                                     const uint32_t *ranges, uint64_t tokens, uint32_t hidden, uint32_t width) {
    pdl_wait();
    pdl_trigger();
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= tokens * hidden) return;
    const uint64_t t = i / hidden, c = i % hidden, h = hidden;
    const uint64_t r_hi = ranges[2 * t + 1], r_lo = ranges[2 * t];
    const int64_t hi = (int64_t)(r_hi < tokens ? r_hi : tokens), lo = (int64_t)r_lo < hi ? (int64_t)r_lo : hi;
    if (hi <= lo) {
        out[i] = 0.0f;
        return;
    }
    float total = 0.0f;
    for (uint32_t tap = 0; tap < width; ++tap) {
        const int64_t other = (int64_t)t + (int64_t)tap - (int64_t)(width / 2);
        if (other < lo || other >= hi) continue;
        const uint64_t base = (uint64_t)other * 3 * h + c;
        total = __fadd_rn(total, __fmul_rn(kernel[c * width + tap], __fmul_rn(projection[base], projection[base + 2 * h])));
    }
    out[i] = __fmul_rn(projection[t * 3 * h + h + c], total);
}

}  // namespace

int32_t encoder_segment_ranges(const uint32_t *ids, uint64_t tokens, uint32_t *ranges) {
    if (tokens && !ids) return fail(MF_INVALID_ARGUMENT, "null segment labels");
    if (tokens > UINT32_MAX) return fail(MF_UNSUPPORTED, "encoder sequence exceeds 2^32 tokens");
    if (tokens == 0) return MF_OK;
    // crates/engine-api/src/encoder.rs:16-45: a nonzero label may start a
    // run only once.
    std::vector<uint32_t> starts;
    uint64_t run = 0;
    for (uint64_t i = 0; i <= tokens; ++i) {
        if (i == tokens || (i > 0 && ids[i] != ids[i - 1])) {
            const uint32_t label = ids[run];
            for (uint64_t j = run; j < i; ++j) {
                ranges[2 * j] = label ? (uint32_t)run : 0u;
                ranges[2 * j + 1] = label ? (uint32_t)i : 0u;
            }
            if (label) starts.push_back(label);
            run = i;
        }
    }
    std::sort(starts.begin(), starts.end());
    if (std::adjacent_find(starts.begin(), starts.end()) != starts.end())
        return fail(MF_INVALID_ARGUMENT, "encoder segment labels must occupy contiguous runs");
    return MF_OK;
}

int32_t bidirectional_gqa(float *out, const float *q, const float *k, const float *v, const uint32_t *ranges,
                          uint64_t tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                          cudaStream_t stream) {
    if (tokens == 0) return MF_OK;
    if (!kv_heads || !q_heads || q_heads % kv_heads)
        return fail(MF_INVALID_SHAPE, "query heads must be a nonzero multiple of key/value heads");
    if (head_dim == 0) return fail(MF_INVALID_SHAPE, "head dimension must be nonzero");
    if (head_dim > (uint32_t)kMaxHeadDim) return fail(MF_UNSUPPORTED, "head dimension above 256 is unsupported");
    const uint32_t group = q_heads / kv_heads;
    if (head_dim == (uint32_t)kEnDim && kEnRows % group == 0) {
        const uint64_t tpc = kEnRows / group;
        const uint64_t blocks = (tokens + tpc - 1) / tpc;
        if (blocks > INT32_MAX || kv_heads > 65535) return fail(MF_UNSUPPORTED, "encoder attention exceeds grid limits");
        const size_t smem = encoder_gqa64_smem_bytes();
        MF_CUDA_TRY(cudaFuncSetAttribute(encoder_gqa64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        return ::mf::launch(encoder_gqa64_kernel, dim3((unsigned)blocks, kv_heads), dim3(256), smem, stream,
                            "encoder_gqa64_kernel", out, q, k, v, ranges, tokens, q_heads, kv_heads);
    }
    if (tokens > INT32_MAX || q_heads > 65535) return fail(MF_UNSUPPORTED, "encoder attention exceeds grid limits");
    return ::mf::launch(encoder_gqa_generic_kernel, dim3((unsigned)tokens, q_heads), dim3(kEgThreads), 0, stream,
                        "encoder_gqa_generic_kernel", out, q, k, v, ranges, q_heads, kv_heads, head_dim);
}

int32_t centered_gated_conv(float *out, const float *projection, const float *kernel, const uint32_t *ranges,
                            uint64_t tokens, uint32_t hidden, uint32_t width, cudaStream_t stream) {
    if (hidden == 0 || width == 0)
        return fail(MF_INVALID_ARGUMENT, "short convolution hidden width and kernel width must be nonzero");
    const uint64_t n = tokens * hidden;
    if (n == 0) return MF_OK;
    return ::mf::launch(centered_conv_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, stream, "centered_conv_kernel",
                        out, projection, kernel, ranges, tokens, hidden, width);
}

}  // namespace mf

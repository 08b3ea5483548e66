// Packed matmul for many tokens (prefill), CUDA-core path.
//
// out[t, r] = sum_g scale[r, g] * sum_{j in g} w(code[r, j]) * x[t, j]
// (crates/backend-cpu/src/packed.rs:96-170).
//
// CTA tile: 64 tokens x 128 weight rows, one 128-wide K group per step, so
// the group structure of the format is the K loop: each step accumulates an
// unscaled partial per output in registers and promotes it with the row's
// group scale (FP32), exactly the per-group order of the reference row dot.
// Codes are decoded to F32 levels once per tile into shared memory (k-major),
// x is staged k-major; each thread owns a 4 x 8 output block.
#include <algorithm>

#include "mf_common.cuh"
#include "packed_kernels.h"

namespace mf {
namespace {

constexpr int BM = 64;    // tokens per CTA tile
constexpr int BN = 128;   // weight rows per CTA tile (per stream)
constexpr int BK = 128;   // = group
constexpr int kThreads = 256;
constexpr int XP = BM + 4;

__device__ __constant__ float kLevels[16] = {
    -0x1.000000p+0f, -0x1.647362p-1f, -0x1.0cd660p-1f, -0x1.946540p-2f,
    -0x1.23449ap-2f, -0x1.7a6a7ep-3f, -0x1.74f0e2p-4f, 0.0f,
    0x1.45f5fep-4f,  0x1.4995c6p-3f,  0x1.f809bap-3f,  0x1.5a0674p-2f,
    0x1.c34970p-2f,  0x1.200f56p-1f,  0x1.722766p-1f,  0x1.000000p+0f,
};

struct GemmParams {
    const float *x, *gate, *up;
    const uint8_t *codes_a, *codes_b;
    const float *scales_a, *scales_b;
    float *out_a, *out_b;
    int T, N, K;
};

// Decode 64 consecutive weights (half a group) of one row into ws[k][col].
template <int FMT>
__device__ __forceinline__ void decode_half_group(const uint8_t *group_codes, int half, float *ws,
                                                  int col, int wp) {
    if constexpr (FMT == MF_TERNARY) {
        const uint4 v = *reinterpret_cast<const uint4 *>(group_codes + half * 16);
        const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 16; ++j)
                ws[(half * 64 + i * 16 + j) * wp + col] =
                    __int_as_float(0x4B000000 | ((words[i] >> (2 * j)) & 3u)) - 8388609.0f;
    } else if constexpr (FMT == MF_NF4) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const uint4 v = *reinterpret_cast<const uint4 *>(group_codes + half * 32 + q * 16);
            const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    ws[(half * 64 + q * 32 + i * 8 + j) * wp + col] =
                        kLevels[(words[i] >> (4 * j)) & 15u];
        }
    } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 v = *reinterpret_cast<const uint4 *>(group_codes + half * 64 + q * 16);
            const uint32_t words[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u,
                                       v.z ^ 0x80808080u, v.w ^ 0x80808080u};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    ws[(half * 64 + q * 16 + i * 4 + j) * wp + col] =
                        __int_as_float(__byte_perm(words[i], 0x4B000000u, 0x7540 + j)) - 8388736.0f;
        }
    }
}

// MODE: 0 single, 1 pair rows (grid covers 2N rows), 2 swiglu pair.
template <int FMT, int MODE, bool SWI_IN>
__global__ void __launch_bounds__(kThreads) packed_gemm_kernel(const GemmParams p) {
    pdl_wait();
    pdl_trigger();
    constexpr int NSTREAM = MODE == 2 ? 2 : 1;
    constexpr int COLS = BN / NSTREAM;          // weight rows per stream in this tile
    constexpr int WP = BN + 4;                  // ws row pitch
    constexpr int TN = 8 / NSTREAM;             // rows per thread per stream
    extern __shared__ __align__(16) float sm[];
    float *xs = sm;                  // [BK][XP]
    float *ws = sm + BK * XP;        // [BK][WP]

    const int T = p.T, N = p.N, K = p.K;
    const int wpb = FMT == MF_TERNARY ? 4 : FMT == MF_NF4 ? 2 : 1;
    const int row_bytes = K / wpb, gbytes = BK / wpb, groups = K / BK;
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;     // tx: rows, ty: tokens
    const int m0 = blockIdx.y * BM;
    const int vrow0 = blockIdx.x * COLS;        // first (virtual) row of this tile

    float acc[NSTREAM][4][TN];
    float part[NSTREAM][4][TN];
#pragma unroll
    for (int s = 0; s < NSTREAM; ++s)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) acc[s][i][j] = 0.0f;

    for (int g = 0; g < groups; ++g) {
        __syncthreads();
        // x tile: BM tokens x BK k, stored k-major.
        for (int e = tid; e < BM * BK; e += kThreads) {
            const int m = e / BK, k = e % BK;
            float v = 0.0f;
            if (m0 + m < T) {
                const size_t gi = (size_t)(m0 + m) * K + (size_t)g * BK + k;
                if constexpr (SWI_IN) v = silu_mul(p.gate[gi], p.up[gi]);
                else v = p.x[gi];
            }
            xs[k * XP + m] = v;
        }
        // weight tile: each thread decodes half a group of one column.
        {
            const int col = tid >> 1, half = tid & 1;   // col in [0, 128)
            const int s = col / COLS, c = col % COLS;
            int vr = vrow0 + c;
            const uint8_t *codes;
            bool ok;
            if constexpr (MODE == 1) {
                ok = vr < 2 * N;
                const bool second = vr >= N;
                codes = (second ? p.codes_b : p.codes_a) + (size_t)(ok ? (second ? vr - N : vr) : 0) * row_bytes;
            } else {
                ok = vr < N;
                codes = (s == 0 ? p.codes_a : p.codes_b) + (size_t)(ok ? vr : 0) * row_bytes;
            }
            if (ok) {
                decode_half_group<FMT>(codes + (size_t)g * gbytes, half, ws, col, WP);
            } else {
                for (int k = 0; k < 64; ++k) ws[(half * 64 + k) * WP + col] = 0.0f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int s = 0; s < NSTREAM; ++s)
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) part[s][i][j] = 0.0f;
#pragma unroll 4
        for (int k = 0; k < BK; ++k) {
            const float4 xv = *reinterpret_cast<const float4 *>(xs + k * XP + ty * 4);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int s = 0; s < NSTREAM; ++s) {
                float wv[TN];
#pragma unroll
                for (int q = 0; q < TN / 4; ++q) {
                    const float4 w4 = *reinterpret_cast<const float4 *>(
                        ws + k * WP + s * COLS + tx * TN + 4 * q);
                    wv[4 * q] = w4.x;
                    wv[4 * q + 1] = w4.y;
                    wv[4 * q + 2] = w4.z;
                    wv[4 * q + 3] = w4.w;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < TN; ++j) part[s][i][j] = fmaf(xa[i], wv[j], part[s][i][j]);
            }
        }
        // promote with the group scales
#pragma unroll
        for (int s = 0; s < NSTREAM; ++s)
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                int vr = vrow0 + tx * TN + j;
                float sc = 0.0f;
                if constexpr (MODE == 1) {
                    if (vr < 2 * N)
                        sc = vr < N ? p.scales_a[(size_t)vr * groups + g]
                                    : p.scales_b[(size_t)(vr - N) * groups + g];
                } else {
                    if (vr < N) sc = (s == 0 ? p.scales_a : p.scales_b)[(size_t)vr * groups + g];
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[s][i][j] = fmaf(sc, part[s][i][j], acc[s][i][j]);
            }
    }
    // epilogue
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= T) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int vr = vrow0 + tx * TN + j;
            if constexpr (MODE == 2) {
                if (vr < N) p.out_a[(size_t)m * N + vr] = silu_mul(acc[0][i][j], acc[1][i][j]);
            } else if constexpr (MODE == 1) {
                if (vr < N) p.out_a[(size_t)m * N + vr] = acc[0][i][j];
                else if (vr < 2 * N) p.out_b[(size_t)m * N + (vr - N)] = acc[0][i][j];
            } else {
                if (vr < N) p.out_a[(size_t)m * N + vr] = acc[0][i][j];
            }
        }
    }
}

template <int FMT, int MODE, bool SWI_IN>
int32_t launch(const GemmParams &p, cudaStream_t stream) {
    auto kernel = packed_gemm_kernel<FMT, MODE, SWI_IN>;
    const size_t smem = (size_t)(BK * XP + BK * (BN + 4)) * sizeof(float);
    MF_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int cols = MODE == 2 ? BN / 2 : BN;
    const int vrows = MODE == 1 ? 2 * p.N : p.N;
    dim3 grid((vrows + cols - 1) / cols, (p.T + BM - 1) / BM);
    if (int32_t e_ = ::mf::launch(kernel, dim3(grid), dim3(kThreads), smem, stream, "packed_gemm_kernel", p)) return e_;
    return MF_OK;
}

template <int MODE, bool SWI_IN>
int32_t by_format(const GemmParams &p, int format, cudaStream_t stream) {
    switch (format) {
    case MF_TERNARY: return launch<MF_TERNARY, MODE, SWI_IN>(p, stream);
    case MF_NF4: return launch<MF_NF4, MODE, SWI_IN>(p, stream);
    case MF_INT8: return launch<MF_INT8, MODE, SWI_IN>(p, stream);
    default: return fail(MF_INVALID_ARGUMENT, "unknown packed format");
    }
}

}  // namespace

int32_t packed_gemm(int mode, bool swiglu_input, float *out_a, float *out_b, const float *x,
                    const float *gate, const float *up, uint64_t t, const uint8_t *codes_a,
                    const float *scales_a, const uint8_t *codes_b, const float *scales_b,
                    uint64_t n, uint64_t k, int format, cudaStream_t stream) {
    if (t == 0 || n == 0) return MF_OK;
    if (k == 0 || k % kGroup) return fail(MF_INVALID_SHAPE, "packed GEMM inner width must be a positive multiple of 128");
    if (t > (1u << 30) || n > (1u << 29) || k > (1u << 24))
        return fail(MF_UNSUPPORTED, "packed matmul dimension exceeds kernel limits");
    if (t > 65535u * BM) return fail(MF_UNSUPPORTED, "packed GEMM token count exceeds grid limit");
    GemmParams p{x, gate, up, codes_a, codes_b, scales_a, scales_b, out_a, out_b,
                 (int)t, (int)n, (int)k};
    if (mode == 0) return swiglu_input ? by_format<0, true>(p, format, stream)
                                       : by_format<0, false>(p, format, stream);
    if (mode == 1) return by_format<1, false>(p, format, stream);
    return by_format<2, false>(p, format, stream);
}

}  // namespace mf

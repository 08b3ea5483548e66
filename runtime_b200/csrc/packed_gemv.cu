// Packed GEMV / small-T packed matmul for sm_100a (the decode hot path).
//
// out[t, r] = sum_g scale[r, g] * sum_{j in g} w(code[r, j]) * x[t, j]
// (crates/backend-cpu/src/packed.rs:96-170, crates/kernels-simd/src/lib.rs:31-208).
//
// Layout and work split
//   * Each row's code stream (K*bits/8 bytes) is read once, in 16-byte chunks,
//     by a team of LPR consecutive lanes (the largest power of two <=
//     min(32, row_bytes/16)): one 128-bit
//     non-allocating load per lane per row, so a warp-wide load covers
//     contiguous bytes.  A 16-byte chunk always lies inside one 128-weight
//     group (32/64/128 bytes for ternary/NF4/INT8).
//   * x for TT tokens is staged once per CTA in shared memory, in 16-byte-chunk
//     order with 4 floats of padding per chunk, so the 128-bit x reads of the
//     lanes of a team (which sit one chunk apart) hit distinct banks.
//   * Each lane keeps R rows in flight and reuses every x value for all R rows
//     and every decoded weight for all TT tokens.
//   * Decode is in registers: ternary and INT8 build exact F32 integers with
//     the 2^23 magic-number trick (one LOP3/PRMT + one FADD per weight); NF4
//     reads a 256-entry byte -> (level_lo, level_hi) table replicated 16x in
//     shared memory (conflict-free 64-bit reads).
//   * Per lane, the chunk's partial dot is multiplied by its group scale and
//     accumulated; a shuffle reduction across the team finishes each row.
//   * CTAs stride over row blocks (grid sized to resident CTAs), so x and the
//     NF4 table are staged once per CTA.
#include <algorithm>
#include <cstdio>

#include "mf_common.cuh"
#include "packed_kernels.h"

namespace mf {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

enum Mode { kSingle = 0, kPairRows = 1, kSwigluPair = 2 };

template <int FMT>
struct Fmt;
template <>
struct Fmt<MF_TERNARY> {
    static constexpr int WPB = 4, GB = 32;
};
template <>
struct Fmt<MF_NF4> {
    static constexpr int WPB = 2, GB = 64;
};
template <>
struct Fmt<MF_INT8> {
    static constexpr int WPB = 1, GB = 128;
};

struct GemvParams {
    const float *x, *gate, *up;
    const uint8_t *codes_a, *codes_b;
    const float *scales_a, *scales_b;
    float *out_a, *out_b;
    int T, N, K;
    int lpr;  // lanes per row team
};

// NF4 byte table: entry b = (L[b & 15], L[b >> 4]); 16 replicas.
__device__ __constant__ float kNf4Levels[16] = {
    -0x1.000000p+0f, -0x1.647362p-1f, -0x1.0cd660p-1f, -0x1.946540p-2f,
    -0x1.23449ap-2f, -0x1.7a6a7ep-3f, -0x1.74f0e2p-4f, 0.0f,
    0x1.45f5fep-4f,  0x1.4995c6p-3f,  0x1.f809bap-3f,  0x1.5a0674p-2f,
    0x1.c34970p-2f,  0x1.200f56p-1f,  0x1.722766p-1f,  0x1.000000p+0f,
};

constexpr int kNf4LutBytes = 256 * 16 * 8;

// Decode one 32-bit code word into 4*WPB F32 weights (unscaled levels).
template <int FMT>
__device__ __forceinline__ void decode_word(uint32_t w, float *out, const float2 *lut, int lane16) {
    if constexpr (FMT == MF_TERNARY) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            // 2^23 + code, minus (2^23 + 1) = code - 1, exact.
            out[j] = __int_as_float(0x4B000000 | ((w >> (2 * j)) & 3u)) - 8388609.0f;
        }
    } else if constexpr (FMT == MF_INT8) {
        const uint32_t biased = w ^ 0x80808080u;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            // bytes [b_j ^ 0x80, 0, 0, 0x4B] = 2^23 + int8 + 128, exact.
            out[j] = __int_as_float(__byte_perm(biased, 0x4B000000u, 0x7540 + j)) - 8388736.0f;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 v = lut[((w >> (8 * j)) & 0xFFu) * 16 + lane16];
            out[2 * j] = v.x;
            out[2 * j + 1] = v.y;
        }
    }
}

template <int FMT, int R, int TT, int MODE, bool SWI_IN>
__global__ void __launch_bounds__(kThreads) packed_gemv_kernel(const GemvParams p) {
    pdl_wait();
    pdl_trigger();
    constexpr int WPB = Fmt<FMT>::WPB;
    constexpr int GB = Fmt<FMT>::GB;
    constexpr int CW = 16 * WPB;  // weights per 16-byte chunk
    constexpr int CS = CW + 4;    // padded chunk stride in shared memory (floats)
    constexpr int WW = 4 * WPB;   // weights per 32-bit word
    constexpr int NB = (MODE == kSwigluPair) ? 2 : 1;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    float2 *lut = reinterpret_cast<float2 *>(smem_raw);
    float *xs = reinterpret_cast<float *>(smem_raw + (FMT == MF_NF4 ? kNf4LutBytes : 0));

    const int T = p.T, N = p.N, K = p.K;
    const int row_bytes = K / WPB;
    const int groups = K / kGroup;
    const int nchunks = K / CW;
    const int xstride = nchunks * CS;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int lpr = p.lpr, slots = 32 / lpr;
    const int slot = lane / lpr, sl = lane % lpr;
    const int lane16 = lane & 15;

    if constexpr (FMT == MF_NF4) {
        for (int e = tid; e < 256 * 16; e += kThreads) {
            const int b = e >> 4;
            lut[e] = make_float2(kNf4Levels[b & 15], kNf4Levels[b >> 4]);
        }
    }

    const int vrows = (MODE == kPairRows) ? 2 * N : N;
    const int rows_per_block = kWarps * slots * R;

    for (int t0 = 0; t0 < T; t0 += TT) {
        const int tn = min(TT, T - t0);
        __syncthreads();
        // Stage x (or silu(gate) * up) for tokens [t0, t0 + TT); pad tokens with 0.
        for (int e = tid; e < TT * K; e += kThreads) {
            const int t = e / K, k = e - t * K;
            float v = 0.0f;
            if (t < tn) {
                const size_t gi = (size_t)(t0 + t) * K + k;
                if constexpr (SWI_IN) v = silu_mul(p.gate[gi], p.up[gi]);
                else v = p.x[gi];
            }
            xs[t * xstride + (k / CW) * CS + (k % CW)] = v;
        }
        __syncthreads();

        for (int rb = blockIdx.x; rb * rows_per_block < vrows; rb += gridDim.x) {
            const int rbase = rb * rows_per_block + (warp * slots + slot) * R;
            const uint8_t *cptr[NB][R];
            const float *sptr[NB][R];
            bool valid[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                int vr = rbase + r;
                valid[r] = vr < vrows;
                if (!valid[r]) vr = 0;
                if constexpr (MODE == kPairRows) {
                    const bool second = vr >= N;
                    const int row = second ? vr - N : vr;
                    cptr[0][r] = (second ? p.codes_b : p.codes_a) + (size_t)row * row_bytes;
                    sptr[0][r] = (second ? p.scales_b : p.scales_a) + (size_t)row * groups;
                } else {
                    cptr[0][r] = p.codes_a + (size_t)vr * row_bytes;
                    sptr[0][r] = p.scales_a + (size_t)vr * groups;
                    if constexpr (NB == 2) {
                        cptr[1][r] = p.codes_b + (size_t)vr * row_bytes;
                        sptr[1][r] = p.scales_b + (size_t)vr * groups;
                    }
                }
            }
            float acc[NB][R][TT];
#pragma unroll
            for (int b = 0; b < NB; ++b)
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int t = 0; t < TT; ++t) acc[b][r][t] = 0.0f;

            for (int off = sl * 16; off < row_bytes; off += lpr * 16) {
                uint4 c[NB][R];
                float sc[NB][R];
#pragma unroll
                for (int b = 0; b < NB; ++b)
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        c[b][r] = valid[r] ? ld_stream_u4(cptr[b][r] + off) : make_uint4(0, 0, 0, 0);
                        sc[b][r] = valid[r] ? __ldg(sptr[b][r] + off / GB) : 0.0f;
                    }
                const float *xc = xs + (off >> 4) * CS;
                float part[NB][R][TT];
#pragma unroll
                for (int b = 0; b < NB; ++b)
#pragma unroll
                    for (int r = 0; r < R; ++r)
#pragma unroll
                        for (int t = 0; t < TT; ++t) part[b][r][t] = 0.0f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float xv[TT][WW];
#pragma unroll
                    for (int t = 0; t < TT; ++t) {
#pragma unroll
                        for (int q = 0; q < WW / 4; ++q) {
                            const float4 v =
                                *reinterpret_cast<const float4 *>(xc + t * xstride + i * WW + 4 * q);
                            xv[t][4 * q] = v.x;
                            xv[t][4 * q + 1] = v.y;
                            xv[t][4 * q + 2] = v.z;
                            xv[t][4 * q + 3] = v.w;
                        }
                    }
#pragma unroll
                    for (int b = 0; b < NB; ++b)
#pragma unroll
                        for (int r = 0; r < R; ++r) {
                            const uint32_t word = i == 0 ? c[b][r].x : i == 1 ? c[b][r].y
                                                : i == 2 ? c[b][r].z : c[b][r].w;
                            float wv[WW];
                            decode_word<FMT>(word, wv, lut, lane16);
#pragma unroll
                            for (int t = 0; t < TT; ++t)
#pragma unroll
                                for (int j = 0; j < WW; ++j)
                                    part[b][r][t] = fmaf(wv[j], xv[t][j], part[b][r][t]);
                        }
                }
#pragma unroll
                for (int b = 0; b < NB; ++b)
#pragma unroll
                    for (int r = 0; r < R; ++r)
#pragma unroll
                        for (int t = 0; t < TT; ++t)
                            acc[b][r][t] = fmaf(sc[b][r], part[b][r][t], acc[b][r][t]);
            }
            // Team reduction (xor offsets stay inside the aligned lpr-lane team).
#pragma unroll
            for (int b = 0; b < NB; ++b)
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int t = 0; t < TT; ++t) {
                        float v = acc[b][r][t];
                        for (int o = lpr >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                        acc[b][r][t] = v;
                    }
            if (sl == 0) {
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if (!valid[r]) continue;
                    const int vr = rbase + r;
#pragma unroll
                    for (int t = 0; t < TT; ++t) {
                        if (t >= tn) continue;
                        const size_t tok = (size_t)(t0 + t);
                        if constexpr (MODE == kSwigluPair) {
                            p.out_a[tok * N + vr] = silu_mul(acc[0][r][t], acc[1][r][t]);
                        } else if constexpr (MODE == kPairRows) {
                            if (vr < N) p.out_a[tok * N + vr] = acc[0][r][t];
                            else p.out_b[tok * N + (vr - N)] = acc[0][r][t];
                        } else {
                            p.out_a[tok * N + vr] = acc[0][r][t];
                        }
                    }
                }
            }
        }
    }
}

template <int FMT>
size_t x_smem_bytes(int K, int TT) {
    constexpr int CW = 16 * Fmt<FMT>::WPB;
    return (size_t)TT * (K / CW) * (CW + 4) * sizeof(float);
}

template <int FMT, int R, int TT, int MODE, bool SWI_IN>
int32_t launch_cfg(const GemvParams &p, cudaStream_t stream) {
    auto kernel = packed_gemv_kernel<FMT, R, TT, MODE, SWI_IN>;
    const size_t smem = x_smem_bytes<FMT>(p.K, TT) + (FMT == MF_NF4 ? kNf4LutBytes : 0);
    MF_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0;
    MF_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem));
    if (per_sm < 1) return fail(MF_RESOURCE_LIMIT, "packed GEMV tile does not fit on an SM");
    const int slots = 32 / p.lpr;
    const int rows_per_block = kWarps * slots * R;
    const int vrows = MODE == kPairRows ? 2 * p.N : p.N;
    const int blocks = (vrows + rows_per_block - 1) / rows_per_block;
    const int grid = std::min(blocks, per_sm * sm_count());
    if (int32_t e_ = ::mf::launch(kernel, dim3(grid), dim3(kThreads), smem, stream, "packed_gemv_kernel", p)) return e_;
    return MF_OK;
}

template <int FMT, int MODE, bool SWI_IN>
int32_t dispatch_tile(const GemvParams &p, int T, cudaStream_t stream) {
    // Token tile TT and rows-per-lane R: keep R*TT <= 4 accumulators per
    // output stream, x staging within ~160 KB, and enough row blocks to fill
    // the GPU at T = 1.
    const size_t budget = 160 * 1024;
    int TT = T >= 8 ? 8 : T >= 4 ? 4 : T >= 2 ? 2 : 1;
    while (TT > 1 && x_smem_bytes<FMT>(p.K, TT) > budget) TT >>= 1;
    if (x_smem_bytes<FMT>(p.K, TT) > budget)
        return fail(MF_UNSUPPORTED, "packed GEMV inner width too large for shared-memory staging");
    if (TT == 1) {
        const int slots = 32 / p.lpr;
        const int vrows = MODE == kPairRows ? 2 * p.N : p.N;
        const int target = 2 * sm_count();
        const int blocks4 = (vrows + kWarps * slots * 4 - 1) / (kWarps * slots * 4);
        const int blocks2 = (vrows + kWarps * slots * 2 - 1) / (kWarps * slots * 2);
        if (MODE != kSwigluPair && blocks4 >= target) return launch_cfg<FMT, 4, 1, MODE, SWI_IN>(p, stream);
        if (blocks2 >= target) return launch_cfg<FMT, 2, 1, MODE, SWI_IN>(p, stream);
        return launch_cfg<FMT, 1, 1, MODE, SWI_IN>(p, stream);
    }
    if (TT == 2) return launch_cfg<FMT, 2, 2, MODE, SWI_IN>(p, stream);
    if (TT == 4) return launch_cfg<FMT, 1, 4, MODE, SWI_IN>(p, stream);
    return launch_cfg<FMT, 1, 8, MODE, SWI_IN>(p, stream);
}

template <int MODE, bool SWI_IN>
int32_t dispatch_format(const GemvParams &p, int format, cudaStream_t stream) {
    switch (format) {
    case MF_TERNARY: return dispatch_tile<MF_TERNARY, MODE, SWI_IN>(p, p.T, stream);
    case MF_NF4: return dispatch_tile<MF_NF4, MODE, SWI_IN>(p, p.T, stream);
    case MF_INT8: return dispatch_tile<MF_INT8, MODE, SWI_IN>(p, p.T, stream);
    default: return fail(MF_INVALID_ARGUMENT, "unknown packed format");
    }
}

}  // namespace

int32_t packed_gemv(int mode, bool swiglu_input, float *out_a, float *out_b, const float *x,
                    const float *gate, const float *up, uint64_t t, const uint8_t *codes_a,
                    const float *scales_a, const uint8_t *codes_b, const float *scales_b,
                    uint64_t n, uint64_t k, int format, cudaStream_t stream) {
    if (t == 0 || n == 0) return MF_OK;
    if (k % kGroup) return fail(MF_INVALID_SHAPE, "packed inner width must be a multiple of 128");
    if (t > (1u << 30) || n > (1u << 30) || k > (1u << 24))
        return fail(MF_UNSUPPORTED, "packed matmul dimension exceeds kernel limits");
    GemvParams p{};
    p.x = x;
    p.gate = gate;
    p.up = up;
    p.codes_a = codes_a;
    p.codes_b = codes_b;
    p.scales_a = scales_a;
    p.scales_b = scales_b;
    p.out_a = out_a;
    p.out_b = out_b;
    p.T = (int)t;
    p.N = (int)n;
    p.K = (int)k;
    if (k == 0) {
        // Empty inner product: every output is +0.
        const size_t bytes = t * n * sizeof(float);
        MF_CUDA_TRY(cudaMemsetAsync(out_a, 0, bytes, stream));
        if (mode == kPairRows) MF_CUDA_TRY(cudaMemsetAsync(out_b, 0, bytes, stream));
        return MF_OK;
    }
    const int row_bytes = (int)(k / (uint64_t)weights_per_byte(format));
    // Team width: the largest power of two <= min(32, 16-byte chunks per row),
    // so teams tile the warp and the xor-shuffle reduction stays in-team.
    int lpr = 1;
    while (lpr * 2 <= std::min(32, row_bytes / 16)) lpr *= 2;
    p.lpr = lpr;
    if (mode == kSingle) {
        return swiglu_input ? dispatch_format<kSingle, true>(p, format, stream)
                            : dispatch_format<kSingle, false>(p, format, stream);
    }
    if (mode == kPairRows) return dispatch_format<kPairRows, false>(p, format, stream);
    return dispatch_format<kSwigluPair, false>(p, format, stream);
}

}  // namespace mf

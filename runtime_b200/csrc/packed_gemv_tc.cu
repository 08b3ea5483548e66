// Decode GEMV (up to 47 tokens) for the packed formats, sm_100a.
//
// out[t, r] = sum_g scale[r, g] * sum_{j in g} w(code[r, j]) * x[t, j]
// (crates/backend-cpu/src/packed.rs:96-170, crates/kernels-simd/src/lib.rs:31-208).
//
// At a few tokens these matmuls stream each weight byte once, so the budget
// is HBM bandwidth: at ~6.5 TB/s and ~1.9 GHz an SM can spend about 5.7
// lane-instructions per code byte.  Ternary packs four weights per byte,
// which an FP32 decode (shift, mask, convert, FMA per weight) cannot afford.
//
// Ternary and INT8: integer tensor cores.  The activations of each
// (token, 128-group) are split exactly into four int8 limbs:
//     x = 2^(e-7) * (l0 + l1 2^-7 + l2 2^-14 + l3 2^-21) + r,  |l_i| <= 64,
// with e chosen so that max|x| * 2^-e lies in [0.25, 0.5); the remainder is
// below 2^-27 of the group maximum.  `mma.sync.m16n8k32.s8.s8.s32` then
// forms exact integer dots of the weights with every limb (the four limbs
// are four columns of the MMA's B operand, two tokens per MMA), and each
// group's dot is promoted in FP32 with its row scale, as the reference's
// per-group `row += scale * group_dot` does.  INT8 codes are the A operand
// as stored; four ternary codes become four int8 weights with one byte
// permute through the table {-1, 0, +1, +2} (code 3 decodes to +2 as in
// crates/kernels-simd/src/lib.rs:22).  Because a dot product does not depend
// on the order of its terms, each lane loads a contiguous run of its rows'
// codes and the limbs are laid out in the matching order by limb_prep_kernel
// (one small launch per matmul; a producer kernel can write them instead).
//
// NF4: an FP32 path.  Each lane keeps 32 activations of the current group
// in registers, reads 16 code bytes of each of its rows, and looks both
// levels of a byte up at once in a 256-entry (level_lo, level_hi) table
// replicated 16 times in shared memory (conflict-free 64-bit reads).  CTAs
// are persistent so the table is built once per CTA.
//
// Work split (both kernels): one warp item is a tile of rows over a chunk of
// K groups; warps never wait on one another.  K is split into chunks only
// when the row tiles alone cannot fill the GPU; then every item writes its
// partial sums and the last item of a tile to finish (an atomic counter)
// adds the chunks in chunk order and runs the epilogue, so results do not
// depend on timing, and resets the counter for the next launch.
#include <algorithm>

#include "mf_common.cuh"
#include "packed_kernels.h"

namespace mf {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTokBlock = 8;         // tokens per grid.y block (4 MMA column blocks)

enum Mode { kSingle = 0, kPairRows = 1, kSwigluPair = 2 };

struct TcParams {
    const float *x, *gate, *up;
    const uint8_t *codes_a, *codes_b;
    const float *scales_a, *scales_b;
    float *out_a, *out_b;
    const uint2 *limbs;              // [T/2 pairs][groups][4][8][4] B fragments
    const float *efac;               // [2 * pairs][groups] 2^(e-7), NaN = poisoned group
    float *partial;                  // [nchunks][T][2N]
    unsigned *counters;              // [vtiles * token blocks]
    int T, N, K, groups;
    int pairs;                       // (T + 1) / 2 token pairs in `limbs`
    int row_tiles, vtiles;           // tiles per matrix; tiles the items cover
    int nchunks, kch;                // chunks; groups per chunk
    int items;                       // vtiles * nchunks
};

__device__ __forceinline__ void imma16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Four ternary codes (nibbles of `sel`, each 0..3) -> four int8 weights.
__device__ __forceinline__ uint32_t ternary4(uint32_t sel) {
    return __byte_perm(0x020100FFu, 0u, sel);  // bytes {-1, 0, +1, +2}
}

// ---------------------------------------------------------------------
// Limb preparation.  B fragment of m16n8k32 for lane (g = lane/4,
// q = lane%4): two words holding k = 4q..4q+3 and 16+4q..16+4q+3 of column
// n = g.  For token pair cb, group G, MMA step s, column n, lane-quad q the
// two words are one uint2 at limbs[((cb * groups + G) * 4 + s) * 32 + n * 4 + q].
// Column n = 4 * (token % 2) + limb.  Word h (0/1) byte i holds the limb of
// the element at group offset
//     INT8:    j = 32q + 8s + 4h + i
//     ternary: j = 32q + 8s + 2i + h
// matching the A operand each lane builds from its own code bytes.
// One warp per (token slot, group); lane = (s, q, h).
// ---------------------------------------------------------------------
template <int FMT, bool SWI_IN>
__global__ void __launch_bounds__(kThreads) limb_prep_kernel(const TcParams p, uint2 *limbs, float *efac) {
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * kWarps + (threadIdx.x >> 5);
    const int tpad = 2 * ((p.T + 1) / 2);
    if (item >= tpad * p.groups) return;
    const int t = item / p.groups, G = item % p.groups;
    const int s = lane >> 3, q = (lane >> 1) & 3, h = lane & 1;
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const bool live = t < p.T;
    if (live) {
        const size_t base = (size_t)t * p.K + (size_t)G * kGroup;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = FMT == MF_INT8 ? 32 * q + 8 * s + 4 * h + i : 32 * q + 8 * s + 2 * i + h;
            if constexpr (SWI_IN) v[i] = silu_mul(p.gate[base + j], p.up[base + j]);
            else v[i] = p.x[base + j];
        }
    }
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    const bool bad = __any_sync(0xffffffffu, !(isfinite(v[0]) && isfinite(v[1]) && isfinite(v[2]) && isfinite(v[3])));
    amax = warp_max(amax);
    // e = exponent of amax + 1 (amax in [2^(e-2), 2^(e-1))), at least -100.
    int e = 0;
    if (amax > 0.0f && !bad) {
        int ex = 0;
        frexpf(amax, &ex);
        e = max(ex + 1, -100);
    }
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (live && !bad) {
        // 2^(7-e) as a product of two normal powers of two (exact scaling).
        const int sh = 7 - e;
        const int sh1 = sh / 2, sh2 = sh - sh / 2;
        const float f1 = __int_as_float((127 + sh1) << 23), f2 = __int_as_float((127 + sh2) << 23);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float y = v[i] * f1 * f2;   // |y| < 64, exact
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const float r = rintf(y);
                w[l] |= ((uint32_t)(int)r & 0xFFu) << (8 * i);
                y = (y - r) * 128.0f;   // exact
            }
        }
    }
    const int cb = t >> 1, n0 = 4 * (t & 1);
    uint32_t *dst = reinterpret_cast<uint32_t *>(limbs + ((size_t)cb * p.groups + G) * 128);
#pragma unroll
    for (int l = 0; l < 4; ++l) dst[(s * 32 + (n0 + l) * 4 + q) * 2 + h] = w[l];
    if (lane == 0) {
        float f = 0.0f;
        if (live) f = bad ? __int_as_float(0x7fc00000) : __int_as_float((127 + e - 7) << 23);
        efac[(size_t)t * p.groups + G] = f;
    }
}

// ---------------------------------------------------------------------
// Warp-level split-K completion.  `v[j][k]` are this lane's values for
// (row, token) pairs listed by `row_of(k)`, `tok_of(k)`; `valid(k)` masks
// them.  Returns true (uniformly across the warp) if this warp must write
// the final outputs, with `v` replaced by the chunk-ordered sums.
// ---------------------------------------------------------------------
template <int J, int NV, typename RowF, typename TokF, typename ValidF>
__device__ __forceinline__ bool splitk_complete(const TcParams &p, float (&v)[J][NV], int mat, int chunk,
                                                unsigned counter_idx, RowF row_of, TokF tok_of, ValidF valid) {
    if (p.nchunks == 1) return true;
    const int lane = threadIdx.x & 31;
    const size_t vstride = 2 * (size_t)p.N;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int m = J == 2 ? j : mat;
#pragma unroll
        for (int k = 0; k < NV; ++k)
            if (valid(k))
                p.partial[((size_t)chunk * p.T + tok_of(k)) * vstride + (size_t)m * p.N + row_of(k)] = v[j][k];
    }
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(&p.counters[counter_idx], 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != (unsigned)(p.nchunks - 1)) return false;
    __threadfence();
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int m = J == 2 ? j : mat;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            if (!valid(k)) continue;
            float a = 0.0f;
            for (int c = 0; c < p.nchunks; ++c)
                a += __ldcg(&p.partial[((size_t)c * p.T + tok_of(k)) * vstride + (size_t)m * p.N + row_of(k)]);
            v[j][k] = a;
        }
    }
    if (lane == 0) p.counters[counter_idx] = 0u;  // ready for the next launch
    return true;
}

template <int MODE>
__device__ __forceinline__ void store_out(const TcParams &p, int mat, int t, int row, float a, float b) {
    const size_t o = (size_t)t * p.N + row;
    if constexpr (MODE == kSwigluPair) p.out_a[o] = silu_mul(a, b);
    else if constexpr (MODE == kPairRows) (mat ? p.out_b : p.out_a)[o] = a;
    else p.out_a[o] = a;
}

// ---------------------------------------------------------------------
// Ternary / INT8 on the integer tensor cores.  grid (items / 4 warps,
// token blocks of 8); item = (16-row tile, chunk of kch groups).
// ---------------------------------------------------------------------
template <int FMT, int MODE, int NCB>
__global__ void __launch_bounds__(kThreads) packed_gemv_imma_kernel(const TcParams p) {
    constexpr int J = MODE == kSwigluPair ? 2 : 1;
    constexpr int GB = FMT == MF_INT8 ? 128 : 32;   // code bytes per row per group
    constexpr int U = FMT == MF_INT8 ? 2 : 4;       // groups loaded per batch
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int item = blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (item >= p.items) return;
    const int vtile = item / p.nchunks, chunk = item % p.nchunks;
    const int tblk = blockIdx.y;
    const int t0 = tblk * kTokBlock;
    const int tb = min(kTokBlock, p.T - t0);
    const int cb0 = t0 / 2;
    const int g0 = chunk * p.kch;
    const int ng = min(p.kch, p.groups - g0);
    const int row_bytes = p.K / (FMT == MF_INT8 ? 1 : 4);
    const int mat = MODE == kPairRows ? (vtile >= p.row_tiles) : 0;
    const int r0 = (MODE == kPairRows && mat ? vtile - p.row_tiles : vtile) * 16;
    const int rg = r0 + g, rg8 = r0 + g + 8;
    const bool ok_g = rg < p.N, ok_g8 = rg8 < p.N;
    // Columns of this lane's MMA results: limb pair (2q, 2q+1) of token 2cb + q/2.
    const float lw0 = (q & 1) ? 0x1p-14f : 1.0f;
    const float lw1 = lw0 * 0x1p-7f;

    float acc[J][NCB][2];
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) acc[j][cb][0] = acc[j][cb][1] = 0.0f;

    for (int gb = 0; gb < ng; gb += U) {
        // Issue every load of the batch first: codes, scales, then limbs.
        uint4 cv[J][U][2][FMT == MF_INT8 ? 2 : 1];
        float sc[J][U][2];
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int m = J == 2 ? j : mat;
            const uint8_t *codes = m ? p.codes_b : p.codes_a;
            const float *scales = m ? p.scales_b : p.scales_a;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int G = g0 + gb + u;
                const bool gok = gb + u < ng;
                const uint8_t *cg = codes + (size_t)G * GB;
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const int row = r ? rg8 : rg;
                    const bool ok = gok && (r ? ok_g8 : ok_g);
                    if constexpr (FMT == MF_INT8) {
                        cv[j][u][r][0] = ok ? ld_stream_u4(cg + (size_t)row * row_bytes + 32 * q) : make_uint4(0, 0, 0, 0);
                        cv[j][u][r][1] = ok ? ld_stream_u4(cg + (size_t)row * row_bytes + 32 * q + 16) : make_uint4(0, 0, 0, 0);
                    } else {
                        const uint2 c2 = ok ? ld_stream_u2(cg + (size_t)row * row_bytes + 8 * q)
                                            : make_uint2(0x55555555u, 0x55555555u);  // weight 0
                        cv[j][u][r][0] = make_uint4(c2.x, c2.y, 0, 0);
                    }
                    sc[j][u][r] = ok ? __ldg(scales + (size_t)row * p.groups + G) : 0.0f;
                }
            }
        }
        uint2 bfr[U][NCB][4];
        float ef[U][NCB];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int G = g0 + min(gb + u, ng - 1);
#pragma unroll
            for (int cb = 0; cb < NCB; ++cb) {
                if (cb0 + cb < p.pairs) {
                    const uint2 *src = p.limbs + ((size_t)(cb0 + cb) * p.groups + G) * 128;
#pragma unroll
                    for (int s = 0; s < 4; ++s) bfr[u][cb][s] = src[s * 32 + g * 4 + q];
                    ef[u][cb] = p.efac[(size_t)(t0 + 2 * cb + (q >> 1)) * p.groups + G];
                } else {
#pragma unroll
                    for (int s = 0; s < 4; ++s) bfr[u][cb][s] = make_uint2(0u, 0u);
                    ef[u][cb] = 0.0f;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (gb + u >= ng) break;
#pragma unroll
            for (int j = 0; j < J; ++j) {
                uint32_t wa[8], wb[8];
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    uint32_t *dst = r ? wb : wa;
                    if constexpr (FMT == MF_INT8) {
                        const uint4 a0 = cv[j][u][r][0], a1 = cv[j][u][r][1];
                        dst[0] = a0.x; dst[1] = a0.y; dst[2] = a0.z; dst[3] = a0.w;
                        dst[4] = a1.x; dst[5] = a1.y; dst[6] = a1.z; dst[7] = a1.w;
                    } else {
                        const uint32_t cw[2] = {cv[j][u][r][0].x, cv[j][u][r][0].y};
#pragma unroll
                        for (int hh = 0; hh < 2; ++hh) {
                            const uint32_t w = cw[hh];
                            dst[4 * hh + 0] = ternary4(w & 0x3333u);
                            dst[4 * hh + 1] = ternary4((w >> 2) & 0x3333u);
                            dst[4 * hh + 2] = ternary4((w >> 16) & 0x3333u);
                            dst[4 * hh + 3] = ternary4((w >> 18) & 0x3333u);
                        }
                    }
                }
#pragma unroll
                for (int cb = 0; cb < NCB; ++cb) {
                    int d[4] = {0, 0, 0, 0};
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint32_t a[4] = {wa[2 * s], wb[2 * s], wa[2 * s + 1], wb[2 * s + 1]};
                        imma16832(d, a, bfr[u][cb][s].x, bfr[u][cb][s].y);
                    }
                    const float vg = fmaf(__int2float_rn(d[1]), lw1, __int2float_rn(d[0]) * lw0) * ef[u][cb];
                    const float vg8 = fmaf(__int2float_rn(d[3]), lw1, __int2float_rn(d[2]) * lw0) * ef[u][cb];
                    acc[j][cb][0] = fmaf(vg, sc[j][u][0], acc[j][cb][0]);
                    acc[j][cb][1] = fmaf(vg8, sc[j][u][1], acc[j][cb][1]);
                }
            }
        }
    }
    // Lanes q and q^1 hold the low and high limb pairs of one token.
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb)
#pragma unroll
            for (int r = 0; r < 2; ++r) acc[j][cb][r] += __shfl_xor_sync(0xffffffffu, acc[j][cb][r], 1);
    // Lane (g, q even) owns tokens 2cb + q/2, rows g and g + 8.
    float v[J][2 * NCB];
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) {
            v[j][2 * cb] = acc[j][cb][0];
            v[j][2 * cb + 1] = acc[j][cb][1];
        }
    const bool mine = !(q & 1);
    auto row_of = [&](int k) { return (k & 1) ? rg8 : rg; };
    auto tok_of = [&](int k) { return t0 + 2 * (k >> 1) + (q >> 1); };
    auto valid = [&](int k) {
        return mine && (2 * (k >> 1) + (q >> 1)) < tb && ((k & 1) ? ok_g8 : ok_g);
    };
    if (!splitk_complete<J, 2 * NCB>(p, v, mat, chunk, (unsigned)(vtile * gridDim.y + tblk), row_of, tok_of, valid))
        return;
#pragma unroll
    for (int k = 0; k < 2 * NCB; ++k)
        if (valid(k)) store_out<MODE>(p, mat, tok_of(k), row_of(k), v[0][k], v[J - 1][k]);
}

// ---------------------------------------------------------------------
// NF4 (FP32), persistent CTAs.  item = (tile of 8 * RS rows, chunk);
// lane (r = lane / 4, q = lane % 4) serves rows r, r + 8, ... of the tile,
// bytes [16q, 16q + 16) of each 64-byte group, i.e. x[32q .. 32q + 31].
// ---------------------------------------------------------------------
__device__ __constant__ float kNf4Levels[16] = {
    -0x1.000000p+0f, -0x1.647362p-1f, -0x1.0cd660p-1f, -0x1.946540p-2f,
    -0x1.23449ap-2f, -0x1.7a6a7ep-3f, -0x1.74f0e2p-4f, 0.0f,
    0x1.45f5fep-4f,  0x1.4995c6p-3f,  0x1.f809bap-3f,  0x1.5a0674p-2f,
    0x1.c34970p-2f,  0x1.200f56p-1f,  0x1.722766p-1f,  0x1.000000p+0f,
};

template <int MODE, int TOK, int RS, bool SWI_IN>
__global__ void __launch_bounds__(kThreads) packed_gemv_nf4_kernel(const TcParams p) {
    constexpr int J = MODE == kSwigluPair ? 2 : 1;
    __shared__ __align__(16) float2 lut[256 * 16];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r = lane >> 2, q = lane & 3, l16 = lane & 15;
    for (int e = tid; e < 256 * 16; e += kThreads) {
        const int b = e >> 4;
        lut[e] = make_float2(kNf4Levels[b & 15], kNf4Levels[b >> 4]);
    }
    __syncthreads();
    const int row_bytes = p.K / 2;
    const int tblk = blockIdx.y;
    const int t0 = tblk * TOK;
    const int tb = min(TOK, p.T - t0);
    for (int item = blockIdx.x * kWarps + warp; item < p.items; item += gridDim.x * kWarps) {
        const int vtile = item / p.nchunks, chunk = item % p.nchunks;
        const int g0 = chunk * p.kch;
        const int ng = min(p.kch, p.groups - g0);
        const int mat = MODE == kPairRows ? (vtile >= p.row_tiles) : 0;
        const int rb0 = (MODE == kPairRows && mat ? vtile - p.row_tiles : vtile) * 8 * RS;
        float acc[J][RS][TOK];
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int i = 0; i < RS; ++i)
#pragma unroll
                for (int t = 0; t < TOK; ++t) acc[j][i][t] = 0.0f;
        for (int gi = 0; gi < ng; ++gi) {
            const int G = g0 + gi;
            uint4 cw[J][RS];
            float sc[J][RS];
#pragma unroll
            for (int j = 0; j < J; ++j) {
                const int m = J == 2 ? j : mat;
                const uint8_t *codes = m ? p.codes_b : p.codes_a;
                const float *scales = m ? p.scales_b : p.scales_a;
#pragma unroll
                for (int i = 0; i < RS; ++i) {
                    const int row = rb0 + r + 8 * i;
                    const bool ok = row < p.N;
                    cw[j][i] = ok ? ld_stream_u4(codes + (size_t)row * row_bytes + (size_t)G * 64 + 16 * q)
                                  : make_uint4(0x77777777u, 0x77777777u, 0x77777777u, 0x77777777u);  // level 0
                    sc[j][i] = ok ? __ldg(scales + (size_t)row * p.groups + G) : 0.0f;
                }
            }
            float xv[TOK][32];
#pragma unroll
            for (int t = 0; t < TOK; ++t) {
                const size_t base = (size_t)(t0 + min(t, tb - 1)) * p.K + (size_t)G * kGroup + 32 * q;
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    if constexpr (SWI_IN) {
#pragma unroll
                        for (int u = 0; u < 4; ++u) xv[t][i + u] = silu_mul(p.gate[base + i + u], p.up[base + i + u]);
                    } else {
                        const float4 v4 = *reinterpret_cast<const float4 *>(p.x + base + i);
                        xv[t][i] = v4.x;
                        xv[t][i + 1] = v4.y;
                        xv[t][i + 2] = v4.z;
                        xv[t][i + 3] = v4.w;
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < J; ++j)
#pragma unroll
                for (int i = 0; i < RS; ++i) {
                    const uint32_t words[4] = {cw[j][i].x, cw[j][i].y, cw[j][i].z, cw[j][i].w};
                    float part[TOK];
#pragma unroll
                    for (int t = 0; t < TOK; ++t) part[t] = 0.0f;
#pragma unroll
                    for (int w = 0; w < 4; ++w)
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const float2 lv = lut[((words[w] >> (8 * b)) & 0xFFu) * 16 + l16];
#pragma unroll
                            for (int t = 0; t < TOK; ++t) {
                                part[t] = fmaf(lv.x, xv[t][8 * w + 2 * b], part[t]);
                                part[t] = fmaf(lv.y, xv[t][8 * w + 2 * b + 1], part[t]);
                            }
                        }
#pragma unroll
                    for (int t = 0; t < TOK; ++t) acc[j][i][t] = fmaf(part[t], sc[j][i], acc[j][i][t]);
                }
        }
        // Sum the four lanes of each row; lane q == 0 owns the row.
        float v[J][RS * TOK];
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int i = 0; i < RS; ++i)
#pragma unroll
                for (int t = 0; t < TOK; ++t) {
                    float a = acc[j][i][t];
                    a += __shfl_xor_sync(0xffffffffu, a, 1);
                    a += __shfl_xor_sync(0xffffffffu, a, 2);
                    v[j][i * TOK + t] = a;
                }
        auto row_of = [&](int k) { return rb0 + r + 8 * (k / TOK); };
        auto tok_of = [&](int k) { return t0 + k % TOK; };
        auto valid = [&](int k) { return q == 0 && (k % TOK) < tb && rb0 + r + 8 * (k / TOK) < p.N; };
        if (!splitk_complete<J, RS * TOK>(p, v, mat, chunk, (unsigned)(vtile * gridDim.y + tblk), row_of, tok_of,
                                          valid))
            continue;
#pragma unroll
        for (int k = 0; k < RS * TOK; ++k)
            if (valid(k)) store_out<MODE>(p, mat, tok_of(k), row_of(k), v[0][k], v[J - 1][k]);
    }
}

// ---------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------
// Chunks: enough (tile, chunk) items to give every SM several warps, each
// chunk at least 4 groups.
void choose_chunks(TcParams &p, int warp_items_target) {
    const int groups = p.groups;
    int nch = std::max(1, (warp_items_target + p.vtiles - 1) / p.vtiles);
    nch = std::min(nch, std::max(1, groups / 4));
    p.kch = (groups + nch - 1) / nch;
    p.nchunks = (groups + p.kch - 1) / p.kch;
    p.items = p.vtiles * p.nchunks;
}

template <int FMT, int MODE, int NCB>
int32_t launch_imma(TcParams p, cudaStream_t stream) {
    const int tblocks = (p.T + kTokBlock - 1) / kTokBlock;
    dim3 grid((p.items + kWarps - 1) / kWarps, tblocks);
    packed_gemv_imma_kernel<FMT, MODE, NCB><<<grid, kThreads, 0, stream>>>(p);
    MF_LAUNCH_CHECK("packed_gemv_imma_kernel");
    return MF_OK;
}

template <int FMT, int MODE, bool SWI>
int32_t dispatch_imma(TcParams p, cudaStream_t stream) {
    p.row_tiles = (p.N + 15) / 16;
    p.vtiles = MODE == kPairRows ? 2 * p.row_tiles : p.row_tiles;
    choose_chunks(p, 8 * sm_count());
    // Limbs of every token (padded to pairs) and group.
    const int tpad = 2 * ((p.T + 1) / 2);
    const int prep_items = tpad * p.groups;
    limb_prep_kernel<FMT, SWI><<<(prep_items + kWarps - 1) / kWarps, kThreads, 0, stream>>>(
        p, const_cast<uint2 *>(p.limbs), const_cast<float *>(p.efac));
    MF_LAUNCH_CHECK("limb_prep_kernel");
    const int tb = std::min(p.T, kTokBlock);
    if (tb <= 2) return launch_imma<FMT, MODE, 1>(p, stream);
    if (tb <= 4) return launch_imma<FMT, MODE, 2>(p, stream);
    if (tb <= 6) return launch_imma<FMT, MODE, 3>(p, stream);
    return launch_imma<FMT, MODE, 4>(p, stream);
}

template <int MODE, int TOK, int RS, bool SWI>
int32_t launch_nf4(TcParams p, cudaStream_t stream) {
    p.row_tiles = (p.N + 8 * RS - 1) / (8 * RS);
    p.vtiles = MODE == kPairRows ? 2 * p.row_tiles : p.row_tiles;
    choose_chunks(p, 8 * sm_count());
    auto kernel = packed_gemv_nf4_kernel<MODE, TOK, RS, SWI>;
    int per_sm = 0;
    MF_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0));
    const int ctas = std::max(1, std::min((p.items + kWarps - 1) / kWarps, std::max(1, per_sm) * sm_count()));
    dim3 grid(ctas, (p.T + TOK - 1) / TOK);
    kernel<<<grid, kThreads, 0, stream>>>(p);
    MF_LAUNCH_CHECK("packed_gemv_nf4_kernel");
    return MF_OK;
}

template <int MODE, bool SWI>
int32_t dispatch_nf4(TcParams p, cudaStream_t stream) {
    // 64-row tiles when they alone give every SM a few warps, else 16.
    const int vmul = MODE == kPairRows ? 2 : 1;
    const bool big = ((p.N + 63) / 64) * vmul >= 4 * sm_count();
    if (p.T == 1) return big ? launch_nf4<MODE, 1, 8, SWI>(p, stream) : launch_nf4<MODE, 1, 2, SWI>(p, stream);
    return big ? launch_nf4<MODE, 2, 8, SWI>(p, stream) : launch_nf4<MODE, 2, 2, SWI>(p, stream);
}

size_t limb_floats(uint64_t t, uint64_t k) {
    const uint64_t pairs = (t + 1) / 2, groups = k / kGroup;
    return (size_t)(pairs * groups * 256 + 2 * pairs * groups);  // 1 KB of limbs + 2 factors per pair-group
}

}  // namespace

bool packed_gemv_tc_supports(int format, uint64_t t) {
    if (format == MF_NF4) return t >= 1 && t <= 2;
    return t >= 1 && t < kGemmMinTokens;
}

size_t packed_gemv_tc_scratch_floats(uint64_t t, uint64_t n, uint64_t k) {
    // Split-K partials for at most k/512 chunks, plus the activation limbs.
    const uint64_t groups = k / kGroup;
    const uint64_t max_chunks = std::max<uint64_t>(1, groups / 4);
    return (size_t)(max_chunks > 1 ? max_chunks * t * 2 * n : 0) + limb_floats(t, k) + 64;
}

size_t packed_gemv_tc_counters(uint64_t t, uint64_t n) {
    // One per (tile, token block) of the larger (pair-rows) tile space.
    return (size_t)(2 * ((n + 15) / 16)) * ((t + kTokBlock - 1) / kTokBlock);
}

int32_t packed_gemv_tc(int mode, bool swiglu_input, float *out_a, float *out_b, const float *x, const float *gate,
                       const float *up, uint64_t t, const uint8_t *codes_a, const float *scales_a,
                       const uint8_t *codes_b, const float *scales_b, uint64_t n, uint64_t k, int format,
                       const SplitScratch &ss, cudaStream_t stream) {
    if (t == 0 || n == 0) return MF_OK;
    if (k == 0 || k % kGroup) return fail(MF_INVALID_SHAPE, "packed inner width must be a positive multiple of 128");
    if (n > (1u << 26) || k > (1u << 24) || t >= kGemmMinTokens)
        return fail(MF_UNSUPPORTED, "packed matmul dimension exceeds decode-GEMV limits");
    if (!packed_gemv_tc_supports(format, t)) return fail(MF_UNSUPPORTED, "decode GEMV does not take this token count");
    if (ss.partial_floats < packed_gemv_tc_scratch_floats(t, n, k) || ss.n_counters < packed_gemv_tc_counters(t, n) ||
        !ss.partial || !ss.counters)
        return fail(MF_RESOURCE_LIMIT, "packed GEMV scratch too small");
    TcParams p{};
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
    p.groups = (int)(k / kGroup);
    p.pairs = (int)((t + 1) / 2);
    // Scratch layout: [limbs (16-byte aligned) | factors | partials].
    float *base = ss.partial;
    const uint64_t pairs = (t + 1) / 2;
    p.limbs = reinterpret_cast<const uint2 *>(base);
    p.efac = base + pairs * p.groups * 256;
    p.partial = base + limb_floats(t, k) + 32;
    p.counters = ss.counters;
#define MF_TC_MODES(DISPATCH, ...)                                                                  \
    do {                                                                                           \
        if (mode == kSingle)                                                                       \
            return swiglu_input ? DISPATCH<__VA_ARGS__ kSingle, true>(p, stream)                   \
                                : DISPATCH<__VA_ARGS__ kSingle, false>(p, stream);                 \
        if (mode == kPairRows) return DISPATCH<__VA_ARGS__ kPairRows, false>(p, stream);           \
        return DISPATCH<__VA_ARGS__ kSwigluPair, false>(p, stream);                                \
    } while (0)
    switch (format) {
    case MF_TERNARY: MF_TC_MODES(dispatch_imma, MF_TERNARY,);
    case MF_INT8: MF_TC_MODES(dispatch_imma, MF_INT8,);
    case MF_NF4: MF_TC_MODES(dispatch_nf4, );
    default: return fail(MF_INVALID_ARGUMENT, "unknown packed format");
    }
#undef MF_TC_MODES
}

}  // namespace mf

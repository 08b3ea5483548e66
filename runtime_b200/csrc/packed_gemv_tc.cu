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
// as stored.  A ternary code c decodes to c - 1 (code 3 to +2, as in
// crates/kernels-simd/src/lib.rs:22), so the dot of a group is
// sum(c * x) - sum(x): the codes enter the MMA as unsigned bytes straight
// from the code word (one mask, and a shift for three of every four, gives
// 64 * c in each byte lane), and the accumulator starts at -64 * sum(limb)
// of the group, which the limb producer computes; the promotion divides the
// 64 out exactly.  Because a dot product does not depend on the order of
// its terms, each lane loads a contiguous run of its rows' codes and the
// limbs are laid out in the matching order by limb_prep_kernel (one small
// launch per matmul; a producer kernel can write them instead).
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
#include <map>
#include <mutex>

#include "mf_common.cuh"
#include "packed_kernels.h"

namespace mf {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTokBlock = 8;         // tokens per grid.y block (4 MMA column blocks)

enum Mode { kSingle = 0, kPairRows = 1, kSwigluPair = 2, kTriple = 3, kConv = 4 };
constexpr int kConvMaxWidth = 4;   // taps of the gated short convolution epilogue (LFM2: 3)
enum Prologue { kFromGlobal = 0, kNorm = 1 };

struct TcParams {
    const float *x, *gate, *up;
    const uint8_t *codes_a, *codes_b, *codes_c;
    const float *scales_a, *scales_b, *scales_c;
    float *out_a, *out_b, *out_c;
    int N2;                          // rows of matrices B and C in kTriple mode
    // kNorm prologue (one token): x = rmsnorm(na + nb) * nw, or rmsnorm of the
    // embedding row of token *eid (ecodes/escales packed, or edense) when na
    // is null; CTA (0, 0) writes the sum to nres.
    const float *na, *nb, *nw;
    float *nres;
    float neps;
    const uint8_t *ecodes;
    const float *escales, *edense, *eid;
    int eformat, erows;
    // Argmax epilogue (kSingle, one token): CTA partials, arrival counter,
    // greedy id, position advanced by one.
    float *aparts;
    unsigned *acount;
    float *asampled;
    uint64_t *apos;
    // Row shard of a split LM head: instead of the greedy id, the merge
    // writes this shard's candidate (value, index + arow0, poisoned) to acand.
    float *acand;
    int arow0;
    const uint2 *limbs;              // [T/2 pairs][groups][4][8][4] B fragments
    const float *efac;               // [2 * pairs][groups] 2^(e-7), NaN = poisoned group
    const int2 *lsum;                // ternary: [pairs][groups][4 quads] -64 * column limb sums
    // Half-group limbs (one token): limbs/efac were written by the producer
    // with token slot 1 holding the upper 64 weights of each group (own
    // exponent); the kernel adds the two slots' sums.  No limb pass.
    int split_halves;
    // SwiGLU-pair epilogue (one token, normalizing prologue): the outputs'
    // half-group limbs for a consumer of format lfmt, lgroups = N / 128.
    uint2 *lout;
    float *lefac;
    int2 *llsum;
    int lfmt, lgroups;
    // Gated short convolution epilogue (kConv, NF4, one token): rows are the
    // B, C and x projections of N channels; out_a gets the conv output and
    // chist ([cwidth - 1][N], oldest first) moves on by one row.
    const float *ckern;
    float *chist;
    int cwidth;
    int T, N, K, groups;
    // Ternary codes in the lane-tiled layout of repack_ternary_lut2 (N a
    // multiple of 16): for 16-row tile t, group G and lane L = 4g + q, the 16
    // bytes at ((t * groups + G) * 32 + L) * 16 are row 16t + g's bytes
    // 8q .. 8q + 7 of group G, then row 16t + g + 8's.
    int lanetiled;
    int pairs;                       // (T + 1) / 2 token pairs in `limbs`
    int row_tiles, vtiles;           // tiles per matrix; tiles the items cover
    int rt, kw;                      // tiles (row groups) per CTA; K parts per CTA
    int kch;                         // groups per K part
};

__device__ __constant__ float kNf4Levels[16] = {
    -0x1.000000p+0f, -0x1.647362p-1f, -0x1.0cd660p-1f, -0x1.946540p-2f,
    -0x1.23449ap-2f, -0x1.7a6a7ep-3f, -0x1.74f0e2p-4f, 0.0f,
    0x1.45f5fep-4f,  0x1.4995c6p-3f,  0x1.f809bap-3f,  0x1.5a0674p-2f,
    0x1.c34970p-2f,  0x1.200f56p-1f,  0x1.722766p-1f,  0x1.000000p+0f,
};

__device__ __forceinline__ void imma16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Unsigned ternary codes (A) against signed limbs (B); C and D distinct, so
// a group's first MMA can start from the limb-sum offset in place.
__device__ __forceinline__ void imma16832_u(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void imma16832_u_c(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int c0,
                                              int c1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%10,%11};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}

// One word of 16 ternary codes (code i in bits 2i, 2i+1) -> four MMA A
// registers: register j holds codes 4b + j of bytes b = 0..3, each as
// 64 * code in its byte lane (bits 6-7).
__device__ __forceinline__ void ternary_u8x4(uint32_t w, uint32_t *r) {
    r[0] = (w << 6) & 0xC0C0C0C0u;
    r[1] = (w << 4) & 0xC0C0C0C0u;
    r[2] = (w << 2) & 0xC0C0C0C0u;
    r[3] = w & 0xC0C0C0C0u;
}

// Group offset of the weight multiplying byte i of B-fragment word h at MMA
// step s for lane quad q: ternary in the order ternary_u8x4 leaves each
// lane's 8 code bytes (word s/2, register 2(s%2) + h); INT8 as stored.
__host__ __device__ __forceinline__ int limb_elem(int fmt, int s, int q, int h, int i) {
    return fmt == MF_INT8 ? 32 * q + 8 * s + 4 * h + i : 32 * q + 16 * (s >> 1) + 4 * i + 2 * (s & 1) + h;
}

// -64 * (sum of limb l's bytes over a warp's group) for l = 0..3, in every
// lane; w[l] holds this lane's four bytes of limb l.
__device__ __forceinline__ void limb_sums64(const uint32_t (&w)[4], int (&sum)[4]) {
#pragma unroll
    for (int l = 0; l < 4; ++l) sum[l] = -64 * __reduce_add_sync(0xffffffffu, __dp4a((int)w[l], 0x01010101, 0));
}

// ---------------------------------------------------------------------
// Limb preparation.  B fragment of m16n8k32 for lane (g = lane/4,
// q = lane%4): two words holding k = 4q..4q+3 and 16+4q..16+4q+3 of column
// n = g.  For token pair cb, group G, MMA step s, column n, lane-quad q the
// two words are one uint2 at limbs[((cb * groups + G) * 4 + s) * 32 + n * 4 + q].
// Column n = 4 * (token % 2) + limb.  Word h (0/1) byte i holds the limb of
// the element at group offset limb_elem(format, s, q, h, i)
//     INT8:    j = 32q + 8s + 4h + i
//     ternary: j = 32q + 16(s/2) + 4i + 2(s%2) + h
// matching the A operand each lane builds from its own code bytes.  For
// ternary, lsum[(pair * groups + G) * 4 + quad] holds -64 times the sums of
// columns 2 quad and 2 quad + 1 (the C fragment columns of that lane quad).
// One warp per (token slot, group); lane = (s, q, h).
// ---------------------------------------------------------------------
template <int FMT, bool SWI_IN>
__global__ void __launch_bounds__(kThreads) limb_prep_kernel(const TcParams p, uint2 *limbs, float *efac, int2 *lsum) {
    pdl_wait();
    pdl_trigger();
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
            const int j = limb_elem(FMT, s, q, h, i);
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
    if constexpr (FMT == MF_TERNARY) {
        int sum[4];
        limb_sums64(w, sum);
        if (lane < 2)
            lsum[((size_t)cb * p.groups + G) * 4 + 2 * (t & 1) + lane] = make_int2(sum[2 * lane], sum[2 * lane + 1]);
    }
    if (lane == 0) {
        float f = 0.0f;
        if (live) f = bad ? __int_as_float(0x7fc00000) : __int_as_float((127 + e - 7) << 23);
        efac[(size_t)t * p.groups + G] = f;
    }
}

template <int MODE>
__device__ __forceinline__ void store_out(const TcParams &p, int mat, int t, int row, float a, float b) {
    if constexpr (MODE == kTriple) {
        float *o = mat == 0 ? p.out_a : mat == 1 ? p.out_b : p.out_c;
        o[(size_t)t * (mat ? p.N2 : p.N) + row] = a;
        return;
    }
    const size_t o = (size_t)t * p.N + row;
    if constexpr (MODE == kSwigluPair) p.out_a[o] = silu_mul(a, b);
    else if constexpr (MODE == kPairRows) (mat ? p.out_b : p.out_a)[o] = a;
    else p.out_a[o] = a;
}

// Matrix, first row and row count of a virtual 16-row tile (IMMA) or of a
// virtual row (NF4, tile = 1): pair-rows stacks B under A, triple stacks
// B and C (N2 rows each) under A.
__device__ __forceinline__ void tile_map(const TcParams &p, int mode, int vt, int tile, int &m, int &r0, int &rows) {
    const int ta = (p.N + tile - 1) / tile, tb = (p.N2 + tile - 1) / tile;
    m = 0;
    r0 = vt * tile;
    rows = p.N;
    if (mode == kPairRows && vt >= ta) {
        m = 1;
        r0 = (vt - ta) * tile;
    } else if (mode == kTriple && vt >= ta) {
        m = vt < ta + tb ? 1 : 2;
        r0 = (vt - ta - (m == 2 ? tb : 0)) * tile;
        rows = p.N2;
    }
}

__device__ __forceinline__ const uint8_t *codes_of(const TcParams &p, int m) {
    return m == 0 ? p.codes_a : m == 1 ? p.codes_b : p.codes_c;
}
__device__ __forceinline__ const float *scales_of(const TcParams &p, int m) {
    return m == 0 ? p.scales_a : m == 1 ? p.scales_b : p.scales_c;
}

// ---------------------------------------------------------------------
// kNorm prologue: one token's input row formed and normalized in shared
// memory by the whole CTA, in the reference's order of rounding
// (crates/backend-cpu/src/normalization_rotary.rs:11-81, :221-235): sum
// a + b (or the dequantized embedding row), sum of squares, reciprocal of
// sqrt(mean + eps), then (v * rec) * w.  Every CTA computes the same values;
// CTA (0, 0) writes the sum.  Call after pdl_wait().
// ---------------------------------------------------------------------
// Starts copying the norm weight p.nw (K floats, a constant) into shared
// memory at nws; called before pdl_wait() so the copy overlaps the
// previous kernel.  norm_prologue waits for it.
__device__ __forceinline__ void nw_prefetch(const TcParams &p, float *nws) {
    if (!p.nw) return;
    for (int e = threadIdx.x; e < p.K / 4; e += blockDim.x) {
        const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(nws + 4 * e));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(p.nw + 4 * e) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// Element k of a row staged with 4 floats of padding after every 32 (PAD):
// lanes that each read 32 consecutive values, 32 apart, then hit distinct
// banks with 128-bit loads.
__host__ __device__ __forceinline__ int pad32(int k) { return k + 4 * (k >> 5); }
__host__ __device__ __forceinline__ size_t padded_row_floats(size_t K) { return K + K / 8; }
// A row of K in the integer-MMA GEMV's staging (padw<2>: 2 floats per 32).
__host__ __device__ __forceinline__ size_t imma_row_floats(size_t K) { return K + K / 16; }

// Element k of a row staged with PADW floats of padding after every 32.
template <int PADW>
__device__ __forceinline__ int padw(int k) { return k + PADW * (k >> 5); }

// Stages the row to normalize in xs (PADW floats of padding after every 32;
// 0, 2 or 4) and, in CTA (0, 0), the sum in p.nres; returns this thread's
// partial sum of squares.
template <int PADW = 0>
__device__ float norm_stage(const TcParams &p, float *xs) {
    const int tid = threadIdx.x;
    const int K = p.K;  // a multiple of 128
    const bool writer = p.nres && blockIdx.x == 0 && blockIdx.y == 0;
    float ss = 0.0f;
    if (p.na) {
        // Eight 16-byte loads of each operand per thread in flight at once.
        constexpr int U = 8;
        const int nvec = K / 4;
        for (int b0 = tid; b0 < nvec; b0 += U * blockDim.x) {
            float4 va[U], vb[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int e = b0 + u * blockDim.x;
                va[u] = e < nvec ? reinterpret_cast<const float4 *>(p.na)[e] : make_float4(0.f, 0.f, 0.f, 0.f);
                vb[u] = (e < nvec && p.nb) ? reinterpret_cast<const float4 *>(p.nb)[e] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int e = b0 + u * blockDim.x;
                if (e >= nvec) continue;
                float4 v = va[u];
                if (p.nb) {
                    v.x = __fadd_rn(v.x, vb[u].x);
                    v.y = __fadd_rn(v.y, vb[u].y);
                    v.z = __fadd_rn(v.z, vb[u].z);
                    v.w = __fadd_rn(v.w, vb[u].w);
                }
                float *dst = xs + padw<PADW>(4 * e);
                if constexpr (PADW % 4 == 0) {
                    *reinterpret_cast<float4 *>(dst) = v;
                } else {
                    reinterpret_cast<float2 *>(dst)[0] = make_float2(v.x, v.y);
                    reinterpret_cast<float2 *>(dst)[1] = make_float2(v.z, v.w);
                }
                if (writer) reinterpret_cast<float4 *>(p.nres)[e] = v;
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
            }
        }
    } else {
        // Embedding row of the device id (packed_gather_rows semantics:
        // level * scale, one rounding; an invalid id gives a NaN row).
        const float idv = *p.eid;
        const long long id = (isfinite(idv) && idv >= 0.0f && floorf(idv) == idv && idv < 16777216.0f &&
                              (long long)idv < p.erows) ? (long long)idv : -1;
        for (int e = tid; e < K; e += blockDim.x) {
            float v;
            if (id < 0) {
                v = __int_as_float(0x7fc00000);
            } else if (p.edense) {
                v = p.edense[(size_t)id * K + e];
            } else {
                const int gw = e / kGroup, w = e % kGroup;
                const uint8_t *c =
                    p.ecodes + (size_t)id * (K / (p.eformat == MF_TERNARY ? 4 : p.eformat == MF_NF4 ? 2 : 1));
                float level;
                if (p.eformat == MF_TERNARY) level = (float)((c[gw * 32 + w / 4] >> (2 * (w % 4))) & 3u) - 1.0f;
                else if (p.eformat == MF_INT8) level = (float)(int8_t)c[e];
                else {
                    const uint8_t b = c[gw * 64 + w / 2];
                    level = kNf4Levels[(w & 1) ? (b >> 4) : (b & 15)];
                }
                v = __fmul_rn(level, p.escales[(size_t)id * (K / kGroup) + gw]);
            }
            xs[padw<PADW>(e)] = v;
            if (writer) p.nres[e] = v;
            ss = fmaf(v, v, ss);
        }
    }
    return ss;
}

// 1 / sqrt(mean(x^2) + eps) from the per-warp partial sums red[0 .. warps),
// summed in lane order: every warp that calls it gets the same value.
__device__ __forceinline__ float norm_reciprocal(const float *red, int K, float eps) {
    const int lane = threadIdx.x & 31;
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
    t = warp_sum(t);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), eps)));
}

// The normalized row in xs, staged with pad32's padding (the NF4 GEMV's
// lanes read 32 consecutive values each).  Every warp forms the reciprocal
// itself from the per-warp sums, so one barrier publishes the sums and one
// the normalized row.
// nw_prefetch into the layout of padw<2> (8-byte copies).
__device__ __forceinline__ void nw_prefetch_pad2(const TcParams &p, float *nws) {
    if (!p.nw) return;
    for (int e = threadIdx.x; e < p.K / 2; e += blockDim.x) {
        const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(nws + padw<2>(2 * e)));
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(d), "l"(p.nw + 2 * e) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ float norm_prologue(const TcParams &p, float *xs, const float *nws) {
    __shared__ float red_ss[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = p.K;
    float ss = norm_stage<4>(p, xs);
    if (!p.nw) {
        // Staged input without normalization (the row as given).
        __syncthreads();
        return 1.0f;
    }
    ss = warp_sum(ss);
    if (lane == 0) red_ss[warp] = ss;
    asm volatile("cp.async.wait_all;" ::: "memory");   // this thread's norm-weight copies
    __syncthreads();
    const float rec = norm_reciprocal(red_ss, K, p.neps);
    for (int e = tid; e < K / 4; e += blockDim.x) {
        float4 *px = reinterpret_cast<float4 *>(xs + pad32(4 * e));
        float4 v = *px;
        const float4 w = reinterpret_cast<const float4 *>(nws)[e];
        v.x = __fmul_rn(__fmul_rn(v.x, rec), w.x);
        v.y = __fmul_rn(__fmul_rn(v.y, rec), w.y);
        v.z = __fmul_rn(__fmul_rn(v.z, rec), w.z);
        v.w = __fmul_rn(__fmul_rn(v.w, rec), w.w);
        *px = v;
    }
    __syncthreads();
    return rec;
}

// Limb fragments of one token (slot 0 of pair 0; slot 1 written as zero)
// from a normalized row in shared memory, in the layout limb_prep_kernel
// writes.  One warp per group.
// With nws: the row in xs is not yet normalized; each value is taken as
// (x * rec) * w on read, the normalizing pass's rounding.
template <int FMT, int PADW = 0>
__device__ void limbs_from_smem(const float *xs, int groups, uint2 *limbs, float *efac, int2 *lsum,
                                const float *nws = nullptr, float rec = 1.0f) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int s = lane >> 3, q = (lane >> 1) & 3, h = lane & 1;
    for (int G = warp; G < groups; G += blockDim.x >> 5) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = limb_elem(FMT, s, q, h, i);
            const int k = padw<PADW>(G * kGroup + j);
            v[i] = xs[k];
            if (nws) v[i] = __fmul_rn(__fmul_rn(v[i], rec), nws[k]);
        }
        float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        const bool bad = __any_sync(0xffffffffu, !(isfinite(v[0]) && isfinite(v[1]) && isfinite(v[2]) && isfinite(v[3])));
        amax = warp_max(amax);
        int e = 0;
        if (amax > 0.0f && !bad) {
            int ex = 0;
            frexpf(amax, &ex);
            e = max(ex + 1, -100);
        }
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (!bad) {
            const int sh = 7 - e;
            const int sh1 = sh / 2, sh2 = sh - sh / 2;
            const float f1 = __int_as_float((127 + sh1) << 23), f2 = __int_as_float((127 + sh2) << 23);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float y = v[i] * f1 * f2;
#pragma unroll
                for (int l = 0; l < 4; ++l) {
                    const float r = rintf(y);
                    w[l] |= ((uint32_t)(int)r & 0xFFu) << (8 * i);
                    y = (y - r) * 128.0f;
                }
            }
        }
        uint32_t *dst = reinterpret_cast<uint32_t *>(limbs + (size_t)G * 128);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            dst[(s * 32 + l * 4 + q) * 2 + h] = w[l];
            dst[(s * 32 + (4 + l) * 4 + q) * 2 + h] = 0u;  // token slot 1: none
        }
        if constexpr (FMT == MF_TERNARY) {
            int sum[4];
            limb_sums64(w, sum);
            if (lane < 4) lsum[(size_t)G * 4 + lane] = lane < 2 ? make_int2(sum[2 * lane], sum[2 * lane + 1]) : make_int2(0, 0);
        }
        if (lane == 0) {
            efac[G] = bad ? __int_as_float(0x7fc00000) : __int_as_float((127 + e - 7) << 23);
            efac[(size_t)groups + G] = 0.0f;
        }
    }
}

// Half-group limbs of one token for a consumer of format LF: the 64 values
// sw[0..63] are weights 64*half .. 64*half + 63 of group G (hg = 2G + half)
// of the consumer's input, split with their own exponent (the split of
// limb_prep_kernel over 64 values instead of 128).  They fill the B columns
// of token slot `half` at the lane quads q = 2*half, 2*half + 1 (the only
// quads whose k slots hold these weights); the same quads of the other slot
// are written as zero, so the two CTAs of a group together write every word
// once.  efac[half][G] is the half's factor.  Lanes 0-15 of one warp.
template <int LF>
__device__ void swiglu_limbs_half(const float *sw, int hg, uint2 *lout, float *lefac, int2 *llsum, int lgroups) {
    const int lane = threadIdx.x & 31;
    const int G = hg >> 1, half = hg & 1;
    const bool act = lane < 16;
    const int s = (lane >> 2) & 3, q = 2 * half + ((lane >> 1) & 1), h = lane & 1;
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (act) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = limb_elem(LF, s, q, h, i);
            v[i] = sw[j - 64 * half];
        }
    }
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    const bool bad = __any_sync(0xffffffffu, !(isfinite(v[0]) && isfinite(v[1]) && isfinite(v[2]) && isfinite(v[3])));
    amax = warp_max(amax);
    int e = 0;
    if (amax > 0.0f && !bad) {
        int ex = 0;
        frexpf(amax, &ex);
        e = max(ex + 1, -100);
    }
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (!bad) {
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
    if (act) {
        uint32_t *dst = reinterpret_cast<uint32_t *>(lout + (size_t)G * 128);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            dst[(s * 32 + (4 * half + l) * 4 + q) * 2 + h] = w[l];
            dst[(s * 32 + (4 * (1 - half) + l) * 4 + q) * 2 + h] = 0u;
        }
    }
    if constexpr (LF == MF_TERNARY) {
        // Inactive lanes hold zero limbs: the sums cover this half's 64 values.
        int sum[4];
        limb_sums64(w, sum);
        if (lane < 2) llsum[(size_t)G * 4 + 2 * half + lane] = make_int2(sum[2 * lane], sum[2 * lane + 1]);
    }
    if (lane == 0) lefac[(size_t)half * lgroups + G] = bad ? __int_as_float(0x7fc00000) : __int_as_float((127 + e - 7) << 23);
}

// Argmax epilogue: `v`/`row` are this thread's candidate (row < 0: none);
// CTA partials are merged by the last CTA to arrive, which
// writes the greedy id (NaN if any logit is non-finite) and advances the
// position.  First strict maximum, as crates/backend-cpu/src/dense.rs:369-411.
__device__ void argmax_epilogue(const TcParams &p, float v, int row, bool poisoned) {
    __shared__ float s_v[32];
    __shared__ int s_i[32], s_p[32];
    __shared__ bool s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    auto merge = [](float &bv, int &bi, int &bp, float ov, int oi, int op) {
        bp |= op;
        if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
            bv = ov;
            bi = oi;
        }
    };
    float bv = v;
    int bi = row, bp = poisoned ? 1 : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        merge(bv, bi, bp, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o),
              __shfl_xor_sync(0xffffffffu, bp, o));
    if (lane == 0) {
        s_v[warp] = bv;
        s_i[warp] = bi;
        s_p[warp] = bp;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < nw; ++w) merge(bv, bi, bp, s_v[w], s_i[w], s_p[w]);
        float *mine = p.aparts + (size_t)blockIdx.x * 3;
        mine[0] = bv;
        mine[1] = __int_as_float(bi);
        mine[2] = __int_as_float(bp);
        __threadfence();
        s_last = atomicAdd(p.acount, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    bv = -INFINITY;
    bi = -1;
    bp = 0;
    // The merge keeps the first strict maximum whatever the order (ties go
    // to the lower row), so each thread takes CTAs tid, tid + blockDim.x, ...
    // with all of a batch's loads in flight before it merges them.
    constexpr int kLoads = 16;
    for (int c0 = tid; c0 < (int)gridDim.x; c0 += kLoads * blockDim.x) {
        float v[kLoads];
        int ix[kLoads], pz[kLoads];
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            const int c = c0 + u * (int)blockDim.x;
            if (c < (int)gridDim.x) {
                const float *pc = p.aparts + (size_t)c * 3;
                v[u] = __ldcg(pc);
                ix[u] = __float_as_int(__ldcg(pc + 1));
                pz[u] = __float_as_int(__ldcg(pc + 2));
            } else {
                v[u] = -INFINITY;
                ix[u] = -1;
                pz[u] = 0;
            }
        }
#pragma unroll
        for (int u = 0; u < kLoads; ++u) merge(bv, bi, bp, v[u], ix[u], pz[u]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        merge(bv, bi, bp, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o),
              __shfl_xor_sync(0xffffffffu, bp, o));
    __syncthreads();
    if (lane == 0) {
        s_v[warp] = bv;
        s_i[warp] = bi;
        s_p[warp] = bp;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < nw; ++w) merge(bv, bi, bp, s_v[w], s_i[w], s_p[w]);
        if (p.acand) {
            p.acand[0] = bv;
            p.acand[1] = bi < 0 ? -1.0f : (float)(bi + p.arow0);
            p.acand[2] = (bp || bi < 0) ? 1.0f : 0.0f;
        } else {
            *p.asampled = (bp || bi < 0) ? __int_as_float(0x7fc00000) : (float)bi;
            if (p.apos) *p.apos += 1;
        }
        *p.acount = 0u;
    }
}

// ---------------------------------------------------------------------
// Ternary / INT8 on the integer tensor cores.
//
// grid (row blocks, token blocks of 8); a CTA of rt * kw warps covers rt
// 16-row tiles over the whole K: warp w serves tile w % rt and K part
// w / rt (p.kch groups).  Each warp first issues every load of its part
// (codes, scales, limb fragments) in batches of U groups, then runs the
// MMAs; the K parts of a tile are added in part order through shared
// memory.  Tiles of a pair-rows call come from A then B.
// ---------------------------------------------------------------------
// Threads per CTA: the one-token ternary SwiGLU pair with the normalizing
// prologue (the decode FFN; 4 row tiles x 4 K parts of 4 groups) and the
// one-token ternary single projection of a plain input (w2; K parts of 4
// groups) run 16 warps, twice the warps of the other variants, to hide
// their dependent latencies; every other variant runs 8.
template <int FMT, int MODE, int UB, int PRO>
constexpr int imma_threads() {
    return FMT == MF_TERNARY && UB == 4 && ((MODE == kSwigluPair && PRO == kNorm) || (MODE == kSingle && PRO == kFromGlobal))
               ? 512 : 256;
}

// LT: ternary codes in the lane-tiled (LUT2) layout.
template <int FMT, int MODE, int NCB, int UB, int PRO, bool LT = false>
__global__ void __launch_bounds__(imma_threads<FMT, MODE, UB, PRO>()) packed_gemv_imma_kernel(const TcParams p) {
    constexpr int J = MODE == kSwigluPair ? 2 : 1;
    constexpr int GB = FMT == MF_INT8 ? 128 : 32;                   // code bytes per row per group
    constexpr int U = UB / (NCB > 2 ? 2 : 1) > 0 ? UB / (NCB > 2 ? 2 : 1) : 1;  // groups per load batch
    extern __shared__ __align__(16) float red[];   // [kw][rt][J][16][8], then (kNorm) x, limbs, factors
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int rt = p.rt, kw = p.kw;
    const int slot = warp % rt, kp = warp / rt;
    const int vtile = blockIdx.x * rt + slot;
    const bool tile_ok = vtile < p.vtiles;
    const int tblk = blockIdx.y;
    const int t0 = tblk * kTokBlock;
    const int tb = min(kTokBlock, p.T - t0);
    const int cb0 = t0 / 2;
    const int g0 = kp * p.kch;
    const int ng = tile_ok ? max(0, min(p.kch, p.groups - g0)) : 0;
    const int row_bytes = p.K / (FMT == MF_INT8 ? 1 : 4);
    int mat = 0, r0 = 0, nrows = p.N;
    tile_map(p, MODE, vtile, 16, mat, r0, nrows);
    const int rg = r0 + g, rg8 = r0 + g + 8;
    const bool ok_g = rg < nrows, ok_g8 = rg8 < nrows;
    // Limb weights of MMA columns 2q, 2q+1 (ternary dots carry a factor 64).
    const float lw0 = ((q & 1) ? 0x1p-14f : 1.0f) * (FMT == MF_TERNARY ? 0x1p-6f : 1.0f);
    const float lw1 = lw0 * 0x1p-7f;

    float acc[J][NCB][2];
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb) acc[j][cb][0] = acc[j][cb][1] = 0.0f;

    uint4 cv[J][U][2][FMT == MF_INT8 ? 2 : 1];
    float sc[J][U][2];
    // The normalizing SwiGLU pair (the decode FFN) stages its group scales in
    // shared memory instead of registers, so a CTA fits on an SM beside the
    // NF4 projection before it and streams its codes before the wait.
    constexpr bool SCS = MODE == kSwigluPair && PRO == kNorm;
    constexpr int kScsStride = 9;   // up to 8 groups per K part (K <= 8192), padded
    auto load_codes = [&](int gb) {
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int m = J == 2 ? j : mat;
            const uint8_t *codes = codes_of(p, m);
            const float *scales = scales_of(p, m);
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
                    } else if constexpr (LT) {
                        // One 16-byte load holds both rows (rows come in whole tiles).
                        if (r == 0) {
                            const uint4 c4 = ok ? ld_stream_u4(codes + (((size_t)(r0 >> 4) * p.groups + G) * 32 + lane) * 16)
                                                : make_uint4(0x55555555u, 0x55555555u, 0x55555555u, 0x55555555u);
                            cv[j][u][0][0] = make_uint4(c4.x, c4.y, 0, 0);
                            cv[j][u][1][0] = make_uint4(c4.z, c4.w, 0, 0);
                        }
                    } else {
                        const uint2 c2 = ok ? ld_stream_u2(cg + (size_t)row * row_bytes + 8 * q)
                                            : make_uint2(0x55555555u, 0x55555555u);  // weight 0
                        cv[j][u][r][0] = make_uint4(c2.x, c2.y, 0, 0);
                    }
                    if constexpr (!SCS) sc[j][u][r] = ok ? ld_stream_f32(scales + (size_t)row * p.groups + G) : 0.0f;
                }
            }
        }
    };
    // Codes and scales are constants: the first batch streams in before the
    // wait for the previous kernel (whose output is the input row or limbs).
    load_codes(0);
    // kNorm layout after the reduction area: x [K], limbs, factors, then the
    // norm weight [K] (16-byte aligned), copied in before the wait.
    // x and the norm weight are staged with 2 floats of padding per 32
    // (padw<2>): the limb split's fragment reads are then conflict-free.
    float *xs = red + (size_t)kw * rt * J * 16 * kTokBlock;
    uint2 *ls = reinterpret_cast<uint2 *>(xs + imma_row_floats(p.K));
    float *es = reinterpret_cast<float *>(ls + (size_t)p.groups * 128);
    int2 *lss = reinterpret_cast<int2 *>(es + ((2 * p.groups + 3) & ~3));
    float *nws = reinterpret_cast<float *>(lss + (size_t)p.groups * 4);
    if constexpr (PRO == kNorm) nw_prefetch_pad2(p, nws);
    // SCS: this warp's scales [J][16 rows][kScsStride], after the norm weight;
    // the prologue's cp.async wait and barrier complete them.
    float *scs = nws + imma_row_floats(p.K) + (size_t)warp * J * 16 * kScsStride;
    if constexpr (SCS) {
        for (int e = lane; e < J * 16 * 8; e += 32) {
            const int j = e / (16 * 8), rr = (e / 8) % 16, u = e % 8;
            const int row = r0 + rr;
            float *dst = scs + (j * 16 + rr) * kScsStride + u;
            if (u < ng && row < nrows) {
                const float *src = scales_of(p, j) + (size_t)row * p.groups + g0 + u;
                const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
            } else {
                *dst = 0.0f;
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    pdl_wait();
    pdl_trigger();
    const uint2 *limbs = p.limbs;
    const float *efac = p.efac;
    const int2 *lsum = p.lsum;
    int pairs = p.pairs;
    if constexpr (PRO == kNorm) {
        // Stage and sum; then every warp forms the reciprocal itself and
        // normalizes while it splits its groups into limbs (two barriers).
        __shared__ float red_ss[32];
        float ss = warp_sum(norm_stage<2>(p, xs));
        if (lane == 0) red_ss[warp] = ss;
        asm volatile("cp.async.wait_all;" ::: "memory");   // this thread's norm-weight (and scale) copies
        __syncthreads();
        if (p.nw) limbs_from_smem<FMT, 2>(xs, p.groups, ls, es, lss, nws, norm_reciprocal(red_ss, p.K, p.neps));
        else limbs_from_smem<FMT, 2>(xs, p.groups, ls, es, lss);
        __syncthreads();
        limbs = ls;
        efac = es;
        lsum = lss;
        pairs = 1;
    }

    // Limb fragments are loaded HB groups at a time (the whole batch for
    // most variants; halves for the staged-scale SwiGLU pair, which keeps its
    // registers low enough to share an SM with the kernel before it).
    constexpr int HB = SCS && U >= 4 ? 2 : U;
    for (int gb = 0; gb < ng; gb += U) {
        if (gb) load_codes(gb);
#pragma unroll
        for (int hb = 0; hb < U; hb += HB) {
        uint2 bfr[HB][NCB][4];
        float ef[HB][NCB];
        // Ternary limb-sum offsets: loaded with the fragments for one token
        // pair, just before their MMAs for more (registers).
        int2 lsv[HB][1];
#pragma unroll
        for (int uh = 0; uh < HB; ++uh) {
            const int u = hb + uh;
            const int G = g0 + min(gb + u, ng - 1);
#pragma unroll
            for (int cb = 0; cb < NCB; ++cb) {
                if (cb0 + cb < pairs) {
                    const uint2 *src = limbs + ((size_t)(cb0 + cb) * p.groups + G) * 128;
#pragma unroll
                    for (int s = 0; s < 4; ++s) bfr[uh][cb][s] = src[s * 32 + g * 4 + q];
                    ef[uh][cb] = efac[(size_t)(t0 + 2 * cb + (q >> 1)) * p.groups + G];
                    if constexpr (FMT == MF_TERNARY && NCB == 1) lsv[uh][0] = lsum[((size_t)cb0 * p.groups + G) * 4 + q];
                } else {
#pragma unroll
                    for (int s = 0; s < 4; ++s) bfr[uh][cb][s] = make_uint2(0u, 0u);
                    ef[uh][cb] = 0.0f;
                    if constexpr (NCB == 1) lsv[uh][0] = make_int2(0, 0);
                }
            }
        }
#pragma unroll
        for (int uh = 0; uh < HB; ++uh) {
            const int u = hb + uh;
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
                        ternary_u8x4(cv[j][u][r][0].x, dst);
                        ternary_u8x4(cv[j][u][r][0].y, dst + 4);
                    }
                }
#pragma unroll
                for (int cb = 0; cb < NCB; ++cb) {
                    int d[4] = {0, 0, 0, 0};
                    int2 lv = make_int2(0, 0);
                    if constexpr (FMT == MF_TERNARY) {
                        if constexpr (NCB == 1) lv = lsv[uh][0];
                        else if (cb0 + cb < pairs) lv = lsum[((size_t)(cb0 + cb) * p.groups + g0 + gb + u) * 4 + q];
                    }
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint32_t a[4] = {wa[2 * s], wb[2 * s], wa[2 * s + 1], wb[2 * s + 1]};
                        if constexpr (FMT == MF_INT8) imma16832(d, a, bfr[uh][cb][s].x, bfr[uh][cb][s].y);
                        else if (s == 0) imma16832_u_c(d, a, bfr[uh][cb][s].x, bfr[uh][cb][s].y, lv.x, lv.y);
                        else imma16832_u(d, a, bfr[uh][cb][s].x, bfr[uh][cb][s].y);
                    }
                    const float vg = fmaf(__int2float_rn(d[1]), lw1, __int2float_rn(d[0]) * lw0) * ef[uh][cb];
                    const float vg8 = fmaf(__int2float_rn(d[3]), lw1, __int2float_rn(d[2]) * lw0) * ef[uh][cb];
                    if constexpr (SCS) {
                        acc[j][cb][0] = fmaf(vg, scs[(j * 16 + g) * kScsStride + gb + u], acc[j][cb][0]);
                        acc[j][cb][1] = fmaf(vg8, scs[(j * 16 + g + 8) * kScsStride + gb + u], acc[j][cb][1]);
                    } else {
                        acc[j][cb][0] = fmaf(vg, sc[j][u][0], acc[j][cb][0]);
                        acc[j][cb][1] = fmaf(vg8, sc[j][u][1], acc[j][cb][1]);
                    }
                }
            }
        }
        }
    }
    // Lanes q and q^1 hold the low and high limb pairs of one token; lane
    // (g, q even) then owns tokens 2cb + q/2 of rows g and g + 8.
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
        for (int cb = 0; cb < NCB; ++cb)
#pragma unroll
            for (int r = 0; r < 2; ++r) acc[j][cb][r] += __shfl_xor_sync(0xffffffffu, acc[j][cb][r], 1);
    if (p.split_halves) {
        // Half-group limbs: slot 1 holds the upper halves of the same token.
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int cb = 0; cb < NCB; ++cb)
#pragma unroll
                for (int r = 0; r < 2; ++r) acc[j][cb][r] += __shfl_xor_sync(0xffffffffu, acc[j][cb][r], 2);
    }
    auto red_at = [&](int part, int sl, int j, int row16, int t) -> float & {
        return red[((((size_t)part * rt + sl) * J + j) * 16 + row16) * kTokBlock + t];
    };
    if (!(q & 1)) {
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int cb = 0; cb < NCB; ++cb) {
                const int t = 2 * cb + (q >> 1);
                red_at(kp, slot, j, g, t) = acc[j][cb][0];
                red_at(kp, slot, j, g + 8, t) = acc[j][cb][1];
            }
    }
    __syncthreads();
    // Sum the K parts in order; one thread per (tile slot, row, token).
    float best = -INFINITY;
    int best_row = -1;
    bool poisoned = false;
    for (int e = threadIdx.x; e < rt * 16 * kTokBlock; e += blockDim.x) {
        const int sl = e / (16 * kTokBlock), row16 = (e / kTokBlock) % 16, t = e % kTokBlock;
        const int vt = blockIdx.x * rt + sl;
        if (vt >= p.vtiles || t >= tb) continue;
        int m, rr0, nr;
        tile_map(p, MODE, vt, 16, m, rr0, nr);
        const int row = rr0 + row16;
        if (row >= nr) continue;
        float v[J];
#pragma unroll
        for (int j = 0; j < J; ++j) {
            float a = red_at(0, sl, j, row16, t);
            for (int part = 1; part < kw; ++part) a += red_at(part, sl, j, row16, t);
            v[j] = a;
        }
        store_out<MODE>(p, m, t0 + t, row, v[0], v[J - 1]);
        if constexpr (MODE == kSwigluPair && PRO == kNorm) {
            // The staged input row is no longer read: it holds the outputs.
            if (p.lout) xs[sl * 16 + row16] = silu_mul(v[0], v[J - 1]);
        }
        if (MODE == kSingle && p.aparts) {
            if (!isfinite(v[0])) poisoned = true;
            else if (best_row < 0 || v[0] > best || (v[0] == best && row < best_row)) {
                best = v[0];
                best_row = row;
            }
        }
    }
    if (MODE == kSingle && p.aparts) argmax_epilogue(p, best, best_row, poisoned);
    if constexpr (MODE == kSwigluPair && PRO == kNorm) {
        // The CTA's rt * 16 outputs (a multiple of 64, aligned) as the
        // consumer's half-group limbs, one warp per half group.
        if (p.lout) {
            __syncthreads();
            const int halves = p.rt * 16 / 64;
            if (warp < halves) {
                const int hg = blockIdx.x * halves + warp;
                if (p.lfmt == MF_INT8) swiglu_limbs_half<MF_INT8>(xs + warp * 64, hg, p.lout, p.lefac, p.llsum, p.lgroups);
                else swiglu_limbs_half<MF_TERNARY>(xs + warp * 64, hg, p.lout, p.lefac, p.llsum, p.lgroups);
            }
        }
    }
}

// ---------------------------------------------------------------------
// One-token single projection of a matrix far larger than one wave (the
// LM head): persistent CTAs of 8 warps.  Warp w takes K part w (KCH groups)
// of 16-row tiles blockIdx.x, blockIdx.x + gridDim.x, ...; the next DEPTH - 1
// tiles' codes and scales are in flight while one tile's MMAs run, and the
// limb fragments of the part stay in registers for every tile.  The 8 parts
// of a tile are added in part order through a double-buffered shared array
// (one barrier per tile); the argmax candidate carries across tiles.
// ---------------------------------------------------------------------
template <int FMT, int KCH, int DEPTH>
__global__ void __launch_bounds__(256, 2) packed_gemv_stream_kernel(const TcParams p) {
    static_assert(DEPTH % 2 == 0, "tiles alternate between the two halves of the part-sum array");
    constexpr int GB = FMT == MF_INT8 ? 128 : 32;   // code bytes per row per group
    constexpr int CW = FMT == MF_INT8 ? 2 : 1;      // uint4 words per row per group per lane
    __shared__ float part[2][8][16];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int g0 = warp * KCH;
    const int ng = max(0, min(KCH, p.groups - g0));
    const int row_bytes = p.K / (FMT == MF_INT8 ? 1 : 4);
    const float lw0 = ((q & 1) ? 0x1p-14f : 1.0f) * (FMT == MF_TERNARY ? 0x1p-6f : 1.0f);
    const float lw1 = lw0 * 0x1p-7f;

    uint4 cv[DEPTH][KCH][2][CW];
    float sc[DEPTH][KCH][2];
    auto load_tile = [&](int vt, uint4 (&c)[KCH][2][CW], float (&s)[KCH][2]) {
        const bool tok = vt < p.row_tiles;
#pragma unroll
        for (int u = 0; u < KCH; ++u) {
            const int G = g0 + u;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int row = vt * 16 + g + 8 * r;
                const bool ok = tok && u < ng && row < p.N;
                const uint8_t *cg = p.codes_a + (size_t)row * row_bytes + (size_t)G * GB;
                if constexpr (FMT == MF_INT8) {
                    c[u][r][0] = ok ? ld_stream_u4(cg + 32 * q) : make_uint4(0, 0, 0, 0);
                    c[u][r][1] = ok ? ld_stream_u4(cg + 32 * q + 16) : make_uint4(0, 0, 0, 0);
                } else {
                    const uint2 c2 = ok ? ld_stream_u2(cg + 8 * q) : make_uint2(0x55555555u, 0x55555555u);
                    c[u][r][0] = make_uint4(c2.x, c2.y, 0, 0);
                }
                s[u][r] = ok ? ld_stream_f32(p.scales_a + (size_t)row * p.groups + G) : 0.0f;
            }
        }
    };
    int vt = blockIdx.x;
    // Constants: the first DEPTH - 1 tiles stream in before the wait.
#pragma unroll
    for (int b = 0; b < DEPTH - 1; ++b) load_tile(vt + b * (int)gridDim.x, cv[b], sc[b]);
    pdl_wait();
    pdl_trigger();
    uint2 bfr[KCH][4];
    float ef[KCH];
    int2 lsv[KCH];
#pragma unroll
    for (int u = 0; u < KCH; ++u) {
        const bool has = u < ng;   // a part past K (K < 8 * KCH groups) has no limbs
        const int G = has ? g0 + u : 0;
#pragma unroll
        for (int st = 0; st < 4; ++st) bfr[u][st] = has ? p.limbs[(size_t)G * 128 + st * 32 + g * 4 + q] : make_uint2(0u, 0u);
        ef[u] = has ? p.efac[(size_t)(q >> 1) * p.groups + G] : 0.0f;
        lsv[u] = (FMT == MF_TERNARY && has) ? p.lsum[(size_t)G * 4 + q] : make_int2(0, 0);
    }
    float best = -INFINITY;
    int best_row = -1;
    bool poisoned = false;
    auto process = [&](int tile, const uint4 (&c)[KCH][2][CW], const float (&s)[KCH][2], int pb) {
        float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
        for (int u = 0; u < KCH; ++u) {
            uint32_t wa[8], wb[8];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                uint32_t *dst = r ? wb : wa;
                if constexpr (FMT == MF_INT8) {
                    const uint4 a0 = c[u][r][0], a1 = c[u][r][1];
                    dst[0] = a0.x; dst[1] = a0.y; dst[2] = a0.z; dst[3] = a0.w;
                    dst[4] = a1.x; dst[5] = a1.y; dst[6] = a1.z; dst[7] = a1.w;
                } else {
                    ternary_u8x4(c[u][r][0].x, dst);
                    ternary_u8x4(c[u][r][0].y, dst + 4);
                }
            }
            int d[4] = {0, 0, 0, 0};
#pragma unroll
            for (int st = 0; st < 4; ++st) {
                const uint32_t a[4] = {wa[2 * st], wb[2 * st], wa[2 * st + 1], wb[2 * st + 1]};
                if constexpr (FMT == MF_INT8) imma16832(d, a, bfr[u][st].x, bfr[u][st].y);
                else if (st == 0) imma16832_u_c(d, a, bfr[u][st].x, bfr[u][st].y, lsv[u].x, lsv[u].y);
                else imma16832_u(d, a, bfr[u][st].x, bfr[u][st].y);
            }
            const float vg = fmaf(__int2float_rn(d[1]), lw1, __int2float_rn(d[0]) * lw0) * ef[u];
            const float vg8 = fmaf(__int2float_rn(d[3]), lw1, __int2float_rn(d[2]) * lw0) * ef[u];
            acc0 = fmaf(vg, s[u][0], acc0);
            acc1 = fmaf(vg8, s[u][1], acc1);
        }
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        if (q == 0) {
            part[pb][warp][g] = acc0;
            part[pb][warp][g + 8] = acc1;
        }
        __syncthreads();   // part[pb] was last read two tiles ago, before the previous barrier
        if (threadIdx.x < 16) {
            const int row = tile * 16 + threadIdx.x;
            if (row < p.N) {
                float v = part[pb][0][threadIdx.x];
#pragma unroll
                for (int w = 1; w < 8; ++w) v += part[pb][w][threadIdx.x];
                p.out_a[row] = v;
                if (p.aparts) {
                    if (!isfinite(v)) poisoned = true;
                    else if (best_row < 0 || v > best || (v == best && row < best_row)) {
                        best = v;
                        best_row = row;
                    }
                }
            }
        }
    };
    // DEPTH - 1 tiles ahead are in flight while one is computed; the buffer
    // index rotates at compile time (the loop body is unrolled DEPTH times).
    while (vt < p.row_tiles) {
#pragma unroll
        for (int b = 0; b < DEPTH; ++b) {
            if (vt < p.row_tiles) {
                load_tile(vt + (DEPTH - 1) * (int)gridDim.x, cv[(b + DEPTH - 1) % DEPTH], sc[(b + DEPTH - 1) % DEPTH]);
                process(vt, cv[b], sc[b], b & 1);
                vt += gridDim.x;
            }
        }
    }
    if (p.aparts) argmax_epilogue(p, best, best_row, poisoned);
}

// ---------------------------------------------------------------------
// One token through a ternary matrix of many waves, K = 128 * KG: every warp
// owns whole 16-row tiles over the full K, so no warp waits on another and
// no tile needs a cross-warp sum.  Lane (g, q) holds its 8 code bytes of
// rows g and g + 8 in every group of the next tile in registers (one
// 16-byte load per group in the lane-tiled layout, two 8-byte loads in the
// raw one) while the current tile's MMAs run.  Each CTA splits the input
// row into limbs itself (shared memory, once), so no limb pass runs.  The
// group scales of a tile come as one 16-byte load per row and lane (groups
// 4q .. 4q + 3) and reach the lanes that promote them by shuffles.
// ---------------------------------------------------------------------
template <int KG, bool SWI, bool LT>
__global__ void __launch_bounds__(256, 1) packed_gemv_tile_kernel(const TcParams p) {
    static_assert(KG == 4 || KG == 8 || KG == 16, "K of 512, 1024 or 2048");
    constexpr int NSV = KG / 4;                  // 16-byte scale vectors per row
    __shared__ __align__(16) float s_x[KG * 128 + KG * 8];   // input row, padw<2>
    __shared__ __align__(16) uint2 s_limbs[KG * 128];
    __shared__ float s_ef[2 * KG];
    __shared__ int2 s_lsum[KG * 4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int row_bytes = KG * 32;
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    const float lw0 = ((q & 1) ? 0x1p-14f : 1.0f) * 0x1p-6f;
    const float lw1 = lw0 * 0x1p-7f;

    auto load_group = [&](int tile, int u) -> uint4 {
        const bool ok = tile < p.row_tiles;
        if constexpr (LT)
            return ok ? ld_stream_u4(p.codes_a + (((size_t)tile * KG + u) * 32 + lane) * 16)
                      : make_uint4(0x55555555u, 0x55555555u, 0x55555555u, 0x55555555u);
        const int r0 = tile * 16;
        const bool oka = ok && r0 + g < p.N, okb = ok && r0 + g + 8 < p.N;
        const uint2 a = oka ? ld_stream_u2(p.codes_a + (size_t)(r0 + g) * row_bytes + 32 * u + 8 * q)
                            : make_uint2(0x55555555u, 0x55555555u);
        const uint2 b = okb ? ld_stream_u2(p.codes_a + (size_t)(r0 + g + 8) * row_bytes + 32 * u + 8 * q)
                            : make_uint2(0x55555555u, 0x55555555u);
        return make_uint4(a.x, a.y, b.x, b.y);
    };
    auto load_scales = [&](int tile, float4 (&sv)[2]) {
        const bool ok = tile < p.row_tiles;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int row = tile * 16 + g + 8 * r;
            sv[r] = (ok && row < p.N && q < NSV) ? ld_stream_f4(p.scales_a + (size_t)row * KG + 4 * q)
                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    int tile = blockIdx.x * (blockDim.x >> 5) + warp;
    // One tile of codes in registers; each group's slot is refilled with the
    // next tile's group as soon as it is decoded, so about one tile per warp
    // stays in flight.
    uint4 c[KG];
    float4 sv[2], svn[2];
#pragma unroll
    for (int u = 0; u < KG; ++u) c[u] = load_group(tile, u);   // constants: before the wait
    load_scales(tile, sv);
    pdl_wait();
    pdl_trigger();
    // The input row (or silu(gate) * up) in shared memory, then its limbs,
    // factors and limb sums: one warp per group.
    for (int e = threadIdx.x; e < KG * 32; e += blockDim.x) {
        float4 v;
        if constexpr (SWI) {
            const float4 a = reinterpret_cast<const float4 *>(p.gate)[e], b = reinterpret_cast<const float4 *>(p.up)[e];
            v = make_float4(silu_mul(a.x, b.x), silu_mul(a.y, b.y), silu_mul(a.z, b.z), silu_mul(a.w, b.w));
        } else {
            v = reinterpret_cast<const float4 *>(p.x)[e];
        }
        float *dst = s_x + padw<2>(4 * e);
        reinterpret_cast<float2 *>(dst)[0] = make_float2(v.x, v.y);
        reinterpret_cast<float2 *>(dst)[1] = make_float2(v.z, v.w);
    }
    __syncthreads();
    limbs_from_smem<MF_TERNARY, 2>(s_x, KG, s_limbs, s_ef, s_lsum);
    __syncthreads();

    float best = -INFINITY;
    int best_row = -1;
    bool poisoned = false;
    while (tile < p.row_tiles) {
        const int next = tile + nwarps;
        load_scales(next, svn);
        float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
        for (int u = 0; u < KG; ++u) {
            uint32_t wa[8], wb[8];
            ternary_u8x4(c[u].x, wa);
            ternary_u8x4(c[u].y, wa + 4);
            ternary_u8x4(c[u].z, wb);
            ternary_u8x4(c[u].w, wb + 4);
            c[u] = load_group(next, u);
            const uint2 *bf = s_limbs + u * 128 + g * 4 + q;
            const int2 ls = s_lsum[u * 4 + q];
            int d[4];
            {
                const uint32_t a[4] = {wa[0], wb[0], wa[1], wb[1]};
                const uint2 b = bf[0];
                imma16832_u_c(d, a, b.x, b.y, ls.x, ls.y);
            }
#pragma unroll
            for (int st = 1; st < 4; ++st) {
                const uint32_t a[4] = {wa[2 * st], wb[2 * st], wa[2 * st + 1], wb[2 * st + 1]};
                const uint2 b = bf[st * 32];
                imma16832_u(d, a, b.x, b.y);
            }
            const float ef = s_ef[(q >> 1) * KG + u];
            // Scale of group u for rows g and g + 8: lane (g, u / 4), element u % 4.
            const int src = (lane & ~3) | (u >> 2);
            const float sa = __shfl_sync(0xffffffffu, (u & 3) == 0 ? sv[0].x : (u & 3) == 1 ? sv[0].y : (u & 3) == 2 ? sv[0].z : sv[0].w, src);
            const float sb = __shfl_sync(0xffffffffu, (u & 3) == 0 ? sv[1].x : (u & 3) == 1 ? sv[1].y : (u & 3) == 2 ? sv[1].z : sv[1].w, src);
            const float vg = fmaf(__int2float_rn(d[1]), lw1, __int2float_rn(d[0]) * lw0) * ef;
            const float vg8 = fmaf(__int2float_rn(d[3]), lw1, __int2float_rn(d[2]) * lw0) * ef;
            acc0 = fmaf(vg, sa, acc0);
            acc1 = fmaf(vg8, sb, acc1);
        }
        // Lanes q and q ^ 1 hold the two limb pairs; q = 2, 3 hold the empty
        // second token slot.
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        if (q == 0) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int row = tile * 16 + g + 8 * r;
                const float v = r ? acc1 : acc0;
                if (row < p.N) {
                    p.out_a[row] = v;
                    if (!isfinite(v)) poisoned = true;
                    else if (best_row < 0 || v > best || (v == best && row < best_row)) {
                        best = v;
                        best_row = row;
                    }
                }
            }
        }
        sv[0] = svn[0];
        sv[1] = svn[1];
        tile = next;
    }
    if (p.aparts) argmax_epilogue(p, best, best_row, poisoned);
}

// ---------------------------------------------------------------------
// NF4 (FP32).  grid (row blocks, token blocks of TOK); a CTA of rw * kw
// warps covers rw * R rows over the whole K: warp w serves rows
// (w % rw) * R .. + R - 1 of the block and K part w / rw, 1024 weights
// wide; lane l reads bytes [16l, 16l + 16) of the part in each row and keeps
// the 32 matching activations in registers.  Every global load is issued
// before the level table is built; parts are added in order through shared
// memory.
// ---------------------------------------------------------------------

constexpr int kNf4PartWeights = 1024;

// Shared floats of the NF4 GEMV's staged input row: the normalizing
// prologue keeps x (pad32 layout) and the norm weight; any other single
// token keeps x.
template <int PRO, int TOK, bool SWI>
__host__ __device__ inline size_t nf4_x_floats(size_t K) {
    return PRO == kNorm ? padded_row_floats(K) + K : TOK == 1 ? padded_row_floats(K) : 0;
}

// The one-token plain-input single projection (the decode out_proj / o)
// runs 16 warps of 2 rows each, the normalizing q/k/v triple 16 warps of 3
// rows; every other variant runs 8.
template <int MODE, int TOK, int R, int PRO>
constexpr int nf4_threads() {
    if (TOK == 1 && R == 8 && MODE == kConv) return 384;   // 12 warps of 8 rows (the conv in_proj)
    return TOK == 1 && ((R == 2 && MODE == kSingle && PRO == kFromGlobal) || (R == 3 && MODE == kTriple && PRO == kNorm))
               ? 512 : 256;
}

template <int MODE, int TOK, int R, bool SWI_IN, int PRO>
__global__ void __launch_bounds__(nf4_threads<MODE, TOK, R, PRO>()) packed_gemv_nf4_kernel(const TcParams p) {
    constexpr int J = MODE == kSwigluPair ? 2 : 1;
    extern __shared__ __align__(16) unsigned char smem_nf4[];
    float2 *lut = reinterpret_cast<float2 *>(smem_nf4);                              // [256][16]
    float *red = reinterpret_cast<float *>(smem_nf4 + 256 * 16 * sizeof(float2));  // [kw][rw*R][J][TOK]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, l16 = lane & 15;
    const int rw = p.rt, kw = p.kw;
    const int wr = warp % rw, kp = warp / rw;
    const int tblk = blockIdx.y;
    const int t0 = tblk * TOK;
    const int tb = min(TOK, p.T - t0);
    const int rows_cta = rw * R;
    const int vrows = MODE == kPairRows ? 2 * p.N : MODE == kTriple ? p.N + 2 * p.N2 : MODE == kConv ? 3 * p.N : p.N;
    const int cch = rows_cta / 3;   // kConv: channels per CTA (B, C and x rows of each)
    const int nblocks = (vrows + rows_cta - 1) / rows_cta;
    const int iters = (nblocks + gridDim.x - 1) / gridDim.x;   // uniform across the CTA
    const int row_bytes = p.K / 2;
    const int k0 = kp * kNf4PartWeights + 32 * lane;  // this lane's 32 weights of each row
    const bool kok = k0 < p.K;
    const int G = k0 / kGroup;

    auto load_rows = [&](int it, uint4 (&cw)[J][R], float (&sc)[J][R]) {
        const int vr0 = (blockIdx.x + it * gridDim.x) * rows_cta + wr * R;
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int i = 0; i < R; ++i) {
                const int vr = vr0 + i;
                int m = 0, row = vr, nr = p.N;
                if constexpr (MODE == kConv) {
                    // Local row l of block blk: projection l / cch of channel blk * cch + l % cch.
                    const int blk = blockIdx.x + it * gridDim.x, l = wr * R + i;
                    row = (l / cch) * p.N + blk * cch + l % cch;
                    nr = 3 * p.N;
                } else if (J == 2) {
                    m = j;
                } else {
                    tile_map(p, MODE, vr, 1, m, row, nr);
                }
                const bool ok = kok && it < iters && vr < vrows && row < nr;
                const uint8_t *codes = codes_of(p, m);
                const float *scales = scales_of(p, m);
                cw[j][i] = ok ? ld_stream_u4(codes + (size_t)row * row_bytes + k0 / 2)
                              : make_uint4(0x77777777u, 0x77777777u, 0x77777777u, 0x77777777u);  // level 0
                sc[j][i] = ok ? ld_stream_f32(scales + (size_t)row * p.groups + G) : 0.0f;
            }
    };
    uint4 cw[J][R], cn[J][R];
    float sc[J][R], sn[J][R];
    load_rows(0, cw, sc);
    // kNorm: x [K + K/8] (pad32 layout), then the norm weight [K].
    float *xs = red + (size_t)kw * rows_cta * J * TOK;
    float *nws = xs + padded_row_floats(p.K);
    if constexpr (PRO == kNorm) nw_prefetch(p, nws);
    // kConv (one pass, block = blockIdx.x): thread e < cch owns channel
    // blockIdx.x * cch + e; its taps and old history rows were written by
    // kernels that completed before this one launched, so they load now.
    float ckw[kConvMaxWidth], chold[kConvMaxWidth];
    if constexpr (MODE == kConv) {
        const int ch = blockIdx.x * cch + tid;
        if (tid < cch && ch < p.N) {
#pragma unroll
            for (int i = 0; i < kConvMaxWidth; ++i) {
                if (i >= p.cwidth) break;
                ckw[i] = p.ckern[(size_t)ch * p.cwidth + i];
                if (i < p.cwidth - 1) chold[i] = p.chist[(size_t)i * p.N + ch];
            }
        }
    }
    // The level table is a constant too: built before the wait.
    for (int e = tid; e < 256 * 16; e += blockDim.x) {
        const int b = e >> 4;
        lut[e] = make_float2(kNf4Levels[b & 15], kNf4Levels[b >> 4]);
    }
    pdl_wait();  // codes and scales are constants; x comes from the previous kernel
    pdl_trigger();
    float xv[TOK][32];
    if constexpr (PRO == kNorm) {
        // One token: x = rmsnorm of the prologue's row, built in shared memory.
        norm_prologue(p, xs, nws);
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            const float4 v4 = kok ? *reinterpret_cast<const float4 *>(xs + pad32(k0) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            xv[0][i] = v4.x;
            xv[0][i + 1] = v4.y;
            xv[0][i + 2] = v4.z;
            xv[0][i + 3] = v4.w;
        }
    } else if constexpr (TOK == 1) {
        // One plain token (or silu(gate) * up of one): the row is staged in
        // shared memory by coalesced 16-byte loads (pad32 layout), then each
        // lane reads its 32 values.
        const size_t row = (size_t)t0 * p.K;
        for (int e = tid; e < p.K / 4; e += blockDim.x) {
            float4 v;
            if constexpr (SWI_IN) {
                const float4 g4 = reinterpret_cast<const float4 *>(p.gate + row)[e];
                const float4 u4 = reinterpret_cast<const float4 *>(p.up + row)[e];
                v = make_float4(silu_mul(g4.x, u4.x), silu_mul(g4.y, u4.y), silu_mul(g4.z, u4.z), silu_mul(g4.w, u4.w));
            } else {
                v = reinterpret_cast<const float4 *>(p.x + row)[e];
            }
            *reinterpret_cast<float4 *>(xs + pad32(4 * e)) = v;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            const float4 v4 = kok ? *reinterpret_cast<const float4 *>(xs + pad32(k0) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            xv[0][i] = v4.x;
            xv[0][i + 1] = v4.y;
            xv[0][i + 2] = v4.z;
            xv[0][i + 3] = v4.w;
        }
    } else {
#pragma unroll
    for (int t = 0; t < TOK; ++t) {
        const size_t base = (size_t)(t0 + min(t, tb - 1)) * p.K + k0;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            if (!kok) {
                xv[t][i] = xv[t][i + 1] = xv[t][i + 2] = xv[t][i + 3] = 0.0f;
            } else if constexpr (SWI_IN) {
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
    }
    __syncthreads();   // the level table (built before the wait) is complete
    for (int it = 0; it < iters; ++it) {
        if (it + 1 < iters) load_rows(it + 1, cn, sn);  // next block's codes stream in meanwhile
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int i = 0; i < R; ++i) {
                const uint32_t words[4] = {cw[j][i].x, cw[j][i].y, cw[j][i].z, cw[j][i].w};
                float part[TOK];
#pragma unroll
                for (int t = 0; t < TOK; ++t) part[t] = 0.0f;
#pragma unroll
                for (int w = 0; w < 4; ++w)
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const float2 lv = lut[__byte_perm(words[w], 0u, 0x4440 + b) * 16 + l16];
#pragma unroll
                        for (int t = 0; t < TOK; ++t) {
                            part[t] = fmaf(lv.x, xv[t][8 * w + 2 * b], part[t]);
                            part[t] = fmaf(lv.y, xv[t][8 * w + 2 * b + 1], part[t]);
                        }
                    }
#pragma unroll
                for (int t = 0; t < TOK; ++t) {
                    const float v = warp_sum(part[t] * sc[j][i]);
                    if (lane == 0) red[(((size_t)kp * rows_cta + wr * R + i) * J + j) * TOK + t] = v;
                }
            }
        __syncthreads();
        const int blk = blockIdx.x + it * gridDim.x;
        float *cb = red + (size_t)kw * rows_cta * J * TOK + nf4_x_floats<PRO, TOK, SWI_IN>(p.K);  // kConv: [rows_cta]
        for (int e = tid; e < rows_cta * TOK; e += blockDim.x) {
            const int ri = e / TOK, t = e % TOK;
            const int vr = blk * rows_cta + ri;
            if (vr >= vrows || t >= tb) continue;
            int m = 0, row = vr, nr = p.N;
            if constexpr (MODE != kConv) {
                tile_map(p, MODE, vr, 1, m, row, nr);
                if (row >= nr) continue;
            }
            float v[J];
#pragma unroll
            for (int j = 0; j < J; ++j) {
                float a = red[((size_t)ri * J + j) * TOK + t];
                for (int part = 1; part < kw; ++part) a += red[(((size_t)part * rows_cta + ri) * J + j) * TOK + t];
                v[j] = a;
            }
            if constexpr (MODE == kConv) cb[ri] = v[0];
            else store_out<MODE>(p, m, t0 + t, row, v[0], v[J - 1]);
        }
        if constexpr (MODE == kConv) {
            // crates/backend-cpu/src/attention_convolution.rs:220-340 for one
            // token, rounded as gated_conv_kernel: u = B * x; the window is the
            // old history then u; sum of tap * window in tap order; times C.
            __syncthreads();
            const int ch = blk * cch + tid;
            if (tid < cch && ch < p.N) {
                const float u = __fmul_rn(cb[tid], cb[2 * cch + tid]);
                float total = 0.0f;
#pragma unroll
                for (int i = 0; i < kConvMaxWidth; ++i) {
                    if (i >= p.cwidth) break;
                    total = __fadd_rn(total, __fmul_rn(ckw[i], i < p.cwidth - 1 ? chold[i] : u));
                }
                p.out_a[ch] = __fmul_rn(total, cb[cch + tid]);
#pragma unroll
                for (int i = 0; i < kConvMaxWidth - 1; ++i) {
                    if (i >= p.cwidth - 1) break;
                    p.chist[(size_t)i * p.N + ch] = i + 1 < p.cwidth - 1 ? chold[i + 1] : u;
                }
            }
        }
        __syncthreads();  // red is rewritten by the next block
#pragma unroll
        for (int j = 0; j < J; ++j)
#pragma unroll
            for (int i = 0; i < R; ++i) {
                cw[j][i] = cn[j][i];
                sc[j][i] = sn[j][i];
            }
    }
}

// ---------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------
template <int FMT, int MODE, int NCB, int UB, int PRO, bool LT = false>
int32_t launch_imma(TcParams p, cudaStream_t stream) {
    constexpr int J = MODE == kSwigluPair ? 2 : 1;
    const int tblocks = (p.T + kTokBlock - 1) / kTokBlock;
    dim3 grid((p.vtiles + p.rt - 1) / p.rt, tblocks);
    size_t smem = (size_t)p.kw * p.rt * J * 16 * kTokBlock * sizeof(float);
    if (PRO == kNorm)
        smem += 2 * imma_row_floats(p.K) * sizeof(float) + (size_t)p.groups * 128 * sizeof(uint2) +
                (size_t)((2 * p.groups + 3) & ~3) * sizeof(float) + (size_t)p.groups * 4 * sizeof(int2);
    if (MODE == kSwigluPair && PRO == kNorm) {
        // staged scales: 8 groups per K part at most (K <= 8192 with 8 parts)
        if (p.kch > 8) return fail(MF_UNSUPPORTED, "staged scales take up to 8 groups per K part");
        smem += (size_t)p.rt * p.kw * J * 16 * 9 * sizeof(float);
    }
    auto kernel = packed_gemv_imma_kernel<FMT, MODE, NCB, UB, PRO, LT>;
    if (smem > 48 * 1024) MF_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (int32_t e_ = ::mf::launch(kernel, dim3(grid), dim3(p.rt * p.kw * 32), smem, stream, "packed_gemv_imma_kernel", p))
        return e_;
    return MF_OK;
}

// K parts of at most UB groups (one load batch), at most 8 parts; tiles
// per CTA: as many as fit in 8 warps while the grid still gives every SM
// two CTAs (a normalizing CTA forms the whole row, so it keeps 8 warps).
void imma_plan(TcParams &p, int ub, bool norm, int max_warps = 8) {
    p.kw = std::min(max_warps, (p.groups + ub - 1) / ub);
    p.kch = (p.groups + p.kw - 1) / p.kw;
    p.kw = (p.groups + p.kch - 1) / p.kch;
    p.rt = std::max(1, max_warps / p.kw);
    if (!norm)
        while (p.rt > 1 && (p.vtiles + p.rt - 1) / p.rt < 2 * sm_count()) p.rt >>= 1;
}

// Groups per load batch: matrices far larger than one wave stream with
// small batches (fewer registers, several CTAs per SM overlapping their
// loads); the rest issue every load of a warp at once.
int imma_ub(int format, int mode, int n, int n2, int k) {
    const double rows = mode == kTriple ? (double)n + 2.0 * n2 : (double)n * (mode == kSingle ? 1 : 2);
    const double bytes = rows * k * (format == MF_INT8 ? 1.0 : 0.25);
    if (bytes > 32e6) return format == MF_INT8 ? 1 : 2;
    return format == MF_INT8 ? 4 : 8;
}

template <int FMT>
int32_t launch_stream(TcParams p, cudaStream_t stream) {
    // K parts of the 8 warps: 1 or 2 groups each (K up to 2048: the codes of
    // the tiles in flight stay in registers).
    const int kch = (p.groups + 7) / 8;
    const int ctas = std::max(1, std::min(p.row_tiles, 2 * sm_count()));
    // Tiles in flight per CTA: INT8 moves 4x the bytes per tile of ternary.
    constexpr int D = FMT == MF_INT8 ? 2 : 4;
    auto go = [&](auto kernel) { return ::mf::launch(kernel, dim3(ctas), dim3(256), 0, stream, "packed_gemv_stream_kernel", p); };
    if (kch <= 1) return go(packed_gemv_stream_kernel<FMT, 1, D>);
    return go(packed_gemv_stream_kernel<FMT, 2, D>);
}

// One token through a ternary matrix of at least two 16-row tiles per warp
// of a full wave (one CTA of 8 warps per SM), K of 512, 1024 or 2048.
bool tile_kernel_fits(const TcParams &p) {
    return p.T == 1 && !p.split_halves && (p.groups == 4 || p.groups == 8 || p.groups == 16) &&
           p.row_tiles >= 2 * 8 * sm_count();
}

template <bool SWI, bool LT>
int32_t launch_tile(TcParams p, cudaStream_t stream) {
    const int ctas = std::max(1, std::min((p.row_tiles + 7) / 8, sm_count()));
    auto go = [&](auto kernel) { return ::mf::launch(kernel, dim3(ctas), dim3(256), 0, stream, "packed_gemv_tile_kernel", p); };
    if (p.groups == 4) return go(packed_gemv_tile_kernel<4, SWI, LT>);
    if (p.groups == 8) return go(packed_gemv_tile_kernel<8, SWI, LT>);
    return go(packed_gemv_tile_kernel<16, SWI, LT>);
}

template <int FMT, int MODE, bool SWI, int UB, int PRO, bool LT = false>
int32_t dispatch_imma_ub(TcParams p, cudaStream_t stream) {
    imma_plan(p, UB, PRO == kNorm, imma_threads<FMT, MODE, UB, PRO>() / 32);
    if constexpr (PRO == kNorm) {
        if (p.lout && (MODE != kSwigluPair || p.T != 1 || (p.rt * 16) % 64 || p.N % (p.rt * 16) || p.N % kGroup))
            return fail(MF_UNSUPPORTED, "SwiGLU limb epilogue does not take this shape");
        return launch_imma<FMT, MODE, 1, UB, PRO, LT>(p, stream);
    } else {
        const int tpad = 2 * ((p.T + 1) / 2);
        const int prep_items = tpad * p.groups;
        if (p.split_halves && p.T != 1) return fail(MF_UNSUPPORTED, "half-group limbs take one token");
        // One token through a many-wave ternary matrix: the warp-tiled kernel,
        // for both layouts, so LUT2 and raw results agree bit for bit.
        if constexpr (FMT == MF_TERNARY && MODE == kSingle)
            if (tile_kernel_fits(p)) return launch_tile<SWI, LT>(p, stream);   // splits its own limbs
        if (!p.split_halves)
            if (int32_t e_ = ::mf::launch(limb_prep_kernel<FMT, SWI>, dim3((prep_items + kWarps - 1) / kWarps), dim3(kThreads), 0, stream, "limb_prep_kernel", p, const_cast<uint2 *>(p.limbs), const_cast<float *>(p.efac), const_cast<int2 *>(p.lsum))) return e_;
        if constexpr (MODE == kSingle) {
            // One token through a many-wave matrix: persistent streaming CTAs.
            if (p.T == 1 && !p.split_halves && !LT && UB <= 2 && p.groups <= 16) return launch_stream<FMT>(p, stream);
        }
        const int tb = std::min(p.T, kTokBlock);
        if (tb <= 2) return launch_imma<FMT, MODE, 1, UB, PRO, LT>(p, stream);
        if (tb <= 4) return launch_imma<FMT, MODE, 2, UB, PRO, LT>(p, stream);
        if (tb <= 6) return launch_imma<FMT, MODE, 3, UB, PRO, LT>(p, stream);
        return launch_imma<FMT, MODE, 4, UB, PRO, LT>(p, stream);
    }
}

template <int FMT, int MODE, bool SWI, int PRO = kFromGlobal, bool LT = false>
int32_t dispatch_imma(TcParams p, cudaStream_t stream) {
    p.row_tiles = (p.N + 15) / 16;
    p.vtiles = MODE == kPairRows ? 2 * p.row_tiles
             : MODE == kTriple   ? p.row_tiles + 2 * ((p.N2 + 15) / 16)
                                 : p.row_tiles;
    if (imma_ub(FMT, MODE, p.N, p.N2, p.K) <= 2)
        return dispatch_imma_ub<FMT, MODE, SWI, FMT == MF_INT8 ? 1 : 2, PRO, LT>(p, stream);
    if constexpr (FMT == MF_TERNARY && MODE == kSwigluPair && PRO == kNorm)
        return dispatch_imma_ub<FMT, MODE, SWI, 4, PRO, LT>(p, stream);   // 16 warps of 4-group parts
    if constexpr (FMT == MF_TERNARY && MODE == kSingle && PRO == kFromGlobal)
        if (p.T <= 2) return dispatch_imma_ub<FMT, MODE, SWI, 4, PRO, LT>(p, stream);   // 16 warps (decode w2)
    return dispatch_imma_ub<FMT, MODE, SWI, FMT == MF_INT8 ? 4 : 8, PRO, LT>(p, stream);
}

template <int MODE, int TOK, int R, bool SWI, int PRO>
size_t nf4_smem(const TcParams &p) {
    constexpr int J = MODE == kSwigluPair ? 2 : 1;
    size_t smem = 256 * 16 * sizeof(float2) + (size_t)p.kw * p.rt * R * J * TOK * sizeof(float);
    smem += nf4_x_floats<PRO, TOK, SWI>(p.K) * sizeof(float);
    if (MODE == kConv) smem += (size_t)p.rt * R * sizeof(float);
    return smem;
}

// Resident CTAs per SM of this variant (shared memory attribute set).
template <int MODE, int TOK, int R, bool SWI, int PRO>
int nf4_per_sm(const TcParams &p) {
    // Cached per (shared memory, block size) of this variant.
    static std::mutex mu;
    static std::map<std::pair<size_t, int>, int> cache;
    const size_t smem = nf4_smem<MODE, TOK, R, SWI, PRO>(p);
    const int threads = p.rt * p.kw * 32;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find({smem, threads});
    if (it != cache.end()) return it->second;
    auto kernel = packed_gemv_nf4_kernel<MODE, TOK, R, SWI, PRO>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess) return 0;
    cache[{smem, threads}] = per_sm;
    return per_sm;
}

template <int MODE, int TOK, int R, bool SWI, int PRO>
int32_t launch_nf4(TcParams p, cudaStream_t stream) {
    const int vrows = MODE == kPairRows ? 2 * p.N : MODE == kTriple ? p.N + 2 * p.N2 : MODE == kConv ? 3 * p.N : p.N;
    const int rows_cta = p.rt * R;
    const size_t smem = nf4_smem<MODE, TOK, R, SWI, PRO>(p);
    auto kernel = packed_gemv_nf4_kernel<MODE, TOK, R, SWI, PRO>;
    const int per_sm = nf4_per_sm<MODE, TOK, R, SWI, PRO>(p);
    if (per_sm == 0) return fail(MF_RESOURCE_LIMIT, "NF4 decode GEMV does not fit on an SM");
    MF_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int nblocks = (vrows + rows_cta - 1) / rows_cta;
    // One pass of resident CTAs; each loops over its row blocks.
    const int grid_x = std::max(1, std::min(nblocks, std::max(1, per_sm) * sm_count()));
    if (MODE == kConv && (rows_cta % 3 || p.N % (rows_cta / 3) || grid_x < nblocks || p.T != 1 ||
                          p.cwidth < 1 || p.cwidth > kConvMaxWidth))
        return fail(MF_UNSUPPORTED, "convolution epilogue does not take this shape");
    if (int32_t e_ = ::mf::launch(kernel, dim3(grid_x, (p.T + TOK - 1) / TOK), dim3(p.rt * p.kw * 32), smem, stream,
                                  "packed_gemv_nf4_kernel", p))
        return e_;
    return MF_OK;
}

template <int MODE, bool SWI, int PRO = kFromGlobal>
int32_t dispatch_nf4(TcParams p, cudaStream_t stream) {
    // K parts of 1024 weights (at most 8: K <= 8192); row groups per CTA up
    // to 8 warps; rows per warp 4, 2 or 1 so the grid gives every SM two CTAs.
    p.kw = (p.K + kNf4PartWeights - 1) / kNf4PartWeights;
    if (p.kw > 8) return fail(MF_UNSUPPORTED, "NF4 decode GEMV takes inner widths up to 8192");
    p.rt = std::max(1, 8 / p.kw);
    const int vrows = MODE == kPairRows ? 2 * p.N : MODE == kTriple ? p.N + 2 * p.N2 : MODE == kConv ? 3 * p.N : p.N;
    auto ctas = [&](int r) { return (vrows + p.rt * r - 1) / (p.rt * r); };
    const int target = 2 * sm_count();
    if constexpr (MODE == kConv) {
        // Rows per CTA a multiple of 3 (B, C and x of each channel), one pass:
        // 12 warps of 8 rows when one CTA per SM covers the rows.
        const int rt8 = p.rt;
        p.rt = std::max(1, 12 / p.kw);
        if ((p.rt * 8) % 3 == 0 && ctas(8) <= sm_count()) return launch_nf4<MODE, 1, 8, SWI, PRO>(p, stream);
        p.rt = rt8;
        if (ctas(12) <= sm_count()) return launch_nf4<MODE, 1, 12, SWI, PRO>(p, stream);
        return launch_nf4<MODE, 1, 6, SWI, PRO>(p, stream);
    }
    if (p.T == 1) {
        // Few, full CTAs (about one per SM, at most ~1.5): with programmatic
        // dependent launch a CTA streams its codes in before the dependency
        // wait only if it is resident while the previous kernel still runs,
        // so every CTA of the grid should fit beside the previous kernel's.
        const int sms = sm_count();
        if constexpr (MODE == kSingle && PRO == kFromGlobal) {
            // 16 warps of 2 rows when one CTA per SM covers the rows.
            const int rt8 = p.rt;
            p.rt = std::max(1, 16 / p.kw);
            if (ctas(2) <= sms) return launch_nf4<MODE, 1, 2, SWI, PRO>(p, stream);
            p.rt = rt8;
        }
        if constexpr (MODE == kTriple && PRO == kNorm) {
            // 16 warps of 3 rows when one CTA per SM covers the rows.
            const int rt8 = p.rt;
            p.rt = std::max(1, 16 / p.kw);
            if (ctas(3) <= sms) return launch_nf4<MODE, 1, 3, SWI, PRO>(p, stream);
            p.rt = rt8;
        }
        if (ctas(4) <= sms * 3 / 2 || ctas(8) * 2 < sms) return launch_nf4<MODE, 1, 4, SWI, PRO>(p, stream);
        return launch_nf4<MODE, 1, 8, SWI, PRO>(p, stream);
    }
    if constexpr (PRO == kNorm) {
        return fail(MF_UNSUPPORTED, "normalizing prologue takes one token");
    } else {
        if (ctas(2) >= target) return launch_nf4<MODE, 2, 2, SWI, PRO>(p, stream);
        return launch_nf4<MODE, 2, 1, SWI, PRO>(p, stream);
    }
}

// The lane-tiled layout from the row-major one: one thread per 16-byte
// output chunk (two 8-byte reads, rows 16t + g and 16t + g + 8).
__global__ void __launch_bounds__(256) ternary_lanetile_kernel(uint4 *out, const uint8_t *codes, uint64_t chunks,
                                                               uint32_t groups, uint64_t row_bytes) {
    pdl_wait();
    pdl_trigger();
    for (uint64_t c = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; c < chunks; c += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t lane = (uint32_t)(c & 31), g = lane >> 2, q = lane & 3;
        const uint64_t tg = c >> 5, tile = tg / groups, G = tg % groups;
        const uint8_t *a = codes + (tile * 16 + g) * row_bytes + G * 32 + 8 * q;
        const uint2 lo = *reinterpret_cast<const uint2 *>(a);
        const uint2 hi = *reinterpret_cast<const uint2 *>(a + 8 * row_bytes);
        out[c] = make_uint4(lo.x, lo.y, hi.x, hi.y);
    }
}

size_t limb_floats(uint64_t t, uint64_t k) {
    const uint64_t pairs = (t + 1) / 2, groups = k / kGroup;
    // 1 KB of limbs, 2 factors and 4 (ternary) limb-sum pairs per pair-group
    return (size_t)(pairs * groups * 256 + 2 * pairs * groups + 8 * pairs * groups);
}

}  // namespace

int32_t ternary_repack_lanetiled(uint8_t *out, const uint8_t *codes, uint64_t rows, uint64_t row_bytes,
                                 cudaStream_t stream) {
    if (rows % 16 || row_bytes % 32) return fail(MF_INVALID_SHAPE, "LUT2 layout needs rows in multiples of 16");
    if (rows == 0 || row_bytes == 0) return MF_OK;
    if (row_bytes / 32 > (1u << 24)) return fail(MF_UNSUPPORTED, "ternary row too wide for the LUT2 layout");
    if (out == codes) return fail(MF_INVALID_ARGUMENT, "LUT2 repack cannot run in place");
    const uint64_t chunks = rows * row_bytes / 16;
    const unsigned blocks = (unsigned)std::min<uint64_t>((chunks + 255) / 256, (uint64_t)sm_count() * 16);
    return ::mf::launch(ternary_lanetile_kernel, dim3(blocks), dim3(256), 0, stream, "ternary_lanetile_kernel",
                        reinterpret_cast<uint4 *>(out), codes, chunks, (uint32_t)(row_bytes / 32), row_bytes);
}

bool packed_gemv_tc_supports(int format, uint64_t t) {
    if (format == MF_NF4) return t >= 1 && t <= 2;
    return t >= 1 && t < kGemmMinTokens;
}

size_t packed_gemv_tc_scratch_floats(uint64_t t, uint64_t n, uint64_t k) {
    (void)n;
    return limb_floats(t, k) + 64;  // activation limbs and group factors
}

size_t packed_gemv_tc_counters(uint64_t t, uint64_t n) {
    (void)t;
    (void)n;
    return 0;
}

int32_t packed_gemv_tc(int mode, bool swiglu_input, float *out_a, float *out_b, const float *x, const float *gate,
                       const float *up, uint64_t t, const uint8_t *codes_a, const float *scales_a,
                       const uint8_t *codes_b, const float *scales_b, uint64_t n, uint64_t k, int format,
                       const SplitScratch &ss, cudaStream_t stream, bool lanetiled) {
    if (t == 0 || n == 0) return MF_OK;
    if (k == 0 || k % kGroup) return fail(MF_INVALID_SHAPE, "packed inner width must be a positive multiple of 128");
    if (n > (1u << 26) || k > (1u << 24) || t >= kGemmMinTokens)
        return fail(MF_UNSUPPORTED, "packed matmul dimension exceeds decode-GEMV limits");
    if (!packed_gemv_tc_supports(format, t)) return fail(MF_UNSUPPORTED, "decode GEMV does not take this token count");
    if (ss.partial_floats < packed_gemv_tc_scratch_floats(t, n, k) || !ss.partial)
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
    if (lanetiled && (format != MF_TERNARY || n % 16))
        return fail(MF_INVALID_ARGUMENT, "LUT2 codes are ternary with rows in multiples of 16");
    p.lanetiled = lanetiled ? 1 : 0;
    // Scratch layout: [limbs (16-byte aligned) | factors | partials].
    float *base = ss.partial;
    const uint64_t pairs = (t + 1) / 2;
    p.limbs = reinterpret_cast<const uint2 *>(base);
    p.efac = base + pairs * p.groups * 256;
    p.lsum = reinterpret_cast<const int2 *>(p.efac + 2 * pairs * p.groups);
#define MF_TC_MODES(DISPATCH, ...)                                                                  \
    do {                                                                                           \
        if (mode == kSingle)                                                                       \
            return swiglu_input ? DISPATCH<__VA_ARGS__ kSingle, true>(p, stream)                   \
                                : DISPATCH<__VA_ARGS__ kSingle, false>(p, stream);                 \
        if (mode == kPairRows) return DISPATCH<__VA_ARGS__ kPairRows, false>(p, stream);           \
        return DISPATCH<__VA_ARGS__ kSwigluPair, false>(p, stream);                                \
    } while (0)
    if (lanetiled) {
        // LUT2 codes: ternary only (checked above), same modes.
        if (mode == kSingle)
            return swiglu_input ? dispatch_imma<MF_TERNARY, kSingle, true, kFromGlobal, true>(p, stream)
                                : dispatch_imma<MF_TERNARY, kSingle, false, kFromGlobal, true>(p, stream);
        if (mode == kPairRows) return dispatch_imma<MF_TERNARY, kPairRows, false, kFromGlobal, true>(p, stream);
        return dispatch_imma<MF_TERNARY, kSwigluPair, false, kFromGlobal, true>(p, stream);
    }
    switch (format) {
    case MF_TERNARY: MF_TC_MODES(dispatch_imma, MF_TERNARY,);
    case MF_INT8: MF_TC_MODES(dispatch_imma, MF_INT8,);
    case MF_NF4: MF_TC_MODES(dispatch_nf4, );
    default: return fail(MF_INVALID_ARGUMENT, "unknown packed format");
    }
#undef MF_TC_MODES
}

bool decode_gemv_conv_supported(const DecodeGemv &d) {
    if (d.mode != kConv || !decode_gemv_supports(d)) return false;
    TcParams p{};
    p.K = (int)d.k;
    p.N = (int)d.n;
    p.kw = (p.K + kNf4PartWeights - 1) / kNf4PartWeights;
    p.rt = std::max(1, 8 / p.kw);
    const int vrows = 3 * p.N, sms = sm_count();
    // The choices of dispatch_nf4: 12 warps of 8 rows, then 8 warps of 12 or 6.
    const int kw = p.kw;
    for (int v = 0; v < 3; ++v) {
        const int r = v == 0 ? 8 : v == 1 ? 12 : 6;
        p.rt = std::max(1, (v == 0 ? 12 : 8) / kw);
        const int rows_cta = p.rt * r, nblocks = (vrows + rows_cta - 1) / rows_cta;
        if (v == 0 && (rows_cta % 3 || nblocks > sms)) continue;
        if (v == 1 && nblocks > sms) continue;
        const int per_sm = v == 0 ? (d.x ? nf4_per_sm<kConv, 1, 8, false, kFromGlobal>(p) : nf4_per_sm<kConv, 1, 8, false, kNorm>(p))
                         : v == 1 ? (d.x ? nf4_per_sm<kConv, 1, 12, false, kFromGlobal>(p) : nf4_per_sm<kConv, 1, 12, false, kNorm>(p))
                                  : (d.x ? nf4_per_sm<kConv, 1, 6, false, kFromGlobal>(p) : nf4_per_sm<kConv, 1, 6, false, kNorm>(p));
        return rows_cta % 3 == 0 && p.N % (rows_cta / 3) == 0 && nblocks <= std::max(1, per_sm) * sms;
    }
    return false;
}

bool decode_gemv_limbs_supported(const DecodeGemv &d) {
    if (d.mode != kSwigluPair || d.x != nullptr || d.sampled || d.cand) return false;
    if (d.format != MF_TERNARY && d.format != MF_INT8) return false;
    if (d.limbs_for != MF_TERNARY && d.limbs_for != MF_INT8) return false;
    if (d.k == 0 || d.k % kGroup || d.k > 8192 || d.n == 0 || d.n % kGroup || d.n > (1u << 26)) return false;
    TcParams p{};
    p.groups = (int)(d.k / kGroup);
    p.vtiles = (int)((d.n + 15) / 16);
    const int ub = imma_ub(d.format, kSwigluPair, (int)d.n, 0, (int)d.k);
    const bool wide = d.format == MF_TERNARY && ub > 2;   // the 16-warp variant (4-group parts)
    imma_plan(p, wide ? 4 : ub, true, wide ? 16 : 8);
    const uint64_t rows = (uint64_t)p.rt * 16;
    return rows % 64 == 0 && d.n % rows == 0;
}

bool decode_gemv_supports(const DecodeGemv &d) {
    if (d.k == 0 || d.k % kGroup || d.n == 0 || d.mode < 0 || d.mode > 4) return false;
    if (d.mode == kConv && (d.format != MF_NF4 || !d.conv_kernel || !d.conv_hist || d.conv_width < 1 ||
                            d.conv_width > (uint32_t)kConvMaxWidth || d.k > 8192 || d.sampled || d.cand))
        return false;
    // The normalizing prologue stages the row in shared memory; NF4 keeps at
    // most eight 1024-wide K parts per CTA.
    if ((d.x == nullptr || d.format == MF_NF4) && d.k > 8192) return false;
    if (d.mode == 3 && d.n2 == 0) return false;
    if ((d.sampled || d.cand) && d.format == MF_NF4) return false;  // argmax epilogue: integer path only
    return d.format == MF_TERNARY || d.format == MF_INT8 || d.format == MF_NF4;
}

int32_t decode_gemv(const DecodeGemv &d, const SplitScratch &ss, cudaStream_t stream) {
    if (!decode_gemv_supports(d)) return fail(MF_UNSUPPORTED, "fused decode projection does not take this shape");
    if ((d.sampled || d.cand) && d.mode != kSingle) return fail(MF_INVALID_ARGUMENT, "argmax epilogue needs a single projection");
    TcParams p{};
    p.x = d.x;
    p.codes_a = d.codes[0];
    p.codes_b = d.codes[1];
    p.codes_c = d.codes[2];
    p.scales_a = d.scales[0];
    p.scales_b = d.scales[1];
    p.scales_c = d.scales[2];
    p.out_a = d.out[0];
    p.out_b = d.out[1];
    p.out_c = d.out[2];
    p.T = 1;
    p.N = (int)d.n;
    p.N2 = (int)d.n2;
    p.K = (int)d.k;
    p.groups = (int)(d.k / kGroup);
    p.pairs = 1;
    p.ckern = d.conv_kernel;
    p.chist = d.conv_hist;
    p.cwidth = (int)d.conv_width;
    const bool norm = d.x == nullptr;
    if (norm) {
        p.na = d.na;
        p.nb = d.nb;
        p.nw = d.nw;
        p.nres = d.nres;
        p.neps = d.eps;
        p.ecodes = d.ecodes;
        p.escales = d.escales;
        p.edense = d.edense;
        p.eid = d.eid;
        p.eformat = d.eformat;
        p.erows = (int)d.erows;
        if ((!d.na && !d.eid) || (!d.na && !d.nw))
            return fail(MF_INVALID_ARGUMENT, "normalizing prologue needs its inputs");
    }
    if (d.format != MF_NF4 && !norm) {
        // Plain input: limbs through the scratch like packed_gemv_tc.
        if (ss.partial_floats < packed_gemv_tc_scratch_floats(1, d.n, d.k) || !ss.partial)
            return fail(MF_RESOURCE_LIMIT, "packed GEMV scratch too small");
        p.limbs = reinterpret_cast<const uint2 *>(ss.partial);
        p.efac = ss.partial + (size_t)p.groups * 256;
        p.lsum = reinterpret_cast<const int2 *>(p.efac + 2 * (size_t)p.groups);
        p.split_halves = d.limbs_ready ? 1 : 0;
    } else if (d.limbs_ready) {
        return fail(MF_INVALID_ARGUMENT, "half-group limbs feed a plain-input integer projection");
    }
    if (d.limbs_for >= 0) {
        // The consumer's limbs go where its plain-input call reads them.
        if (!decode_gemv_limbs_supported(d)) return fail(MF_UNSUPPORTED, "SwiGLU limb epilogue does not take this shape");
        if (ss.partial_floats < packed_gemv_tc_scratch_floats(1, d.k, d.n) || !ss.partial)
            return fail(MF_RESOURCE_LIMIT, "packed GEMV scratch too small");
        p.lout = reinterpret_cast<uint2 *>(ss.partial);
        p.lgroups = (int)(d.n / kGroup);
        p.lefac = ss.partial + (size_t)p.lgroups * 256;
        p.llsum = reinterpret_cast<int2 *>(p.lefac + 2 * (size_t)p.lgroups);
        p.lfmt = d.limbs_for;
    }
    if (d.sampled || d.cand) {
        // One (value, index, poisoned) triple per CTA (at most one CTA per
        // 16-row tile), after the limbs when the input is plain.
        const size_t off = norm ? 0 : packed_gemv_tc_scratch_floats(1, d.n, d.k);
        if (!ss.partial || !ss.counters || ss.n_counters < 1 || ss.partial_floats < off + 3 * ((d.n + 15) / 16))
            return fail(MF_RESOURCE_LIMIT, "argmax epilogue needs scratch");
        p.aparts = ss.partial + off;
        p.acount = ss.counters;
        p.asampled = d.sampled;
        p.acand = d.cand;
        p.arow0 = (int)d.row0;
        p.apos = d.pos;
    }
    if (d.mode == kConv && d.format != MF_NF4) return fail(MF_UNSUPPORTED, "convolution epilogue needs NF4 rows");
    if (d.lanetiled && (d.format != MF_TERNARY || d.n % 16 || (d.mode == kTriple && d.n2 % 16)))
        return fail(MF_INVALID_ARGUMENT, "LUT2 codes are ternary with rows in multiples of 16");
    p.lanetiled = d.lanetiled ? 1 : 0;
#define MF_DG(FMT, LT)                                                                               \
    do {                                                                                             \
        if (norm) {                                                                                  \
            switch (d.mode) {                                                                        \
            case kSingle: return dispatch_imma<FMT, kSingle, false, kNorm, LT>(p, stream);           \
            case kPairRows: return dispatch_imma<FMT, kPairRows, false, kNorm, LT>(p, stream);       \
            case kSwigluPair: return dispatch_imma<FMT, kSwigluPair, false, kNorm, LT>(p, stream);   \
            default: return dispatch_imma<FMT, kTriple, false, kNorm, LT>(p, stream);                \
            }                                                                                        \
        }                                                                                            \
        switch (d.mode) {                                                                            \
        case kSingle: return dispatch_imma<FMT, kSingle, false, kFromGlobal, LT>(p, stream);         \
        case kPairRows: return dispatch_imma<FMT, kPairRows, false, kFromGlobal, LT>(p, stream);     \
        case kSwigluPair: return dispatch_imma<FMT, kSwigluPair, false, kFromGlobal, LT>(p, stream); \
        default: return dispatch_imma<FMT, kTriple, false, kFromGlobal, LT>(p, stream);              \
        }                                                                                            \
    } while (0)
    if (d.format == MF_TERNARY && d.lanetiled) MF_DG(MF_TERNARY, true);
    if (d.format == MF_TERNARY) MF_DG(MF_TERNARY, false);
    if (d.format == MF_INT8) MF_DG(MF_INT8, false);
#undef MF_DG
    if (norm) {
        switch (d.mode) {
        case kSingle: return dispatch_nf4<kSingle, false, kNorm>(p, stream);
        case kPairRows: return dispatch_nf4<kPairRows, false, kNorm>(p, stream);
        case kSwigluPair: return dispatch_nf4<kSwigluPair, false, kNorm>(p, stream);
        case kConv: return dispatch_nf4<kConv, false, kNorm>(p, stream);
        default: return dispatch_nf4<kTriple, false, kNorm>(p, stream);
        }
    }
    switch (d.mode) {
    case kSingle: return dispatch_nf4<kSingle, false>(p, stream);
    case kPairRows: return dispatch_nf4<kPairRows, false>(p, stream);
    case kSwigluPair: return dispatch_nf4<kSwigluPair, false>(p, stream);
    case kConv: return dispatch_nf4<kConv, false>(p, stream);
    default: return dispatch_nf4<kTriple, false>(p, stream);
    }
}

}  // namespace mf

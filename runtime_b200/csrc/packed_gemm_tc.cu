// Packed matmul for many tokens (prefill) on the 5th-generation tensor
// cores: tcgen05.mma with F32 accumulators in TMEM, activations fed by TMA,
// packed weights dequantised into shared memory by the CTA itself.
//
// out[t, r] = sum_g scale[r, g] * sum_{j in g} w(code[r, j]) * x[t, j]
// (crates/backend-cpu/src/packed.rs:121-195).  Modes: single, pair rows
// (two matrices on one input, packed.rs:251-297), SwiGLU pair
// (silu(A x) * (B x), packed.rs:303-397) and SwiGLU input (the input is
// silu(gate) * up, packed.rs:402-490).
//
// Precision.  A BF16 operand carries 8 significant bits; the contract asks
// for F32-accumulate accuracy (1e-3 max relative error and reorder-sized
// error per element).  Each operand is split into a BF16 pair v = hi + lo,
// hi = bf16(v), lo = bf16(v - hi), which keeps 16 significant bits
// (relative error <= 2^-17), and every product is accumulated from three
// MMAs: Wh*Xh + Wh*Xl + Wl*Xh (the dropped Wl*Xl is <= 2^-16 relative).
// The weight operand is the dequantised, scale-folded weight
// scale[r, g] * level(code) rounded once to F32, so the per-group scale
// needs no separate promotion step.  BF16 keeps the F32 exponent range:
// magnitudes from 1e-30 to 1e30 and non-finite inputs behave as in F32
// (an infinite input makes its lo part NaN, so its token's outputs are NaN).
//
// Tiling.  One CTA computes 128 weight rows x 256 tokens (M = 128,
// N = 256: 256 TMEM columns of F32) over K in 64-wide stages (one
// 128-byte swizzle row of BF16), two stages in flight:
//   warp 0     TMA producer: the Xh and Xl tiles (256 x 64 each) per stage
//   warp 1     TMEM allocation; one lane issues 12 MMAs per stage and
//              commits each stage back to the producers
//   warps 2-5  dequantise 128 rows x 64 weights per stage into the swizzled
//              Wh and Wl tiles (one row per thread, codes loaded one stage
//              ahead), then the epilogue: TMEM -> registers -> global.
// In the SwiGLU-pair mode tile rows 0-63 are rows r0..r0+63 of A and rows
// 64-127 the same rows of B; the epilogue pairs them through shared memory.
#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "mf_common.cuh"
#include "packed_kernels.h"
#include "tc_sm100.cuh"

namespace mf {

// Set (bit 0) by a tensor-core GEMM whose pipeline wait timed out.
__device__ unsigned int g_tc_gemm_fault = 0;

// Ternary / INT8 GEMMs: 0 (default) and 2 run the group-scaled two-pass
// kernel, 3 the scale-folded three-pass one (comparison runs;
// mf_set_gemm_passes).
std::atomic<int> g_gemm_passes{0};
void set_gemm_passes(int passes) { g_gemm_passes.store(passes, std::memory_order_relaxed); }

namespace {

using namespace sm100;

constexpr int TM = 128;   // weight rows per tile (MMA M)
constexpr int TN = 256;   // tokens per tile (MMA N)
constexpr int TK = 64;    // K per stage
constexpr int kStages = 2;
constexpr int kThreads = 320;   // TMA, MMA, 4 dequantising warps, 4 epilogue warps
constexpr uint32_t kXBytes = TN * TK * 2;                         // 32 KB per BF16 plane
constexpr uint32_t kWBytes = TM * TK * 2;                         // 16 KB per BF16 plane
constexpr uint32_t kStageBytes = 2 * kXBytes + 2 * kWBytes;        // 96 KB
constexpr uint32_t kPairBytes = 64 * 33 * 4;                       // SwiGLU pairing buffer
constexpr uint32_t kBarBytes = 128;
constexpr size_t kSmemBytes = kStages * kStageBytes + kPairBytes + kBarBytes + 1024;  // + alignment slack
constexpr uint32_t kAccCols = 256;                                  // one F32 accumulator tile
constexpr uint32_t kTmemCols = 2 * kAccCols;                        // double-buffered
constexpr uint32_t kIdesc = idesc_bf16_f32(TM, TN);

__device__ __constant__ float kNf4[16] = {
    -0x1.000000p+0f, -0x1.647362p-1f, -0x1.0cd660p-1f, -0x1.946540p-2f,
    -0x1.23449ap-2f, -0x1.7a6a7ep-3f, -0x1.74f0e2p-4f, 0.0f,
    0x1.45f5fep-4f,  0x1.4995c6p-3f,  0x1.f809bap-3f,  0x1.5a0674p-2f,
    0x1.c34970p-2f,  0x1.200f56p-1f,  0x1.722766p-1f,  0x1.000000p+0f,
};

struct TcGemmParams {
    const uint8_t *codes_a, *codes_b;
    const float *scales_a, *scales_b;
    float *out_a, *out_b;
    int T, N, K;
    // Split-K (grid.z splits of kb_per_split 64-wide stages): each split
    // writes its raw sums to partial[z][T][VR] (VR virtual rows: N, or 2N
    // for the pair modes with B's rows after A's) for split_reduce_kernel.
    float *partial;
    int kb_per_split, VR;
    // Tile grid walked by the persistent CTAs: tile = (z * tiles_x + x) *
    // tiles_y + y (token tiles of one row tile are neighbours, so CTAs that
    // run at the same time share weight rows in L2).
    int tiles_x, tiles_y, splits;
    // Ternary codes in the lane-tiled layout (see ternary_repack_lanetiled).
    int lanetiled;
};

template <int FMT>
struct CodeChunk {
    // Bytes of one 64-weight chunk: 16 ternary, 32 NF4, 64 INT8.
    static constexpr int kVec = FMT == MF_TERNARY ? 1 : FMT == MF_NF4 ? 2 : 4;
    uint4 v[kVec];
};

template <int FMT>
__device__ __forceinline__ void load_chunk(CodeChunk<FMT> &c, const uint8_t *row, int kb, bool valid) {
    if (!valid) {
#pragma unroll
        for (int i = 0; i < CodeChunk<FMT>::kVec; ++i) c.v[i] = make_uint4(0, 0, 0, 0);
        return;
    }
    const uint4 *src = reinterpret_cast<const uint4 *>(row) + (size_t)kb * CodeChunk<FMT>::kVec;
#pragma unroll
    for (int i = 0; i < CodeChunk<FMT>::kVec; ++i) c.v[i] = __ldg(src + i);
}

// One 64-weight stage of a lane-tiled ternary row: `base` is the row's
// first byte in its tile (lane (r % 8) * 4 chunk, upper half for r % 16 >= 8);
// stage kb is group kb / 2, q-chunks 2 (kb % 2) and 2 (kb % 2) + 1.
__device__ __forceinline__ void load_chunk_lanetiled(CodeChunk<MF_TERNARY> &c, const uint8_t *base, int kb, bool valid) {
    if (!valid) {
        c.v[0] = make_uint4(0, 0, 0, 0);
        return;
    }
    const uint8_t *b = base + (size_t)(kb >> 1) * 512 + (kb & 1) * 32;
    const uint2 lo = __ldg(reinterpret_cast<const uint2 *>(b));
    const uint2 hi = __ldg(reinterpret_cast<const uint2 *>(b + 16));
    c.v[0] = make_uint4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// The 8 dequantised, scale-folded weights of 16-byte output chunk c
// (weights 8c .. 8c+7 of the 64-weight stage).
template <int FMT>
__device__ __forceinline__ void weights8(const CodeChunk<FMT> &cc, int c, float sc, const float *lut,
                                         float (&w)[8]) {
    if constexpr (FMT == MF_TERNARY) {
        // ternary-format-v1: 4 codes per byte, LSB first; level = code - 1.
        const uint32_t bits = word_of(cc.v[0], c >> 1) >> (16 * (c & 1));
#pragma unroll
        for (int e = 0; e < 8; ++e)
            w[e] = (__int_as_float(0x4B000000u | ((bits >> (2 * e)) & 3u)) - 8388609.0f) * sc;
    } else if constexpr (FMT == MF_NF4) {
        // nf4-format-v1: 2 codes per byte, low nibble first.
        const uint32_t bits = word_of(cc.v[c >> 2], c & 3);
#pragma unroll
        for (int e = 0; e < 8; ++e) w[e] = lut[(bits >> (4 * e)) & 15u] * sc;
    } else {
        // int8-format-v1: signed two's-complement bytes.
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int wi = 2 * c + h;   // word 0..15 of the 64-byte chunk
            const uint32_t word = word_of(cc.v[wi >> 2], wi & 3) ^ 0x80808080u;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                w[4 * h + j] = (__int_as_float(__byte_perm(word, 0x4B000000u, 0x7540 + j)) - 8388736.0f) * sc;
        }
    }
}

__device__ __forceinline__ uint32_t bf16x2_bits(__nv_bfloat162 v) {
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
    __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162 *>(&a), y = *reinterpret_cast<__nv_bfloat162 *>(&b);
    return bf16x2_bits(__hsub2(x, y));
}

// The two-pass GEMM's K order: in every 16-element block, position 2m holds
// element m and position 2m + 1 element m + 8 (m < 8).  Both operands use it
// (split_bf16_kernel<.., true> for the activation), so each dot is the same
// sum; it lets a BF16 pair come from one shift and mask of the codes.
//
// The 8 levels (BF16, exact) at positions 8c .. 8c+7 of a 64-weight stage,
// as 4 pairs.  Integer bit tricks, no float conversion: 0x4300 | u is the
// BF16 of 128 + u for u < 128.
template <int FMT>
__device__ __forceinline__ void levels8_p16(const CodeChunk<FMT> &cc, int c, uint32_t (&h)[4]) {
    static_assert(FMT == MF_TERNARY || FMT == MF_INT8, "integer levels only");
    const int j = c >> 1, m0 = 4 * (c & 1);   // block j, pairs m0 .. m0+3
    if constexpr (FMT == MF_TERNARY) {
        // Element e of the block sits at bits 2e of word j: the pair
        // (m, m + 8) is bits 2m and 2m + 16.  level = code - 1.
        const uint32_t w = word_of(cc.v[0], j);
#pragma unroll
        for (int e = 0; e < 4; ++e)
            h[e] = bf16x2_sub(((w >> (2 * (m0 + e))) & 0x00030003u) | 0x43004300u, 0x43014301u);   // - 129
    } else {
        // Element e of the block is byte e % 4 of word e / 4 (two's
        // complement): 128 + (b & 127) minus 128 (b >= 0) or 256 (b < 0).
        const uint32_t lo = word_of(cc.v[j], c & 1), hi = word_of(cc.v[j], 2 + (c & 1));
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t x = __byte_perm(lo, hi, 0x0400u + 0x0101u * e);   // bytes e of lo and hi at 0 and 2
            h[e] = bf16x2_sub((x & 0x007F007Fu) | 0x43004300u, (x & 0x00800080u) | 0x43004300u);
        }
    }
}

// hi = bf16(w), lo = bf16(w - hi), packed 8 per 16 bytes.
__device__ __forceinline__ void split8(const float (&w)[8], uint4 &hi, uint4 &lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 hv = __floats2bfloat162_rn(w[2 * i], w[2 * i + 1]);
        const float2 hf = __bfloat1622float2(hv);
        const __nv_bfloat162 lv = __floats2bfloat162_rn(w[2 * i] - hf.x, w[2 * i + 1] - hf.y);
        h[i] = bf16x2_bits(hv);
        l[i] = bf16x2_bits(lv);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// MODE: 0 single, 1 pair rows (virtual rows 0..2N-1), 2 SwiGLU pair.
// Persistent: CTA c computes tiles c, c + gridDim.x, ...; the MMA warp
// fills accumulator (j & 1) for the CTA's j-th tile while the epilogue
// warps drain the other one.
template <int FMT, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    packed_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl,
                          const TcGemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ float lut[16];
    __shared__ volatile int s_fail;   // any role's wait timed out
    __shared__ volatile int e_fail;   // an epilogue warp's wait timed out
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *gbase = smem_raw + (base - raw);
    auto xh_s = [&](int s) { return base + s * kStageBytes; };
    auto xl_s = [&](int s) { return base + s * kStageBytes + kXBytes; };
    auto wh_off = [&](int s) { return s * kStageBytes + 2 * kXBytes; };
    auto wl_off = [&](int s) { return s * kStageBytes + 2 * kXBytes + kWBytes; };
    float *xb = reinterpret_cast<float *>(gbase + kStages * kStageBytes);   // [64][33] pairing buffer
    const uint32_t bars = base + kStages * kStageBytes + kPairBytes;
    auto full_x = [&](int s) { return bars + 8u * s; };
    auto full_w = [&](int s) { return bars + 8u * (kStages + s); };
    auto empty = [&](int s) { return bars + 8u * (2 * kStages + s); };
    auto tmem_full = [&](int b) { return bars + 8u * (3 * kStages + b); };
    auto tmem_empty = [&](int b) { return bars + 8u * (3 * kStages + 2 + b); };
    const uint32_t tmem_slot = bars + 8u * (3 * kStages + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = p.K / TK;
    const int ntiles = p.tiles_x * p.tiles_y * p.splits;
    // Weight-row tiles fastest: the CTAs of one wave share a few token
    // tiles' activation planes (128 tokens x K x 4 bytes each, 16x a ternary
    // row tile's codes), which then stay in L2 while every row tile reads
    // them; the packed weights are small enough to stay there too.
    auto coords = [&](int tile, int &tx, int &ty, int &z) {
        tx = tile % p.tiles_x;
        const int r = tile / p.tiles_x;
        ty = r % p.tiles_y;
        z = r / p.tiles_y;
    };

    if (threadIdx.x == 0) {
#pragma unroll
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full_x(s), 1);
            mbar_init(full_w(s), 4);
            mbar_init(empty(s), 1);
        }
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            mbar_init(tmem_full(b), 1);
            mbar_init(tmem_empty(b), 4);
        }
        mbar_init_fence();
        s_fail = 0;
        e_fail = 0;
    }
    if (threadIdx.x < 16) lut[threadIdx.x] = kNf4[threadIdx.x];
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&tm_xh);
        tma_prefetch_map(&tm_xl);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(gbase + (tmem_slot - base));
    pdl_wait();
    pdl_trigger();

    if (warp == 0) {
        // ------------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t it = 0;   // stage counter across this CTA's tiles
            for (int tile = blockIdx.x; tile < ntiles && !s_fail; tile += gridDim.x) {
                int tx, ty, z;
                coords(tile, tx, ty, z);
                const int kb0 = z * p.kb_per_split, nkl = min(nk - kb0, p.kb_per_split);
                bool ok = true;
                for (int i = 0; i < nkl; ++i, ++it) {
                    const int s = it % kStages;
                    if (it >= kStages && !mbar_wait(empty(s), ((it / kStages) - 1) & 1)) {
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_x(s), 2 * kXBytes);
                    tma_load_2d(xh_s(s), &tm_xh, (kb0 + i) * TK, ty * TN, full_x(s));
                    tma_load_2d(xl_s(s), &tm_xl, (kb0 + i) * TK, ty * TN, full_x(s));
                }
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t it = 0;
            int j = 0;
            for (int tile = blockIdx.x; tile < ntiles && !s_fail; tile += gridDim.x, ++j) {
                int tx, ty, z;
                coords(tile, tx, ty, z);
                const int kb0 = z * p.kb_per_split, nkl = min(nk - kb0, p.kb_per_split);
                const int b = j & 1;
                if (j >= 2 && !mbar_wait(tmem_empty(b), ((j >> 1) - 1) & 1)) {
                    s_fail = 1;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t acc = tmem + b * kAccCols;
                bool ok = true;
                for (int i = 0; i < nkl; ++i, ++it) {
                    const int s = it % kStages;
                    const uint32_t par = (it / kStages) & 1;
                    if (!mbar_wait(full_x(s), par) || !mbar_wait(full_w(s), par)) {
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
#pragma unroll
                    for (int kk = 0; kk < TK / 16; ++kk) {
                        const uint64_t ah = sw128_kmajor_desc(base + wh_off(s) + kk * 32);
                        const uint64_t al = sw128_kmajor_desc(base + wl_off(s) + kk * 32);
                        const uint64_t bh = sw128_kmajor_desc(xh_s(s) + kk * 32);
                        const uint64_t bl = sw128_kmajor_desc(xl_s(s) + kk * 32);
                        mma_bf16_ss(acc, ah, bh, kIdesc, (i | kk) != 0);
                        mma_bf16_ss(acc, ah, bl, kIdesc, 1);
                        mma_bf16_ss(acc, al, bh, kIdesc, 1);
                    }
                    mma_commit(empty(s));
                }
                mma_commit(tmem_full(b));   // arrives when the tile's MMAs are done (also after a failure)
                if (!ok) break;
            }
        }
        __syncwarp();
    } else if (warp < 6) {
        // ------------------------------------------------- dequantisation
        const int d = threadIdx.x - 64;   // tile row 0..127
        const int wrow_bytes = FMT == MF_TERNARY ? p.K / 4 : FMT == MF_NF4 ? p.K / 2 : p.K;
        const int groups = p.K / kGroup;
        // First code byte of row r (row-major, or its place in a lane tile).
        auto row_base = [&](const uint8_t *codes, int r) -> const uint8_t * {
            if (FMT == MF_TERNARY && p.lanetiled)
                return codes + (size_t)(r >> 4) * groups * 512 + (r & 7) * 64 + ((r >> 3) & 1) * 8;
            return codes + (size_t)r * wrow_bytes;
        };
        auto load = [&](CodeChunk<FMT> &c, const uint8_t *row, int kb, bool valid) {
            if constexpr (FMT == MF_TERNARY) {
                if (p.lanetiled) {
                    load_chunk_lanetiled(c, row, kb, valid);
                    return;
                }
            }
            load_chunk<FMT>(c, row, kb, valid);
        };
        const uint32_t swz = d & 7;
        uint32_t it = 0;
        for (int tile = blockIdx.x; tile < ntiles && !s_fail; tile += gridDim.x) {
            int tx, ty, z;
            coords(tile, tx, ty, z);
            const int kb0 = z * p.kb_per_split, nkl = min(nk - kb0, p.kb_per_split);
            const uint8_t *crow = nullptr;
            const float *srow = nullptr;
            bool valid;
            if constexpr (MODE == 2) {
                const int r = tx * (TM / 2) + (d & (TM / 2 - 1));
                valid = r < p.N;
                const bool second = d >= TM / 2;
                if (valid) {
                    crow = row_base(second ? p.codes_b : p.codes_a, r);
                    srow = (second ? p.scales_b : p.scales_a) + (size_t)r * groups;
                }
            } else if constexpr (MODE == 1) {
                const int v = tx * TM + d;
                valid = v < 2 * p.N;
                if (valid) {
                    const bool second = v >= p.N;
                    const int r = second ? v - p.N : v;
                    crow = row_base(second ? p.codes_b : p.codes_a, r);
                    srow = (second ? p.scales_b : p.scales_a) + (size_t)r * groups;
                }
            } else {
                const int v = tx * TM + d;
                valid = v < p.N;
                if (valid) {
                    crow = row_base(p.codes_a, v);
                    srow = p.scales_a + (size_t)v * groups;
                }
            }
            CodeChunk<FMT> cur;
            load(cur, crow, kb0, valid);
            bool ok = true;
            for (int i = 0; i < nkl; ++i, ++it) {
                const int kb = kb0 + i, s = it % kStages;
                CodeChunk<FMT> nxt;
                load(nxt, crow, i + 1 < nkl ? kb + 1 : kb, valid);
                const float sc = valid ? __ldg(srow + (kb >> 1)) : 0.0f;
                // Every lane waits (each needs the acquire); the verdict is made
                // warp-uniform so the warp leaves the loop together.
                if (it >= kStages && !__all_sync(0xffffffffu, mbar_wait(empty(s), ((it / kStages) - 1) & 1))) {
                    s_fail = 1;
                    ok = false;
                    break;
                }
                uint8_t *wh = gbase + wh_off(s) + d * 128;
                uint8_t *wl = gbase + wl_off(s) + d * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    float w[8];
                    weights8<FMT>(cur, c, sc, lut, w);
                    uint4 hi, lo;
                    split8(w, hi, lo);
                    *reinterpret_cast<uint4 *>(wh + ((c ^ swz) << 4)) = hi;
                    *reinterpret_cast<uint4 *>(wl + ((c ^ swz) << 4)) = lo;
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(full_w(s));
                cur = nxt;
            }
            if (!ok) break;
        }
    } else {
        // ------------------------------------------------------- epilogue
        const int q = warp & 3;            // TMEM lane quarter of this warp
        const int row = 32 * q + lane;     // tile row of this thread
        int j = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++j) {
            int tx, ty, z;
            coords(tile, tx, ty, z);
            const int b = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(tmem_full(b), (j >> 1) & 1)) && lane == 0) e_fail = 1;
            // The four epilogue warps agree before any pairing exchange.
            named_barrier(1, 128);
            if (e_fail) {
                s_fail = 1;
                break;
            }
            tc_fence_after_sync();
            const bool poison = s_fail;
            const uint32_t taddr = tmem + b * kAccCols + ((uint32_t)(32 * q) << 16);
            const int t0 = ty * TN;
            for (int cb = 0; cb < TN / 32; ++cb) {
                uint32_t r[32];
                tmem_ld_32x32(taddr + cb * 32, r);
                const int tb = t0 + cb * 32;
                if (p.partial) {
                    // Split-K: raw sums of this split, virtual-row layout.
                    int vr;
                    if constexpr (MODE == 2) {
                        const int rr = tx * (TM / 2) + (row & (TM / 2 - 1));
                        vr = rr < p.N ? (row < TM / 2 ? rr : p.N + rr) : -1;
                    } else {
                        vr = tx * TM + row;
                        if (vr >= p.VR) vr = -1;
                    }
                    if (vr >= 0) {
                        float *dst = p.partial + (size_t)z * p.T * p.VR + vr;
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (tb + i < p.T)
                                dst[(size_t)(tb + i) * p.VR] = poison ? __int_as_float(0x7fc00000) : __uint_as_float(r[i]);
                    }
                    continue;
                }
                if constexpr (MODE == 2) {
                    if (q >= 2) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) xb[(row - 64) * 33 + i] = __uint_as_float(r[i]);
                    }
                    named_barrier(1, 128);
                    if (q < 2) {
                        const int n = tx * (TM / 2) + row;
                        if (n < p.N) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                if (tb + i < p.T) {
                                    const float v = silu_mul(__uint_as_float(r[i]), xb[row * 33 + i]);
                                    p.out_a[(size_t)(tb + i) * p.N + n] = poison ? __int_as_float(0x7fc00000) : v;
                                }
                            }
                        }
                    }
                    named_barrier(1, 128);
                } else {
                    const int v = tx * TM + row;
                    float *out = p.out_a;
                    int n = v;
                    if constexpr (MODE == 1) {
                        if (v >= p.N) {
                            out = p.out_b;
                            n = v - p.N;
                        }
                        if (v >= 2 * p.N) n = -1;
                    } else {
                        if (v >= p.N) n = -1;
                    }
                    if (n >= 0) {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (tb + i < p.T)
                                out[(size_t)(tb + i) * p.N + n] = poison ? __int_as_float(0x7fc00000) : __uint_as_float(r[i]);
                    }
                }
            }
            // The accumulator may be refilled once all four warps have read it.
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(tmem_empty(b));
        }
    }
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (threadIdx.x == 0 && s_fail) atomicOr(&g_tc_gemm_fault, 1u);
}

// ---------------------------------------------------------------------
// Group-scaled GEMM for ternary and INT8 codes (two MMA passes).  Their
// levels are small integers, exact in BF16, so the weight operand is the
// level itself and only the activation is split (hi + lo): each 128-weight
// K group's dot is accumulated by two MMAs per K step, W * Xh + W * Xl, into
// one of three 128-column TMEM accumulators, and the epilogue warps fold it
// into the tile's running sums (registers: 64 columns per thread) as sum +=
// scale[r, g] * dot, group by group in K order (the reference's per-group
// promotion), while the next groups accumulate into the other buffers (so
// the MMAs run on through most of a tile's store).  Tiles are 128 weight
// rows x 128 tokens.  The weight operand lives in TMEM: the dequantisers
// write each stage's levels (integer bit tricks, the levels8_p16 K order)
// with tcgen05.st into one of four 32-column TMEM stages, so shared memory
// holds only the activation planes, four 32 KB stages deep.
// Roles: warp 0 TMA, warp 1 MMA issuer, warps 2-5 dequantise (levels only),
// warps 6-13 fold and store (two warps per TMEM lane quarter, one per
// 64-column half).  Every wait is bounded; a timed-out CTA writes NaN for
// its tiles and sets the fault word.
// ---------------------------------------------------------------------
constexpr int GS_TN = 128;
constexpr int GS_STAGES = 4;
constexpr int GS_ACCS = 3;   // group accumulators: the MMAs run up to three groups ahead of the fold
constexpr uint32_t kGsXBytes = GS_TN * TK * 2;                       // 16 KB per BF16 plane
constexpr uint32_t kGsStageBytes = 2 * kGsXBytes;                      // 32 KB: Xh, Xl
constexpr uint32_t kGsBarBytes = 256;                                   // 14 mbarriers + the TMEM slot
constexpr uint32_t kGsPairBytes = 4 * kPairBytes;                       // two hand-over buffers per column half
constexpr size_t kGsSmemBytes = GS_STAGES * kGsStageBytes + kGsPairBytes + kGsBarBytes + 1024;
static_assert(kGsSmemBytes + 64 <= 227 * 1024, "two-pass GEMM shared memory");
constexpr uint32_t kGsAccCols = GS_TN;                                 // one group: W.Xh + W.Xl
constexpr uint32_t kGsACol = GS_ACCS * kGsAccCols;                      // weight stages from here
constexpr uint32_t kGsAStageCols = TK / 2;                              // 64 BF16 levels a row
constexpr uint32_t kGsTmemCols = 512;
static_assert(kGsACol + GS_STAGES * kGsAStageCols <= kGsTmemCols, "two-pass GEMM TMEM");
// TMA, MMA, 4 dequantising warps, 8 fold/epilogue warps (two per TMEM lane
// quarter, 64 columns each, their running sums in registers).
constexpr int kGsThreads = 448;
constexpr uint32_t kGsIdesc = idesc_bf16_f32(TM, GS_TN);

// silu(g) * u for the two-pass kernel's SwiGLU epilogue, with the hardware
// exponential and an approximate quotient (a few ulp from silu_mul).  That
// epilogue runs once per 128 x 128 tile, between two tiles' MMAs, and with
// the exact forms it was long enough to stall the tensor pipe.
__device__ __forceinline__ float silu_mul_fast(float g, float u) {
    return __fdividef(g, 1.0f + __expf(-g)) * u;
}

template <int FMT, int MODE>
__global__ void __launch_bounds__(kGsThreads, 1)
    packed_gemm_gs_kernel(const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl,
                          const TcGemmParams p) {
    static_assert(FMT == MF_TERNARY || FMT == MF_INT8, "integer levels only");
    extern __shared__ uint8_t smem_raw[];
    __shared__ volatile int s_fail;
    __shared__ volatile int e_fail;
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *gbase = smem_raw + (base - raw);
    auto xh_s = [&](int s) { return base + s * kGsStageBytes; };
    auto xl_s = [&](int s) { return base + s * kGsStageBytes + kGsXBytes; };
    float *xb0 = reinterpret_cast<float *>(gbase + GS_STAGES * kGsStageBytes);   // [2][2][64][33] pairing buffers
    const uint32_t bars = base + GS_STAGES * kGsStageBytes + kGsPairBytes;
    // full(s): the stage's activation tiles (TMA bytes) and levels (four
    // dequantising warps) are in place, one wait for the MMA issuer.
    // empty(s): the stage's MMAs are done.
    // pfull(b) / pempty(b): a group's dot is complete in TMEM buffer b / the
    // fold warps have read it.
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (GS_STAGES + s); };
    auto pempty = [&](int b) { return bars + 8u * (2 * GS_STAGES + b); };
    auto pfull = [&](int b) { return bars + 8u * (2 * GS_STAGES + GS_ACCS + b); };   // group dot in buffer b
    const uint32_t tmem_slot = bars + 8u * (2 * GS_STAGES + 2 * GS_ACCS);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = p.K / TK;
    const int ntiles = p.tiles_x * p.tiles_y * p.splits;
    // Weight-row tiles fastest: the CTAs of one wave share a few token
    // tiles' activation planes (128 tokens x K x 4 bytes each, 16x a ternary
    // row tile's codes), which then stay in L2 while every row tile reads
    // them; the packed weights are small enough to stay there too.
    auto coords = [&](int tile, int &tx, int &ty, int &z) {
        tx = tile % p.tiles_x;
        const int r = tile / p.tiles_x;
        ty = r % p.tiles_y;
        z = r / p.tiles_y;
    };

    if (threadIdx.x == 0) {
#pragma unroll
        for (int s = 0; s < GS_STAGES; ++s) {
            mbar_init(full(s), 5);
            mbar_init(empty(s), 1);
        }
#pragma unroll
        for (int b = 0; b < GS_ACCS; ++b) {
            mbar_init(pempty(b), 8);
            mbar_init(pfull(b), 1);
        }
        mbar_init_fence();
        s_fail = 0;
        e_fail = 0;
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_map(&tm_xh);
        tma_prefetch_map(&tm_xl);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kGsTmemCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(gbase + (tmem_slot - base));
    pdl_wait();
    pdl_trigger();

    if (warp == 0) {
        // ------------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            for (int tile = blockIdx.x; tile < ntiles && !s_fail; tile += gridDim.x) {
                int tx, ty, z;
                coords(tile, tx, ty, z);
                const int kb0 = z * p.kb_per_split, nkl = min(nk - kb0, p.kb_per_split);
                bool ok = true;
                for (int i = 0; i < nkl; ++i, ++it) {
                    const int s = it % GS_STAGES;
                    if (it >= GS_STAGES && !mbar_wait(empty(s), ((it / GS_STAGES) - 1) & 1)) {
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full(s), 2 * kGsXBytes);
                    tma_load_2d(xh_s(s), &tm_xh, (kb0 + i) * TK, ty * GS_TN, full(s));
                    tma_load_2d(xl_s(s), &tm_xl, (kb0 + i) * TK, ty * GS_TN, full(s));
                }
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t it = 0, gi = 0;   // stages and groups across this CTA's tiles
            bool ok = true;
            for (int tile = blockIdx.x; tile < ntiles && ok && !s_fail; tile += gridDim.x) {
                int tx, ty, z;
                coords(tile, tx, ty, z);
                const int kb0 = z * p.kb_per_split, nkl = min(nk - kb0, p.kb_per_split);
                // One 128-wide K group (two stages) per iteration, into the
                // TMEM buffer the fold warps freed.
                for (int i = 0; i < nkl && ok; i += 2, ++gi) {
                    const int b = gi % GS_ACCS;
                    if (gi >= GS_ACCS && !mbar_wait(pempty(b), ((gi / GS_ACCS) - 1) & 1)) {
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t acc = tmem + b * kGsAccCols;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t u = it + h;
                        const int s = u % GS_STAGES;
                        if (!mbar_wait(full(s), (u / GS_STAGES) & 1)) {
                            s_fail = 1;
                            ok = false;
                            mma_commit(pfull(b));   // release the fold warps' wait on this group
                            break;
                        }
                        tc_fence_after_sync();
#pragma unroll
                        for (int kk = 0; kk < TK / 16; ++kk) {
                            const uint32_t aw = tmem + kGsACol + s * kGsAStageCols + kk * 8;
                            mma_bf16_ts(acc, aw, sw128_kmajor_desc(xh_s(s) + kk * 32), kGsIdesc, (h | kk) != 0);
                            mma_bf16_ts(acc, aw, sw128_kmajor_desc(xl_s(s) + kk * 32), kGsIdesc, 1);
                        }
                        mma_commit(empty(s));
                    }
                    if (ok) mma_commit(pfull(b));   // the group's dot is complete
                    it += 2;
                }
            }
        }
        __syncwarp();
    } else if (warp < 6) {
        // ------------------------------------------ dequantisation (levels)
        // Tile row = TMEM lane: a warp reaches only its lane quarter.
        const int d = 32 * (warp & 3) + lane;
        const int wrow_bytes = FMT == MF_TERNARY ? p.K / 4 : p.K;
        const int groups = p.K / kGroup;
        auto row_base = [&](const uint8_t *codes, int r) -> const uint8_t * {
            if (FMT == MF_TERNARY && p.lanetiled)
                return codes + (size_t)(r >> 4) * groups * 512 + (r & 7) * 64 + ((r >> 3) & 1) * 8;
            return codes + (size_t)r * wrow_bytes;
        };
        auto load = [&](CodeChunk<FMT> &c, const uint8_t *row, int kb, bool valid) {
            if constexpr (FMT == MF_TERNARY) {
                if (p.lanetiled) {
                    load_chunk_lanetiled(c, row, kb, valid);
                    return;
                }
            }
            load_chunk<FMT>(c, row, kb, valid);
        };
        const uint32_t arow = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + kGsACol;
        uint32_t it = 0;
        for (int tile = blockIdx.x; tile < ntiles && !s_fail; tile += gridDim.x) {
            int tx, ty, z;
            coords(tile, tx, ty, z);
            const int kb0 = z * p.kb_per_split, nkl = min(nk - kb0, p.kb_per_split);
            const uint8_t *crow = nullptr;
            bool valid;
            if constexpr (MODE == 2) {
                const int r = tx * (TM / 2) + (d & (TM / 2 - 1));
                valid = r < p.N;
                if (valid) crow = row_base(d >= TM / 2 ? p.codes_b : p.codes_a, r);
            } else if constexpr (MODE == 1) {
                const int v = tx * TM + d;
                valid = v < 2 * p.N;
                if (valid) crow = v >= p.N ? row_base(p.codes_b, v - p.N) : row_base(p.codes_a, v);
            } else {
                const int v = tx * TM + d;
                valid = v < p.N;
                if (valid) crow = row_base(p.codes_a, v);
            }
            // Codes four stages ahead in a register ring (a stage's MMAs take
            // a third of the scale-folded kernel's, so one stage of
            // prefetch no longer covers the load latency).
            constexpr int kRing = 4;
            CodeChunk<FMT> ring[kRing];
#pragma unroll
            for (int u = 0; u < kRing; ++u) load(ring[u], crow, kb0 + min(u, nkl - 1), valid);
            bool ok = true;
            for (int i0 = 0; i0 < nkl && ok; i0 += kRing) {
#pragma unroll
                for (int u = 0; u < kRing; ++u) {
                    const int i = i0 + u;
                    if (i >= nkl) break;
                    const int s = it % GS_STAGES;
                    if (it >= GS_STAGES &&
                        !__all_sync(0xffffffffu, mbar_wait(empty(s), ((it / GS_STAGES) - 1) & 1))) {
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();   // the stage's last MMAs are complete
                    uint32_t lv[32];
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        uint32_t h[4];
                        levels8_p16<FMT>(ring[u], c, h);
#pragma unroll
                        for (int e = 0; e < 4; ++e) lv[4 * c + e] = h[e];
                    }
                    tmem_st_32x32(arow + s * kGsAStageCols, lv);
                    tc_fence_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(full(s));
                    if (i + kRing < nkl) load(ring[u], crow, kb0 + i + kRing, valid);
                    ++it;
                }
            }
            if (!ok) break;
        }
    } else {
        // ------------------------------------------ group fold and epilogue
        const int q = warp & 3;            // TMEM lane quarter of this warp
        const int h = (warp - 6) >> 2;     // column half: tokens 64h .. 64h + 63 of the tile
        const int row = 32 * q + lane;     // tile row of this thread
        const int groups = p.K / kGroup;
        float *xb = xb0 + h * (2 * 64 * 33);   // this half's two hand-over buffers
        uint32_t gi = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            int tx, ty, z;
            coords(tile, tx, ty, z);
            const int kb0 = z * p.kb_per_split, nkl = min(nk - kb0, p.kb_per_split);
            // This row's group scales.
            const float *srow = nullptr;
            if constexpr (MODE == 2) {
                const int r = tx * (TM / 2) + (row & (TM / 2 - 1));
                if (r < p.N) srow = (row >= TM / 2 ? p.scales_b : p.scales_a) + (size_t)r * groups;
            } else if constexpr (MODE == 1) {
                const int v = tx * TM + row;
                if (v < 2 * p.N) srow = v >= p.N ? p.scales_b + (size_t)(v - p.N) * groups : p.scales_a + (size_t)v * groups;
            } else {
                const int v = tx * TM + row;
                if (v < p.N) srow = p.scales_a + (size_t)v * groups;
            }
            float acc[64];
            bool fail = false;
            const uint32_t pcol = ((uint32_t)(32 * q) << 16) + 64 * h;
            float sc = srow ? __ldg(srow + (kb0 >> 1)) : 0.0f;
            for (int g = 0; g < nkl / 2; ++g, ++gi) {
                const int b = gi % GS_ACCS;
                const float sc_next = (srow && g + 1 < nkl / 2) ? __ldg(srow + (kb0 >> 1) + g + 1) : 0.0f;
                if (!__all_sync(0xffffffffu, mbar_wait(pfull(b), (gi / GS_ACCS) & 1))) {
                    fail = true;
                    break;
                }
                tc_fence_after_sync();
                // One 32-column chunk at a time (the SM's 14 warps leave 128
                // registers a thread: 64 sums + 32 loaded + addressing).
#pragma unroll
                for (int cb = 0; cb < 2; ++cb) {
                    uint32_t r[32];
                    tmem_ld_32x32(tmem + b * kGsAccCols + pcol + 32 * cb, r);
                    if (cb == 1) {
                        // The group's dot is in registers: the buffer can refill.
                        tc_fence_before_sync();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(pempty(b));
                    }
                    float *a = acc + 32 * cb;
                    if (g == 0) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) a[i] = sc * __uint_as_float(r[i]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) a[i] = fmaf(sc, __uint_as_float(r[i]), a[i]);
                    }
                }
                sc = sc_next;
            }
            if (fail && lane == 0) e_fail = 1;
            // The eight epilogue warps agree before any pairing exchange.
            named_barrier(1, 256);
            if (e_fail) {
                s_fail = 1;
                break;
            }
            const bool poison = s_fail;
            const int t0 = ty * GS_TN + 64 * h;
            if (p.partial) {
                // Split-K: this split's scaled sums, virtual-row layout.
                int vr;
                if constexpr (MODE == 2) {
                    const int rr = tx * (TM / 2) + (row & (TM / 2 - 1));
                    vr = rr < p.N ? (row < TM / 2 ? rr : p.N + rr) : -1;
                } else {
                    vr = tx * TM + row;
                    if (vr >= p.VR) vr = -1;
                }
                if (vr >= 0) {
                    float *dst = p.partial + (size_t)z * p.T * p.VR + vr;
#pragma unroll
                    for (int i = 0; i < 64; ++i)
                        if (t0 + i < p.T)
                            dst[(size_t)(t0 + i) * p.VR] = poison ? __int_as_float(0x7fc00000) : acc[i];
                }
            } else if constexpr (MODE == 2) {
                // SwiGLU pairing, the work split evenly: gate rows (q < 2)
                // finish the first 32 tokens of the half, up rows (q >= 2)
                // the last 32, each taking its partner's values for those
                // tokens through shared memory.
                const int pr = row & (TM / 2 - 1);
                const bool gate_row = q < 2;
                float *mine = xb + (gate_row ? 1 : 0) * (64 * 33);    // what this thread hands over
                const float *theirs = xb + (gate_row ? 0 : 1) * (64 * 33) + pr * 33;
                // (Branches, not a runtime offset into acc: it stays in registers.)
                if (gate_row) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) mine[pr * 33 + i] = acc[32 + i];
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) mine[pr * 33 + i] = acc[i];
                }
                named_barrier(1, 256);
                const int n = tx * (TM / 2) + pr;
                const int tb = t0 + (gate_row ? 0 : 32);
                float *dst = p.out_a + (size_t)tb * p.N + n;
                if (n < p.N) {
                    // Every partner value is read before the first store:
                    // the compiler cannot tell the shared reads from the
                    // global writes apart, and interleaved they made each
                    // token a serial load-compute-store chain.
                    float v[32];
                    if (gate_row) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = theirs[i];
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = silu_mul_fast(acc[i], v[i]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = theirs[i];
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = silu_mul_fast(v[i], acc[32 + i]);
                    }
                    const int lim = min(32, p.T - tb);
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (i < lim) dst[(size_t)i * p.N] = poison ? __int_as_float(0x7fc00000) : v[i];
                }
            } else {
                const int v = tx * TM + row;
                float *out = p.out_a;
                int n = v;
                if constexpr (MODE == 1) {
                    if (v >= p.N) {
                        out = p.out_b;
                        n = v - p.N;
                    }
                    if (v >= 2 * p.N) n = -1;
                } else {
                    if (v >= p.N) n = -1;
                }
                if (n >= 0) {
#pragma unroll
                    for (int i = 0; i < 64; ++i)
                        if (t0 + i < p.T)
                            out[(size_t)(t0 + i) * p.N + n] = poison ? __int_as_float(0x7fc00000) : acc[i];
                }
            }
        }
    }
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, kGsTmemCols);
    }
    if (threadIdx.x == 0 && s_fail) atomicOr(&g_tc_gemm_fault, 1u);
}

// x (or silu(gate) * up) -> BF16 hi and lo planes, 4 elements per thread.
template <bool SWI_IN>
__device__ __forceinline__ float4 split_input(const float4 *x, const float4 *gate, const float4 *up, size_t i) {
    if constexpr (SWI_IN) {
        const float4 g = gate[i], u = up[i];
        return make_float4(silu_mul(g.x, u.x), silu_mul(g.y, u.y), silu_mul(g.z, u.z), silu_mul(g.w, u.w));
    } else {
        return x[i];
    }
}

// The two-pass kernel's planes: the same split, each 16-element block in the
// levels8_p16 order (position 2m = element m, 2m + 1 = element m + 8).
template <bool SWI_IN>
__global__ void __launch_bounds__(256) split_bf16_p16_kernel(const float4 *x, const float4 *gate, const float4 *up,
                                                             uint4 *xh, uint4 *xl, size_t n16) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x) {
        float v[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 f = split_input<SWI_IN>(x, gate, up, 4 * i + q);
            v[4 * q] = f.x;
            v[4 * q + 1] = f.y;
            v[4 * q + 2] = f.z;
            v[4 * q + 3] = f.w;
        }
        uint32_t h[8], l[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const __nv_bfloat162 hv = __floats2bfloat162_rn(v[m], v[m + 8]);
            const float2 hf = __bfloat1622float2(hv);
            h[m] = bf16x2_bits(hv);
            l[m] = bf16x2_bits(__floats2bfloat162_rn(v[m] - hf.x, v[m + 8] - hf.y));
        }
        xh[2 * i] = make_uint4(h[0], h[1], h[2], h[3]);
        xh[2 * i + 1] = make_uint4(h[4], h[5], h[6], h[7]);
        xl[2 * i] = make_uint4(l[0], l[1], l[2], l[3]);
        xl[2 * i + 1] = make_uint4(l[4], l[5], l[6], l[7]);
    }
}

template <bool SWI_IN>
__global__ void __launch_bounds__(256) split_bf16_kernel(const float4 *x, const float4 *gate, const float4 *up,
                                                         uint2 *xh, uint2 *xl, size_t n4) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = split_input<SWI_IN>(x, gate, up, i);
        const __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y), h1 = __floats2bfloat162_rn(v.z, v.w);
        const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
        const __nv_bfloat162 l0 = __floats2bfloat162_rn(v.x - f0.x, v.y - f0.y);
        const __nv_bfloat162 l1 = __floats2bfloat162_rn(v.z - f1.x, v.w - f1.y);
        xh[i] = make_uint2(bf16x2_bits(h0), bf16x2_bits(h1));
        xl[i] = make_uint2(bf16x2_bits(l0), bf16x2_bits(l1));
    }
}

// out = sum over splits of partial[z][t][vr] in split order, then the mode's
// epilogue: single, pair rows (B's rows at N..2N-1), SwiGLU pair.
template <int MODE>
__global__ void __launch_bounds__(256) split_reduce_kernel(const float *partial, float *out_a, float *out_b, int T,
                                                           int N, int VR, int splits) {
    pdl_wait();
    pdl_trigger();
    const size_t total = (size_t)T * N;
    const size_t plane = (size_t)T * VR;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const size_t t = e / N, n = e - t * N;
        const float *pa = partial + t * VR + n;
        float a = 0.0f, b = 0.0f;
        for (int z = 0; z < splits; ++z) {
            a += pa[(size_t)z * plane];
            if (MODE != 0) b += pa[(size_t)z * plane + N];
        }
        if constexpr (MODE == 0) {
            out_a[e] = a;
        } else if constexpr (MODE == 1) {
            out_a[e] = a;
            out_b[e] = b;
        } else {
            out_a[e] = silu_mul(a, b);
        }
    }
}

// Split-K plan: a grid of fewer tiles than ~60% of the SMs splits K (at
// least 8 stages of 64 per split, at most 4 splits).
struct TcPlan {
    int tiles_x, tiles_y, splits, kb_per_split, vr;
};

// tn: tokens per tile (TN, or GS_TN for the group-scaled kernel, whose
// splits hold whole 128-wide groups).
TcPlan tc_plan(int mode, uint64_t t, uint64_t n, uint64_t k, int tn = TN) {
    TcPlan pl{};
    const int rows_per_tile = mode == kPackedSwigluPair ? TM / 2 : TM;
    const uint64_t vrows = mode == kPackedPairRows ? 2 * n : n;
    pl.tiles_x = (int)((vrows + rows_per_tile - 1) / rows_per_tile);
    pl.tiles_y = (int)((t + tn - 1) / tn);
    pl.vr = (int)(mode == kPackedSingle ? n : 2 * n);
    const int nk = (int)(k / TK);
    const int tiles = pl.tiles_x * pl.tiles_y;
    const int sms = sm_count();
    int splits = 1;
    if (tiles * 10 < sms * 6) splits = std::min({4, std::max(1, sms / tiles), std::max(1, nk / 8)});
    pl.kb_per_split = (nk + splits - 1) / splits;
    if (tn == GS_TN) pl.kb_per_split = (pl.kb_per_split + 1) & ~1;   // whole groups per split
    pl.splits = (nk + pl.kb_per_split - 1) / pl.kb_per_split;
    return pl;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

// [T, K] BF16 plane, boxes of 64 (K) x box_tokens, 128-byte swizzle.
int32_t plane_map(CUtensorMap *map, const void *plane, uint64_t t, uint64_t k, int box_tokens = TN) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return fail(MF_UNSUPPORTED, "driver entry point cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {k, t};
    const cuuint64_t strides[1] = {k * 2};
    const cuuint32_t box[2] = {(cuuint32_t)TK, (cuuint32_t)box_tokens};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(plane), dims, strides, box,
                          elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MF_BACKEND_FAILURE, "cuTensorMapEncodeTiled rejected the activation plane");
    return MF_OK;
}

template <int FMT, int MODE>
int32_t launch_tc(const CUtensorMap &mh, const CUtensorMap &ml, const TcGemmParams &p, const TcPlan &pl,
                  cudaStream_t stream) {
    auto kernel = packed_gemm_tc_kernel<FMT, MODE>;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [&] {
        attr = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    });
    MF_CUDA_TRY(attr);
    const int ntiles = pl.tiles_x * pl.tiles_y * pl.splits;
    const dim3 grid(std::min(ntiles, sm_count()));   // one persistent CTA per SM
    if (int32_t e_ = ::mf::launch(kernel, grid, dim3(kThreads), kSmemBytes, stream, "packed_gemm_tc_kernel", mh, ml, p))
        return e_;
    if (pl.splits == 1) return MF_OK;
    const size_t total = (size_t)p.T * p.N;
    const unsigned blocks = (unsigned)std::min<size_t>((total + 255) / 256, 148 * 16);
    return ::mf::launch(split_reduce_kernel<MODE>, dim3(blocks), dim3(256), 0, stream, "split_reduce_kernel",
                        (const float *)p.partial, p.out_a, p.out_b, p.T, p.N, p.VR, pl.splits);
}

template <int FMT, int MODE>
int32_t launch_gs(const CUtensorMap &mh, const CUtensorMap &ml, const TcGemmParams &p, const TcPlan &pl,
                  cudaStream_t stream) {
    auto kernel = packed_gemm_gs_kernel<FMT, MODE>;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [&] {
        attr = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGsSmemBytes);
    });
    MF_CUDA_TRY(attr);
    const int ntiles = pl.tiles_x * pl.tiles_y * pl.splits;
    const dim3 grid(std::min(ntiles, sm_count()));   // one persistent CTA per SM
    if (int32_t e_ = ::mf::launch(kernel, grid, dim3(kGsThreads), kGsSmemBytes, stream, "packed_gemm_gs_kernel", mh, ml,
                                  p))
        return e_;
    if (pl.splits == 1) return MF_OK;
    const size_t total = (size_t)p.T * p.N;
    const unsigned blocks = (unsigned)std::min<size_t>((total + 255) / 256, 148 * 16);
    return ::mf::launch(split_reduce_kernel<MODE>, dim3(blocks), dim3(256), 0, stream, "split_reduce_kernel",
                        (const float *)p.partial, p.out_a, p.out_b, p.T, p.N, p.VR, pl.splits);
}

template <int MODE>
int32_t by_format(const CUtensorMap &mh, const CUtensorMap &ml, const TcGemmParams &p, const TcPlan &pl, int format,
                  cudaStream_t stream) {
    switch (format) {
    case MF_TERNARY: return launch_tc<MF_TERNARY, MODE>(mh, ml, p, pl, stream);
    case MF_NF4: return launch_tc<MF_NF4, MODE>(mh, ml, p, pl, stream);
    case MF_INT8: return launch_tc<MF_INT8, MODE>(mh, ml, p, pl, stream);
    default: return fail(MF_INVALID_ARGUMENT, "unknown packed format");
    }
}

}  // namespace

// Split-K partial floats of a call (0 without a split).
size_t split_floats(int mode, uint64_t t, uint64_t n, uint64_t k) {
    // The larger of the two kernels' split-K partials.
    size_t out = 0;
    for (int tn : {TN, GS_TN}) {
        const TcPlan pl = tc_plan(mode, t, n, k, tn);
        if (pl.splits > 1) out = std::max(out, (size_t)pl.splits * t * pl.vr);
    }
    return out;
}

size_t packed_gemm_tc_scratch_floats(uint64_t t, uint64_t n, uint64_t k) {
    // Two BF16 planes of [t, k] (4 bytes per element), then the split-K
    // partials of the largest mode.
    size_t part = 0;
    for (int mode : {(int)kPackedSingle, (int)kPackedPairRows, (int)kPackedSwigluPair})
        part = std::max(part, split_floats(mode, t, n, k));
    return (size_t)t * (size_t)k + part;
}

int32_t packed_gemm_tc(int mode, bool swiglu_input, float *out_a, float *out_b, const float *x, const float *gate,
                       const float *up, uint64_t t, const uint8_t *codes_a, const float *scales_a,
                       const uint8_t *codes_b, const float *scales_b, uint64_t n, uint64_t k, int format,
                       const SplitScratch &ss, cudaStream_t stream, bool lanetiled) {
    if (t == 0 || n == 0) return MF_OK;
    if (k == 0 || k % kGroup) return fail(MF_INVALID_SHAPE, "packed GEMM inner width must be a positive multiple of 128");
    if (t > (1u << 24) || n > (1u << 28) || k > (1u << 20))
        return fail(MF_UNSUPPORTED, "packed matmul dimension exceeds kernel limits");
    if ((t + TN - 1) / TN > 65535u) return fail(MF_UNSUPPORTED, "packed GEMM token count exceeds grid limit");
    if (lanetiled && (format != MF_TERNARY || n % 16))
        return fail(MF_INVALID_ARGUMENT, "LUT2 codes are ternary with rows in multiples of 16");
    if (!ss.partial || ss.partial_floats < (size_t)t * k + split_floats(mode, t, n, k))
        return fail(MF_RESOURCE_LIMIT, "tensor-core GEMM needs activation and split-K scratch");
    uint16_t *xh = reinterpret_cast<uint16_t *>(ss.partial);
    uint16_t *xl = xh + (size_t)t * k;
    // Ternary and INT8 levels are exact in BF16: the group-scaled two-pass
    // kernel (measured faster than the three-pass one at every token count,
    // 64 to 4,096).  NF4 levels are not: it takes the three-pass kernel.
    const bool gs = format != MF_NF4 && g_gemm_passes.load(std::memory_order_relaxed) != 3;
    const float4 *xf = reinterpret_cast<const float4 *>(x);
    const float4 *gf = reinterpret_cast<const float4 *>(swiglu_input ? gate : nullptr);
    const float4 *uf = reinterpret_cast<const float4 *>(swiglu_input ? up : nullptr);
    if (gs) {
        const size_t n16 = (size_t)t * k / 16;
        const unsigned blocks = (unsigned)std::min<size_t>((n16 + 255) / 256, 148 * 16);
        auto kernel = swiglu_input ? split_bf16_p16_kernel<true> : split_bf16_p16_kernel<false>;
        if (int32_t e_ = ::mf::launch(kernel, dim3(blocks), dim3(256), 0, stream, "split_bf16_p16_kernel", xf, gf, uf,
                                      reinterpret_cast<uint4 *>(xh), reinterpret_cast<uint4 *>(xl), n16))
            return e_;
    } else {
        const size_t n4 = (size_t)t * k / 4;
        const unsigned blocks = (unsigned)std::min<size_t>((n4 + 255) / 256, 148 * 16);
        auto kernel = swiglu_input ? split_bf16_kernel<true> : split_bf16_kernel<false>;
        if (int32_t e_ = ::mf::launch(kernel, dim3(blocks), dim3(256), 0, stream, "split_bf16_kernel", xf, gf, uf,
                                      reinterpret_cast<uint2 *>(xh), reinterpret_cast<uint2 *>(xl), n4))
            return e_;
    }
    CUtensorMap mh, ml;
    if (int32_t e_ = plane_map(&mh, xh, t, k, gs ? GS_TN : TN)) return e_;
    if (int32_t e_ = plane_map(&ml, xl, t, k, gs ? GS_TN : TN)) return e_;
    const TcPlan pl = tc_plan(mode, t, n, k, gs ? GS_TN : TN);
    TcGemmParams p{codes_a, codes_b, scales_a, scales_b, out_a, out_b, (int)t, (int)n, (int)k, nullptr,
                   pl.kb_per_split, pl.vr, pl.tiles_x, pl.tiles_y, pl.splits};
    if (pl.splits > 1) p.partial = ss.partial + (size_t)t * k;
    p.lanetiled = lanetiled ? 1 : 0;
    if (gs) {
        if (format == MF_TERNARY) {
            if (mode == kPackedSingle) return launch_gs<MF_TERNARY, 0>(mh, ml, p, pl, stream);
            if (mode == kPackedPairRows) return launch_gs<MF_TERNARY, 1>(mh, ml, p, pl, stream);
            return launch_gs<MF_TERNARY, 2>(mh, ml, p, pl, stream);
        }
        if (mode == kPackedSingle) return launch_gs<MF_INT8, 0>(mh, ml, p, pl, stream);
        if (mode == kPackedPairRows) return launch_gs<MF_INT8, 1>(mh, ml, p, pl, stream);
        return launch_gs<MF_INT8, 2>(mh, ml, p, pl, stream);
    }
    if (mode == kPackedSingle) return by_format<0>(mh, ml, p, pl, format, stream);
    if (mode == kPackedPairRows) return by_format<1>(mh, ml, p, pl, format, stream);
    return by_format<2>(mh, ml, p, pl, format, stream);
}

int32_t packed_gemm_tc_faults(uint32_t *flags) {
    unsigned v = 0;
    MF_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_tc_gemm_fault, sizeof(v)));
    const unsigned zero = 0;
    MF_CUDA_TRY(cudaMemcpyToSymbol(g_tc_gemm_fault, &zero, sizeof(zero)));
    *flags = v;
    return MF_OK;
}

}  // namespace mf

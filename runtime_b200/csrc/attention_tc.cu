// Many-token causal GQA (prefill) on the tcgen05 tensor cores, head
// dimension 64: the scores S = Q K^T and the products P V as BF16 MMAs with
// F32 accumulators in TMEM, the online softmax in F32 between them.
//
// The reference computes attention in F32
// (crates/backend-cpu/src/attention_convolution.rs:11-187: scores
// dot(q, k) / sqrt(head_dim), causal mask, softmax, weighted sum of v).  A
// BF16 operand carries 8 significant bits, so each F32 operand is split
// into three BF16 parts v = h + m + l (24 bits) and each product of two
// operands sums the six part products of order <= 2 (h*h, h*m, m*h, h*l,
// l*h, m*m; the rest are below 2^-24 relative), for Q K^T and for P V.
// Two parts (16 bits) were not enough: for rows that see only a few keys
// they left errors of ~2e-5 on unit-scale outputs, twice the 1e-5 the F32
// kernel meets.
//
// One CTA owns 128 query rows: 128 / group tokens times the `group` query
// heads that share one kv head (row r = token r / group, head r % group),
// and walks the visible keys in tiles of 64.  Roles (352 threads):
//   warps 4-9  load each K and V tile (F32, from the cache), split it and
//              write K [key][dim] and V^T [dim][key] as swizzled BF16 part
//              tiles, two stages deep (the Q tile once, the same way);
//   warps 0-3  one query row per thread (= its TMEM lane): read the tile's
//              scores from TMEM, mask and scale them, update the running
//              max and sum, write P = exp(s - max) as three BF16 parts into
//              TMEM (the A operand of P V), and fold the previous tile's
//              P V into the row's output, kept in 64 registers as
//              O = O * correction + P V with F32 adds; at the end O / sum
//              to global memory;
//   warp 10    one lane issues the MMAs: S(j+1) = Q K(j+1)^T into the
//              other of two score buffers while the softmax works on S(j),
//              then P(j) V(j) into TMEM from zero once P(j) is written.
// Each tile's P V starts from zero and is added to the output in F32
// registers, so no accumulator sums over the whole key range inside the
// tensor cores.  Scores, P and P V are double-buffered in TMEM (2 x 64,
// 2 x 3 x 32 and 2 x 64 columns; P two BF16 per column), so the softmax of
// one tile overlaps the MMAs of the one before.  Every wait is bounded; a
// CTA whose wait expires writes NaN for its rows and sets the fault word.
#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "mf_common.cuh"
#include "packed_kernels.h"
#include "tc_sm100.cuh"

namespace mf {

// Set (bit 0) by a tensor-core attention whose pipeline wait timed out.
__device__ unsigned int g_tc_attn_fault = 0;

// Many-token attention on the tensor cores (default) or the F32 kernel.
std::atomic<bool> g_attn_tc{true};
void set_attention_tc(bool on) { g_attn_tc.store(on, std::memory_order_relaxed); }
bool attention_tc_enabled() { return g_attn_tc.load(std::memory_order_relaxed); }

namespace {

using namespace sm100;

constexpr int AT_ROWS = 128;    // query rows per CTA (MMA M)
constexpr int AT_KEYS = 64;     // keys per tile (N of Q K^T, K of P V)
constexpr int AT_DIM = 64;      // head dimension (K of Q K^T, N of P V)
constexpr int AT_STAGES = 2;
constexpr int AT_LOADERS = 6;                      // loader warps 4 .. 3 + AT_LOADERS
constexpr int AT_MMA_WARP = 4 + AT_LOADERS;
constexpr int AT_THREADS = 32 * (AT_MMA_WARP + 1);
constexpr int AT_PARTS = 3;     // BF16 parts of every operand
constexpr uint32_t kQPart = AT_ROWS * AT_DIM * 2;                  // 16 KB: [128 rows][64 dims]
constexpr uint32_t kKPart = AT_KEYS * AT_DIM * 2;                  // 8 KB: [64 keys][64 dims]
constexpr uint32_t kVPart = AT_DIM * AT_KEYS * 2;                  // 8 KB: V^T [64 dims][64 keys]
constexpr uint32_t kQBytes = AT_PARTS * kQPart;
constexpr uint32_t kStageBytes = AT_PARTS * (kKPart + kVPart);     // 48 KB
constexpr int kRawPitch = AT_DIM + 4;                               // floats per staged row (conflict-free columns)
constexpr uint32_t kRawBytes = AT_ROWS * kRawPitch * 4;             // 34 KB: Q, or one tile's K and V
constexpr uint32_t kBarBytes = 128;
constexpr size_t kAtSmemBytes = kQBytes + AT_STAGES * kStageBytes + 2 * kRawBytes + kBarBytes + 1024;
static_assert(kAtSmemBytes + 64 <= 227 * 1024, "attention shared memory");
constexpr uint32_t kSCol = 0;       // two score buffers of 64 columns
constexpr uint32_t kPCol = 128;     // two P buffers: 3 parts x 32 columns (64 keys, two per column)
constexpr uint32_t kPBuf = AT_PARTS * 32;
constexpr uint32_t kXCol = 320;     // two P V buffers of 64 columns
constexpr uint32_t kAtTmemCols = 512;
constexpr uint32_t kIdescS = idesc_bf16_f32(AT_ROWS, AT_KEYS);
constexpr uint32_t kIdescO = idesc_bf16_f32(AT_ROWS, AT_DIM);
// The part products of order <= 2, as (part of the A operand, part of B).
constexpr int kPairs = 6;
__host__ __device__ constexpr int pair_a(int i) { return i == 2 ? 1 : i == 4 ? 2 : i == 5 ? 1 : 0; }
__host__ __device__ constexpr int pair_b(int i) { return i == 1 ? 1 : i == 3 ? 2 : i == 5 ? 1 : 0; }

// x = h + m + l exactly: each part is the next 8 significant bits of x
// (truncated to BF16; every remainder is exact in F32), for a pair of
// values, packed two per word (a in the low half).
__device__ __forceinline__ void split3(float a, float b, uint32_t (&w)[3]) {
#pragma unroll
    for (int p = 0; p < AT_PARTS; ++p) {
        const uint32_t ha = __float_as_uint(a) & 0xffff0000u, hb = __float_as_uint(b) & 0xffff0000u;
        w[p] = __byte_perm(ha, hb, 0x7632);
        a -= __uint_as_float(ha);
        b -= __uint_as_float(hb);
    }
}

// 16-byte asynchronous copy to shared memory; `bytes` 0 writes zeros.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Byte offset of element `col` (BF16) of row `row` in a [rows][64] tile in
// the 128-byte swizzled K-major layout the MMA descriptors describe.
__device__ __forceinline__ uint32_t sw_off(uint32_t row, uint32_t col) {
    return row * 128u + ((((col * 2u) >> 4) ^ (row & 7u)) << 4) + ((col * 2u) & 15u);
}

// 32 TMEM lanes x 8 columns from 8 registers (no wait).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(AT_THREADS, 1)
    gqa_prefill_tc_kernel(float *out, const float *q, const float *key_cache, const float *value_cache, uint64_t len,
                          const uint64_t *len_dev, uint64_t tokens, uint32_t q_heads, uint32_t kv_heads,
                          uint64_t cache_stride) {
    extern __shared__ uint8_t at_smem_raw[];
    __shared__ volatile int s_fail;
    const uint32_t raw = smem_u32(at_smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *gbase = at_smem_raw + (base - raw);
    auto q_s = [&](int p) { return base + p * kQPart; };
    auto k_s = [&](int s, int p) { return base + kQBytes + s * kStageBytes + p * kKPart; };
    auto v_s = [&](int s, int p) { return base + kQBytes + s * kStageBytes + AT_PARTS * kKPart + p * kVPart; };
    const uint32_t raw0 = base + kQBytes + AT_STAGES * kStageBytes;   // two F32 staging buffers
    const uint32_t bars = raw0 + 2 * kRawBytes;
    auto q_full = [&]() { return bars; };
    auto kv_full = [&](int s) { return bars + 8u * (1 + s); };
    auto kv_empty = [&](int s) { return bars + 8u * (3 + s); };
    auto s_full = [&](int b) { return bars + 8u * (5 + b); };
    auto p_full = [&](int b) { return bars + 8u * (7 + b); };    // P buffer b written
    auto pv_done = [&](int b) { return bars + 8u * (9 + b); };   // P V into buffer b complete
    const uint32_t ld_bar = bars + 8u * 11;                       // the loader warps meet
    const uint32_t tmem_slot = bars + 8u * 12;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(q_full(), AT_LOADERS);
        mbar_init(ld_bar, AT_LOADERS);
#pragma unroll
        for (int s = 0; s < AT_STAGES; ++s) {
            mbar_init(kv_full(s), AT_LOADERS);
            mbar_init(kv_empty(s), 1);
            mbar_init(s_full(s), 1);
            mbar_init(p_full(s), 4);   // the four softmax warps
            mbar_init(pv_done(s), 1);
        }
        mbar_init_fence();
        s_fail = 0;
    }
    if (warp == AT_MMA_WARP) {
        tmem_alloc(tmem_slot, kAtTmemCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(gbase + (tmem_slot - base));
    pdl_wait();
    pdl_trigger();

    // blockIdx.z: sequence of a batch (tokens rows each, caches cache_stride
    // floats apart, its own length).
    const uint64_t qw = (uint64_t)q_heads * AT_DIM, kvw = (uint64_t)kv_heads * AT_DIM;
    {
        const uint64_t b = blockIdx.z;
        q += b * tokens * qw;
        out += b * tokens * qw;
        key_cache += b * cache_stride;
        value_cache += b * cache_stride;
        if (len_dev) len_dev += b;
    }
    const uint32_t group = q_heads / kv_heads;
    const uint32_t tpc = AT_ROWS / group;                      // tokens per CTA
    const uint32_t kvh = blockIdx.y;
    const uint64_t tb = (uint64_t)(gridDim.x - 1 - blockIdx.x) * tpc;   // longest blocks first
    const uint64_t base_len = len_dev ? *len_dev : len;
    const uint64_t t_last = min(tb + tpc, tokens) - 1;
    const uint64_t kend = base_len + t_last + 1;                // keys any row of the block sees
    const int ntiles = (int)((kend + AT_KEYS - 1) / AT_KEYS);

    if (warp >= 4 && warp < 4 + AT_LOADERS) {
        // ------------------------------------------- loaders: Q once, K / V tiles
        // The F32 rows arrive by cp.async in two staging buffers (padded
        // rows, conflict-free column reads), one tile ahead of the split;
        // the split then reads shared memory and writes each BF16 part with
        // 128-bit stores.  Loops stay rolled: with the four roles' code
        // fully unrolled the instruction cache missed more than anything
        // else stalled.
        constexpr int kLt = 32 * AT_LOADERS;
        const int tid = threadIdx.x - 128;   // 0..kLt-1
        auto raw = [&](int b) { return raw0 + (uint32_t)b * kRawBytes; };
        auto rawf = [&](int b) { return reinterpret_cast<const float *>(gbase + (raw(b) - base)); };
        // The loader warps meet on an mbarrier with a bounded wait (a
        // warp that left on a failed wait cannot hold the others forever).
        uint32_t ld_phase = 0;
        auto loader_sync = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(ld_bar);
            const bool ok = __all_sync(0xffffffffu, mbar_wait(ld_bar, ld_phase & 1));
            ++ld_phase;
            if (!ok) s_fail = 1;
            return ok;
        };
        // Staged tile j: K rows 0..63, V rows 64..127 of buffer (j + 1) & 1.
        auto fetch = [&](int j) {
            const uint64_t k0 = (uint64_t)j * AT_KEYS;
            const uint32_t rb = raw((j + 1) & 1);
#pragma unroll 2
            for (int e = tid; e < 2 * AT_KEYS * 16; e += kLt) {
                const int row = e >> 4, c4 = e & 15, key = row & (AT_KEYS - 1);
                const float *src = row < AT_KEYS ? key_cache : value_cache;
                const bool in = k0 + key < kend;
                cp_async16(rb + (uint32_t)(row * kRawPitch + 4 * c4) * 4,
                           src + (in ? (k0 + key) * kvw + (uint64_t)kvh * AT_DIM + 4 * c4 : 0), in ? 16u : 0u);
            }
            cp_async_commit();
        };
        // Q: 128 rows into buffer 0.
#pragma unroll 2
        for (int e = tid; e < AT_ROWS * 16; e += kLt) {
            const int r = e >> 4, c4 = e & 15;
            const uint64_t t = tb + r / group;
            cp_async16(raw(0) + (uint32_t)(r * kRawPitch + 4 * c4) * 4,
                       q + (t < tokens ? t * qw + (uint64_t)(kvh * group + r % group) * AT_DIM + 4 * c4 : 0),
                       t < tokens ? 16u : 0u);
        }
        cp_async_commit();
        fetch(0);
        // Split 8 staged values of one row (F32, 16-byte aligned) into the
        // three parts and store them at `off` of each part tile.
        auto split8 = [&](const float *src, uint32_t part0, uint32_t pitch_bytes, uint32_t off) {
            const float4 a = *reinterpret_cast<const float4 *>(src), b = *reinterpret_cast<const float4 *>(src + 4);
            uint32_t w0[3], w1[3], w2[3], w3[3];
            split3(a.x, a.y, w0);
            split3(a.z, a.w, w1);
            split3(b.x, b.y, w2);
            split3(b.z, b.w, w3);
#pragma unroll
            for (int p = 0; p < AT_PARTS; ++p)
                *reinterpret_cast<uint4 *>(gbase + (part0 - base) + p * pitch_bytes + off) =
                    make_uint4(w0[p], w1[p], w2[p], w3[p]);
        };
        cp_async_wait<1>();
        bool lok = loader_sync();
#pragma unroll 1
        for (int e = tid; lok && e < AT_ROWS * 8; e += kLt) {
            const int r = e >> 3, g = e & 7;
            split8(rawf(0) + r * kRawPitch + 8 * g, q_s(0), kQPart, sw_off(r, 8 * g));
        }
        lok = lok && loader_sync();   // buffer 0 free for tile 1
        if (lok && ntiles > 1) fetch(1);
        fence_async_smem();
        __syncwarp();
        if (lok && lane == 0) mbar_arrive(q_full());
        for (int j = 0; lok && j < ntiles; ++j) {
            const int s = j & 1;
            if (j + 1 < ntiles)
                cp_async_wait<1>();
            else
                cp_async_wait<0>();
            if (!loader_sync()) break;
            if (j >= AT_STAGES && !__all_sync(0xffffffffu, mbar_wait(kv_empty(s), ((j >> 1) - 1) & 1))) {
                s_fail = 1;
                break;
            }
            const float *rk = rawf((j + 1) & 1), *rv = rk + AT_KEYS * kRawPitch;
            // K [key][dim]: one item is 8 dims of one key.
#pragma unroll 1
            for (int e = tid; e < AT_KEYS * 8; e += kLt) {
                const int key = e >> 3, g = e & 7;
                split8(rk + key * kRawPitch + 8 * g, k_s(s, 0), kKPart, sw_off(key, 8 * g));
            }
            // V^T [dim][key]: one item is 8 keys of one dim (column reads).
#pragma unroll 1
            for (int e = tid; e < AT_DIM * 8; e += kLt) {
                const int d = e & (AT_DIM - 1), g = e >> 6;
                float f[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) f[i] = rv[(8 * g + i) * kRawPitch + d];
                uint32_t w0[3], w1[3], w2[3], w3[3];
                split3(f[0], f[1], w0);
                split3(f[2], f[3], w1);
                split3(f[4], f[5], w2);
                split3(f[6], f[7], w3);
#pragma unroll
                for (int p = 0; p < AT_PARTS; ++p)
                    *reinterpret_cast<uint4 *>(gbase + (v_s(s, p) - base) + sw_off(d, 8 * g)) =
                        make_uint4(w0[p], w1[p], w2[p], w3[p]);
            }
            if (!loader_sync()) break;   // staging buffer read by all: refill it
            if (j + 2 < ntiles) fetch(j + 2);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(kv_full(s));
        }
        cp_async_wait<0>();
    } else if (warp < 4) {
        // ------------------------------------------------ softmax, one row per thread
        const uint32_t r = 32u * warp + lane;                       // = TMEM lane
        const uint32_t lq = (uint32_t)(32 * warp) << 16;            // lane-quarter address bits
        const uint64_t t = tb + r / group;
        const uint64_t lim = base_len + min(t, t_last) + 1;        // keys below lim are visible
        const float scale = 0.125f;                                 // 1 / sqrt(64), exact
        float m = -INFINITY, l = 0.0f, c_prev = 0.0f;
        float o[AT_DIM];
#pragma unroll
        for (int i = 0; i < AT_DIM; ++i) o[i] = 0.0f;
        // o = o * c + (P V of tile jj), read from its TMEM buffer.
        auto fold = [&](int jj, float c) {
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t xv[32];
                tmem_ld_32x32(tmem + lq + kXCol + (uint32_t)(jj & 1) * AT_DIM + 32 * hf, xv);
#pragma unroll
                for (int i = 0; i < 32; ++i) o[32 * hf + i] = fmaf(o[32 * hf + i], c, __uint_as_float(xv[i]));
            }
        };
        bool ok = true;
        for (int j = 0; j < ntiles && ok; ++j) {
            if (!__all_sync(0xffffffffu, mbar_wait(s_full(j & 1), (j >> 1) & 1))) {
                ok = false;
                break;
            }
            tc_fence_after_sync();
            const uint64_t k0 = (uint64_t)j * AT_KEYS;
            const uint32_t sb = tmem + lq + kSCol + (uint32_t)(j & 1) * AT_KEYS;
            float mx = -INFINITY;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t sv[32];
                tmem_ld_32x32(sb + 32 * hf, sv);
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (k0 + 32 * hf + i < lim) mx = fmaxf(mx, __fmul_rn(__uint_as_float(sv[i]), scale));
            }
            const float m_new = fmaxf(m, mx);                        // finite: key 0 is visible to every row
            const float corr = m == -INFINITY ? 0.0f : __expf(m - m_new);
            // P buffer j & 1 was last read by P(j-2) V(j-2).
            if (j >= 2) {
                if (!__all_sync(0xffffffffu, mbar_wait(pv_done(j & 1), ((j - 2) >> 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
            }
            float sum = 0.0f;
            const uint32_t pb = tmem + lq + kPCol + (uint32_t)(j & 1) * kPBuf;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t sv[32];
                tmem_ld_32x32(sb + 32 * hf, sv);
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t pw[AT_PARTS][8];
#pragma unroll
                    for (int i = 0; i < 16; i += 2) {
                        const int k = 16 * c + i;
                        const uint64_t key = k0 + 32 * hf + k;
                        const float p0 = key < lim ? __expf(__fmul_rn(__uint_as_float(sv[k]), scale) - m_new) : 0.0f;
                        const float p1 = key + 1 < lim ? __expf(__fmul_rn(__uint_as_float(sv[k + 1]), scale) - m_new) : 0.0f;
                        sum += p0 + p1;
                        uint32_t w[3];
                        split3(p0, p1, w);
#pragma unroll
                        for (int p = 0; p < AT_PARTS; ++p) pw[p][i / 2] = w[p];
                    }
#pragma unroll
                    for (int p = 0; p < AT_PARTS; ++p) tmem_st8(pb + 32 * p + 16 * hf + 8 * c, pw[p]);
                }
            }
            tmem_wait_st();
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full(j & 1));
            // Fold the previous tile's P V (its buffer is next written by
            // P(j+1) V(j+1), after this warp's next arrival).
            if (j > 0) {
                if (!__all_sync(0xffffffffu, mbar_wait(pv_done((j - 1) & 1), ((j - 1) >> 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                fold(j - 1, c_prev);
            }
            l = l * corr + sum;
            m = m_new;
            c_prev = corr;
        }
        if (ok) {
            if (__all_sync(0xffffffffu, mbar_wait(pv_done((ntiles - 1) & 1), ((ntiles - 1) >> 1) & 1))) {
                tc_fence_after_sync();
                fold(ntiles - 1, c_prev);
            } else {
                ok = false;
            }
        }
        if (!ok) s_fail = 1;
        const bool poison = !ok || s_fail;
        if (t < tokens) {
            float *dst = out + t * qw + (uint64_t)(kvh * group + r % group) * AT_DIM;
            const float nan = __int_as_float(0x7fc00000);
#pragma unroll
            for (int i = 0; i < AT_DIM; i += 4) {
                const float4 v = poison ? make_float4(nan, nan, nan, nan)
                                        : make_float4(o[i] / l, o[i + 1] / l, o[i + 2] / l, o[i + 3] / l);
                *reinterpret_cast<float4 *>(dst + i) = v;
            }
        }
    } else if (warp == AT_MMA_WARP) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0) {
            bool ok = mbar_wait(q_full(), 0) && mbar_wait(kv_full(0), 0);
            auto issue_s = [&](int j) {
                const int s = j & 1;
                const uint32_t d = tmem + kSCol + (uint32_t)s * AT_KEYS;
#pragma unroll
                for (int kk = 0; kk < AT_DIM / 16; ++kk)
#pragma unroll
                    for (int i = 0; i < kPairs; ++i)
                        mma_bf16_ss(d, sw128_kmajor_desc(q_s(pair_a(i)) + kk * 32),
                                    sw128_kmajor_desc(k_s(s, pair_b(i)) + kk * 32), kIdescS, (kk | i) != 0);
                mma_commit(s_full(s));
            };
            if (ok) {
                tc_fence_after_sync();
                issue_s(0);
            }
            for (int j = 0; j < ntiles && ok; ++j) {
                if (j + 1 < ntiles) {
                    if (!mbar_wait(kv_full((j + 1) & 1), ((j + 1) >> 1) & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    issue_s(j + 1);
                }
                const int s = j & 1;
                if (!mbar_wait(p_full(s), (j >> 1) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t x = tmem + kXCol + (uint32_t)s * AT_DIM;   // this tile's P V, from zero
                const uint32_t pa = tmem + kPCol + (uint32_t)s * kPBuf;
#pragma unroll
                for (int kk = 0; kk < AT_KEYS / 16; ++kk)
#pragma unroll
                    for (int i = 0; i < kPairs; ++i)
                        mma_bf16_ts(x, pa + 32 * pair_a(i) + 8 * kk, sw128_kmajor_desc(v_s(s, pair_b(i)) + kk * 32),
                                    kIdescO, (kk | i) != 0);
                mma_commit(pv_done(s));
                mma_commit(kv_empty(s));
            }
            if (!ok) {
                s_fail = 1;
                // release the softmax warps' waits
                mma_commit(pv_done(0));
                mma_commit(pv_done(1));
                mma_commit(s_full(0));
                mma_commit(s_full(1));
            }
        }
        __syncwarp();
    }
    tc_fence_before_sync();
    __syncthreads();
    if (warp == AT_MMA_WARP) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, kAtTmemCols);
    }
    if (threadIdx.x == 0 && s_fail) atomicOr(&g_tc_attn_fault, 1u);
}

}  // namespace

bool gqa_prefill_tc_fits(uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim) {
    const uint32_t group = kv_heads ? q_heads / kv_heads : 0;
    return head_dim == (uint32_t)AT_DIM && group && q_heads % kv_heads == 0 && AT_ROWS % group == 0;
}

int32_t gqa_prefill_tc(float *out, const float *q, const float *key_cache, const float *value_cache, uint64_t len,
                       const uint64_t *len_dev, uint64_t tokens, uint32_t q_heads, uint32_t kv_heads,
                       uint64_t cache_stride, uint32_t seqs, cudaStream_t stream) {
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(gqa_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kAtSmemBytes);
    });
    MF_CUDA_TRY(attr);
    const uint64_t tpc = AT_ROWS / (q_heads / kv_heads);
    const dim3 grid((unsigned)((tokens + tpc - 1) / tpc), kv_heads, seqs);
    return ::mf::launch(gqa_prefill_tc_kernel, grid, dim3(AT_THREADS), kAtSmemBytes, stream, "gqa_prefill_tc_kernel",
                        out, q, key_cache, value_cache, len, len_dev, tokens, q_heads, kv_heads, cache_stride);
}

int32_t attention_tc_faults(uint32_t *flags) {
    unsigned v = 0;
    MF_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_tc_attn_fault, sizeof(v)));
    const unsigned zero = 0;
    MF_CUDA_TRY(cudaMemcpyToSymbol(g_tc_attn_fault, &zero, sizeof(zero)));
    *flags = v;
    return MF_OK;
}

}  // namespace mf

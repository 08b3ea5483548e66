// Persistent single-token decode step, sm_100a: one launch per greedy token.
//
// The reference's one-token pass (crates/executor-core/src/lfm2/executor/
// execution.rs:35-627, then sample_epilogue :591-614) is a chain of ~70
// dependent matrix-vector products whose weights (487 MB for the 1.2B-shaped
// model) far exceed anything a chain of separate launches can stream: each
// launch drains, and the next one refills, the machine.  Here every SM runs
// one CTA for the whole token:
//
//  * a producer warp streams the CTA's share of every stage's weights (and,
//    for attention, of the cached K/V rows) into a ring of shared-memory slots
//    with bulk copies (cp.async.bulk into this CTA only), running ahead of the
//    compute by as many slots as fit: weights do not depend on activations,
//    so the HBM stream is limited by the ring, not by the chain;
//  * 16 consumer warps wait for the stage's input vector, compute the CTA's
//    rows from the ring and publish them.
//
// Stages exchange vectors through global memory as 64-bit words
// (value bits | tag << 32), the tag naming the token (a per-state epoch) and
// the stage: a reader spins on exactly the words it needs until their tags
// match, so waiting for the producers and loading their data is one round
// trip, and no grid-wide barrier exists.  A CTA can only be one stage ahead
// of another (every stage's input is written by all CTAs of the stage
// before), and every stage writes its own buffer, so no word is overwritten
// while a reader may still want its old value.
//
// Arithmetic per stage is that of the separate kernels: ternary and INT8
// rows on the integer tensor cores with the activation split exactly into
// four int8 limbs per 128-group (promoted per group with the row's scale),
// NF4 and dense F32 rows on FP32 FMAs, RMSNorm / SwiGLU / the gated short
// convolution / RoPE rounded as the reference rounds them.
//
// Every wait is bounded (2 s of globaltimer): a CTA whose wait expires sets
// the fault word, stops, lets its own bulk copies land and returns; CTAs
// waiting on it expire the same way, and later launches return at once
// until the host reads and clears the word (mf_device_faults).
#include <algorithm>
#include <vector>

#include "mf_common.cuh"
#include "packed_kernels.h"
#include "tc_sm100.cuh"

namespace mf {
namespace {

using sm100::globaltimer_ns;
using sm100::mbar_arrive;
using sm100::mbar_arrive_expect_tx;
using sm100::mbar_init;
using sm100::mbar_init_fence;
using sm100::mbar_try_wait;
using sm100::smem_u32;

constexpr int kCW = 8;                     // consumer warps (224 registers each)
constexpr int kCThreads = kCW * 32;
constexpr int kPThreads = kCThreads + 32;  // + the producer warp
constexpr uint32_t kSlotCode = 33792;      // code (or K/V) bytes per ring slot
constexpr uint32_t kSlotScale = 4096;      // scale bytes per ring slot
constexpr uint32_t kSlotBytes = kSlotCode + kSlotScale;
constexpr int kMaxRows = 64;               // physical rows per chunk (4 MMA tiles)
constexpr int kRedPerSlot = 256;           // partial sums per chunk: K parts x rows <= 256
constexpr int kTblReplicas = 8;            // NF4 byte table copies (lane % 8 picks one)
constexpr int kAttD = 64;                  // head dimension of the attention stage
constexpr int kKPitch = 68;                // staged key row pitch (floats)
constexpr int kKeysPerChunk = 64;
constexpr int kMaxGroup = 8;
constexpr int kMaxConvW = 4;
constexpr int kDenseFmt = 3;
constexpr uint32_t kStagesPerEpoch = 256;  // tag = epoch * 256 + stage
constexpr int kMaxSlots = 6;
constexpr int kMaxPerThread = 8;           // tagged input words one consumer thread polls at once
constexpr int kMaxCh = 32;                 // conv channels per CTA (hidden <= 4096 over >= 128 CTAs)
constexpr int kMaxAttChunks = 32;          // attention chunks per kv head (partials merged in one trip)
// Attention scratch in the xs region: q rows, normed q, new k, new v, raw k,
// scores, running max / sum / rescale; then the prefetched q/k norm weights
// and RoPE row (192 floats) and the merge's (m, l) pairs.
constexpr int kAttScratch = kMaxGroup * kAttD * 2 + 3 * kAttD + kMaxGroup * kKeysPerChunk + 3 * kMaxGroup;
constexpr int kAttFloats = kAttScratch + 192 + 2 * kMaxAttChunks * kMaxGroup;
constexpr uint32_t kDynSmemLimit = 227 * 1024 - 1024;   // 227 KB per CTA less the kernel's static arrays

enum PKind { PK_MIXCONV = 0, PK_QKV = 1, PK_PROJ = 2, PK_FFN = 3, PK_ATTN = 4, PK_HEAD = 5 };

// NF4 levels (crates/kernels-simd/src/lib.rs:113-130, bitsandbytes order).
__device__ __constant__ float kPNf4[16] = {
    -0x1.000000p+0f, -0x1.647362p-1f, -0x1.0cd660p-1f, -0x1.946540p-2f,
    -0x1.23449ap-2f, -0x1.7a6a7ep-3f, -0x1.74f0e2p-4f, 0.0f,
    0x1.45f5fep-4f,  0x1.4995c6p-3f,  0x1.f809bap-3f,  0x1.5a0674p-2f,
    0x1.c34970p-2f,  0x1.200f56p-1f,  0x1.722766p-1f,  0x1.000000p+0f,
};

__device__ unsigned int g_persist_fault = 0;

}  // namespace

// One matrix of a stage.
struct PMat {
    const uint8_t *codes;
    const float *scales;
    const float *dense;
    uint32_t rows;
    uint32_t pad;
};

// One stage of the step (host-built, one array per state).
struct PStage {
    int32_t kind, fmt, K, comps;
    uint32_t V;        // virtual rows (conv: channels; FFN: pair rows; attention: unused)
    uint32_t cv;       // virtual rows per ring chunk
    uint32_t pitch;    // shared-memory pitch of a staged code row
    uint32_t tiles;    // 16-row MMA tiles per full chunk
    PMat mat[3];       // QKV: q, k, v; FFN: w1, w3; conv / PROJ / HEAD: one
    uint32_t split0, split1;   // QKV: first k row, first v row; conv: hidden (row offset per comp)
    int32_t in_stage;  // stage whose output is this stage's input (-1: embedding row)
    uint32_t in_off;   // element offset into that output
    int32_t norm;      // residual update + RMSNorm prologue
    float eps;
    const float *norm_w;
    const unsigned long long *in;   // tagged input words (in_stage's output + in_off)
    unsigned long long *out;   // tagged output words
    const float *conv_k;
    float *conv_hist;
    int32_t conv_w;
    int32_t att_index;
    const float *q_norm, *k_norm;
    float *kcache, *vcache;
    uint64_t pad_;
};
static_assert(sizeof(PStage) % 16 == 0, "stage descriptors are copied in 16-byte pieces");

struct PParams {
    const PStage *stages;
    int n_stages;
    int hidden, q_heads, kv_heads, group, vocab;
    int att_chunks;            // CTAs per kv head in an attention stage
    uint64_t capacity;
    const float2 *rope;        // [capacity][kAttD / 2] (sin, cos)
    float att_eps;
    // embedding (layer-0 input)
    const uint8_t *ecodes;
    const float *escales, *edense;
    int efmt;
    uint32_t erows;
    // state
    uint64_t *pos;
    float *sampled, *logits;
    uint32_t *epoch;
    float *att_part;           // [n_att][kv_heads][att_chunks][group][kAttD + 2]
    unsigned *att_count;       // [n_att][kv_heads]
    float *arg_part;           // [grid][3]
    unsigned *arg_count;
    int nslots;
    uint32_t off_bar, off_res, off_xs, off_limb, off_efac, off_red, off_conv, off_desc, off_ring;
    uint64_t timeout_ns;
};

namespace {

__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_tagged(unsigned long long *p, float v, uint32_t tag) {
    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint32_t stage_tag(uint32_t epoch, int s) { return epoch * kStagesPerEpoch + (uint32_t)s; }

// Shared control: the CTA-wide abort flag and the norm partial sums.
struct Ctl {
    volatile int *abort_flag;
    uint64_t timeout;
    __device__ bool aborted() const { return *abort_flag != 0; }
    __device__ void abort() const {
        *abort_flag = 1;
        atomicOr(&g_persist_fault, 1u);
    }
};

// Spins until the word's tag matches; NaN after the time limit or an abort.
__device__ float wait_tagged(const unsigned long long *p, uint32_t tag, const Ctl &c) {
    unsigned long long v = ld_tagged(p);
    if ((uint32_t)(v >> 32) == tag) return __uint_as_float((uint32_t)v);
    const uint64_t t0 = globaltimer_ns();
    for (int i = 0;; ++i) {
        v = ld_tagged(p);
        if ((uint32_t)(v >> 32) == tag) return __uint_as_float((uint32_t)v);
        if ((i & 15) == 15) {
            if (c.aborted()) break;
            if (globaltimer_ns() - t0 > c.timeout) {
                c.abort();
                break;
            }
        }
    }
    return __int_as_float(0x7fc00000);
}

// Up to N tagged words at base[i * stride] (i < count), all loads in flight
// at once; only the words whose tag does not match yet are loaded again, all
// of them together each round.  Values land in out[i]; NaN for any word
// still missing at the time limit.  Not inlined: it runs in stage prologues
// only, and inlined it pushes the kernel past its register budget.
template <int N>
__device__ __noinline__ void wait_tagged_n(const unsigned long long *base, int stride, int count, uint32_t tag, float (&out)[N],
                                           const Ctl &c) {
    unsigned long long v[N];
#pragma unroll
    for (int i = 0; i < N; ++i)
        if (i < count) v[i] = ld_tagged(base + (size_t)i * stride);
    bool all = true;
#pragma unroll
    for (int i = 0; i < N; ++i) all &= i >= count || (uint32_t)(v[i] >> 32) == tag;
    if (!all) {
        const uint64_t t0 = globaltimer_ns();
        for (int it = 0;; ++it) {
            all = true;
#pragma unroll
            for (int i = 0; i < N; ++i) {
                if (i < count && (uint32_t)(v[i] >> 32) != tag) {
                    v[i] = ld_tagged(base + (size_t)i * stride);
                    all &= (uint32_t)(v[i] >> 32) == tag;
                }
            }
            if (all) break;
            if ((it & 15) == 15 && (c.aborted() || globaltimer_ns() - t0 > c.timeout)) {
                if (!c.aborted()) c.abort();
#pragma unroll
                for (int i = 0; i < N; ++i) v[i] = 0x7fc00000ull;   // NaN values, tags ignored below
                break;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = i < count ? __uint_as_float((uint32_t)v[i]) : 0.0f;
}

// NO x NI tagged words at base[o * so + i * si] (o < count_o, i < NI), all in
// flight at once; out[o * NI + i].  As wait_tagged_n otherwise.
template <int NO, int NI>
__device__ __noinline__ void wait_tagged_2d(const unsigned long long *base, int so, int si, int count_o, uint32_t tag,
                                            float (&out)[NO * NI], const Ctl &c) {
    constexpr int N = NO * NI;
    unsigned long long v[N];
#pragma unroll
    for (int k = 0; k < N; ++k)
        if (k / NI < count_o) v[k] = ld_tagged(base + (size_t)(k / NI) * so + (size_t)(k % NI) * si);
    bool all = true;
#pragma unroll
    for (int k = 0; k < N; ++k) all &= k / NI >= count_o || (uint32_t)(v[k] >> 32) == tag;
    if (!all) {
        const uint64_t t0 = globaltimer_ns();
        for (int it = 0;; ++it) {
            all = true;
#pragma unroll
            for (int k = 0; k < N; ++k) {
                if (k / NI < count_o && (uint32_t)(v[k] >> 32) != tag) {
                    v[k] = ld_tagged(base + (size_t)(k / NI) * so + (size_t)(k % NI) * si);
                    all &= (uint32_t)(v[k] >> 32) == tag;
                }
            }
            if (all) break;
            if ((it & 15) == 15 && (c.aborted() || globaltimer_ns() - t0 > c.timeout)) {
                if (!c.aborted()) c.abort();
#pragma unroll
                for (int k = 0; k < N; ++k) v[k] = 0x7fc00000ull;
                break;
            }
        }
    }
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = k / NI < count_o ? __uint_as_float((uint32_t)v[k]) : 0.0f;
}

__device__ bool wait_full(uint32_t bar, uint32_t parity, const Ctl &c) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 16; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (c.aborted()) return false;
        if (globaltimer_ns() - t0 > c.timeout) {
            c.abort();
            return false;
        }
    }
}

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory"); }

// Consumer barrier that also agrees on the abort flag: every consumer
// thread gets the OR of what each saw when it arrived, so all of them leave
// at the same barrier (a flag set after some thread looked cannot split
// them between leaving and waiting at the next barrier).
__device__ __forceinline__ bool cbar_aborted(const Ctl &c) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.or.pred po, 1, %2, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)c.aborted()), "n"(kCThreads)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(pol)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t pol;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t pol;
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void imma16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Four ternary codes (nibbles of `sel`, each 0..3) -> int8 {-1, 0, +1, +2}
// (code 3 decodes to +2, crates/kernels-simd/src/lib.rs:22).
__device__ __forceinline__ uint32_t ternary4(uint32_t sel) { return __byte_perm(0x020100FFu, 0u, sel); }

__host__ __device__ __forceinline__ int pad32(int k) { return k + 4 * (k >> 5); }

// Work split helpers (identical on the producer and the consumers).
__device__ __forceinline__ void cta_rows(uint32_t V, uint32_t &v0, uint32_t &v1) {
    v0 = (uint32_t)((uint64_t)V * blockIdx.x / gridDim.x);
    v1 = (uint32_t)((uint64_t)V * (blockIdx.x + 1) / gridDim.x);
}

// Attention unit of this CTA: kv head, chunk index, and the cached keys
// [k0, k1) it reads (the new key, index pos, is the last chunk's).
__device__ __forceinline__ bool att_unit(const PParams &p, uint64_t pos, int &h, int &ci, uint64_t &k0, uint64_t &k1,
                                         uint64_t &kend) {
    const int C = p.att_chunks;
    if ((int)blockIdx.x >= p.kv_heads * C) return false;
    h = blockIdx.x / C;
    ci = blockIdx.x % C;
    const uint64_t ctx = pos + 1;
    k0 = ctx * (uint64_t)ci / (uint64_t)C;
    kend = ctx * (uint64_t)(ci + 1) / (uint64_t)C;
    k1 = min(kend, pos);
    if (k1 < k0) k1 = k0;
    return true;
}

// Physical code row `pr` (comp-major within a chunk of nv virtual rows
// starting at va) -> matrix and row.
__device__ __forceinline__ void phys_row(const PStage &S, uint32_t va, uint32_t nv, uint32_t pr, int &m, uint32_t &row) {
    const uint32_t comp = pr / nv, v = va + (pr - comp * nv);
    if (S.kind == PK_QKV) {
        if (v < S.split0) { m = 0; row = v; }
        else if (v < S.split1) { m = 1; row = v - S.split0; }
        else { m = 2; row = v - S.split1; }
    } else if (S.kind == PK_MIXCONV) {
        m = 0;
        row = comp * S.split0 + v;
    } else {
        m = S.kind == PK_FFN ? (int)comp : 0;
        row = v;
    }
}

// Number of physical rows from `pr` on (within its component) whose matrix
// rows are consecutive in one matrix.
__device__ __forceinline__ uint32_t phys_run(const PStage &S, uint32_t va, uint32_t nv, uint32_t pr) {
    const uint32_t comp = pr / nv, v = va + (pr - comp * nv);
    uint32_t end = va + nv;   // end of this component's virtual rows
    if (S.kind == PK_QKV) {
        if (v < S.split0) end = min(end, S.split0);
        else if (v < S.split1) end = min(end, S.split1);
    }
    return end - v;
}

__device__ __forceinline__ uint32_t row_bytes_of(int fmt, int K) {
    return fmt == MF_TERNARY ? K / 4 : fmt == MF_NF4 ? K / 2 : fmt == MF_INT8 ? K : K * 4;
}

// ---------------------------------------------------------------------
// Producer warp: the CTA's chunks of every stage, in the consumers' order.
// ---------------------------------------------------------------------
__device__ __forceinline__ void producer(const PParams &p, unsigned char *sm, uint64_t pos, const Ctl &c) {
    const int lane = threadIdx.x & 31;
    const uint32_t bar0 = smem_u32(sm + p.off_bar);
    const uint32_t ring = smem_u32(sm + p.off_ring);
    const int NS = p.nslots;
    const uint64_t pol_w = policy_evict_first(), pol_kv = policy_evict_last();
    uint32_t n = 0;   // chunks issued
    bool ok = true;
    for (int s = 0; s < p.n_stages && ok; ++s) {
        const PStage &S = p.stages[s];
        uint32_t nchunks = 0, per = 0;
        uint64_t base = 0, count = 0;
        int h = 0, ci = 0;
        if (S.kind == PK_ATTN) {
            uint64_t k0, k1, kend;
            if (att_unit(p, pos, h, ci, k0, k1, kend)) {
                base = k0;
                count = k1 - k0;
            }
            per = kKeysPerChunk;
        } else {
            uint32_t v0, v1;
            cta_rows(S.V, v0, v1);
            base = v0;
            count = v1 - v0;
            per = S.cv;
        }
        nchunks = (uint32_t)((count + per - 1) / per);
        for (uint32_t ch = 0; ch < nchunks; ++ch, ++n) {
            const uint32_t slot = n % NS, round = n / NS;
            const uint32_t full = bar0 + 8 * slot, empty = bar0 + 8 * (NS + slot);
            if (round > 0 && !wait_full(empty, (round - 1) & 1, c)) {
                ok = false;
                break;
            }
            const uint32_t dst = ring + slot * kSlotBytes;
            uint32_t bytes = 0;
            if (S.kind == PK_ATTN) {
                const uint64_t key0 = base + (uint64_t)ch * per;
                const uint32_t nk = (uint32_t)min((uint64_t)per, base + count - key0);
                const uint64_t kvw = (uint64_t)p.kv_heads * kAttD;
                for (uint32_t j = lane; j < nk; j += 32) {
                    const uint64_t off = (key0 + j) * kvw + (uint64_t)h * kAttD;
                    bulk_g2s(dst + j * kKPitch * 4, S.kcache + off, kAttD * 4, full, pol_kv);
                    bulk_g2s(dst + kKeysPerChunk * kKPitch * 4 + j * kAttD * 4, S.vcache + off, kAttD * 4, full, pol_kv);
                }
                bytes = nk * 2 * kAttD * 4;
            } else {
                const uint32_t va = (uint32_t)(base + (uint64_t)ch * per);
                const uint32_t nv = (uint32_t)min((uint64_t)per, base + count - va);
                const uint32_t P = nv * (uint32_t)S.comps;
                const uint32_t rb = row_bytes_of(S.fmt, S.K);
                for (uint32_t pr = lane; pr < P; pr += 32) {
                    int m;
                    uint32_t row;
                    phys_row(S, va, nv, pr, m, row);
                    const void *src = S.fmt == kDenseFmt ? (const void *)(S.mat[m].dense + (size_t)row * S.K)
                                                         : (const void *)(S.mat[m].codes + (size_t)row * rb);
                    bulk_g2s(dst + pr * S.pitch, src, rb, full, pol_w);
                }
                bytes = P * rb;
                if (S.fmt != kDenseFmt) {
                    // Group scales [P][K / 128]: one bulk copy per run of rows
                    // contiguous in one matrix (16-byte rows), else through
                    // registers (narrow rows of small models only).
                    const uint32_t G = (uint32_t)S.K / 128;
                    const uint32_t sdst = dst + kSlotCode;
                    if ((G * 4) % 16 == 0) {
                        if (lane == 0) {
                            for (uint32_t pr = 0; pr < P;) {
                                int m;
                                uint32_t row;
                                phys_row(S, va, nv, pr, m, row);
                                const uint32_t run = phys_run(S, va, nv, pr);
                                bulk_g2s(sdst + pr * G * 4, S.mat[m].scales + (size_t)row * G, run * G * 4, full, pol_w);
                                pr += run;
                            }
                        }
                        bytes += P * G * 4;
                    } else {
                        float *sp = reinterpret_cast<float *>(sm + p.off_ring + slot * kSlotBytes + kSlotCode);
                        for (uint32_t e = lane; e < P * G; e += 32) {
                            const uint32_t pr = e / G, g = e - pr * G;
                            int m;
                            uint32_t row;
                            phys_row(S, va, nv, pr, m, row);
                            sp[e] = ld_stream_f32(S.mat[m].scales + (size_t)row * G + g);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_expect_tx(full, bytes);
        }
    }
    if (!ok) {
        // Let the copies already issued land before the CTA can exit.
        const uint32_t first = n > (uint32_t)NS ? n - NS : 0;
        for (uint32_t k = first; k < n; ++k) {
            const uint32_t slot = k % NS, round = k / NS;
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(bar0 + 8 * slot, round & 1))
                if (globaltimer_ns() - t0 > c.timeout) break;
        }
    }
}

// ---------------------------------------------------------------------
// Consumer side.
// ---------------------------------------------------------------------
struct Smem {
    float2 *tbl;       // NF4 byte -> (level of low nibble, level of high nibble)
    float *res;        // residual stream [hidden]
    float *xs;         // staged input row, pad32 layout (attention: its scratch)
    uint2 *limbs;      // B fragments: [groups][4 k-steps][16 lanes]
    float *nws;        // norm weight [hidden] (aliases limbs: dead once xs is formed)
    float *efac;       // [groups] 2^(e-7) (NaN: poisoned group)
    float *red;        // [kMaxSlots][kRedPerSlot] cross-warp partial sums per ring slot
    float *red_ss;     // [32]
    float *cvk, *cvh;  // conv taps [kMaxCh][kMaxConvW], history [kMaxConvW - 1][kMaxCh]
    PStage *desc;      // [3] stage descriptors
    unsigned *cnt;     // [kMaxSlots] warps done with each slot's chunk
    unsigned char *ring;
    uint32_t bar0;
};

// Shared-memory regions of the kernel, derived from the dynamic shared array
// in the calling function so that every pointer is known to be shared.
__device__ __forceinline__ Smem make_smem(const PParams &p, float *red_ss) {
    extern __shared__ __align__(1024) unsigned char sm[];
    Smem S;
    S.tbl = reinterpret_cast<float2 *>(sm);
    S.bar0 = smem_u32(sm + p.off_bar);
    S.res = reinterpret_cast<float *>(sm + p.off_res);
    S.xs = reinterpret_cast<float *>(sm + p.off_xs);
    S.limbs = reinterpret_cast<uint2 *>(sm + p.off_limb);
    S.efac = reinterpret_cast<float *>(sm + p.off_efac);
    S.red = reinterpret_cast<float *>(sm + p.off_red);
    S.red_ss = red_ss;
    S.nws = reinterpret_cast<float *>(sm + p.off_limb);
    S.cvk = reinterpret_cast<float *>(sm + p.off_conv);
    S.cvh = S.cvk + kMaxCh * kMaxConvW;
    S.desc = reinterpret_cast<PStage *>(sm + p.off_desc);
    S.cnt = reinterpret_cast<unsigned *>(sm + p.off_bar + 8 * 2 * kMaxSlots);
    S.ring = sm + p.off_ring;
    return S;
}

// Splits the 128 values v (this lane's four) of group G into four int8
// limbs and stores the token-0 B-fragment words (see limb layout below).
// Lane (s = lane / 8, q = (lane / 2) % 4, h = lane % 2) holds the elements
// at group offsets j(i) = 32q + 8s + 2i + h (ternary) or 32q + 8s + 4h + i
// (INT8), i = 0..3: the order in which a lane's A fragment holds its
// weights.  Exact: x = 2^(e-7) (l0 + l1 2^-7 + l2 2^-14 + l3 2^-21) + r with
// |l| <= 64 and |r| < 2^-27 max|x|.
__device__ __forceinline__ void store_limbs(const Smem &S, int G, const float (&v)[4]) {
    const int lane = threadIdx.x & 31;
    const int s = lane >> 3, q = (lane >> 1) & 3, h = lane & 1;
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
    // B fragment of m16n8k32 for lane L = 4n + q (n = MMA column = limb):
    // words k = 4q..4q+3 (.x) and 16+4q..16+4q+3 (.y) of k-step s.
    uint32_t *dst = reinterpret_cast<uint32_t *>(S.limbs + (size_t)G * 64);
#pragma unroll
    for (int l = 0; l < 4; ++l) dst[(s * 16 + l * 4 + q) * 2 + h] = w[l];
    if (lane == 0) S.efac[G] = bad ? __int_as_float(0x7fc00000) : __int_as_float((127 + e - 7) << 23);
}

__device__ __forceinline__ int limb_j(int fmt, int lane, int i) {
    const int s = lane >> 3, q = (lane >> 1) & 3, h = lane & 1;
    return fmt == MF_INT8 ? 32 * q + 8 * s + 4 * h + i : 32 * q + 8 * s + 2 * i + h;
}

// Embedding row value e of the token in p.sampled (packed_gather_rows
// semantics: level * scale, one rounding; an invalid id gives NaN).
__device__ __forceinline__ float embed_value(const PParams &p, long long id, int e, int K) {
    if (id < 0) return __int_as_float(0x7fc00000);
    if (p.edense) return p.edense[(size_t)id * K + e];
    const int gw = e / 128, w = e % 128;
    float level;
    if (p.efmt == MF_TERNARY) {
        const uint8_t *c = p.ecodes + (size_t)id * (K / 4);
        level = (float)((c[gw * 32 + w / 4] >> (2 * (w % 4))) & 3u) - 1.0f;
    } else if (p.efmt == MF_INT8) {
        level = (float)(int8_t)p.ecodes[(size_t)id * K + e];
    } else {
        const uint8_t b = p.ecodes[(size_t)id * (K / 2) + gw * 64 + w / 2];
        level = kPNf4[(w & 1) ? (b >> 4) : (b & 15)];
    }
    return __fmul_rn(level, p.escales[(size_t)id * (K / 128) + gw]);
}

__device__ __forceinline__ long long sampled_id(const PParams &p) {
    const float idv = *p.sampled;
    return (isfinite(idv) && idv >= 0.0f && floorf(idv) == idv && idv < 16777216.0f && (long long)idv < (long long)p.erows)
               ? (long long)idv : -1;
}

// Argmax candidate merge: first strict maximum (ties to the lower row),
// poison flag sticky (crates/backend-cpu/src/dense.rs:369-411).
__device__ __forceinline__ void am_merge(float &bv, int &bi, int &bp, float ov, int oi, int op) {
    bp |= op;
    if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
        bv = ov;
        bi = oi;
    }
}

// Attention: warp-cooperative head RMSNorm + split-half RoPE of one head row
// (crates/backend-cpu/src/normalization_rotary.rs:246-369 rounding).
__device__ void norm_rope64(const float *x, const float *w, float eps, const float2 *rot, float *dst, int lane) {
    float v0 = x[lane], v1 = x[lane + 32];
    float ss = fmaf(v1, v1, v0 * v0);
    ss = warp_sum(ss);
    const float rec = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 64.0f), eps)));
    v0 = __fmul_rn(__fmul_rn(v0, rec), w[lane]);
    v1 = __fmul_rn(__fmul_rn(v1, rec), w[lane + 32]);
    const float2 r = rot[lane];   // pair c = lane: elements lane and lane + 32
    dst[lane] = __fsub_rn(__fmul_rn(v0, r.y), __fmul_rn(v1, r.x));
    dst[lane + 32] = __fadd_rn(__fmul_rn(v1, r.y), __fmul_rn(v0, r.x));
}

// One chunk of keys for the attention stage: scores, online softmax, PV.
// K rows at kr (pitch kp floats), V rows at vr (pitch 64); nk keys.
__device__ void att_chunk(const float *kr, int kp, const float *vr, int nk, const float *qs, float *sp, float *mrun,
                          float *lrun, float *crr, int group, float scale, float &o_run, int tid) {
    const int lane = tid & 31, warp = tid >> 5;
    for (int idx = tid; idx < group * kKeysPerChunk; idx += kCThreads) {
        const int gh = idx / kKeysPerChunk, j = idx % kKeysPerChunk;
        float sc = -INFINITY;
        if (j < nk) {
            const float4 *q4 = reinterpret_cast<const float4 *>(qs + gh * kAttD);
            const float4 *k4 = reinterpret_cast<const float4 *>(kr + j * kp);
            float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
            for (int d4 = 0; d4 < kAttD / 4; ++d4) {
                const float4 a = q4[d4], b = k4[d4];
                d0 = fmaf(a.x, b.x, d0);
                d1 = fmaf(a.y, b.y, d1);
                d2 = fmaf(a.z, b.z, d2);
                d3 = fmaf(a.w, b.w, d3);
            }
            sc = __fmul_rn((d0 + d1) + (d2 + d3), scale);
        }
        sp[gh * kKeysPerChunk + j] = sc;
    }
    cbar();
    if (warp < group) {
        const int gh = warp;
        const float s0 = sp[gh * kKeysPerChunk + lane], s1 = sp[gh * kKeysPerChunk + 32 + lane];
        const float m_old = mrun[gh];
        const float m_new = fmaxf(m_old, warp_max(fmaxf(s0, s1)));
        const float p0 = s0 == -INFINITY ? 0.0f : expf(s0 - m_new);
        const float p1 = s1 == -INFINITY ? 0.0f : expf(s1 - m_new);
        const float corr = m_old == -INFINITY ? 0.0f : expf(m_old - m_new);
        const float psum = warp_sum(p0 + p1);
        sp[gh * kKeysPerChunk + lane] = p0;
        sp[gh * kKeysPerChunk + 32 + lane] = p1;
        if (lane == 0) {
            lrun[gh] = lrun[gh] * corr + psum;
            mrun[gh] = m_new;
            crr[gh] = corr;
        }
    }
    cbar();
    if (tid < group * kAttD) {
        const int gh = tid / kAttD, d = tid % kAttD;
        const float *pr = sp + gh * kKeysPerChunk;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        for (int j = 0; j < nk; j += 4) {
            a0 = fmaf(pr[j], vr[j * kAttD + d], a0);
            if (j + 1 < nk) a1 = fmaf(pr[j + 1], vr[(j + 1) * kAttD + d], a1);
            if (j + 2 < nk) a2 = fmaf(pr[j + 2], vr[(j + 2) * kAttD + d], a2);
            if (j + 3 < nk) a3 = fmaf(pr[j + 3], vr[(j + 3) * kAttD + d], a3);
        }
        o_run = fmaf(o_run, crr[gh], (a0 + a1) + (a2 + a3));
    }
}

// cp.async of 16 / 4 bytes into shared memory (completed by cp_wait_all).
__device__ __forceinline__ void cp16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Stage constants copied into shared memory at the start of a stage, before
// its input is waited for, so that nothing after the wait goes to global
// memory but the input itself: the next stage's descriptor (triple-buffered:
// every stage passes at least one consumer barrier, so the buffer being
// overwritten was last read two stages ago), the norm weight, the conv taps
// and histories of this CTA's channels, and the attention's q/k norm
// weights and RoPE row.
__device__ __forceinline__ void stage_prefetch(const PParams &p, const Smem &S, int s, const PStage &St, uint64_t pos, int tid) {
    constexpr int kDescChunks = (int)(sizeof(PStage) / 16);
    if (s + 1 < p.n_stages && tid < kDescChunks)
        cp16(reinterpret_cast<unsigned char *>(S.desc + (s + 1) % 3) + 16 * tid,
             reinterpret_cast<const unsigned char *>(p.stages + s + 1) + 16 * tid);
    if (St.norm)
        for (int e = tid; e < p.hidden / 4; e += kCThreads) cp16(S.nws + 4 * e, St.norm_w + 4 * e);
    if (St.kind == PK_MIXCONV) {
        uint32_t v0, v1;
        cta_rows(St.V, v0, v1);
        const int nch = (int)(v1 - v0), W = St.conv_w;
        for (int e = tid; e < nch * (2 * W - 1); e += kCThreads) {
            if (e < nch * W) {
                const int ch = e / W, tap = e % W;
                cp4(S.cvk + ch * kMaxConvW + tap, St.conv_k + (size_t)(v0 + ch) * W + tap);
            } else {
                const int f = e - nch * W, i = f / nch, ch = f % nch;
                cp4(S.cvh + i * kMaxCh + ch, St.conv_hist + (size_t)i * p.hidden + v0 + ch);
            }
        }
    }
    if (St.kind == PK_ATTN) {
        float *aw = S.xs + kAttScratch;   // q_norm [64], k_norm [64], rot [32] (sin, cos)
        if (tid < 16) cp16(aw + 4 * tid, St.q_norm + 4 * tid);
        else if (tid < 32) cp16(aw + 64 + 4 * (tid - 16), St.k_norm + 4 * (tid - 16));
        else if (tid < 48) cp16(aw + 128 + 4 * (tid - 32), reinterpret_cast<const float *>(p.rope + pos * (kAttD / 2)) + 4 * (tid - 32));
    }
    cp_commit();
}

// Kernel parameters, copied into shared memory once per launch so that the
// stage functions below (not inlined: each gets its own register budget)
// read them without a global or local-memory trip.
__shared__ PParams sP;
__shared__ float sRedSS[32];
__shared__ unsigned sLast;
__shared__ float sAmV[kCW];
__shared__ int sAmI[kCW], sAmP[kCW];

__device__ __forceinline__ Smem smem() { return make_smem(sP, sRedSS); }

// Residual update + RMSNorm prologue of stage s (in the stage's shared
// descriptor St): the embedding row of the sampled id for layer 0, else the
// previous stage's tagged output added to the residual; then the normalized
// row split into limbs (integer formats, each warp its own groups) or staged
// in xs (NF4, dense).  Returns true when the CTA is aborting.
__device__ __noinline__ bool prologue_norm(const PStage &St, uint32_t epoch, Ctl c) {
    const Smem S = smem();
    const PParams &p = sP;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hidden = p.hidden;
    const unsigned long long *in = St.in;
    const uint32_t tin = St.in_stage >= 0 ? stage_tag(epoch, St.in_stage) : 0u;
    float ss = 0.0f;
    const long long id = St.in_stage < 0 ? sampled_id(p) : -1;
    for (int e0 = tid; e0 < hidden; e0 += kCThreads * kMaxPerThread) {
        const int per = min(kMaxPerThread, (hidden - e0 + kCThreads - 1) / kCThreads);
        float dv[kMaxPerThread];
        if (St.in_stage < 0) {
#pragma unroll
            for (int i = 0; i < kMaxPerThread; ++i)
                if (i < per) dv[i] = embed_value(p, id, e0 + i * kCThreads, hidden);
        } else {
            wait_tagged_n<kMaxPerThread>(in + e0, kCThreads, per, tin, dv, c);
        }
#pragma unroll
        for (int i = 0; i < kMaxPerThread; ++i) {
            if (i >= per) break;
            const int e = e0 + i * kCThreads;
            const float v = St.in_stage < 0 ? dv[i] : __fadd_rn(S.res[e], dv[i]);
            S.res[e] = v;
            ss = fmaf(v, v, ss);
        }
    }
    ss = warp_sum(ss);
    if (lane == 0) S.red_ss[warp] = ss;
    cp_wait_all();
    if (cbar_aborted(c)) return true;
    float t = lane < kCW ? S.red_ss[lane] : 0.0f;
    t = warp_sum(t);
    const float rec = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)hidden), St.eps)));
    const int fmt = St.fmt;
    if (fmt == MF_TERNARY || fmt == MF_INT8) {
        const int step = fmt == MF_INT8 ? 1 : 2, j0 = limb_j(fmt, lane, 0);
        for (int Gi = warp; Gi < St.K / 128; Gi += kCW) {
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int k = Gi * 128 + j0 + i * step;
                v[i] = __fmul_rn(__fmul_rn(S.res[k], rec), S.nws[k]);
            }
            store_limbs(S, Gi, v);
        }
    } else {
        for (int e = tid; e < hidden; e += kCThreads) S.xs[pad32(e)] = __fmul_rn(__fmul_rn(S.res[e], rec), S.nws[e]);
    }
    cbar();
    return false;
}

// Prologue of a stage whose input is a previous stage's tagged output used as
// is: limbs for the integer formats (each warp gathers its groups, up to
// eight per round trip), the staged row for NF4 and dense.
__device__ __noinline__ bool prologue_plain(const PStage &St, uint32_t epoch, Ctl c) {
    const Smem S = smem();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned long long *in = St.in;
    const uint32_t tin = stage_tag(epoch, St.in_stage);
    const int fmt = St.fmt, K = St.K, G = K / 128;
    if (fmt == MF_TERNARY || fmt == MF_INT8) {
        const int step = fmt == MF_INT8 ? 1 : 2, j0 = limb_j(fmt, lane, 0);
        for (int gb = warp; gb < G; gb += 8 * kCW) {
            const int ng = min(8, (G - gb + kCW - 1) / kCW);
            float v[32];
            wait_tagged_2d<8, 4>(in + gb * 128 + j0, kCW * 128, step, ng, tin, v, c);
            for (int gg = 0; gg < ng; ++gg) {
                float w4[4] = {v[4 * gg], v[4 * gg + 1], v[4 * gg + 2], v[4 * gg + 3]};
                store_limbs(S, gb + gg * kCW, w4);
            }
        }
    } else {
        for (int e0 = tid; e0 < K; e0 += kCThreads * 16) {
            const int per = min(16, (K - e0 + kCThreads - 1) / kCThreads);
            float xv[16];
            wait_tagged_n<16>(in + e0, kCThreads, per, tin, xv, c);
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (i < per) S.xs[pad32(e0 + i * kCThreads)] = xv[i];
        }
    }
    cp_wait_all();
    return cbar_aborted(c);
}

// One warp's share of an integer-format chunk: 16-row tile `tile`, groups
// [gb, ge) of K, every row's partial sum into red[kp * P + row].
__device__ __noinline__ void chunk_imma(const PStage &St, int slot, int P, int tile, int kp, int gb, int ge) {
    const Smem S = smem();
    const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
    const int fmt = St.fmt, G = St.K / 128;
    const unsigned char *codes = S.ring + slot * kSlotBytes;
    const float *scl = reinterpret_cast<const float *>(codes + kSlotCode);
    float *red = S.red + slot * kRedPerSlot;
    const int p0 = tile * 16 + g, p1 = p0 + 8;
    const bool ok0 = p0 < P, ok1 = p1 < P;
    const float lw0 = (q & 1) ? 0x1p-14f : 1.0f, lw1 = lw0 * 0x1p-7f;
    float acc0 = 0.0f, acc1 = 0.0f;
    const unsigned char *r0 = codes + (size_t)(ok0 ? p0 : 0) * St.pitch;
    const unsigned char *r1 = codes + (size_t)(ok1 ? p1 : 0) * St.pitch;
#pragma unroll 2
    for (int Gi = gb; Gi < ge; ++Gi) {
        uint32_t wa[8], wb[8];
        if (fmt == MF_INT8) {
            const uint4 a0 = *reinterpret_cast<const uint4 *>(r0 + Gi * 128 + 32 * q);
            const uint4 a1 = *reinterpret_cast<const uint4 *>(r0 + Gi * 128 + 32 * q + 16);
            const uint4 b0 = *reinterpret_cast<const uint4 *>(r1 + Gi * 128 + 32 * q);
            const uint4 b1 = *reinterpret_cast<const uint4 *>(r1 + Gi * 128 + 32 * q + 16);
            wa[0] = a0.x; wa[1] = a0.y; wa[2] = a0.z; wa[3] = a0.w;
            wa[4] = a1.x; wa[5] = a1.y; wa[6] = a1.z; wa[7] = a1.w;
            wb[0] = b0.x; wb[1] = b0.y; wb[2] = b0.z; wb[3] = b0.w;
            wb[4] = b1.x; wb[5] = b1.y; wb[6] = b1.z; wb[7] = b1.w;
        } else {
            const uint2 ca = *reinterpret_cast<const uint2 *>(r0 + Gi * 32 + 8 * q);
            const uint2 cb = *reinterpret_cast<const uint2 *>(r1 + Gi * 32 + 8 * q);
            const uint32_t cwa[2] = {ca.x, ca.y}, cwb[2] = {cb.x, cb.y};
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                wa[4 * hh + 0] = ternary4(cwa[hh] & 0x3333u);
                wa[4 * hh + 1] = ternary4((cwa[hh] >> 2) & 0x3333u);
                wa[4 * hh + 2] = ternary4((cwa[hh] >> 16) & 0x3333u);
                wa[4 * hh + 3] = ternary4((cwa[hh] >> 18) & 0x3333u);
                wb[4 * hh + 0] = ternary4(cwb[hh] & 0x3333u);
                wb[4 * hh + 1] = ternary4((cwb[hh] >> 2) & 0x3333u);
                wb[4 * hh + 2] = ternary4((cwb[hh] >> 16) & 0x3333u);
                wb[4 * hh + 3] = ternary4((cwb[hh] >> 18) & 0x3333u);
            }
        }
        // The four k-steps into separate accumulators (independent MMAs),
        // then exact int32 sums.
        int d[4][4];
        const uint2 *lb = S.limbs + (size_t)Gi * 64;
#pragma unroll
        for (int st = 0; st < 4; ++st) {
            d[st][0] = d[st][1] = d[st][2] = d[st][3] = 0;
            const uint2 b = lane < 16 ? lb[st * 16 + lane] : make_uint2(0u, 0u);
            const uint32_t a[4] = {wa[2 * st], wb[2 * st], wa[2 * st + 1], wb[2 * st + 1]};
            imma16832(d[st], a, b.x, b.y);
        }
        const int s0 = (d[0][0] + d[1][0]) + (d[2][0] + d[3][0]);
        const int s1 = (d[0][1] + d[1][1]) + (d[2][1] + d[3][1]);
        const int s2 = (d[0][2] + d[1][2]) + (d[2][2] + d[3][2]);
        const int s3 = (d[0][3] + d[1][3]) + (d[2][3] + d[3][3]);
        const float ef = S.efac[Gi];
        const float vg = fmaf(__int2float_rn(s1), lw1, __int2float_rn(s0) * lw0) * ef;
        const float vg8 = fmaf(__int2float_rn(s3), lw1, __int2float_rn(s2) * lw0) * ef;
        acc0 = fmaf(vg, ok0 ? scl[p0 * G + Gi] : 0.0f, acc0);
        acc1 = fmaf(vg8, ok1 ? scl[p1 * G + Gi] : 0.0f, acc1);
    }
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    if (q == 0) {
        if (ok0) red[kp * P + p0] = acc0;
        if (ok1) red[kp * P + p1] = acc1;
    }
}

// One warp's share of an NF4 or dense chunk: rows rg, rg + wpk, ... of the
// chunk over K part kp (1024 weights: lane = 32-weight unit u, its 32
// activations loaded from xs once per chunk); partial sums into red.
__device__ __noinline__ void chunk_fp32(const PStage &St, int slot, int P, int kp, int rg, int wpk) {
    const Smem S = smem();
    const int lane = threadIdx.x & 31;
    const int fmt = St.fmt, K = St.K, G = K / 128, U = K / 32;
    const unsigned char *codes = S.ring + slot * kSlotBytes;
    const float *scl = reinterpret_cast<const float *>(codes + kSlotCode);
    float *red = S.red + slot * kRedPerSlot;
    const int u = kp * 32 + lane;
    float xr[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v4 = u < U ? *reinterpret_cast<const float4 *>(S.xs + pad32(32 * u) + 4 * i)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        xr[4 * i] = v4.x;
        xr[4 * i + 1] = v4.y;
        xr[4 * i + 2] = v4.z;
        xr[4 * i + 3] = v4.w;
    }
    const float2 *tbl = S.tbl + (lane & (kTblReplicas - 1));   // this lane's copy of the table
    for (int pr = rg; pr < P; pr += wpk) {
        const unsigned char *row = codes + (size_t)pr * St.pitch;
        float acc = 0.0f;
        if (u < U) {
            if (fmt == MF_NF4) {
                const uint4 cw4 = *reinterpret_cast<const uint4 *>(row + 16 * u);
                const uint32_t cw[4] = {cw4.x, cw4.y, cw4.z, cw4.w};
                float lo = 0.0f, hi = 0.0f;
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
#pragma unroll
                    for (int bi = 0; bi < 4; ++bi) {
                        const float2 l = tbl[((cw[wi] >> (8 * bi)) & 0xFFu) * kTblReplicas];
                        lo = fmaf(l.x, xr[8 * wi + 2 * bi], lo);
                        hi = fmaf(l.y, xr[8 * wi + 2 * bi + 1], hi);
                    }
                }
                acc = (lo + hi) * scl[pr * G + u / 4];
            } else {
                const float4 *w4 = reinterpret_cast<const float4 *>(row) + 8 * u;
                float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 w = w4[i];
                    a0 = fmaf(w.x, xr[4 * i], a0);
                    a1 = fmaf(w.y, xr[4 * i + 1], a1);
                    a2 = fmaf(w.z, xr[4 * i + 2], a2);
                    a3 = fmaf(w.w, xr[4 * i + 3], a3);
                }
                acc = (a0 + a1) + (a2 + a3);
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) red[kp * P + pr] = acc;
    }
}

// The chunk's epilogue, by the one warp that finished it last: K parts summed
// in order, then the stage's output (tagged word, SwiGLU, convolution, or
// logits with the argmax candidate of the lane).
__device__ __noinline__ void chunk_finalize(const PStage &St, int slot, uint32_t va, uint32_t nv, uint32_t v0, int KP,
                                            uint32_t tag, float *am) {
    const Smem S = smem();
    const int lane = threadIdx.x & 31;
    const int comps = St.comps, kind = St.kind, P = (int)nv * comps;
    const float *red = S.red + slot * kRedPerSlot;
    const int hidden = sP.hidden;
    for (int r = lane; r < (int)nv; r += 32) {
        float val[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int cc = 0; cc < 3; ++cc) {
            if (cc >= comps) break;
            float a = 0.0f;
            for (int k = 0; k < KP; ++k) a += red[k * P + cc * (int)nv + r];
            val[cc] = a;
        }
        const uint32_t v = va + r;
        if (kind == PK_FFN) {
            st_tagged(St.out + v, silu_mul(val[0], val[1]), tag);
        } else if (kind == PK_MIXCONV) {
            // crates/backend-cpu/src/attention_convolution.rs:220-340, one
            // token; taps and history were prefetched for channels v0..v1.
            const int W = St.conv_w, ch = (int)(v - v0);
            const float uu = __fmul_rn(val[0], val[2]);
            float win[kMaxConvW];
#pragma unroll
            for (int i = 0; i < kMaxConvW - 1; ++i)
                if (i < W - 1) win[i] = S.cvh[i * kMaxCh + ch];
            win[W - 1] = uu;
            float total = 0.0f;
#pragma unroll
            for (int tap = 0; tap < kMaxConvW; ++tap)
                if (tap < W) total = __fadd_rn(total, __fmul_rn(S.cvk[ch * kMaxConvW + tap], win[tap]));
#pragma unroll
            for (int i = 0; i < kMaxConvW - 1; ++i)
                if (i < W - 1) St.conv_hist[(size_t)i * hidden + v] = win[i + 1];
            st_tagged(St.out + v, __fmul_rn(total, val[1]), tag);
        } else if (kind == PK_HEAD) {
            sP.logits[v] = val[0];
            float bv = am[0];
            int bi = __float_as_int(am[1]), bp = __float_as_int(am[2]);
            am_merge(bv, bi, bp, val[0], (int)v, isfinite(val[0]) ? 0 : 1);
            am[0] = bv;
            am[1] = __int_as_float(bi);
            am[2] = __int_as_float(bp);
        } else {
            st_tagged(St.out + v, val[0], tag);
        }
    }
}

// Attention stage (one token): this CTA's (kv head, key chunk) unit; partial
// softmax sums merged by the last chunk CTA of the kv head.
__device__ __noinline__ bool stage_attention(const PStage &St, uint32_t tag, uint64_t pos, uint32_t epoch, uint32_t *n_io,
                                             Ctl c) {
    const Smem S = smem();
    const PParams &p = sP;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int NS = p.nslots, hidden = p.hidden;
    int h = 0, ci = 0;
    uint64_t k0 = 0, k1 = 0, kend = 0;
    if (!att_unit(p, pos, h, ci, k0, k1, kend)) {
        // Idle CTA: still one barrier, for the descriptor buffer rule.
        cp_wait_all();
        cbar();
        return false;
    }
    uint32_t n = *n_io;
    const int group = p.group;
    const uint32_t tin = stage_tag(epoch, St.in_stage);
    const unsigned long long *qkv = St.in;
    float *qraw = S.xs;                         // [group][64]
    float *qs = qraw + kMaxGroup * kAttD;       // [group][64] normed + rotated
    float *kn = qs + kMaxGroup * kAttD;         // [64] new key (normed + rotated)
    float *vn = kn + kAttD;                     // [64] new value
    float *kraw = vn + kAttD;                   // [64]
    float *sp = kraw + kAttD;                   // [group][64]
    float *mrun = sp + kMaxGroup * kKeysPerChunk, *lrun = mrun + kMaxGroup, *crr = lrun + kMaxGroup;
    const float *aw = S.xs + kAttScratch;       // prefetched q_norm, k_norm, rot
    float *ml = S.xs + kAttScratch + 192;       // merge: [C][group] (m, l)
    const bool has_new = kend > pos;            // this chunk holds key `pos`
    for (int e = tid; e < group * kAttD + 2 * kAttD; e += kCThreads) {
        uint32_t src;
        float *dst;
        if (e < group * kAttD) {
            src = (uint32_t)(h * group * kAttD + e);
            dst = qraw + e;
        } else if (e < group * kAttD + kAttD) {
            const int d = e - group * kAttD;
            src = (uint32_t)(hidden + h * kAttD + d);
            dst = kraw + d;
        } else {
            const int d = e - group * kAttD - kAttD;
            src = (uint32_t)(hidden + p.kv_heads * kAttD + h * kAttD + d);
            dst = vn + d;
        }
        *dst = wait_tagged(qkv + src, tin, c);
    }
    if (tid < kMaxGroup) {
        mrun[tid] = -INFINITY;
        lrun[tid] = 0.0f;
        crr[tid] = 0.0f;
    }
    cp_wait_all();
    if (cbar_aborted(c)) return true;
    const float2 *rot = reinterpret_cast<const float2 *>(aw + 128);
    if (warp < group) norm_rope64(qraw + warp * kAttD, aw, p.att_eps, rot, qs + warp * kAttD, lane);
    else if (warp == group) norm_rope64(kraw, aw + 64, p.att_eps, rot, kn, lane);
    cbar();
    if (has_new && tid < kAttD) {
        const uint64_t kvw = (uint64_t)p.kv_heads * kAttD;
        St.kcache[pos * kvw + (uint64_t)h * kAttD + tid] = kn[tid];
        St.vcache[pos * kvw + (uint64_t)h * kAttD + tid] = vn[tid];
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)kAttD));
    float o_run = 0.0f;
    const uint32_t nch = (uint32_t)((k1 - k0 + kKeysPerChunk - 1) / kKeysPerChunk);
    for (uint32_t ch = 0; ch < nch; ++ch, ++n) {
        const uint32_t slot = n % NS, round = n / NS;
        const bool got = wait_full(S.bar0 + 8 * slot, round & 1, c);
        const int nk = (int)min((uint64_t)kKeysPerChunk, k1 - (k0 + (uint64_t)ch * kKeysPerChunk));
        const float *kr = reinterpret_cast<const float *>(S.ring + slot * kSlotBytes);
        const float *vr = kr + kKeysPerChunk * kKPitch;
        if (got) att_chunk(kr, kKPitch, vr, nk, qs, sp, mrun, lrun, crr, group, scale, o_run, tid);
        else { cbar(); cbar(); }
        __syncwarp();
        if (lane == 0) mbar_arrive(S.bar0 + 8 * (NS + slot));
        if (cbar_aborted(c)) {
            *n_io = n + 1;
            return true;
        }
    }
    *n_io = n;
    if (has_new) {
        att_chunk(kn, kAttD, vn, 1, qs, sp, mrun, lrun, crr, group, scale, o_run, tid);
        cbar();
    }
    // Partial (m, l, o) of each query head, then the last chunk CTA of this
    // kv head merges all chunks in chunk order.
    const int C = p.att_chunks;
    float *part = p.att_part + (((size_t)St.att_index * p.kv_heads + h) * C) * group * (kAttD + 2);
    if (tid < group * kAttD) {
        const int gh = tid / kAttD, d = tid % kAttD;
        float *pr = part + ((size_t)ci * group + gh) * (kAttD + 2);
        pr[2 + d] = o_run;
        if (d == 0) {
            pr[0] = mrun[gh];
            pr[1] = lrun[gh];
        }
    }
    __threadfence();
    cbar();
    if (tid == 0) {
        unsigned *cnt = p.att_count + (size_t)St.att_index * p.kv_heads + h;
        sLast = atomicAdd(cnt, 1u) == (unsigned)(C - 1);
    }
    cbar();
    if (sLast) {
        // One round trip: (m, l) of every chunk into shared memory, and each
        // thread's weighted-V values of every chunk into registers, all loads
        // in flight together.
        __threadfence();
        if (tid < C * group) {
            const float *pr = part + (size_t)tid * (kAttD + 2);
            ml[2 * tid] = __ldcg(pr);
            ml[2 * tid + 1] = __ldcg(pr + 1);
        }
        const int gh = tid / kAttD, d = tid % kAttD;
        float ov[kMaxAttChunks];
#pragma unroll
        for (int i = 0; i < kMaxAttChunks; ++i)
            ov[i] = (gh < group && i < C) ? __ldcg(part + ((size_t)i * group + gh) * (kAttD + 2) + 2 + d) : 0.0f;
        cbar();
        if (gh < group) {
            float M = -INFINITY;
            for (int cc = 0; cc < C; ++cc) M = fmaxf(M, ml[2 * (cc * group + gh)]);
            float L = 0.0f, O = 0.0f;
#pragma unroll
            for (int i = 0; i < kMaxAttChunks; ++i) {
                if (i >= C) break;
                const float m = ml[2 * (i * group + gh)];
                if (m == -INFINITY) continue;
                const float w = expf(m - M);
                L = fmaf(ml[2 * (i * group + gh) + 1], w, L);
                O = fmaf(ov[i], w, O);
            }
            st_tagged(St.out + (size_t)(h * group + gh) * kAttD + d, __fdiv_rn(O, L), tag);
        }
        if (tid == 0) p.att_count[(size_t)St.att_index * p.kv_heads + h] = 0u;
    }
    cbar();
    return false;
}

// End of the LM head stage: the CTA's argmax candidate, then the last CTA
// merges every CTA's (first strict maximum, NaN poisoning), writes the greedy
// id, and advances the position and the epoch.
__device__ __noinline__ void head_reduce(uint64_t pos, uint32_t epoch, const float *am) {
    const PParams &p = sP;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float bv = am[0];
    int bi = __float_as_int(am[1]), bp = __float_as_int(am[2]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        am_merge(bv, bi, bp, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o),
                 __shfl_xor_sync(0xffffffffu, bp, o));
    if (lane == 0) {
        sAmV[warp] = bv;
        sAmI[warp] = bi;
        sAmP[warp] = bp;
    }
    cbar();
    if (tid == 0) {
        for (int w = 1; w < kCW; ++w) am_merge(bv, bi, bp, sAmV[w], sAmI[w], sAmP[w]);
        float *mine = p.arg_part + (size_t)blockIdx.x * 3;
        mine[0] = bv;
        mine[1] = __int_as_float(bi);
        mine[2] = __int_as_float(bp);
        __threadfence();
        sLast = atomicAdd(p.arg_count, 1u) == gridDim.x - 1;
    }
    cbar();
    if (!sLast) return;
    __threadfence();
    bv = -INFINITY;
    bi = -1;
    bp = 0;
    for (int cc = tid; cc < (int)gridDim.x; cc += kCThreads) {
        const float *pc = p.arg_part + (size_t)cc * 3;
        am_merge(bv, bi, bp, __ldcg(pc), __float_as_int(__ldcg(pc + 1)), __float_as_int(__ldcg(pc + 2)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        am_merge(bv, bi, bp, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o),
                 __shfl_xor_sync(0xffffffffu, bp, o));
    cbar();
    if (lane == 0) {
        sAmV[warp] = bv;
        sAmI[warp] = bi;
        sAmP[warp] = bp;
    }
    cbar();
    if (tid == 0) {
        for (int w = 1; w < kCW; ++w) am_merge(bv, bi, bp, sAmV[w], sAmI[w], sAmP[w]);
        *p.sampled = (bp || bi < 0) ? __int_as_float(0x7fc00000) : (float)bi;
        *p.pos = pos + 1;
        *p.epoch = epoch + 1;
        *p.arg_count = 0u;
    }
}

__device__ __forceinline__ void consumer(uint64_t pos, uint32_t epoch, Ctl c) {
    const Smem S = smem();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int NS = sP.nslots, n_stages = sP.n_stages;
    uint32_t n = 0;   // chunks consumed (the producer's order)
    float am[3] = {-INFINITY, __int_as_float(-1), __int_as_float(0)};   // argmax candidate (head)
    for (int s = 0; s < n_stages; ++s) {
        const PStage &St = S.desc[s % 3];
        const uint32_t tag = stage_tag(epoch, s);
        stage_prefetch(sP, S, s, St, pos, tid);
        const int kind = St.kind;
        if (kind == PK_ATTN) {
            if (stage_attention(St, tag, pos, epoch, &n, c)) return;
            continue;
        }
        const int fmt = St.fmt;
        const bool imma = fmt == MF_TERNARY || fmt == MF_INT8;
        if (St.norm ? prologue_norm(St, epoch, c) : prologue_plain(St, epoch, c)) return;
        uint32_t v0, v1;
        cta_rows(St.V, v0, v1);
        const uint32_t per = St.cv;
        const uint32_t nch = (v1 - v0 + per - 1) / per;
        const int G = St.K / 128, U = St.K / 32;
        // Integer formats: warp = (16-row tile, K part); NF4 / dense: warp =
        // (K part of 1024 weights, row group).
        const int T = (int)St.tiles;
        const int KP = imma ? kCW / T : max(1, (U + 31) / 32);
        const int WPK = kCW / KP;
        const int gpp = (G + KP - 1) / KP;
        const int tile = warp % T;
        const int kp = imma ? warp / T : warp % KP;
        const int rg = warp / KP;
        const bool active = imma ? kp < KP : rg < WPK;
        for (uint32_t ch = 0; ch < nch; ++ch, ++n) {
            const uint32_t slot = n % NS, round = n / NS;
            const bool got = wait_full(S.bar0 + 8 * slot, round & 1, c);
            const uint32_t va = v0 + ch * per;
            const uint32_t nv = min(per, v1 - va);
            const int P = (int)nv * St.comps;
            if (got && active) {
                if (imma) chunk_imma(St, (int)slot, P, tile, kp, kp * gpp, min(G, (kp + 1) * gpp));
                else chunk_fp32(St, (int)slot, P, kp, rg, WPK);
            }
            // The last warp to finish the chunk finalizes it; the others
            // release the slot at once (the finalizing warp releases it after
            // reading the partials, so no warp reaches the chunk that reuses
            // this slot's partial sums before then).
            __syncwarp();
            unsigned last = 0;
            if (lane == 0) {
                __threadfence_block();
                last = atomicAdd(S.cnt + slot, 1u) == (unsigned)(kCW - 1);
                if (!last) mbar_arrive(S.bar0 + 8 * (NS + slot));
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) continue;
            __threadfence_block();
            chunk_finalize(St, (int)slot, va, nv, v0, KP, tag, am);
            __syncwarp();
            if (lane == 0) {
                S.cnt[slot] = 0u;
                mbar_arrive(S.bar0 + 8 * (NS + slot));
            }
        }
        if (kind == PK_HEAD) {
            cbar();   // every chunk finalized
            head_reduce(pos, epoch, am);
        }
    }
}

__global__ void __launch_bounds__(kPThreads, 1) decode_persistent_kernel(const PParams p) {
    __shared__ int s_abort;
    __shared__ int s_skip;
    const int tid = threadIdx.x;
    if (tid == 0) sP = p;
    __syncthreads();
    const Smem S = smem();
    for (int e = tid; e < 256 * kTblReplicas; e += blockDim.x) {
        const int b = e / kTblReplicas;
        S.tbl[e] = make_float2(kPNf4[b & 15], kPNf4[b >> 4]);
    }
    if (tid < kMaxSlots) S.cnt[tid] = 0u;
    if (tid < (int)(sizeof(PStage) / 4))   // stage 0's descriptor
        reinterpret_cast<uint32_t *>(S.desc)[tid] = reinterpret_cast<const uint32_t *>(p.stages)[tid];
    if (tid == 0) {
        for (int i = 0; i < p.nslots; ++i) {
            mbar_init(S.bar0 + 8 * i, 1);
            mbar_init(S.bar0 + 8 * (p.nslots + i), kCW);
        }
        mbar_init_fence();
        s_abort = 0;
        s_skip = *reinterpret_cast<volatile unsigned *>(&g_persist_fault) != 0;
    }
    __syncthreads();
    if (s_skip) return;   // an earlier step faulted: nothing runs until the host clears it
    Ctl c;
    c.abort_flag = &s_abort;
    c.timeout = p.timeout_ns;
    const uint64_t pos = *p.pos;
    const uint32_t epoch = *p.epoch;
    if (tid >= kCThreads) producer(p, reinterpret_cast<unsigned char *>(S.tbl), pos, c);
    else consumer(pos, epoch, c);
}

}  // namespace

// ---------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------
namespace {

uint32_t code_pitch(int fmt, int K) {
    const uint32_t rb = fmt == MF_TERNARY ? K / 4 : fmt == MF_NF4 ? K / 2 : fmt == MF_INT8 ? K : K * 4;
    if (fmt == MF_TERNARY) return rb + ((32 - (int)(rb % 128)) + 128) % 128;   // = 32 mod 128
    if (fmt == MF_INT8) return rb + ((16 - (int)(rb % 128)) + 128) % 128;      // = 16 mod 128
    return rb;
}

struct Layout {
    uint32_t off_bar, off_res, off_xs, off_limb, off_efac, off_red, off_conv, off_desc, off_ring, total;
    int nslots;
};

uint32_t al(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

}  // namespace

struct PersistPlan {
    std::vector<PStage> stages;
    PParams params{};
    Layout lay{};
    size_t out_words = 0;
    int n_att = 0;
};

bool persistent_geometry_ok(const PersistModelDesc &d) {
    if (d.hidden % 128 || d.hidden > 4096 || d.intermediate % 128 || d.intermediate > 16384) return false;
    if (d.head_dim != kAttD || d.kv_heads == 0 || d.q_heads % d.kv_heads) return false;
    // Query group: at most 4 heads (one consumer thread per (head, dim) pair
    // of a kv head's group).
    if (d.q_heads / d.kv_heads > 4 || d.conv_width < 1 || d.conv_width > kMaxConvW) return false;
    if ((uint64_t)d.q_heads * kAttD != d.hidden) return false;
    if (d.hidden > 128u * kMaxCh) return false;   // conv channels per CTA (>= 128 CTAs)
    if (d.vocab == 0 || d.vocab > (1u << 24)) return false;
    const uint32_t stages = (uint32_t)d.layers.size() * 5 + 1;
    if (stages >= kStagesPerEpoch) return false;
    for (const PersistLayerDesc &L : d.layers) {
        auto packed = [](const PersistMat &m) { return m.codes && m.scales; };
        if (L.kind == MF_LAYER_ATTENTION && !d.rope) return false;
        if (L.kind == MF_LAYER_CONV) {
            if (!packed(L.in_proj) || !packed(L.out_proj)) return false;
        } else {
            if (!packed(L.q) || !packed(L.k) || !packed(L.v) || !packed(L.o)) return false;
            if (L.q.format != L.k.format || L.k.format != L.v.format) return false;
        }
        if (!packed(L.w1) || !packed(L.w2) || !packed(L.w3) || L.w1.format != L.w3.format) return false;
    }
    if (!d.emb.dense && !(d.emb.codes && d.emb.scales)) return false;
    return true;
}

// Builds the stage program and the shared-memory layout.  Output words,
// partials and counters are addressed inside `ws` (persistent_ws_bytes).
int32_t persistent_plan(const PersistModelDesc &d, const PersistStateDesc &s, int sms, void *ws, PersistPlan **out) {
    if (!persistent_geometry_ok(d)) return fail(MF_UNSUPPORTED, "persistent decode step does not take this model");
    PersistPlan *pl = new (std::nothrow) PersistPlan();
    if (!pl) return fail(MF_RESOURCE_LIMIT, "host allocation failed");
    const uint32_t h = d.hidden, f = d.intermediate, kvw = d.kv_heads * kAttD;
    const int group = (int)(d.q_heads / d.kv_heads);
    const int C = std::min(sms / (int)d.kv_heads, kMaxAttChunks);
    // Workspace: [epoch u32 x 64][arg count u32 x 64][att counts][arg partials][att partials][outputs]
    unsigned char *w = static_cast<unsigned char *>(ws);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        unsigned char *r = w + off;
        off += (bytes + 255) / 256 * 256;
        return r;
    };
    pl->params.epoch = reinterpret_cast<uint32_t *>(take(256));
    pl->params.arg_count = reinterpret_cast<unsigned *>(take(256));
    int n_att = 0;
    for (const PersistLayerDesc &L : d.layers) n_att += L.kind == MF_LAYER_ATTENTION;
    pl->n_att = n_att;
    pl->params.att_count = reinterpret_cast<unsigned *>(take(sizeof(unsigned) * std::max(1, n_att) * d.kv_heads));
    pl->params.arg_part = reinterpret_cast<float *>(take(sizeof(float) * 3 * sms));
    pl->params.att_part =
        reinterpret_cast<float *>(take(sizeof(float) * std::max(1, n_att) * d.kv_heads * C * group * (kAttD + 2)));

    auto mat = [](const PersistMat &m) {
        PMat r{};
        r.codes = m.codes;
        r.scales = m.scales;
        r.dense = m.dense;
        r.rows = m.rows;
        return r;
    };
    auto outbuf = [&](size_t n) { return reinterpret_cast<unsigned long long *>(take(n * 8)); };
    auto chunking = [&](PStage &S) {
        S.pitch = code_pitch(S.fmt, S.K);
        const uint32_t G = S.K / 128;
        uint32_t cap = kSlotCode / (S.pitch * S.comps);
        cap = std::min<uint32_t>(cap, kMaxRows / S.comps);
        if (S.fmt != kDenseFmt) cap = std::min<uint32_t>(cap, kSlotScale / (4 * G * S.comps));
        S.cv = std::max<uint32_t>(1, cap);
        S.tiles = (S.cv * S.comps + 15) / 16;
    };
    std::vector<PStage> &st = pl->stages;
    int prev_down = -1;   // stage producing the residual delta for the next norm
    int att_i = 0;
    for (size_t li = 0; li < d.layers.size(); ++li) {
        const PersistLayerDesc &L = d.layers[li];
        int mixer_out;
        if (L.kind == MF_LAYER_CONV) {
            PStage a{};
            a.kind = PK_MIXCONV;
            a.fmt = L.in_proj.format;
            a.K = h;
            a.comps = 3;
            a.V = h;
            a.mat[0] = mat(L.in_proj);
            a.split0 = h;
            a.in_stage = prev_down;
            a.norm = 1;
            a.eps = d.block_eps;
            a.norm_w = L.operator_norm;
            a.out = outbuf(h);
            a.conv_k = L.conv_kernel;
            a.conv_hist = s.history[li];
            a.conv_w = d.conv_width;
            chunking(a);
            st.push_back(a);
            PStage b{};
            b.kind = PK_PROJ;
            b.fmt = L.out_proj.format;
            b.K = h;
            b.comps = 1;
            b.V = h;
            b.mat[0] = mat(L.out_proj);
            b.in_stage = (int)st.size() - 1;
            b.out = outbuf(h);
            chunking(b);
            st.push_back(b);
            mixer_out = (int)st.size() - 1;
        } else {
            PStage a{};
            a.kind = PK_QKV;
            a.fmt = L.q.format;
            a.K = h;
            a.comps = 1;
            a.V = h + 2 * kvw;
            a.mat[0] = mat(L.q);
            a.mat[1] = mat(L.k);
            a.mat[2] = mat(L.v);
            a.split0 = h;
            a.split1 = h + kvw;
            a.in_stage = prev_down;
            a.norm = 1;
            a.eps = d.block_eps;
            a.norm_w = L.operator_norm;
            a.out = outbuf(h + 2 * kvw);
            chunking(a);
            st.push_back(a);
            PStage b{};
            b.kind = PK_ATTN;
            b.in_stage = (int)st.size() - 1;
            b.out = outbuf(h);
            b.q_norm = L.q_norm;
            b.k_norm = L.k_norm;
            b.kcache = s.kcache[li];
            b.vcache = s.vcache[li];
            b.att_index = att_i++;
            st.push_back(b);
            PStage o{};
            o.kind = PK_PROJ;
            o.fmt = L.o.format;
            o.K = h;
            o.comps = 1;
            o.V = h;
            o.mat[0] = mat(L.o);
            o.in_stage = (int)st.size() - 1;
            o.out = outbuf(h);
            chunking(o);
            st.push_back(o);
            mixer_out = (int)st.size() - 1;
        }
        PStage fp{};
        fp.kind = PK_FFN;
        fp.fmt = L.w1.format;
        fp.K = h;
        fp.comps = 2;
        fp.V = f;
        fp.mat[0] = mat(L.w1);
        fp.mat[1] = mat(L.w3);
        fp.in_stage = mixer_out;
        fp.norm = 1;
        fp.eps = d.block_eps;
        fp.norm_w = L.ffn_norm;
        fp.out = outbuf(f);
        chunking(fp);
        st.push_back(fp);
        PStage dn{};
        dn.kind = PK_PROJ;
        dn.fmt = L.w2.format;
        dn.K = f;
        dn.comps = 1;
        dn.V = h;
        dn.mat[0] = mat(L.w2);
        dn.in_stage = (int)st.size() - 1;
        dn.out = outbuf(h);
        chunking(dn);
        st.push_back(dn);
        prev_down = (int)st.size() - 1;
    }
    PStage hd{};
    hd.kind = PK_HEAD;
    hd.fmt = d.emb.dense ? kDenseFmt : d.emb.format;
    hd.K = h;
    hd.comps = 1;
    hd.V = d.vocab;
    hd.mat[0] = mat(d.emb);
    hd.in_stage = prev_down;
    hd.norm = 1;
    hd.eps = d.norm_eps;
    hd.norm_w = d.emb_norm;
    chunking(hd);
    st.push_back(hd);
    for (PStage &S : st)
        if (S.in_stage >= 0) S.in = st[S.in_stage].out + S.in_off;
    // Stage program at the end of the workspace.
    PStage *dev_stages = reinterpret_cast<PStage *>(take(sizeof(PStage) * st.size()));
    pl->out_words = off;

    // Shared-memory layout.
    uint32_t kmax_imma = 128, kmax_x = h;
    for (const PStage &S : st) {
        if (S.kind == PK_ATTN) continue;
        if (S.fmt == MF_TERNARY || S.fmt == MF_INT8) kmax_imma = std::max<uint32_t>(kmax_imma, S.K);
        else kmax_x = std::max<uint32_t>(kmax_x, S.K);
    }
    Layout &ly = pl->lay;
    uint32_t o = 256 * 8 * kTblReplicas;   // NF4 byte table, kTblReplicas copies
    ly.off_bar = o;
    o += 8 * 2 * kMaxSlots + 4 * kMaxSlots;   // mbarriers, then the slots' warp counters
    ly.off_res = o = al(o, 16);
    o += 4 * h;
    ly.off_xs = o = al(o, 16);
    o += 4 * std::max<uint32_t>(pad32((int)kmax_x), kAttFloats);
    ly.off_limb = o = al(o, 16);
    o += std::max<uint32_t>((kmax_imma / 128) * 512, 4 * h);   // limbs, or the norm weight
    ly.off_efac = o = al(o, 16);
    o += 4 * (kmax_imma / 128);
    ly.off_red = o = al(o, 16);
    o += 4 * kMaxSlots * kRedPerSlot;
    ly.off_conv = o = al(o, 16);
    o += 4 * kMaxCh * (2 * kMaxConvW - 1);
    ly.off_desc = o = al(o, 16);
    o += 3 * sizeof(PStage);
    ly.off_ring = o = al(o, 1024);
    const uint32_t limit = kDynSmemLimit;
    if (o + 2 * kSlotBytes > limit) {
        delete pl;
        return fail(MF_UNSUPPORTED, "persistent decode step: shared memory too small for this model");
    }
    ly.nslots = (int)std::min<uint32_t>(kMaxSlots, (limit - o) / kSlotBytes);
    ly.total = o + ly.nslots * kSlotBytes;

    PParams &pp = pl->params;
    pp.stages = dev_stages;
    pp.n_stages = (int)st.size();
    pp.hidden = (int)h;
    pp.q_heads = (int)d.q_heads;
    pp.kv_heads = (int)d.kv_heads;
    pp.group = group;
    pp.vocab = (int)d.vocab;
    pp.att_chunks = C;
    pp.capacity = d.max_tokens;
    pp.rope = d.rope;
    pp.att_eps = d.block_eps;
    pp.ecodes = d.emb.codes;
    pp.escales = d.emb.scales;
    pp.edense = d.emb.dense;
    pp.efmt = d.emb.format;
    pp.erows = d.emb.rows;
    pp.pos = s.pos;
    pp.sampled = s.sampled;
    pp.logits = s.logits;
    pp.nslots = ly.nslots;
    pp.off_bar = ly.off_bar;
    pp.off_res = ly.off_res;
    pp.off_xs = ly.off_xs;
    pp.off_limb = ly.off_limb;
    pp.off_efac = ly.off_efac;
    pp.off_red = ly.off_red;
    pp.off_conv = ly.off_conv;
    pp.off_desc = ly.off_desc;
    pp.off_ring = ly.off_ring;
    pp.timeout_ns = 2000000000ull;
    *out = pl;
    return MF_OK;
}

size_t persistent_ws_bytes(const PersistModelDesc &d, int sms) {
    // Mirror of persistent_plan's `take` sequence (an upper bound).
    const size_t h = d.hidden, f = d.intermediate, kvw = (size_t)d.kv_heads * kAttD;
    const size_t group = d.kv_heads ? d.q_heads / d.kv_heads : 1;
    const size_t C = d.kv_heads ? sms / d.kv_heads : 1;
    size_t n_att = 0;
    for (const PersistLayerDesc &L : d.layers) n_att += L.kind == MF_LAYER_ATTENTION;
    size_t words = 0;
    for (const PersistLayerDesc &L : d.layers)
        words += (L.kind == MF_LAYER_CONV ? 2 * h : (h + 2 * kvw) + 2 * h) + f + h;
    auto r = [](size_t b) { return (b + 255) / 256 * 256; };
    size_t total = 256 + 256 + r(4 * std::max<size_t>(1, n_att) * d.kv_heads) + r(4 * 3 * (size_t)sms) +
                   r(4 * std::max<size_t>(1, n_att) * d.kv_heads * C * group * (kAttD + 2));
    total += 8 * words + 256 * 6 * d.layers.size() + r(sizeof(PStage) * (d.layers.size() * 5 + 1)) + 4096;
    return total;
}

// Uploads the program, zeroes the workspace and sets the epoch to 1 (tags of
// zeroed words never match).  Stream-ordered.
int32_t persistent_init(PersistPlan *pl, void *ws, size_t ws_bytes, cudaStream_t stream) {
    if (pl->out_words > ws_bytes) return fail(MF_RESOURCE_LIMIT, "persistent workspace too small");
    MF_CUDA_TRY(cudaMemsetAsync(ws, 0, ws_bytes, stream));
    static const uint32_t kOne = 1;
    MF_CUDA_TRY(cudaMemcpyAsync(pl->params.epoch, &kOne, sizeof(kOne), cudaMemcpyHostToDevice, stream));
    MF_CUDA_TRY(cudaMemcpyAsync(const_cast<PStage *>(pl->params.stages), pl->stages.data(),
                                sizeof(PStage) * pl->stages.size(), cudaMemcpyHostToDevice, stream));
    // The host program must outlive the async copy: callers synchronize.
    MF_CUDA_TRY(cudaStreamSynchronize(stream));
    MF_CUDA_TRY(cudaFuncSetAttribute(decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kDynSmemLimit));
    return MF_OK;
}

int32_t persistent_launch(const PersistPlan *pl, int sms, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)sms);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = pl->lay.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    const cudaError_t err = cudaLaunchKernelEx(&cfg, decode_persistent_kernel, pl->params);
    if (err != cudaSuccess) return cuda_fail(err, "decode_persistent_kernel");
    return MF_OK;
}

void persistent_free(PersistPlan *pl) { delete pl; }

int persistent_slots(const PersistPlan *pl) { return pl->lay.nslots; }

int32_t persistent_faults(uint32_t *flags) {
    uint32_t v = 0, zero = 0;
    MF_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_persist_fault, sizeof(v)));
    MF_CUDA_TRY(cudaMemcpyToSymbol(g_persist_fault, &zero, sizeof(zero)));
    *flags = v;
    return MF_OK;
}

}  // namespace mf

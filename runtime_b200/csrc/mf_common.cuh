// Shared helpers for the sm_100a kernels and the C-ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/mfcuda.h"

namespace mf {

constexpr int kGroup = 128;       // K elements per scale group (all formats)
constexpr int kSmCount = 148;     // B200: 2 dies x 74 SMs (queried at runtime too)

// Thread-local last error message (static strings only).
void set_error(const char *message);
int32_t fail(int32_t status, const char *message);
int32_t cuda_fail(cudaError_t err, const char *where);

inline int weights_per_byte(int format) { return format == MF_TERNARY ? 4 : format == MF_NF4 ? 2 : 1; }
inline uint64_t code_cols(int format, uint64_t k) { return k / (uint64_t)weights_per_byte(format); }

// Number of SMs of the current device (cached per device).
int sm_count();

// Launch accounting: every kernel launch through this library bumps this
// counter (read by the backend's dispatch counts and the bench).
void count_launch(int64_t n = 1);
uint64_t launches();

// Whether launches carry the programmatic-dependent-launch attribute (on by
// default; mf_set_pdl turns it off for comparison runs).
bool pdl_enabled();

// Per-launch timing of the executor's step (mf_lfm2_time_step): while a
// recorder is set on this thread, every launch records an event after
// itself on its stream, with the current label (or the kernel's name).
// The events serialize the launches they separate.
struct LaunchRecorder {
    cudaEvent_t *events = nullptr;
    const char **names = nullptr;
    size_t cap = 0, n = 0;
    const char *label = nullptr;
};
LaunchRecorder *&launch_recorder();

// Every kernel of this library is launched through here.  With PDL the
// next kernel in the stream may start while this one runs; each kernel
// therefore executes pdl_wait() before it reads anything an earlier kernel
// wrote or writes anything at all (weights and other constants may be read
// before it), so completion stays transitive along the stream, and calls
// pdl_trigger() only after its own wait, so at most one kernel is launched
// ahead of the one running.
template <typename... KArgs, typename... Args>
int32_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               const char *name, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    count_launch();
    const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (err != cudaSuccess) return cuda_fail(err, name);
    if (LaunchRecorder *r = launch_recorder()) {
        if (r->n < r->cap) {
            cudaEventRecord(r->events[r->n], stream);
            r->names[r->n] = r->label ? r->label : name;
        }
        r->n++;
    }
    return MF_OK;
}

}  // namespace mf

#define MF_CUDA_TRY(expr)                                         \
    do {                                                          \
        cudaError_t mf_err_ = (expr);                             \
        if (mf_err_ != cudaSuccess) return mf::cuda_fail(mf_err_, #expr); \
    } while (0)

#define MF_LAUNCH_CHECK(where)                                    \
    do {                                                          \
        mf::count_launch();                                       \
        cudaError_t mf_err_ = cudaGetLastError();                 \
        if (mf_err_ != cudaSuccess) return mf::cuda_fail(mf_err_, where); \
    } while (0)

// ---------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------
namespace mf {

// Programmatic dependent launch: let the next kernel in the stream start
// launching, and wait for the previous kernel's completion (and memory).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Non-caching 16-byte global load for streamed weights (read exactly once).
// Streamed weights (codes and scales read once per step) are loaded with an
// L2 evict-first policy: the decode step reads more weight bytes than L2
// holds, and evicting them first keeps the activations, the KV cache and the
// kernels' code resident for the next kernel in the chain.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p), "l"(l2_evict_first()));
    return r;
}

__device__ __forceinline__ uint2 ld_stream_u2(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;"
                 : "=r"(r.x), "=r"(r.y)
                 : "l"(p), "l"(l2_evict_first()));
    return r;
}

__device__ __forceinline__ float4 ld_stream_f4(const float *p) {
    const uint4 u = ld_stream_u4(p);
    return make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w));
}

__device__ __forceinline__ float ld_stream_f32(const float *p) {
    float r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(r) : "l"(p), "l"(l2_evict_first()));
    return r;
}

// IEEE-rounded silu(g) * u as the reference computes it:
// sigmoid = 1 / (1 + exp(-g)); (g * sigmoid) * u, each op rounded.
__device__ __forceinline__ float silu_mul(float g, float u) {
    float sigmoid = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    return __fmul_rn(__fmul_rn(g, sigmoid), u);
}

}  // namespace mf

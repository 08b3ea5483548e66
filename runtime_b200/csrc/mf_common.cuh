// Shared helpers for the sm_100a kernels and the C-ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

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
__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint2 ld_stream_u2(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

// IEEE-rounded silu(g) * u as the reference computes it:
// sigmoid = 1 / (1 + exp(-g)); (g * sigmoid) * u, each op rounded.
__device__ __forceinline__ float silu_mul(float g, float u) {
    float sigmoid = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    return __fmul_rn(__fmul_rn(g, sigmoid), u);
}

}  // namespace mf

// Backend and buffer records behind the opaque C-ABI handles.
#pragma once

#include <vector>

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <unordered_set>

#include "../../include/mfcuda.h"
#include "packed_kernels.h"

struct mf_buffer {
    mf_backend *owner;
    uint64_t generation;
    uint64_t id;
    int32_t dtype;
    uint32_t rank;
    uint64_t shape[MF_MAX_RANK];
    uint64_t elements;
    uint64_t bytes;
    int32_t alloc_class;
    void *ptr;
    // U8 streams only: some byte equals 0x80 (the reserved INT8 code -128).
    // Recorded at upload so INT8 admission needs no per-call device scan.
    bool has_int8_reserved;
    // U8 ternary codes in the backend's LUT2 (lane-tiled) layout, as written
    // by mf_repack_ternary_lut2: only the *_lut2 ops accept them.
    bool lut2;
};

struct mf_backend {
    int32_t ordinal;
    uint64_t owner;
    uint64_t generation;
    cudaStream_t stream;
    mf_limits limits;
    uint64_t live_by_class[4];
    uint64_t live_total;
    uint64_t peak;
    uint64_t next_id;
    uint32_t pending_ops;
    uint64_t pending_bytes;
    int32_t inject;  // 0 none, 1 fence, 2 allocation, 3 readback
    mf_dispatch_counts counts;
    std::unordered_set<const mf_buffer *> live;
    // Stream-ordered scratch for per-call staging (host ids, positions,
    // masks, attention partials).  Reused call after call in stream order.
    void *scratch;
    size_t scratch_bytes;
    // Split-K arrival counters of the decode GEMV (kept zero between calls).
    unsigned *splitk_counters;
    size_t splitk_counters_n;
    // Actual-instance token of the lease (process-unique, never reused).
    uint64_t instance;
    // Fence retirement queue: abandoned fences and the buffers their
    // submissions still reference, released once the fence is terminal.
    struct Retired {
        mf_fence *fence;
        std::vector<mf_buffer *> buffers;
    };
    std::vector<Retired> retired;
};

struct mf_fence {
    mf_backend *backend;
    cudaEvent_t event;
    bool failed;
};

struct mf_readback {
    mf_backend *backend;
    cudaEvent_t event;
    float *host;
    uint64_t length;
    bool failed;
    bool consumed;
};

namespace mf {
// Shared by the executor: device scratch of at least `bytes` (stream-ordered).
int32_t backend_scratch(mf_backend *b, size_t bytes, void **out);
// Host -> device copy into backend scratch at byte offset `offset`.
int32_t backend_stage(mf_backend *b, const void *host, size_t bytes, size_t offset, void **dev);
int32_t check_buffer(const mf_backend *b, const mf_buffer *buf);
// NCCL, loaded on first use (nccl_dyn.cpp): the LM-head row split's
// all-gather of shard candidates.
int32_t nccl_unique_id(uint8_t *out, size_t capacity);
int32_t nccl_comm_init(void **comm, const uint8_t *id_bytes, int rank, int world);
int32_t nccl_all_gather_f32(const float *send, float *recv, size_t count, void *comm, cudaStream_t stream);
void nccl_comm_destroy(void *comm);
// A new backend-owned buffer (accounted in its allocation class).
int32_t backend_alloc_buffer(mf_backend *b, int32_t dtype, const uint64_t *shape, uint32_t rank, int32_t alloc_class,
                             mf_buffer **out);
// Split-K scratch for a packed matmul of t tokens over an [n, k] matrix
// (partials in the stream-ordered scratch, counters zeroed once).
int32_t backend_splitk(mf_backend *b, uint64_t t, uint64_t n, uint64_t k, SplitScratch *out);
// The model releases these buffers when it is destroyed (bundle loader).
void lfm2_adopt_buffers(mf_lfm2 *m, const std::vector<mf_buffer *> &bufs);
// At least `n` zeroed arrival counters (shared by split kernels; every
// launch leaves them zero).
int32_t backend_counters(mf_backend *b, size_t n, unsigned **out);
}  // namespace mf

// C-ABI backend: the InferenceOps mirror (crates/engine-api/src/inference.rs:33-425).
//
// Every entry point validates all operands (ownership, generation, dtype,
// shape, format) before it enqueues anything, mirroring the admission rules
// of the CPU backend (crates/backend-cpu/src/*.rs), then enqueues kernels on
// the backend's stream.  Messages are the reference's where one exists.
#include <atomic>
#include <cuda_runtime.h>
#include <string.h>

#include <algorithm>
#include <vector>
#include <new>

#include "backend_internal.h"
#include "mf_common.cuh"
#include "packed_kernels.h"

namespace mf {

static thread_local const char *t_last_error = "";

void set_error(const char *message) { t_last_error = message ? message : ""; }

int32_t fail(int32_t status, const char *message) {
    set_error(message);
    return status;
}

int32_t cuda_fail(cudaError_t err, const char *where) {
    (void)where;
    set_error(cudaGetErrorString(err));
    return err == cudaErrorMemoryAllocation ? MF_RESOURCE_LIMIT : MF_BACKEND_FAILURE;
}

int sm_count() {
    static thread_local int cached_dev = -1, cached = kSmCount;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return kSmCount;
    if (dev != cached_dev) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) cached = v;
        cached_dev = dev;
    }
    return cached;
}

static uint64_t g_launches = 0;
static std::mutex g_launch_mu;
namespace {
std::atomic<bool> g_pdl{true};
}  // namespace

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed); }

LaunchRecorder *&launch_recorder() {
    static thread_local LaunchRecorder *r = nullptr;
    return r;
}

void count_launch(int64_t n) {
    std::lock_guard<std::mutex> lock(g_launch_mu);
    g_launches += (uint64_t)n;
}
uint64_t launches() {
    std::lock_guard<std::mutex> lock(g_launch_mu);
    return g_launches;
}

int32_t check_buffer(const mf_backend *b, const mf_buffer *buf) {
    if (!b || !buf) return fail(MF_INVALID_ARGUMENT, "null buffer handle");
    if (buf->owner != b || !b->live.count(buf)) return fail(MF_WRONG_BACKEND, "buffer belongs to another backend");
    if (buf->generation != b->generation)
        return fail(MF_STALE_BUFFER, "buffer belongs to an earlier backend generation");
    return MF_OK;
}

int32_t backend_scratch(mf_backend *b, size_t bytes, void **out) {
    if (bytes <= b->scratch_bytes && b->scratch) {
        *out = b->scratch;
        return MF_OK;
    }
    size_t want = std::max<size_t>(bytes, std::max<size_t>(1 << 20, b->scratch_bytes * 2));
    if (b->scratch) MF_CUDA_TRY(cudaFreeAsync(b->scratch, b->stream));
    b->scratch = nullptr;
    b->scratch_bytes = 0;
    MF_CUDA_TRY(cudaMallocAsync(&b->scratch, want, b->stream));
    b->scratch_bytes = want;
    *out = b->scratch;
    return MF_OK;
}

int32_t backend_counters(mf_backend *b, size_t n, unsigned **out) {
    if (n > b->splitk_counters_n) {
        const size_t want = std::max<size_t>(n, std::max<size_t>(4096, 2 * b->splitk_counters_n));
        if (b->splitk_counters) MF_CUDA_TRY(cudaFreeAsync(b->splitk_counters, b->stream));
        b->splitk_counters = nullptr;
        b->splitk_counters_n = 0;
        MF_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void **>(&b->splitk_counters), want * sizeof(unsigned), b->stream));
        MF_CUDA_TRY(cudaMemsetAsync(b->splitk_counters, 0, want * sizeof(unsigned), b->stream));
        b->splitk_counters_n = want;
    }
    *out = b->splitk_counters;
    return MF_OK;
}

int32_t backend_splitk(mf_backend *b, uint64_t t, uint64_t n, uint64_t k, SplitScratch *out) {
    *out = SplitScratch{};
    if (k == 0 || k % 128) return MF_OK;
    if (t >= kGemmMinTokens) {
        // The tensor-core GEMM's BF16 activation planes.
        if (!g_gemm_tc.load(std::memory_order_relaxed)) return MF_OK;
        const size_t floats = packed_gemm_tc_scratch_floats(t, n, k);
        void *planes = nullptr;
        int32_t st = backend_scratch(b, floats * sizeof(float), &planes);
        if (st) return st;
        out->partial = static_cast<float *>(planes);
        out->partial_floats = floats;
        return MF_OK;
    }
    if (!packed_gemv_tc_supports(MF_TERNARY, t)) return MF_OK;
    size_t floats = packed_gemv_tc_scratch_floats(t, n, k);
    // From kNf4GemmMinTokens an NF4 matmul runs the tensor-core GEMM.
    if (t >= kNf4GemmMinTokens && g_gemm_tc.load(std::memory_order_relaxed))
        floats = std::max(floats, packed_gemm_tc_scratch_floats(t, n, k));
    const size_t counters = packed_gemv_tc_counters(t, n);
    int32_t cst = backend_counters(b, counters, &out->counters);
    if (cst) return cst;
    void *partial = nullptr;
    int32_t st = backend_scratch(b, floats * sizeof(float), &partial);
    if (st) return st;
    out->partial = static_cast<float *>(partial);
    out->partial_floats = floats;
    out->counters = b->splitk_counters;
    out->n_counters = b->splitk_counters_n;
    return MF_OK;
}

int32_t backend_stage(mf_backend *b, const void *host, size_t bytes, size_t offset, void **dev) {
    void *base = nullptr;
    int32_t st = backend_scratch(b, offset + bytes, &base);
    if (st) return st;
    *dev = static_cast<char *>(base) + offset;
    if (bytes) {
        MF_CUDA_TRY(cudaMemcpyAsync(*dev, host, bytes, cudaMemcpyHostToDevice, b->stream));
        b->counts.copies++;
    }
    return MF_OK;
}

}  // namespace mf

using namespace mf;

namespace {

constexpr size_t kAlign = 256;

inline size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

int32_t check_f32(const mf_backend *b, const mf_buffer *buf) {
    int32_t st = check_buffer(b, buf);
    if (st) return st;
    if (buf->dtype != MF_DTYPE_F32) return fail(MF_INVALID_DTYPE, "expected an f32 operand");
    return MF_OK;
}

int32_t check_u8(const mf_backend *b, const mf_buffer *buf) {
    int32_t st = check_buffer(b, buf);
    if (st) return st;
    if (buf->dtype != MF_DTYPE_U8) return fail(MF_INVALID_DTYPE, "expected a u8 operand");
    return MF_OK;
}

bool same_shape(const mf_buffer *a, const mf_buffer *b) {
    if (a->rank != b->rank) return false;
    for (uint32_t i = 0; i < a->rank; ++i)
        if (a->shape[i] != b->shape[i]) return false;
    return true;
}

bool has_shape(const mf_buffer *a, std::initializer_list<uint64_t> dims) {
    if (a->rank != dims.size()) return false;
    uint32_t i = 0;
    for (uint64_t d : dims)
        if (a->shape[i++] != d) return false;
    return true;
}

// crates/backend-cpu/src/storage.rs:363-375.
int32_t check_output(const mf_backend *b, const mf_buffer *out, std::initializer_list<uint64_t> dims) {
    int32_t st = check_f32(b, out);
    if (st) return st;
    if (!has_shape(out, dims)) return fail(MF_INVALID_SHAPE, "output layout differs from required contiguous shape");
    return MF_OK;
}

int32_t check_output_like(const mf_backend *b, const mf_buffer *out, const mf_buffer *like) {
    int32_t st = check_f32(b, out);
    if (st) return st;
    if (!same_shape(out, like)) return fail(MF_INVALID_SHAPE, "output layout differs from required contiguous shape");
    return MF_OK;
}

struct PackedInfo {
    uint64_t rows, inner;
    int format;
};

// crates/backend-cpu/src/packed.rs:177-220.
int32_t check_packed_operands(const mf_backend *b, const mf_buffer *codes, const mf_buffer *scales,
                              PackedInfo *info, bool lut2 = false) {
    int32_t st = check_u8(b, codes);
    if (!st) st = check_f32(b, scales);
    if (st) return st;
    if (codes->lut2 && !lut2)
        return fail(MF_INVALID_ARGUMENT, "packed codes are in the LUT2 layout; only the LUT2 ops take them");
    if (lut2 && !codes->lut2)
        return fail(MF_INVALID_ARGUMENT, "LUT2 ops take codes returned by repack_ternary_lut2");
    if (codes->rank != 2 || scales->rank != 2)
        return fail(MF_INVALID_SHAPE, "packed weight streams must be rank two");
    const uint64_t rows = codes->shape[0], code_width = codes->shape[1], groups = scales->shape[1];
    if (groups > UINT64_MAX / 128) return fail(MF_OVERFLOW, "packed inner width overflows usize");
    const uint64_t inner = groups * 128;
    int format;
    if (code_width == inner / 4) {
        format = MF_TERNARY;
    } else if (code_width == inner / 2) {
        format = MF_NF4;
    } else if (code_width == inner) {
        if (codes->has_int8_reserved) return fail(MF_INVALID_ARGUMENT, "INT8 -128 code is reserved");
        format = MF_INT8;
    } else {
        return fail(MF_INVALID_SHAPE,
                    "packed code width must be inner/4 (ternary), inner/2 (nf4), or inner (int8)");
    }
    if (scales->shape[0] != rows) return fail(MF_INVALID_SHAPE, "packed codes and scales disagree on row count");
    if (lut2 && format != MF_TERNARY) return fail(MF_INVALID_DTYPE, "LUT2 ops take ternary code streams");
    info->rows = rows;
    info->inner = inner;
    info->format = format;
    return MF_OK;
}

int32_t alloc_buffer(mf_backend *b, int32_t dtype, const uint64_t *shape, uint32_t rank,
                     int32_t alloc_class, mf_buffer **out) {
    if (!b || !out || (rank && !shape)) return fail(MF_INVALID_ARGUMENT, "null argument");
    if (rank > MF_MAX_RANK) return fail(MF_INVALID_SHAPE, "rank exceeds backend capability");
    if (alloc_class < 0 || alloc_class > 3) return fail(MF_INVALID_ARGUMENT, "unknown allocation class");
    if (b->inject == 2) {
        b->inject = 0;
        return fail(MF_BACKEND_FAILURE, "injected allocation failure");
    }
    uint64_t elements = 1;
    for (uint32_t i = 0; i < rank; ++i) {
        if (shape[i] && elements > UINT64_MAX / shape[i]) return fail(MF_OVERFLOW, "element count overflows u64");
        elements *= shape[i];
    }
    const uint64_t esize = dtype == MF_DTYPE_F32 ? 4 : 1;
    if (elements > UINT64_MAX / esize) return fail(MF_OVERFLOW, "byte length overflows u64");
    const uint64_t bytes = elements * esize;
    if (bytes > b->limits.max_allocation_bytes)
        return fail(MF_RESOURCE_LIMIT, "allocation exceeds configured per-buffer limit");
    if (b->live_total + bytes > b->limits.max_total_bytes)
        return fail(MF_RESOURCE_LIMIT, "allocation exceeds configured total resource limit");
    mf_buffer *buf = new (std::nothrow) mf_buffer();
    if (!buf) return fail(MF_RESOURCE_LIMIT, "host allocation failed");
    buf->owner = b;
    buf->generation = b->generation;
    buf->id = ++b->next_id;
    buf->dtype = dtype;
    buf->rank = rank;
    for (uint32_t i = 0; i < rank; ++i) buf->shape[i] = shape[i];
    buf->elements = elements;
    buf->bytes = bytes;
    buf->alloc_class = alloc_class;
    buf->ptr = nullptr;
    buf->has_int8_reserved = false;
    if (bytes) {
        cudaError_t err = cudaMallocAsync(&buf->ptr, align_up(bytes), b->stream);
        if (err != cudaSuccess) {
            delete buf;
            return cuda_fail(err, "cudaMallocAsync");
        }
    }
    b->live.insert(buf);
    b->live_by_class[alloc_class] += bytes;
    b->live_total += bytes;
    b->peak = std::max(b->peak, b->live_total + b->pending_bytes);
    *out = buf;
    return MF_OK;
}

float *fptr(const mf_buffer *b) { return static_cast<float *>(b->ptr); }
const uint8_t *uptr(const mf_buffer *b) { return static_cast<const uint8_t *>(b->ptr); }

// Resolve a TokenIds argument: host ids (validated, staged to device) or a
// device f32 [T] buffer.
int32_t resolve_ids(mf_backend *b, const uint32_t *host_ids, uint64_t n_ids, const mf_buffer *device_ids,
                    uint64_t rows, const float **ids_f32, const uint32_t **ids_u32, uint64_t *count) {
    *ids_f32 = nullptr;
    *ids_u32 = nullptr;
    if (device_ids) {
        int32_t st = check_f32(b, device_ids);
        if (st) return st;
        if (device_ids->rank != 1) return fail(MF_INVALID_SHAPE, "device token-id buffer must be rank one");
        *ids_f32 = fptr(device_ids);
        *count = device_ids->shape[0];
        return MF_OK;
    }
    if (n_ids && !host_ids) return fail(MF_INVALID_ARGUMENT, "null host ids");
    for (uint64_t i = 0; i < n_ids; ++i)
        if (host_ids[i] >= rows) return fail(MF_OUT_OF_BOUNDS, "gather identifier exceeds row count");
    *count = n_ids;
    return MF_OK;
}

int32_t stage_host_ids(mf_backend *b, const uint32_t *host_ids, uint64_t n_ids, const uint32_t **dev) {
    void *p = nullptr;
    int32_t st = backend_stage(b, host_ids, n_ids * sizeof(uint32_t), 0, &p);
    *dev = static_cast<const uint32_t *>(p);
    return st;
}

}  // namespace

int32_t mf::backend_alloc_buffer(mf_backend *b, int32_t dtype, const uint64_t *shape, uint32_t rank,
                                 int32_t alloc_class, mf_buffer **out) {
    return alloc_buffer(b, dtype, shape, rank, alloc_class, out);
}

// ---------------------------------------------------------------------
// Lifecycle
// ---------------------------------------------------------------------
extern "C" {

int32_t mf_set_pdl(int32_t enabled) {
    g_pdl.store(enabled != 0, std::memory_order_relaxed);
    return MF_OK;
}

int32_t mf_set_gemm_tc(int32_t enabled) {
    mf::g_gemm_tc.store(enabled != 0, std::memory_order_relaxed);
    return MF_OK;
}

int32_t mf_set_attention_tc(int32_t enabled) {
    mf::set_attention_tc(enabled != 0);
    return MF_OK;
}

int32_t mf_set_gemm_passes(int32_t passes) {
    if (passes != 0 && passes != 2 && passes != 3) return fail(MF_INVALID_ARGUMENT, "GEMM passes must be 0, 2 or 3");
    mf::set_gemm_passes(passes);
    return MF_OK;
}

int32_t mf_device_faults(uint32_t *flags) {
    if (!flags) return fail(MF_INVALID_ARGUMENT, "null output");
    uint32_t gemm = 0, attn = 0, step = 0;
    int32_t st = mf::packed_gemm_tc_faults(&gemm);
    if (!st) st = mf::attention_tc_faults(&attn);
    if (!st) st = mf::persistent_faults(&step);
    if (st) return st;
    *flags = (gemm || attn ? 1u : 0u) | (step ? 2u : 0u);
    return MF_OK;
}

int32_t mf_abi_version(void) { return MF_ABI_VERSION; }
const char *mf_last_error(void) { return t_last_error; }

int32_t mf_backend_create(int32_t ordinal, uint64_t owner, const mf_limits *limits, mf_backend **out) {
    if (!out) return fail(MF_INVALID_ARGUMENT, "null output handle");
    int count = 0;
    MF_CUDA_TRY(cudaGetDeviceCount(&count));
    if (ordinal < 0 || ordinal >= count) return fail(MF_INVALID_ARGUMENT, "device ordinal out of range");
    MF_CUDA_TRY(cudaSetDevice(ordinal));
    cudaDeviceProp prop;
    MF_CUDA_TRY(cudaGetDeviceProperties(&prop, ordinal));
    if (prop.major != 10) return fail(MF_UNSUPPORTED, "libmfcuda is built for sm_100a (B200) only");
    mf_backend *b = new (std::nothrow) mf_backend();
    if (!b) return fail(MF_RESOURCE_LIMIT, "host allocation failed");
    b->ordinal = ordinal;
    b->owner = owner;
    b->generation = 1;
    b->limits.max_allocation_bytes = limits ? limits->max_allocation_bytes : UINT64_MAX;
    b->limits.max_total_bytes = limits ? limits->max_total_bytes : UINT64_MAX;
    b->limits.max_pending_operations = limits ? limits->max_pending_operations : UINT32_MAX;
    static std::atomic<uint64_t> g_instances{0};
    b->instance = ++g_instances;
    cudaError_t err = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking);
    if (err != cudaSuccess) {
        delete b;
        return cuda_fail(err, "cudaStreamCreate");
    }
    // Keep freed stream-ordered memory cached in the pool (no OS round trip).
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, ordinal) == cudaSuccess) {
        uint64_t threshold = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
    }
    *out = b;
    return MF_OK;
}

int32_t mf_backend_destroy(mf_backend *b) {
    if (!b) return MF_OK;
    cudaSetDevice(b->ordinal);
    // Retired fences: their buffers are among `live` (freed below).
    for (mf_backend::Retired &r : b->retired) {
        cudaEventSynchronize(r.fence->event);
        cudaEventDestroy(r.fence->event);
        delete r.fence;
    }
    b->retired.clear();
    for (const mf_buffer *buf : b->live) {
        if (buf->ptr) cudaFreeAsync(buf->ptr, b->stream);
        delete buf;
    }
    b->live.clear();
    if (b->scratch) cudaFreeAsync(b->scratch, b->stream);
    if (b->splitk_counters) cudaFreeAsync(b->splitk_counters, b->stream);
    cudaStreamSynchronize(b->stream);
    cudaStreamDestroy(b->stream);
    delete b;
    return MF_OK;
}

int32_t mf_identity_get(const mf_backend *b, mf_identity *out) {
    if (!b || !out) return fail(MF_INVALID_ARGUMENT, "null argument");
    out->kind = 2;  // BackendKind::Cuda
    out->ordinal = (uint32_t)b->ordinal;
    out->owner = b->owner;
    out->generation = b->generation;
    return MF_OK;
}

int32_t mf_capabilities_get(const mf_backend *b, mf_capabilities *out) {
    if (!b || !out) return fail(MF_INVALID_ARGUMENT, "null argument");
    out->dtypes = 0x3;
    // Every OperationKind (backend.rs:75-99) except LmProjection (bit 12),
    // which no executor path issues.
    out->operations = ((1ull << 22) - 1) & ~(1ull << 12);
    out->max_rank = MF_MAX_RANK;
    out->max_elements = 1ull << 40;
    out->max_allocation_bytes = b->limits.max_allocation_bytes;
    out->supports_nonblocking_completion = 1;
    return MF_OK;
}

int32_t mf_resource_report_get(const mf_backend *b, mf_resource_report *out) {
    if (!b || !out) return fail(MF_INVALID_ARGUMENT, "null argument");
    out->resident_weight_bytes = b->live_by_class[MF_CLASS_WEIGHT];
    out->cache_bytes = b->live_by_class[MF_CLASS_CACHE];
    out->scratch_bytes = b->live_by_class[MF_CLASS_SCRATCH] + b->scratch_bytes;
    out->staged_branch_bytes = b->live_by_class[MF_CLASS_BRANCH];
    out->pending_operation_bytes = b->pending_bytes;
    out->pending_operations = b->pending_ops;
    return MF_OK;
}

int32_t mf_peak_accounted_bytes(const mf_backend *b, uint64_t *out) {
    if (!b || !out) return fail(MF_INVALID_ARGUMENT, "null argument");
    *out = b->peak;
    return MF_OK;
}

int32_t mf_advance_generation(mf_backend *b) {
    if (!b) return fail(MF_INVALID_ARGUMENT, "null backend");
    b->generation++;
    return MF_OK;
}

int32_t mf_dispatch_counts_get(const mf_backend *b, mf_dispatch_counts *out) {
    if (!b || !out) return fail(MF_INVALID_ARGUMENT, "null argument");
    *out = b->counts;
    out->kernels = launches();
    return MF_OK;
}

void *mf_backend_stream(const mf_backend *b) { return b ? (void *)b->stream : nullptr; }

int32_t mf_inject_failure(mf_backend *b, int32_t kind) {
    if (!b || kind < 0 || kind > 3) return fail(MF_INVALID_ARGUMENT, "unknown failure kind");
    b->inject = kind;
    return MF_OK;
}

// ---------------------------------------------------------------------
// Buffers
// ---------------------------------------------------------------------
int32_t mf_allocate_f32(mf_backend *b, const uint64_t *shape, uint32_t rank, int32_t alloc_class,
                        int32_t uninit, mf_buffer **out) {
    int32_t st = alloc_buffer(b, MF_DTYPE_F32, shape, rank, alloc_class, out);
    if (st) return st;
    if (!uninit && (*out)->bytes) MF_CUDA_TRY(cudaMemsetAsync((*out)->ptr, 0, (*out)->bytes, b->stream));
    return MF_OK;
}

int32_t mf_upload_f32(mf_backend *b, const uint64_t *shape, uint32_t rank, const float *values,
                      int32_t alloc_class, mf_buffer **out) {
    mf_buffer *buf = nullptr;
    int32_t st = alloc_buffer(b, MF_DTYPE_F32, shape, rank, alloc_class, &buf);
    if (st) return st;
    if (buf->bytes) {
        if (!values) {
            mf_buffer_release(b, buf);
            return fail(MF_INVALID_ARGUMENT, "null upload values");
        }
        MF_CUDA_TRY(cudaMemcpyAsync(buf->ptr, values, buf->bytes, cudaMemcpyHostToDevice, b->stream));
        b->counts.copies++;
    }
    *out = buf;
    return MF_OK;
}

int32_t mf_upload_u8(mf_backend *b, const uint64_t *shape, uint32_t rank, const uint8_t *bytes,
                     int32_t alloc_class, mf_buffer **out) {
    mf_buffer *buf = nullptr;
    int32_t st = alloc_buffer(b, MF_DTYPE_U8, shape, rank, alloc_class, &buf);
    if (st) return st;
    if (buf->bytes) {
        if (!bytes) {
            mf_buffer_release(b, buf);
            return fail(MF_INVALID_ARGUMENT, "null upload bytes");
        }
        buf->has_int8_reserved = memchr(bytes, 0x80, buf->bytes) != nullptr;
        MF_CUDA_TRY(cudaMemcpyAsync(buf->ptr, bytes, buf->bytes, cudaMemcpyHostToDevice, b->stream));
        b->counts.copies++;
    }
    *out = buf;
    return MF_OK;
}

namespace {
bool retired_holds_buffer(const mf_backend *b, const mf_buffer *buf) {
    for (const mf_backend::Retired &r : b->retired)
        for (const mf_buffer *o : r.buffers)
            if (o == buf) return true;
    return false;
}
bool retired_holds_fence(const mf_backend *b, const mf_fence *f) {
    for (const mf_backend::Retired &r : b->retired)
        if (r.fence == f) return true;
    return false;
}
int32_t release_buffer(mf_backend *b, mf_buffer *buf) {
    if (buf->ptr) MF_CUDA_TRY(cudaFreeAsync(buf->ptr, b->stream));
    b->live.erase(buf);
    b->live_by_class[buf->alloc_class] -= buf->bytes;
    b->live_total -= buf->bytes;
    delete buf;
    return MF_OK;
}
void release_fence(mf_fence *f) {
    cudaEventDestroy(f->event);
    if (f->backend->pending_ops) f->backend->pending_ops--;
    delete f;
}
}  // namespace

int32_t mf_buffer_release(mf_backend *b, mf_buffer *buf) {
    if (!b || !buf) return fail(MF_INVALID_ARGUMENT, "null argument");
    if (buf->owner != b || !b->live.count(buf)) return fail(MF_WRONG_BACKEND, "buffer belongs to another backend");
    if (retired_holds_buffer(b, buf)) return fail(MF_INVALID_ARGUMENT, "buffer is retained by a retired fence");
    return release_buffer(b, buf);
}

int32_t mf_buffer_info(const mf_buffer *buf, int32_t *dtype, uint32_t *rank, uint64_t *shape,
                       int32_t *alloc_class) {
    if (!buf) return fail(MF_INVALID_ARGUMENT, "null buffer");
    if (dtype) *dtype = buf->dtype;
    if (rank) *rank = buf->rank;
    if (shape)
        for (uint32_t i = 0; i < buf->rank; ++i) shape[i] = buf->shape[i];
    if (alloc_class) *alloc_class = buf->alloc_class;
    return MF_OK;
}

void *mf_buffer_device_ptr(const mf_buffer *buf) { return buf ? buf->ptr : nullptr; }

// ---------------------------------------------------------------------
// Completions
// ---------------------------------------------------------------------
int32_t mf_fence_submit(mf_backend *b, mf_fence **out) {
    if (!b || !out) return fail(MF_INVALID_ARGUMENT, "null argument");
    if (b->pending_ops >= b->limits.max_pending_operations)
        return fail(MF_RESOURCE_LIMIT, "pending operation count exceeds configured limit");
    mf_fence *f = new (std::nothrow) mf_fence();
    if (!f) return fail(MF_RESOURCE_LIMIT, "host allocation failed");
    f->backend = b;
    f->failed = false;
    if (b->inject == 1) {
        b->inject = 0;
        f->failed = true;
    }
    cudaError_t err = cudaEventCreateWithFlags(&f->event, cudaEventDisableTiming);
    if (err == cudaSuccess) err = cudaEventRecord(f->event, b->stream);
    if (err != cudaSuccess) {
        delete f;
        return cuda_fail(err, "fence");
    }
    b->pending_ops++;
    b->counts.fences++;
    *out = f;
    return MF_OK;
}

int32_t mf_fence_poll(mf_fence *f) {
    if (!f) return fail(MF_INVALID_ARGUMENT, "null fence");
    cudaError_t err = cudaEventQuery(f->event);
    if (err == cudaErrorNotReady) return MF_PENDING;
    if (err != cudaSuccess) return cuda_fail(err, "fence");
    if (f->failed) return fail(MF_BACKEND_FAILURE, "injected fence failure");
    return MF_OK;
}

int32_t mf_fence_release(mf_fence *f) {
    if (!f) return MF_OK;
    if (retired_holds_fence(f->backend, f)) return fail(MF_INVALID_ARGUMENT, "fence is owned by the retirement queue");
    release_fence(f);
    return MF_OK;
}

// crates/engine-api/src/backend.rs:25-62: identity plus an actual-instance
// token that distinguishes backends whose public identity fields collide.
int32_t mf_lease_get(const mf_backend *b, mf_lease *out) {
    if (!b || !out) return fail(MF_INVALID_ARGUMENT, "null argument");
    int32_t st = mf_identity_get(b, &out->identity);
    if (st) return st;
    out->instance = b->instance;
    return MF_OK;
}

// crates/engine-api/src/resources.rs:143-170 (FenceRetirement::retire):
// ownership is checked for the fence and every buffer before anything
// changes; a rejection leaves the whole payload with the caller.
int32_t mf_fence_retire(mf_backend *b, mf_fence *f, mf_buffer *const *retained, uint64_t n_retained) {
    if (!b || !f || (n_retained && !retained)) return fail(MF_INVALID_ARGUMENT, "null argument");
    if (f->backend != b) return fail(MF_WRONG_BACKEND, "fence belongs to another backend");
    for (uint64_t i = 0; i < n_retained; ++i) {
        const mf_buffer *buf = retained[i];
        if (!buf) return fail(MF_INVALID_ARGUMENT, "null retained buffer");
        if (buf->owner != b || !b->live.count(buf)) return fail(MF_WRONG_BACKEND, "retained buffer belongs to another backend");
        if (retired_holds_buffer(b, buf)) return fail(MF_INVALID_ARGUMENT, "buffer is already retained by a retired fence");
        for (uint64_t j = 0; j < i; ++j)
            if (retained[j] == buf) return fail(MF_INVALID_ARGUMENT, "buffer retained twice");
    }
    if (retired_holds_fence(b, f)) return fail(MF_INVALID_ARGUMENT, "fence is already retired");
    try {
        b->retired.push_back(mf_backend::Retired{f, std::vector<mf_buffer *>(retained, retained + n_retained)});
    } catch (...) {
        return fail(MF_RESOURCE_LIMIT, "host allocation failed");
    }
    return MF_OK;
}

// crates/engine-api/src/inference.rs:45-46 and resources.rs:175-176: one
// nonblocking pass; every terminal fence (success or failure) releases its
// buffers and itself.
int32_t mf_poll_retired_fences(mf_backend *b) {
    if (!b) return fail(MF_INVALID_ARGUMENT, "null backend");
    size_t keep = 0;
    for (size_t i = 0; i < b->retired.size(); ++i) {
        mf_backend::Retired &r = b->retired[i];
        const cudaError_t err = cudaEventQuery(r.fence->event);
        if (err == cudaErrorNotReady) {
            if (keep != i) b->retired[keep] = std::move(r);
            ++keep;
            continue;
        }
        for (mf_buffer *buf : r.buffers) release_buffer(b, buf);
        release_fence(r.fence);
    }
    b->retired.resize(keep);
    return MF_OK;
}

// FenceRetirement::has_unresolved (resources.rs:178-184): the number of
// retired fences not yet observed terminal.
int32_t mf_retired_fences_unresolved(const mf_backend *b, uint64_t *count) {
    if (!b || !count) return fail(MF_INVALID_ARGUMENT, "null argument");
    *count = b->retired.size();
    return MF_OK;
}

int32_t mf_read_f32_async(mf_backend *b, const mf_buffer *buf, mf_readback **out) {
    if (!out) return fail(MF_INVALID_ARGUMENT, "null argument");
    int32_t st = check_f32(b, buf);
    if (st) return st;
    if (b->pending_ops >= b->limits.max_pending_operations)
        return fail(MF_RESOURCE_LIMIT, "pending operation count exceeds configured limit");
    mf_readback *r = new (std::nothrow) mf_readback();
    if (!r) return fail(MF_RESOURCE_LIMIT, "host allocation failed");
    r->backend = b;
    r->length = buf->elements;
    r->failed = false;
    r->consumed = false;
    if (b->inject == 3) {
        b->inject = 0;
        r->failed = true;
    }
    r->host = nullptr;
    cudaError_t err = cudaSuccess;
    if (buf->bytes) err = cudaMallocHost(&r->host, buf->bytes);
    if (err == cudaSuccess && buf->bytes)
        err = cudaMemcpyAsync(r->host, buf->ptr, buf->bytes, cudaMemcpyDeviceToHost, b->stream);
    if (err == cudaSuccess) err = cudaEventCreateWithFlags(&r->event, cudaEventDisableTiming);
    if (err == cudaSuccess) err = cudaEventRecord(r->event, b->stream);
    if (err != cudaSuccess) {
        if (r->host) cudaFreeHost(r->host);
        delete r;
        return cuda_fail(err, "readback");
    }
    b->pending_ops++;
    b->pending_bytes += buf->bytes;
    b->peak = std::max(b->peak, b->live_total + b->pending_bytes);
    b->counts.readbacks++;
    b->counts.copies++;
    *out = r;
    return MF_OK;
}

int32_t mf_readback_poll(mf_readback *r, float *out, uint64_t capacity, uint64_t *length) {
    if (!r) return fail(MF_INVALID_ARGUMENT, "null readback");
    if (r->consumed) return fail(MF_COMPLETION_CONSUMED, "completion result was already consumed");
    cudaError_t err = cudaEventQuery(r->event);
    if (err == cudaErrorNotReady) return MF_PENDING;
    if (err != cudaSuccess) return cuda_fail(err, "readback");
    if (r->failed) return fail(MF_BACKEND_FAILURE, "injected readback failure");
    if (length) *length = r->length;
    if (capacity < r->length || (r->length && !out)) return fail(MF_INVALID_ARGUMENT, "readback destination too small");
    if (r->length) memcpy(out, r->host, r->length * sizeof(float));
    r->consumed = true;
    return MF_OK;
}

int32_t mf_readback_release(mf_readback *r) {
    if (!r) return MF_OK;
    cudaEventSynchronize(r->event);
    cudaEventDestroy(r->event);
    if (r->host) cudaFreeHost(r->host);
    mf_backend *b = r->backend;
    if (b->pending_ops) b->pending_ops--;
    b->pending_bytes -= std::min<uint64_t>(b->pending_bytes, r->length * sizeof(float));
    delete r;
    return MF_OK;
}

// ---------------------------------------------------------------------
// Operations
// ---------------------------------------------------------------------
int32_t mf_copy(mf_backend *b, mf_buffer *output, const mf_buffer *input) {
    int32_t st = check_f32(b, input);
    if (!st) st = check_output_like(b, output, input);
    if (st) return st;
    if (input->bytes && output != input)
        MF_CUDA_TRY(cudaMemcpyAsync(output->ptr, input->ptr, input->bytes, cudaMemcpyDeviceToDevice, b->stream));
    b->counts.copies++;
    return MF_OK;
}

// crates/backend-cpu/src/dense.rs:272-341 and backend.rs RectCopy2d::validate.
int32_t mf_copy_rect_2d(mf_backend *b, mf_buffer *output, const mf_buffer *input, const mf_rect_copy_2d *r) {
    int32_t st = check_f32(b, input);
    if (!st) st = check_f32(b, output);
    if (st) return st;
    if (!r) return fail(MF_INVALID_ARGUMENT, "null rectangle");
    if (input == output)
        return fail(MF_UNSUPPORTED, "rectangular copy does not permit overlapping source and destination allocation");
    if (input->rank != 2 || output->rank != 2) return fail(MF_INVALID_SHAPE, "rectangular copy requires rank-two buffers");
    auto fits = [](uint64_t start, uint64_t len, uint64_t dim) { return start <= dim && len <= dim - start; };
    if (!fits(r->source_row, r->rows, input->shape[0]) || !fits(r->source_column, r->columns, input->shape[1]) ||
        !fits(r->destination_row, r->rows, output->shape[0]) ||
        !fits(r->destination_column, r->columns, output->shape[1]))
        return fail(MF_OUT_OF_BOUNDS, "rectangular copy exceeds buffer bounds");
    return copy_rect_2d(fptr(output), output->shape[1], fptr(input), input->shape[1], r->source_row,
                        r->source_column, r->destination_row, r->destination_column, r->rows, r->columns,
                        b->stream);
}

static int32_t argmax_common(mf_backend *b, mf_buffer *output, const mf_buffer *input, const uint64_t *mask,
                             uint64_t mask_words, bool masked) {
    int32_t st = check_f32(b, input);
    if (st) return st;
    if (input->rank != 2) return fail(MF_INVALID_SHAPE, "argmax input must be rank two");
    const uint64_t rows = input->shape[0], width = input->shape[1];
    if (width == 0 || width > (1ull << 24))
        return fail(MF_UNSUPPORTED, "argmax width must be in [1, 2^24] for exact f32 indices");
    if (masked && mask_words != (width + 63) / 64)
        return fail(MF_INVALID_ARGUMENT, "masked argmax mask length must be ceil(width / 64)");
    if (masked && !mask) return fail(MF_INVALID_ARGUMENT, "null mask");
    st = check_output(b, output, {rows});
    if (st) return st;
    // Scratch: [staged mask | per-CTA partials], sized once before staging.
    const size_t mask_bytes = masked ? ((mask_words * sizeof(uint64_t) + 255) & ~size_t(255)) : 0;
    const size_t part_floats = argmax_scratch_floats(rows, width);
    void *base = nullptr;
    st = backend_scratch(b, mask_bytes + part_floats * sizeof(float) + 256, &base);
    if (st) return st;
    const uint64_t *dmask = nullptr;
    if (masked) {
        void *p = nullptr;
        st = backend_stage(b, mask, mask_words * sizeof(uint64_t), 0, &p);
        if (st) return st;
        dmask = static_cast<const uint64_t *>(p);
    }
    SplitScratch ss;
    st = backend_counters(b, rows, &ss.counters);
    if (st) return st;
    ss.n_counters = rows;
    ss.partial = reinterpret_cast<float *>(static_cast<char *>(base) + mask_bytes);
    ss.partial_floats = part_floats;
    return argmax(fptr(output), fptr(input), rows, width, dmask, &ss, b->stream);
}

int32_t mf_argmax(mf_backend *b, mf_buffer *output, const mf_buffer *input) {
    return argmax_common(b, output, input, nullptr, 0, false);
}

int32_t mf_argmax_masked(mf_backend *b, mf_buffer *output, const mf_buffer *input, const uint64_t *mask,
                         uint64_t mask_words) {
    return argmax_common(b, output, input, mask, mask_words, true);
}

int32_t mf_gather_rows(mf_backend *b, mf_buffer *output, const mf_buffer *table, const uint32_t *host_ids,
                       uint64_t n_ids, const mf_buffer *device_ids) {
    int32_t st = check_f32(b, table);
    if (st) return st;
    if (table->rank != 2) return fail(MF_INVALID_SHAPE, "gather table must be rank two");
    const float *idf = nullptr;
    const uint32_t *idu = nullptr;
    uint64_t count = 0;
    st = resolve_ids(b, host_ids, n_ids, device_ids, table->shape[0], &idf, &idu, &count);
    if (!st) st = check_output(b, output, {count, table->shape[1]});
    if (st) return st;
    if (!device_ids) {
        st = stage_host_ids(b, host_ids, count, &idu);
        if (st) return st;
    }
    return gather_rows(fptr(output), fptr(table), table->shape[0], table->shape[1], idf, idu, count, b->stream);
}

int32_t mf_gather_columns(mf_backend *b, mf_buffer *output, const mf_buffer *input, const uint32_t *columns,
                          uint64_t n_columns) {
    int32_t st = check_f32(b, input);
    if (st) return st;
    if (input->rank != 2) return fail(MF_INVALID_SHAPE, "column gather input must be rank two");
    if (n_columns && !columns) return fail(MF_INVALID_ARGUMENT, "null columns");
    for (uint64_t i = 0; i < n_columns; ++i)
        if (columns[i] >= input->shape[1])
            return fail(MF_OUT_OF_BOUNDS, "column gather identifier exceeds input width");
    st = check_output(b, output, {input->shape[0], n_columns});
    if (st) return st;
    const uint32_t *dev = nullptr;
    st = stage_host_ids(b, columns, n_columns, &dev);
    if (st) return st;
    return gather_columns(fptr(output), fptr(input), input->shape[0], input->shape[1], dev, n_columns, b->stream);
}

int32_t mf_packed_gather_rows(mf_backend *b, mf_buffer *output, const mf_buffer *codes, const mf_buffer *scales,
                              const uint32_t *host_ids, uint64_t n_ids, const mf_buffer *device_ids) {
    PackedInfo pi;
    int32_t st = check_packed_operands(b, codes, scales, &pi);
    if (!st) st = check_f32(b, output);
    if (st) return st;
    const float *idf = nullptr;
    const uint32_t *idu = nullptr;
    uint64_t count = 0;
    st = resolve_ids(b, host_ids, n_ids, device_ids, pi.rows, &idf, &idu, &count);
    if (st) return st;
    if (!has_shape(output, {count, pi.inner}))
        return fail(MF_INVALID_SHAPE, "packed gather output layout differs from required shape");
    if (!device_ids) {
        st = stage_host_ids(b, host_ids, count, &idu);
        if (st) return st;
    }
    return packed_gather_rows(fptr(output), uptr(codes), fptr(scales), pi.rows, pi.inner, pi.format, idf, idu,
                              count, b->stream);
}

// crates/backend-cpu/src/packed.rs:96-170.
int32_t mf_packed_linear(mf_backend *b, mf_buffer *output, const mf_buffer *input, const mf_buffer *codes,
                         const mf_buffer *scales) {
    int32_t st = check_f32(b, input);
    if (st) return st;
    PackedInfo pi;
    st = check_packed_operands(b, codes, scales, &pi);
    if (st) return st;
    if (input->rank != 2) return fail(MF_INVALID_SHAPE, "packed linear input must be rank two");
    if (input->shape[1] != pi.inner) return fail(MF_INVALID_SHAPE, "packed linear input width differs from weight width");
    st = check_output(b, output, {input->shape[0], pi.rows});
    if (st) return st;
    SplitScratch ss;
    st = backend_splitk(b, input->shape[0], pi.rows, pi.inner, &ss);
    if (st) return st;
    return packed_matmul(kPackedSingle, false, fptr(output), nullptr, fptr(input), nullptr, nullptr,
                         input->shape[0], uptr(codes), fptr(scales), nullptr, nullptr, pi.rows, pi.inner,
                         pi.format, &ss, b->stream);
}

// packed.rs:222-272.
int32_t mf_packed_linear_pair(mf_backend *b, mf_buffer *out_a, mf_buffer *out_b, const mf_buffer *input,
                              const mf_buffer *codes_a, const mf_buffer *scales_a, const mf_buffer *codes_b,
                              const mf_buffer *scales_b) {
    int32_t st = check_buffer(b, codes_a);
    if (!st) st = check_buffer(b, codes_b);
    if (!st) st = check_buffer(b, scales_a);
    if (!st) st = check_buffer(b, scales_b);
    if (!st) st = check_buffer(b, out_a);
    if (!st) st = check_buffer(b, out_b);
    if (st) return st;
    if (!same_shape(codes_a, codes_b) || !same_shape(scales_a, scales_b) || !same_shape(out_a, out_b))
        return fail(MF_INVALID_SHAPE, "packed linear pair requires equal weight and output shapes");
    st = check_f32(b, input);
    if (st) return st;
    PackedInfo pa, pb;
    st = check_packed_operands(b, codes_a, scales_a, &pa);
    if (!st) st = check_packed_operands(b, codes_b, scales_b, &pb);
    if (st) return st;
    if (input->rank != 2) return fail(MF_INVALID_SHAPE, "packed linear input must be rank two");
    if (input->shape[1] != pa.inner) return fail(MF_INVALID_SHAPE, "packed linear input width differs from weight width");
    st = check_output(b, out_a, {input->shape[0], pa.rows});
    if (!st) st = check_output(b, out_b, {input->shape[0], pa.rows});
    if (st) return st;
    if (out_a == out_b) return fail(MF_INVALID_ARGUMENT, "pair outputs must be distinct buffers");
    SplitScratch ss;
    st = backend_splitk(b, input->shape[0], pa.rows, pa.inner, &ss);
    if (st) return st;
    return packed_matmul(kPackedPairRows, false, fptr(out_a), fptr(out_b), fptr(input), nullptr, nullptr,
                         input->shape[0], uptr(codes_a), fptr(scales_a), uptr(codes_b), fptr(scales_b), pa.rows,
                         pa.inner, pa.format, &ss, b->stream);
}

// packed.rs:377-465.
int32_t mf_packed_swiglu_linear(mf_backend *b, mf_buffer *output, const mf_buffer *gate, const mf_buffer *up,
                                const mf_buffer *codes, const mf_buffer *scales) {
    int32_t st = check_f32(b, gate);
    if (!st) st = check_f32(b, up);
    if (st) return st;
    PackedInfo pi;
    st = check_packed_operands(b, codes, scales, &pi);
    if (st) return st;
    if (gate->rank != 2 || !same_shape(gate, up))
        return fail(MF_INVALID_SHAPE, "packed SwiGLU gate and up layouts must match and be rank two");
    if (gate->shape[1] != pi.inner) return fail(MF_INVALID_SHAPE, "packed SwiGLU input width differs from weight width");
    st = check_output(b, output, {gate->shape[0], pi.rows});
    if (st) return st;
    SplitScratch ss;
    st = backend_splitk(b, gate->shape[0], pi.rows, pi.inner, &ss);
    if (st) return st;
    return packed_matmul(kPackedSingle, true, fptr(output), nullptr, nullptr, fptr(gate), fptr(up),
                         gate->shape[0], uptr(codes), fptr(scales), nullptr, nullptr, pi.rows, pi.inner,
                         pi.format, &ss, b->stream);
}

// packed.rs:278-372.
int32_t mf_packed_swiglu_pair(mf_backend *b, mf_buffer *output, const mf_buffer *input, const mf_buffer *codes_a,
                              const mf_buffer *scales_a, const mf_buffer *codes_b, const mf_buffer *scales_b) {
    int32_t st = check_f32(b, input);
    if (!st) st = check_buffer(b, codes_a);
    if (!st) st = check_buffer(b, codes_b);
    if (!st) st = check_buffer(b, scales_a);
    if (!st) st = check_buffer(b, scales_b);
    if (st) return st;
    if (!same_shape(codes_a, codes_b) || !same_shape(scales_a, scales_b))
        return fail(MF_INVALID_SHAPE, "packed SwiGLU pair requires equal weight shapes");
    PackedInfo pa, pb;
    st = check_packed_operands(b, codes_a, scales_a, &pa);
    if (!st) st = check_packed_operands(b, codes_b, scales_b, &pb);
    if (st) return st;
    if (input->rank != 2) return fail(MF_INVALID_SHAPE, "packed SwiGLU pair input must be rank two");
    if (input->shape[1] != pa.inner)
        return fail(MF_INVALID_SHAPE, "packed SwiGLU pair input width differs from weight width");
    st = check_output(b, output, {input->shape[0], pa.rows});
    if (st) return st;
    SplitScratch ss;
    st = backend_splitk(b, input->shape[0], pa.rows, pa.inner, &ss);
    if (st) return st;
    return packed_matmul(kPackedSwigluPair, false, fptr(output), nullptr, fptr(input), nullptr, nullptr,
                         input->shape[0], uptr(codes_a), fptr(scales_a), uptr(codes_b), fptr(scales_b), pa.rows,
                         pa.inner, pa.format, &ss, b->stream);
}

// inference.rs:253-311.  This backend's LUT2 layout is a lane-tiled
// rearrangement of the ternary bytes (ternary_repack_lanetiled): for each
// 16-row tile and 128-weight group, the 16 bytes one lane of the decode
// GEMV's integer MMA consumes (8 code bytes of each of its two rows) are
// contiguous, and a warp's 32 lanes read one contiguous 512-byte block.  Same
// byte count, lossless; raw streams stay valid for every other op.
int32_t mf_supports_ternary_lut2(const mf_backend *) { return 1; }

int32_t mf_repack_ternary_lut2(mf_backend *b, const mf_buffer *codes, mf_buffer **out) {
    if (!out) return fail(MF_INVALID_ARGUMENT, "null argument");
    int32_t st = check_u8(b, codes);
    if (st) return st;
    if (codes->lut2) return fail(MF_INVALID_ARGUMENT, "codes are already in the LUT2 layout");
    if (codes->rank != 2) return fail(MF_INVALID_SHAPE, "packed weight streams must be rank two");
    // A shape this layout cannot take is a resource limit, which the
    // reference's loader answers by keeping the raw stream for that role
    // (crates/executor-core/src/lfm2/executor/construction.rs:435-440).
    if (codes->shape[0] % 16 || codes->shape[1] % 32)
        return fail(MF_RESOURCE_LIMIT, "LUT2 layout needs rows in multiples of 16 and whole 128-weight groups");
    mf_buffer *buf = nullptr;
    st = alloc_buffer(b, MF_DTYPE_U8, codes->shape, 2, codes->alloc_class, &buf);
    if (st) return st;
    st = ternary_repack_lanetiled(static_cast<uint8_t *>(buf->ptr), static_cast<const uint8_t *>(codes->ptr),
                                  codes->shape[0], codes->shape[1], b->stream);
    if (st) {
        mf_buffer_release(b, buf);
        return st;
    }
    buf->lut2 = true;
    buf->has_int8_reserved = codes->has_int8_reserved;
    *out = buf;
    return MF_OK;
}

// packed_linear over LUT2 codes (inference.rs:283-296): same contract and
// results as mf_packed_linear on the raw stream.
int32_t mf_packed_linear_lut2(mf_backend *b, mf_buffer *output, const mf_buffer *input, const mf_buffer *codes,
                              const mf_buffer *scales) {
    int32_t st = check_f32(b, input);
    if (st) return st;
    PackedInfo pi;
    st = check_packed_operands(b, codes, scales, &pi, true);
    if (st) return st;
    if (input->rank != 2) return fail(MF_INVALID_SHAPE, "packed linear input must be rank two");
    if (input->shape[1] != pi.inner) return fail(MF_INVALID_SHAPE, "packed linear input width differs from weight width");
    st = check_output(b, output, {input->shape[0], pi.rows});
    if (st) return st;
    SplitScratch ss;
    st = backend_splitk(b, input->shape[0], pi.rows, pi.inner, &ss);
    if (st) return st;
    return packed_matmul(kPackedSingle, false, fptr(output), nullptr, fptr(input), nullptr, nullptr,
                         input->shape[0], uptr(codes), fptr(scales), nullptr, nullptr, pi.rows, pi.inner,
                         pi.format, &ss, b->stream, true);
}

// packed_swiglu_pair over LUT2 codes (inference.rs:298-311).
int32_t mf_packed_swiglu_pair_lut2(mf_backend *b, mf_buffer *output, const mf_buffer *input,
                                   const mf_buffer *codes_a, const mf_buffer *scales_a, const mf_buffer *codes_b,
                                   const mf_buffer *scales_b) {
    int32_t st = check_f32(b, input);
    if (!st) st = check_buffer(b, codes_a);
    if (!st) st = check_buffer(b, codes_b);
    if (!st) st = check_buffer(b, scales_a);
    if (!st) st = check_buffer(b, scales_b);
    if (st) return st;
    if (!same_shape(codes_a, codes_b) || !same_shape(scales_a, scales_b))
        return fail(MF_INVALID_SHAPE, "packed SwiGLU pair requires equal weight shapes");
    PackedInfo pa, pb;
    st = check_packed_operands(b, codes_a, scales_a, &pa, true);
    if (!st) st = check_packed_operands(b, codes_b, scales_b, &pb, true);
    if (st) return st;
    if (input->rank != 2) return fail(MF_INVALID_SHAPE, "packed SwiGLU pair input must be rank two");
    if (input->shape[1] != pa.inner)
        return fail(MF_INVALID_SHAPE, "packed SwiGLU pair input width differs from weight width");
    st = check_output(b, output, {input->shape[0], pa.rows});
    if (st) return st;
    SplitScratch ss;
    st = backend_splitk(b, input->shape[0], pa.rows, pa.inner, &ss);
    if (st) return st;
    return packed_matmul(kPackedSwigluPair, false, fptr(output), nullptr, fptr(input), nullptr, nullptr,
                         input->shape[0], uptr(codes_a), fptr(scales_a), uptr(codes_b), fptr(scales_b), pa.rows,
                         pa.inner, pa.format, &ss, b->stream, true);
}

static int32_t check_eps(float eps) {
    if (!(eps > 0.0f) || eps != eps || eps == INFINITY)
        return fail(MF_INVALID_ARGUMENT, "RMS epsilon must be finite and positive");
    return MF_OK;
}

static int32_t rms_common(mf_backend *b, mf_buffer *sum, mf_buffer *normed, const mf_buffer *left,
                          const mf_buffer *right, const mf_buffer *weight, float eps) {
    int32_t st = check_eps(eps);
    if (!st) st = check_f32(b, left);
    if (!st && right) st = check_f32(b, right);
    if (!st) st = check_f32(b, weight);
    if (st) return st;
    if (right && !same_shape(left, right)) return fail(MF_INVALID_SHAPE, "elementwise operands have different layouts");
    if (left->rank != 2 || weight->rank != 1)
        return fail(MF_INVALID_SHAPE, "RMS input must be rank two and weight rank one");
    if (left->shape[1] != weight->shape[0]) return fail(MF_INVALID_SHAPE, "RMS input width differs from weight width");
    if (sum) {
        st = check_output_like(b, sum, left);
        if (st) return st;
    }
    st = check_output_like(b, normed, left);
    if (st) return st;
    if (left->shape[1] > (1ull << 24)) return fail(MF_UNSUPPORTED, "RMS width exceeds exact f32 divisor range");
    if (sum && (sum == normed)) return fail(MF_INVALID_ARGUMENT, "sum and normed outputs must be distinct");
    return row_rms_norm(sum ? fptr(sum) : nullptr, fptr(normed), fptr(left), right ? fptr(right) : nullptr,
                        left->shape[0], left->shape[1], fptr(weight), eps, b->stream);
}

int32_t mf_add_row_rms_norm(mf_backend *b, mf_buffer *sum, mf_buffer *normed, const mf_buffer *left,
                            const mf_buffer *right, const mf_buffer *weight, float epsilon) {
    if (!sum || !right) return fail(MF_INVALID_ARGUMENT, "null argument");
    return rms_common(b, sum, normed, left, right, weight, epsilon);
}

int32_t mf_row_rms_norm(mf_backend *b, mf_buffer *output, const mf_buffer *input, const mf_buffer *weight,
                        float epsilon) {
    return rms_common(b, nullptr, output, input, nullptr, weight, epsilon);
}

// PackedHeadSpec::validate_packed: [tokens, heads * head_dim].
static int32_t check_heads(const mf_buffer *buf, uint32_t heads, uint32_t head_dim, uint64_t *tokens) {
    if (heads == 0 || head_dim == 0)
        return fail(MF_INVALID_ARGUMENT, "head count and head dimension must be nonzero");
    if (buf->rank != 2 || buf->shape[1] != (uint64_t)heads * head_dim)
        return fail(MF_INVALID_SHAPE, "packed head rows must be [tokens, heads * head_dim]");
    *tokens = buf->shape[0];
    return MF_OK;
}

int32_t mf_head_rms_norm(mf_backend *b, mf_buffer *output, const mf_buffer *input, const mf_buffer *weight,
                         uint32_t heads, uint32_t head_dim, float epsilon) {
    int32_t st = check_eps(epsilon);
    if (!st) st = check_f32(b, input);
    if (!st) st = check_f32(b, weight);
    if (st) return st;
    uint64_t tokens = 0;
    st = check_heads(input, heads, head_dim, &tokens);
    if (st) return st;
    if (!has_shape(weight, {head_dim})) return fail(MF_INVALID_SHAPE, "head RMS weight must have head_dim entries");
    st = check_output_like(b, output, input);
    if (st) return st;
    return head_norm_rope(fptr(output), fptr(input), tokens, heads, head_dim, fptr(weight), epsilon, false, nullptr,
                          nullptr, 0.0f, b->stream);
}

static int32_t check_rope(uint32_t head_dim, float theta) {
    if (head_dim % 2) return fail(MF_INVALID_SHAPE, "split-half RoPE requires an even head dimension");
    if (!(theta > 0.0f) || theta == INFINITY) return fail(MF_INVALID_ARGUMENT, "RoPE theta must be finite and positive");
    return MF_OK;
}

int32_t mf_split_half_rotary(mf_backend *b, mf_buffer *output, const mf_buffer *input, const uint64_t *positions,
                             uint64_t n_positions, uint32_t heads, uint32_t head_dim, float theta) {
    int32_t st = check_f32(b, input);
    if (st) return st;
    uint64_t tokens = 0;
    st = check_heads(input, heads, head_dim, &tokens);
    if (!st) st = check_rope(head_dim, theta);
    if (st) return st;
    if (n_positions != tokens) return fail(MF_INVALID_SHAPE, "RoPE position count differs from token count");
    if (n_positions && !positions) return fail(MF_INVALID_ARGUMENT, "null positions");
    st = check_output_like(b, output, input);
    if (st) return st;
    void *dpos = nullptr;
    st = backend_stage(b, positions, n_positions * sizeof(uint64_t), 0, &dpos);
    if (st) return st;
    return head_norm_rope(fptr(output), fptr(input), tokens, heads, head_dim, nullptr, 1.0f, true,
                          static_cast<const uint64_t *>(dpos), nullptr, theta, b->stream);
}

// normalization_rotary.rs:246-369.
int32_t mf_qk_norm_rope(mf_backend *b, mf_buffer *query_out, mf_buffer *key_out, const mf_buffer *query,
                        const mf_buffer *key, const mf_buffer *query_weight, const mf_buffer *key_weight,
                        const uint64_t *positions, uint64_t n_positions, uint32_t query_heads, uint32_t head_dim,
                        float theta, uint32_t key_value_heads, float epsilon) {
    int32_t st = check_rope(head_dim, theta);
    if (!st) st = check_eps(epsilon);
    if (!st) st = check_f32(b, query);
    if (!st) st = check_f32(b, key);
    if (!st) st = check_f32(b, query_weight);
    if (!st) st = check_f32(b, key_weight);
    if (st) return st;
    uint64_t qt = 0, kt = 0;
    st = check_heads(query, query_heads, head_dim, &qt);
    if (!st) st = check_heads(key, key_value_heads, head_dim, &kt);
    if (st) return st;
    if (qt != kt) return fail(MF_INVALID_SHAPE, "RoPE query and key token counts differ");
    if (n_positions != qt) return fail(MF_INVALID_SHAPE, "RoPE position count differs from token count");
    if (n_positions && !positions) return fail(MF_INVALID_ARGUMENT, "null positions");
    st = check_output_like(b, query_out, query);
    if (!st) st = check_output_like(b, key_out, key);
    if (st) return st;
    if (!has_shape(query_weight, {head_dim})) return fail(MF_INVALID_SHAPE, "query");
    if (!has_shape(key_weight, {head_dim})) return fail(MF_INVALID_SHAPE, "key");
    void *dpos = nullptr;
    st = backend_stage(b, positions, n_positions * sizeof(uint64_t), 0, &dpos);
    if (st) return st;
    const uint64_t *pos = static_cast<const uint64_t *>(dpos);
    st = head_norm_rope(fptr(query_out), fptr(query), qt, query_heads, head_dim, fptr(query_weight), epsilon, true,
                        pos, nullptr, theta, b->stream);
    if (st) return st;
    return head_norm_rope(fptr(key_out), fptr(key), kt, key_value_heads, head_dim, fptr(key_weight), epsilon, true,
                          pos, nullptr, theta, b->stream);
}

static int32_t binary(mf_backend *b, mf_buffer *output, const mf_buffer *left, const mf_buffer *right, int op) {
    int32_t st = check_f32(b, left);
    if (!st) st = check_f32(b, right);
    if (st) return st;
    if (!same_shape(left, right))
        return fail(MF_INVALID_SHAPE, op == 2 ? "SwiGLU gate and up layouts differ" : "elementwise operands have different layouts");
    st = check_output_like(b, output, left);
    if (st) return st;
    return elementwise(op, fptr(output), fptr(left), fptr(right), left->elements, b->stream);
}

int32_t mf_add(mf_backend *b, mf_buffer *o, const mf_buffer *l, const mf_buffer *r) { return binary(b, o, l, r, 0); }
int32_t mf_multiply(mf_backend *b, mf_buffer *o, const mf_buffer *l, const mf_buffer *r) { return binary(b, o, l, r, 1); }
int32_t mf_swiglu(mf_backend *b, mf_buffer *o, const mf_buffer *g, const mf_buffer *u) { return binary(b, o, g, u, 2); }

// crates/backend-cpu/src/dense.rs:200-270.
int32_t mf_linear(mf_backend *b, mf_buffer *output, const mf_buffer *input, const mf_buffer *weight) {
    int32_t st = check_f32(b, input);
    if (!st) st = check_f32(b, weight);
    if (st) return st;
    if (input->rank != 2 || weight->rank != 2) return fail(MF_INVALID_SHAPE, "linear input and weight must be rank two");
    if (input->shape[1] != weight->shape[1]) return fail(MF_INVALID_SHAPE, "linear input width differs from weight width");
    st = check_output(b, output, {input->shape[0], weight->shape[0]});
    if (st) return st;
    return dense_linear(fptr(output), fptr(input), input->shape[0], fptr(weight), weight->shape[0], weight->shape[1],
                        b->stream);
}

// crates/backend-cpu/src/attention_convolution.rs:11-187.
int32_t mf_causal_gqa(mf_backend *b, mf_buffer *output, const mf_buffer *query, const mf_buffer *key,
                      const mf_buffer *value, mf_buffer *key_cache, mf_buffer *value_cache, uint64_t *cache_len,
                      uint32_t query_heads, uint32_t key_value_heads, uint32_t head_dim) {
    if (!cache_len) return fail(MF_INVALID_ARGUMENT, "null cache length");
    if (key_value_heads == 0 || query_heads == 0 || query_heads % key_value_heads)
        return fail(MF_INVALID_SHAPE, "query heads must be a nonzero multiple of key/value heads");
    int32_t st = check_f32(b, query);
    if (!st) st = check_f32(b, key);
    if (!st) st = check_f32(b, value);
    if (!st) st = check_f32(b, key_cache);
    if (!st) st = check_f32(b, value_cache);
    if (st) return st;
    if (key_cache == value_cache) return fail(MF_INVALID_ARGUMENT, "key and value caches must have distinct storage");
    uint64_t tokens = 0, kt = 0, vt = 0;
    st = check_heads(query, query_heads, head_dim, &tokens);
    if (!st) st = check_heads(key, key_value_heads, head_dim, &kt);
    if (!st) st = check_heads(value, key_value_heads, head_dim, &vt);
    if (st) return st;
    if (kt != tokens || vt != tokens) return fail(MF_INVALID_SHAPE, "GQA query, key, and value token counts differ");
    st = check_output_like(b, output, query);
    if (st) return st;
    const uint64_t kvw = (uint64_t)key_value_heads * head_dim;
    if (key_cache->rank != 2 || key_cache->shape[1] != kvw || !same_shape(key_cache, value_cache))
        return fail(MF_INVALID_SHAPE, "GQA caches must have matching [capacity, kv_heads * head_dim] shape");
    const uint64_t capacity = key_cache->shape[0];
    if (*cache_len > capacity || tokens > capacity - *cache_len)
        return fail(MF_OUT_OF_BOUNDS, "GQA append exceeds cache capacity");
    const size_t need = causal_gqa_scratch_bytes(tokens, query_heads, key_value_heads, head_dim, *cache_len + tokens);
    void *scratch = nullptr;
    if (need) {
        st = backend_scratch(b, need, &scratch);
        if (st) return st;
    }
    st = causal_gqa(fptr(output), fptr(query), fptr(key), fptr(value), fptr(key_cache), fptr(value_cache), capacity,
                    *cache_len, nullptr, false, tokens, query_heads, key_value_heads, head_dim,
                    static_cast<float *>(scratch), need, b->stream);
    if (st) return st;
    *cache_len += tokens;
    return MF_OK;
}

// crates/backend-cpu/src/attention_convolution.rs:218-340.
int32_t mf_gated_short_convolution(mf_backend *b, mf_buffer *output, const mf_buffer *projection,
                                   const mf_buffer *kernel, mf_buffer *history, uint32_t hidden, uint32_t width) {
    if (hidden == 0 || width == 0)
        return fail(MF_INVALID_ARGUMENT, "short convolution hidden width and kernel width must be nonzero");
    int32_t st = check_f32(b, projection);
    if (!st) st = check_f32(b, kernel);
    if (!st) st = check_f32(b, history);
    if (st) return st;
    if (projection->rank != 2 || projection->shape[1] != 3ull * hidden)
        return fail(MF_INVALID_SHAPE, "short convolution projection must be [tokens, 3 * hidden]");
    const uint64_t tokens = projection->shape[0];
    st = check_output(b, output, {tokens, hidden});
    if (st) return st;
    if (!has_shape(kernel, {hidden, width})) return fail(MF_INVALID_SHAPE, "short convolution kernel must be [hidden, width]");
    if (!has_shape(history, {(uint64_t)width - 1, hidden}))
        return fail(MF_INVALID_SHAPE, "short convolution history must be [width - 1, hidden]");
    return gated_short_conv(fptr(output), fptr(projection), tokens, hidden, fptr(kernel), width, fptr(history),
                            b->stream);
}

// ---------------------------------------------------------------------
// EncoderOps (crates/engine-api/src/encoder.rs:80-103)
// ---------------------------------------------------------------------
// The labels' runs (validated, encoder.rs:16-45), as the kernels take them.
static int32_t segment_ranges(const uint32_t *segment_ids, uint64_t n, std::vector<uint32_t> *ranges) {
    if (n && !segment_ids) return fail(MF_INVALID_ARGUMENT, "null segment labels");
    ranges->assign(2 * n, 0u);
    return encoder_segment_ranges(segment_ids, n, ranges->data());
}

static int32_t stage_ranges(mf_backend *b, const std::vector<uint32_t> &ranges, const uint32_t **dev) {
    void *p = nullptr;
    int32_t st = backend_stage(b, ranges.data(), ranges.size() * sizeof(uint32_t), 0, &p);
    *dev = static_cast<const uint32_t *>(p);
    return st;
}

int32_t mf_bidirectional_gqa(mf_backend *b, mf_buffer *output, const mf_buffer *query, const mf_buffer *key,
                             const mf_buffer *value, const uint32_t *segment_ids, uint64_t n_segments,
                             uint32_t query_heads, uint32_t key_value_heads, uint32_t head_dim) {
    if (key_value_heads == 0 || query_heads == 0 || query_heads % key_value_heads)
        return fail(MF_INVALID_SHAPE, "query heads must be a nonzero multiple of key/value heads");
    std::vector<uint32_t> host_ranges;
    int32_t st = segment_ranges(segment_ids, n_segments, &host_ranges);
    if (st) return st;
    st = check_f32(b, query);
    if (!st) st = check_f32(b, key);
    if (!st) st = check_f32(b, value);
    if (st) return st;
    uint64_t tokens = 0, kt = 0, vt = 0;
    st = check_heads(query, query_heads, head_dim, &tokens);
    if (st) return st;
    if (n_segments != tokens) return fail(MF_INVALID_SHAPE, "encoder segments must match the token count");
    st = check_heads(key, key_value_heads, head_dim, &kt);
    if (!st) st = check_heads(value, key_value_heads, head_dim, &vt);
    if (st) return st;
    if (kt != tokens || vt != tokens) return fail(MF_INVALID_SHAPE, "encoder GQA token counts differ");
    st = check_output_like(b, output, query);
    if (st) return st;
    if (output == query || output == key || output == value)
        return fail(MF_INVALID_ARGUMENT, "encoder GQA output must not alias an input");
    if (tokens == 0) return MF_OK;
    const uint32_t *ranges = nullptr;
    st = stage_ranges(b, host_ranges, &ranges);
    if (st) return st;
    return bidirectional_gqa(fptr(output), fptr(query), fptr(key), fptr(value), ranges, tokens, query_heads,
                             key_value_heads, head_dim, b->stream);
}

int32_t mf_centered_gated_convolution(mf_backend *b, mf_buffer *output, const mf_buffer *projection,
                                      const mf_buffer *kernel, const uint32_t *segment_ids, uint64_t n_segments,
                                      uint32_t hidden, uint32_t width) {
    if (hidden == 0 || width == 0)
        return fail(MF_INVALID_ARGUMENT, "short convolution hidden width and kernel width must be nonzero");
    std::vector<uint32_t> host_ranges;
    int32_t st = segment_ranges(segment_ids, n_segments, &host_ranges);
    if (st) return st;
    st = check_f32(b, projection);
    if (!st) st = check_f32(b, kernel);
    if (st) return st;
    if (projection->rank != 2 || projection->shape[1] != 3ull * hidden)
        return fail(MF_INVALID_SHAPE, "centered convolution projection must be [tokens,3*hidden]");
    const uint64_t tokens = projection->shape[0];
    if (n_segments != tokens) return fail(MF_INVALID_SHAPE, "encoder segments must match the token count");
    st = check_output(b, output, {tokens, hidden});
    if (st) return st;
    if (!has_shape(kernel, {hidden, width})) return fail(MF_INVALID_SHAPE, "centered convolution kernel must be [hidden,width]");
    if (output == projection || output == kernel)
        return fail(MF_INVALID_ARGUMENT, "centered convolution output must not alias an input");
    if (tokens == 0) return MF_OK;
    const uint32_t *ranges = nullptr;
    st = stage_ranges(b, host_ranges, &ranges);
    if (st) return st;
    return centered_gated_conv(fptr(output), fptr(projection), fptr(kernel), ranges, tokens, hidden, width,
                               b->stream);
}

// ---------------------------------------------------------------------
// Raw-pointer tier
// ---------------------------------------------------------------------
static int32_t raw_packed_check(uint64_t k, int32_t format) {
    if (format < MF_TERNARY || format > MF_INT8) return fail(MF_INVALID_ARGUMENT, "unknown packed format");
    if (k % 128) return fail(MF_INVALID_SHAPE, "packed inner width must be a multiple of 128");
    return MF_OK;
}

// The kernels read codes with 128-bit loads and F32 data with 32/128-bit
// loads: code streams must be 16-byte aligned, F32 arrays 16-byte aligned.
static int32_t raw_align_check(std::initializer_list<const void *> ptrs) {
    for (const void *p : ptrs)
        if (p && (reinterpret_cast<uintptr_t>(p) & 15u))
            return fail(MF_INVALID_LAYOUT, "device operands must be 16-byte aligned");
    return MF_OK;
}

int32_t mfk_packed_linear(float *out, const float *x, uint64_t t, const uint8_t *codes, const float *scales,
                          uint64_t n, uint64_t k, int32_t format, void *stream) {
    int32_t st = raw_packed_check(k, format);
    if (st) return st;
    if (t && n && (!out || !x || (k && (!codes || !scales)))) return fail(MF_INVALID_ARGUMENT, "null pointer");
    if ((st = raw_align_check({out, x, codes, scales}))) return st;
    return packed_matmul(kPackedSingle, false, out, nullptr, x, nullptr, nullptr, t, codes, scales, nullptr, nullptr, n,
                         k, format, nullptr, (cudaStream_t)stream);
}

int32_t mfk_repack_ternary_lut2(uint8_t *out, const uint8_t *codes, uint64_t rows, uint64_t row_bytes, void *stream) {
    if (rows && row_bytes && (!out || !codes)) return fail(MF_INVALID_ARGUMENT, "null pointer");
    if (rows % 16 || row_bytes % 32)
        return fail(MF_RESOURCE_LIMIT, "LUT2 layout needs rows in multiples of 16 and whole 128-weight groups");
    if (rows > UINT64_MAX / (row_bytes ? row_bytes : 1)) return fail(MF_OVERFLOW, "byte length overflows u64");
    int32_t st = raw_align_check({out, codes});
    if (st) return st;
    const uint8_t *o = out, *c = codes;
    const uint64_t n = rows * row_bytes;
    if (n && o < c + n && c < o + n) return fail(MF_INVALID_ARGUMENT, "LUT2 repack output overlaps its input");
    return ternary_repack_lanetiled(out, codes, rows, row_bytes, (cudaStream_t)stream);
}

int32_t mfk_packed_linear_pair(float *out_a, float *out_b, const float *x, uint64_t t, const uint8_t *codes_a,
                               const float *scales_a, const uint8_t *codes_b, const float *scales_b, uint64_t n,
                               uint64_t k, int32_t format, void *stream) {
    int32_t st = raw_packed_check(k, format);
    if (st) return st;
    if (t && n && (!out_a || !out_b || !x || (k && (!codes_a || !scales_a || !codes_b || !scales_b))))
        return fail(MF_INVALID_ARGUMENT, "null pointer");
    if ((st = raw_align_check({out_a, out_b, x, codes_a, scales_a, codes_b, scales_b}))) return st;
    return packed_matmul(kPackedPairRows, false, out_a, out_b, x, nullptr, nullptr, t, codes_a, scales_a, codes_b,
                         scales_b, n, k, format, nullptr, (cudaStream_t)stream);
}

int32_t mfk_packed_swiglu_pair(float *out, const float *x, uint64_t t, const uint8_t *codes_a, const float *scales_a,
                               const uint8_t *codes_b, const float *scales_b, uint64_t n, uint64_t k, int32_t format,
                               void *stream) {
    int32_t st = raw_packed_check(k, format);
    if (st) return st;
    if (t && n && (!out || !x || (k && (!codes_a || !scales_a || !codes_b || !scales_b))))
        return fail(MF_INVALID_ARGUMENT, "null pointer");
    if ((st = raw_align_check({out, x, codes_a, scales_a, codes_b, scales_b}))) return st;
    return packed_matmul(kPackedSwigluPair, false, out, nullptr, x, nullptr, nullptr, t, codes_a, scales_a, codes_b,
                         scales_b, n, k, format, nullptr, (cudaStream_t)stream);
}

int32_t mfk_packed_swiglu_linear(float *out, const float *gate, const float *up, uint64_t t, const uint8_t *codes,
                                 const float *scales, uint64_t n, uint64_t k, int32_t format, void *stream) {
    int32_t st = raw_packed_check(k, format);
    if (st) return st;
    if (t && n && (!out || !gate || !up || (k && (!codes || !scales)))) return fail(MF_INVALID_ARGUMENT, "null pointer");
    if ((st = raw_align_check({out, gate, up, codes, scales}))) return st;
    return packed_matmul(kPackedSingle, true, out, nullptr, nullptr, gate, up, t, codes, scales, nullptr, nullptr, n, k,
                         format, nullptr, (cudaStream_t)stream);
}

int32_t mfk_packed_gather_rows(float *out, const uint8_t *codes, const float *scales, uint64_t rows, uint64_t k,
                               int32_t format, const float *ids, uint64_t n_ids, void *stream) {
    int32_t st = raw_packed_check(k, format);
    if (st) return st;
    if (n_ids && k && (!out || !codes || !scales || !ids)) return fail(MF_INVALID_ARGUMENT, "null pointer");
    if ((st = raw_align_check({out, codes, scales, ids}))) return st;
    return packed_gather_rows(out, codes, scales, rows, k, format, ids, nullptr, n_ids, (cudaStream_t)stream);
}

int32_t mfk_argmax(float *out, const float *logits, uint64_t rows, uint64_t width, void *stream) {
    if (width == 0 || width > (1ull << 24))
        return fail(MF_UNSUPPORTED, "argmax width must be in [1, 2^24] for exact f32 indices");
    if (rows && (!out || !logits)) return fail(MF_INVALID_ARGUMENT, "null pointer");
    return argmax(out, logits, rows, width, nullptr, nullptr, (cudaStream_t)stream);
}

int32_t mfk_encoder_segment_ranges(const uint32_t *segment_ids, uint64_t tokens, uint32_t *ranges) {
    if (tokens && (!segment_ids || !ranges)) return fail(MF_INVALID_ARGUMENT, "null pointer");
    return encoder_segment_ranges(segment_ids, tokens, ranges);
}

int32_t mfk_bidirectional_gqa(float *out, const float *q, const float *k, const float *v, const uint32_t *ranges,
                              uint64_t tokens, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                              void *stream) {
    if (tokens && (!out || !q || !k || !v || !ranges)) return fail(MF_INVALID_ARGUMENT, "null device pointer");
    int32_t st = raw_align_check({out, q, k, v});
    if (st) return st;
    return bidirectional_gqa(out, q, k, v, ranges, tokens, q_heads, kv_heads, head_dim, (cudaStream_t)stream);
}

int32_t mfk_centered_gated_convolution(float *out, const float *projection, const float *kernel,
                                       const uint32_t *ranges, uint64_t tokens, uint32_t hidden, uint32_t width,
                                       void *stream) {
    if (tokens && (!out || !projection || !kernel || !ranges)) return fail(MF_INVALID_ARGUMENT, "null device pointer");
    return centered_gated_conv(out, projection, kernel, ranges, tokens, hidden, width, (cudaStream_t)stream);
}

}  // extern "C"

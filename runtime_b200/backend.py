"""Python mirror of the reference's ``InferenceOps`` contract over libmfcuda.

Method names, argument order and meaning, and error kinds follow
crates/engine-api/src/inference.rs:33-425 so that tests read like the
reference's own.  Every method calls straight into the C ABI; nothing here
computes.  Errors raise :class:`ExecutorError` with the variant name of
crates/engine-api/src/error.rs:10-28 in ``.kind``.
"""
from __future__ import annotations

import ctypes as C
import time
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import P, U64

KINDS = {
    1: "InvalidArgument", 2: "InvalidShape", 3: "InvalidLayout", 4: "InvalidDType", 5: "Overflow",
    6: "OutOfBounds", 7: "Unsupported", 8: "ResourceLimit", 9: "WrongBackend", 10: "StaleBuffer",
    11: "DuplicateName", 12: "MissingRequiredTensor", 13: "UnexpectedTensor", 14: "InvalidTie",
    15: "Cancelled", 16: "CompletionConsumed", 17: "BackendFailure",
}
PENDING = 100
F32, U8 = 0, 1
WEIGHT, CACHE, SCRATCH, BRANCH = 0, 1, 2, 3


class ExecutorError(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = status
        self.kind = KINDS.get(status, f"status {status}")
        self.message = message
        super().__init__(f"{self.kind}: {message}")


def _check(status: int):
    if status != 0:
        raise ExecutorError(status, (_lib.load().mf_last_error() or b"").decode())


def _shape_arr(shape):
    shape = tuple(int(d) for d in shape)
    arr = (U64 * max(1, len(shape)))(*shape)
    return arr, len(shape)


class CudaBuffer:
    """A backend-owned device buffer handle (BufferDescriptor analogue)."""

    def __init__(self, backend: "CudaBackend", handle: int, shape, dtype: int, cls: int):
        self.backend = backend
        self.handle = handle
        self.shape = tuple(int(d) for d in shape)
        self.dtype = dtype
        self.alloc_class = cls

    @property
    def ptr(self) -> int:
        return _lib.load().mf_buffer_device_ptr(self.handle) or 0

    def release(self):
        if self.handle and self.backend.handle:
            _check(_lib.load().mf_buffer_release(self.backend.handle, self.handle))
        self.handle = None

    def __repr__(self):
        return f"CudaBuffer(shape={self.shape}, dtype={'f32' if self.dtype == F32 else 'u8'})"


def _h(buf):
    return None if buf is None else buf.handle


class Completion:
    """Pollable fence / readback (crates/engine-api/src/resources.rs:89-99)."""

    def __init__(self, handle, kind: str, length: int = 0, shape=None):
        self.handle = handle
        self.kind = kind
        self.length = length
        self.shape = shape

    def poll(self):
        """None while pending; () for a fence, np.ndarray for a readback."""
        L = _lib.load()
        if self.kind == "fence":
            st = L.mf_fence_poll(self.handle)
            if st == PENDING:
                return None
            _check(st)
            return ()
        out = np.empty(max(1, self.length), np.float32)
        n = U64(0)
        st = L.mf_readback_poll(self.handle, out.ctypes.data, out.size, C.byref(n))
        if st == PENDING:
            return None
        _check(st)
        return out[: n.value].reshape(self.shape)

    def wait(self, timeout_s: float = 120.0):
        deadline = time.monotonic() + timeout_s
        while True:
            r = self.poll()
            if r is not None:
                return r
            if time.monotonic() > deadline:
                raise TimeoutError(f"{self.kind} did not complete in {timeout_s}s")
            time.sleep(0)

    def release(self):
        if self.handle:
            L = _lib.load()
            (L.mf_fence_release if self.kind == "fence" else L.mf_readback_release)(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


@dataclass
class Identity:
    kind: int
    ordinal: int
    owner: int
    generation: int


class CudaBackend:
    """One device backend (InferenceOps implementor) on CUDA device `ordinal`."""

    def __init__(self, ordinal: int = 0, owner: int = 0, limits: dict | None = None):
        L = _lib.load()
        lim = None
        if limits:
            lim = _lib.Limits(limits.get("max_allocation_bytes", 2**64 - 1),
                              limits.get("max_total_bytes", 2**64 - 1),
                              limits.get("max_pending_operations", 2**32 - 1))
        h = P()
        _check(L.mf_backend_create(ordinal, owner, C.byref(lim) if lim else None, C.byref(h)))
        self.handle = h.value
        self.ordinal = ordinal

    def close(self):
        if self.handle:
            _lib.load().mf_backend_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- identity, accounting --------------------------------------------
    def identity(self) -> Identity:
        out = _lib.Identity()
        _check(_lib.load().mf_identity_get(self.handle, C.byref(out)))
        return Identity(out.kind, out.ordinal, out.owner, out.generation)

    def lease(self) -> tuple[Identity, int]:
        """(identity, actual-instance token): crates/engine-api/src/backend.rs:25-62."""
        out = _lib.Lease()
        _check(_lib.load().mf_lease_get(self.handle, C.byref(out)))
        i = out.identity
        return Identity(i.kind, i.ordinal, i.owner, i.generation), out.instance

    def retire_fence(self, fence: "Completion", retained=()):
        """FenceRetirement::retire (crates/engine-api/src/resources.rs:143-170):
        on success the backend owns the fence and the buffers; a rejection
        raises before anything changes and the caller keeps them."""
        arr = (P * max(1, len(retained)))(*[b.handle for b in retained])
        _check(_lib.load().mf_fence_retire(self.handle, fence.handle, arr, len(retained)))
        fence.handle = None
        for b in retained:
            b.handle = None

    def poll_retired_fences(self):
        _check(_lib.load().mf_poll_retired_fences(self.handle))

    def retired_fences_unresolved(self) -> int:
        v = U64()
        _check(_lib.load().mf_retired_fences_unresolved(self.handle, C.byref(v)))
        return v.value

    def capabilities(self) -> _lib.Capabilities:
        out = _lib.Capabilities()
        _check(_lib.load().mf_capabilities_get(self.handle, C.byref(out)))
        return out

    def resource_report(self) -> dict:
        out = _lib.ResourceReport()
        _check(_lib.load().mf_resource_report_get(self.handle, C.byref(out)))
        return {f: getattr(out, f) for f, _ in out._fields_}

    def peak_accounted_bytes(self) -> int:
        v = U64()
        _check(_lib.load().mf_peak_accounted_bytes(self.handle, C.byref(v)))
        return v.value

    def advance_generation(self):
        _check(_lib.load().mf_advance_generation(self.handle))

    def dispatch_counts(self) -> dict:
        out = _lib.DispatchCounts()
        _check(_lib.load().mf_dispatch_counts_get(self.handle, C.byref(out)))
        return {f: getattr(out, f) for f, _ in out._fields_}

    def inject_failure(self, kind: str):
        _check(_lib.load().mf_inject_failure(self.handle, {"fence": 1, "allocation": 2,
                                                           "readback": 3}[kind]))

    @property
    def stream(self) -> int:
        return _lib.load().mf_backend_stream(self.handle)

    # ---- buffers -----------------------------------------------------------
    def allocate_f32_classified(self, shape, cls: int = SCRATCH, uninit: bool = False) -> CudaBuffer:
        arr, rank = _shape_arr(shape)
        h = P()
        _check(_lib.load().mf_allocate_f32(self.handle, arr, rank, cls, int(uninit), C.byref(h)))
        return CudaBuffer(self, h.value, shape, F32, cls)

    def allocate_f32(self, shape) -> CudaBuffer:
        return self.allocate_f32_classified(shape, SCRATCH)

    def upload_f32_classified(self, shape, values, cls: int = SCRATCH) -> CudaBuffer:
        v = np.ascontiguousarray(values, dtype=np.float32)
        arr, rank = _shape_arr(shape)
        h = P()
        _check(_lib.load().mf_upload_f32(self.handle, arr, rank, v.ctypes.data if v.size else None,
                                         cls, C.byref(h)))
        return CudaBuffer(self, h.value, shape, F32, cls)

    def upload_f32(self, values, shape=None, cls: int = SCRATCH) -> CudaBuffer:
        v = np.ascontiguousarray(values, dtype=np.float32)
        return self.upload_f32_classified(v.shape if shape is None else shape, v, cls)

    def upload_u8_classified(self, shape, values, cls: int = WEIGHT) -> CudaBuffer:
        v = np.ascontiguousarray(values, dtype=np.uint8)
        arr, rank = _shape_arr(shape)
        h = P()
        _check(_lib.load().mf_upload_u8(self.handle, arr, rank, v.ctypes.data if v.size else None,
                                        cls, C.byref(h)))
        return CudaBuffer(self, h.value, shape, U8, cls)

    def upload_u8(self, values, shape=None, cls: int = WEIGHT) -> CudaBuffer:
        v = np.ascontiguousarray(values, dtype=np.uint8)
        return self.upload_u8_classified(v.shape if shape is None else shape, v, cls)

    # ---- completions -------------------------------------------------------
    def fence(self) -> Completion:
        h = P()
        _check(_lib.load().mf_fence_submit(self.handle, C.byref(h)))
        return Completion(h.value, "fence")

    def read_f32_async(self, buf: CudaBuffer) -> Completion:
        h = P()
        _check(_lib.load().mf_read_f32_async(self.handle, _h(buf), C.byref(h)))
        return Completion(h.value, "readback", int(np.prod(buf.shape)) if buf.shape else 1, buf.shape)

    def read_f32(self, buf: CudaBuffer) -> np.ndarray:
        c = self.read_f32_async(buf)
        try:
            return c.wait()
        finally:
            c.release()

    # ---- operations (inference.rs:113-425) --------------------------------
    def copy(self, output, input):
        _check(_lib.load().mf_copy(self.handle, _h(output), _h(input)))

    def copy_rect_2d(self, output, input, rect):
        r = _lib.RectCopy2d(*[int(v) for v in rect])
        _check(_lib.load().mf_copy_rect_2d(self.handle, _h(output), _h(input), C.byref(r)))

    def argmax(self, output, input):
        _check(_lib.load().mf_argmax(self.handle, _h(output), _h(input)))

    def argmax_masked(self, output, input, mask):
        m = np.ascontiguousarray(mask, dtype=np.uint64)
        _check(_lib.load().mf_argmax_masked(self.handle, _h(output), _h(input),
                                            m.ctypes.data if m.size else None, m.size))

    @staticmethod
    def _ids(ids):
        """TokenIds: a sequence of host u32 ids, or a CudaBuffer of device f32 ids."""
        if isinstance(ids, CudaBuffer):
            return None, 0, ids.handle, None
        a = np.ascontiguousarray(ids, dtype=np.uint32)
        return (a.ctypes.data if a.size else None), a.size, None, a

    def gather_rows(self, output, table, ids):
        hp, n, dev, keep = self._ids(ids)
        _check(_lib.load().mf_gather_rows(self.handle, _h(output), _h(table), hp, n, dev))

    def gather_columns(self, output, input, columns):
        a = np.ascontiguousarray(columns, dtype=np.uint32)
        _check(_lib.load().mf_gather_columns(self.handle, _h(output), _h(input),
                                             a.ctypes.data if a.size else None, a.size))

    def packed_gather_rows(self, output, codes, scales, ids):
        hp, n, dev, keep = self._ids(ids)
        _check(_lib.load().mf_packed_gather_rows(self.handle, _h(output), _h(codes), _h(scales),
                                                 hp, n, dev))

    def packed_linear(self, output, input, codes, scales):
        _check(_lib.load().mf_packed_linear(self.handle, _h(output), _h(input), _h(codes), _h(scales)))

    def packed_linear_pair(self, out_a, out_b, input, codes_a, scales_a, codes_b, scales_b):
        _check(_lib.load().mf_packed_linear_pair(self.handle, _h(out_a), _h(out_b), _h(input),
                                                 _h(codes_a), _h(scales_a), _h(codes_b),
                                                 _h(scales_b)))

    def packed_swiglu_linear(self, output, gate, up, codes, scales):
        _check(_lib.load().mf_packed_swiglu_linear(self.handle, _h(output), _h(gate), _h(up),
                                                   _h(codes), _h(scales)))

    def packed_swiglu_pair(self, output, input, codes_a, scales_a, codes_b, scales_b):
        _check(_lib.load().mf_packed_swiglu_pair(self.handle, _h(output), _h(input), _h(codes_a),
                                                 _h(scales_a), _h(codes_b), _h(scales_b)))

    def supports_ternary_lut2(self) -> bool:
        return bool(_lib.load().mf_supports_ternary_lut2(self.handle))

    def repack_ternary_lut2(self, codes) -> CudaBuffer:
        """The backend's LUT2 layout of a ternary code stream (a new buffer,
        same shape and allocation class; only the *_lut2 ops take it)."""
        h = P()
        _check(_lib.load().mf_repack_ternary_lut2(self.handle, _h(codes), C.byref(h)))
        return CudaBuffer(self, h.value, codes.shape, U8, codes.alloc_class)

    def packed_linear_lut2(self, output, input, codes, scales):
        _check(_lib.load().mf_packed_linear_lut2(self.handle, _h(output), _h(input), _h(codes), _h(scales)))

    def packed_swiglu_pair_lut2(self, output, input, codes_a, scales_a, codes_b, scales_b):
        _check(_lib.load().mf_packed_swiglu_pair_lut2(self.handle, _h(output), _h(input), _h(codes_a),
                                                      _h(scales_a), _h(codes_b), _h(scales_b)))

    def add_row_rms_norm(self, sum, normed, left, right, weight, epsilon):
        _check(_lib.load().mf_add_row_rms_norm(self.handle, _h(sum), _h(normed), _h(left), _h(right),
                                               _h(weight), epsilon))

    def qk_norm_rope(self, query_out, key_out, query, key, query_weight, key_weight, positions,
                     rope, key_value_heads, epsilon):
        """rope = (query_heads, head_dim, theta); key_value_heads = (heads, head_dim)."""
        pos = np.ascontiguousarray(positions, dtype=np.uint64)
        qh, hd, theta = rope
        _check(_lib.load().mf_qk_norm_rope(self.handle, _h(query_out), _h(key_out), _h(query),
                                           _h(key), _h(query_weight), _h(key_weight),
                                           pos.ctypes.data if pos.size else None, pos.size, qh, hd,
                                           theta, key_value_heads[0], epsilon))

    def add(self, output, left, right):
        _check(_lib.load().mf_add(self.handle, _h(output), _h(left), _h(right)))

    def multiply(self, output, left, right):
        _check(_lib.load().mf_multiply(self.handle, _h(output), _h(left), _h(right)))

    def linear(self, output, input, weight):
        _check(_lib.load().mf_linear(self.handle, _h(output), _h(input), _h(weight)))

    def row_rms_norm(self, output, input, weight, epsilon):
        _check(_lib.load().mf_row_rms_norm(self.handle, _h(output), _h(input), _h(weight), epsilon))

    def head_rms_norm(self, output, input, weight, heads, epsilon):
        """heads = (heads, head_dim)."""
        _check(_lib.load().mf_head_rms_norm(self.handle, _h(output), _h(input), _h(weight),
                                            heads[0], heads[1], epsilon))

    def split_half_rotary(self, output, input, positions, spec):
        """spec = (heads, head_dim, theta)."""
        pos = np.ascontiguousarray(positions, dtype=np.uint64)
        _check(_lib.load().mf_split_half_rotary(self.handle, _h(output), _h(input),
                                                pos.ctypes.data if pos.size else None, pos.size,
                                                spec[0], spec[1], spec[2]))

    def causal_gqa(self, output, query, key, value, key_cache, value_cache, cache_len: int, spec):
        """spec = (query_heads, kv_heads, head_dim).  Returns the new cache length."""
        n = U64(cache_len)
        _check(_lib.load().mf_causal_gqa(self.handle, _h(output), _h(query), _h(key), _h(value),
                                         _h(key_cache), _h(value_cache), C.byref(n), spec[0],
                                         spec[1], spec[2]))
        return n.value

    def gated_short_convolution(self, output, projection, kernel, history, spec):
        """spec = (hidden, width)."""
        _check(_lib.load().mf_gated_short_convolution(self.handle, _h(output), _h(projection),
                                                      _h(kernel), _h(history), spec[0], spec[1]))

    # EncoderOps (crates/engine-api/src/encoder.rs:80-103).  `segments`:
    # one label per token, every nonzero label on one contiguous run, 0 = padding.
    def bidirectional_gqa(self, output, query, key, value, segments, spec):
        """spec = (query_heads, kv_heads, head_dim); noncausal attention within
        each token's segment, zero rows for padding."""
        ids = np.ascontiguousarray(segments, np.uint32)
        _check(_lib.load().mf_bidirectional_gqa(self.handle, _h(output), _h(query), _h(key), _h(value),
                                                ids.ctypes.data if ids.size else None, ids.size,
                                                spec[0], spec[1], spec[2]))

    def centered_gated_convolution(self, output, projection, kernel, segments, spec):
        """spec = (hidden, width); C[t] * sum_j kernel[j] * (B*V)[t + j - width/2]
        within each token's segment, zero rows for padding."""
        ids = np.ascontiguousarray(segments, np.uint32)
        _check(_lib.load().mf_centered_gated_convolution(self.handle, _h(output), _h(projection), _h(kernel),
                                                         ids.ctypes.data if ids.size else None, ids.size,
                                                         spec[0], spec[1]))

    def swiglu(self, output, gate, up):
        _check(_lib.load().mf_swiglu(self.handle, _h(output), _h(gate), _h(up)))

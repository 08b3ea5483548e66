"""Loader for libmfcuda.so and its C signatures.

The library is built in-tree (``python -m runtime_b200.build``).  There is no
fallback: if the shared library is missing or fails to load, every entry
point raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmfcuda.so")

P = C.c_void_p
I32 = C.c_int32
U32 = C.c_uint32
U64 = C.c_uint64
F32 = C.c_float
PU64 = C.POINTER(U64)
PU32 = C.POINTER(U32)
PF32 = C.POINTER(F32)


class Limits(C.Structure):
    _fields_ = [("max_allocation_bytes", U64), ("max_total_bytes", U64),
                ("max_pending_operations", U32)]


class Identity(C.Structure):
    _fields_ = [("kind", U32), ("ordinal", U32), ("owner", U64), ("generation", U64)]


class Lease(C.Structure):
    _fields_ = [("identity", Identity), ("instance", U64)]


class ResourceReport(C.Structure):
    _fields_ = [("resident_weight_bytes", U64), ("cache_bytes", U64), ("scratch_bytes", U64),
                ("staged_branch_bytes", U64), ("pending_operation_bytes", U64),
                ("pending_operations", U32)]


class Capabilities(C.Structure):
    _fields_ = [("dtypes", U32), ("operations", U64), ("max_rank", U32), ("max_elements", U64),
                ("max_allocation_bytes", U64), ("supports_nonblocking_completion", I32)]


class RectCopy2d(C.Structure):
    _fields_ = [("source_row", U64), ("source_column", U64), ("destination_row", U64),
                ("destination_column", U64), ("rows", U64), ("columns", U64)]


class DispatchCounts(C.Structure):
    _fields_ = [("kernels", U64), ("copies", U64), ("fences", U64), ("readbacks", U64)]


class Lfm2Config(C.Structure):
    _fields_ = [("hidden", U32), ("intermediate", U32), ("q_heads", U32), ("kv_heads", U32),
                ("head_dim", U32), ("conv_width", U32), ("vocab", U32), ("n_layers", U32),
                ("layer_kinds", P), ("rope_theta", F32), ("block_eps", F32), ("norm_eps", F32),
                ("max_tokens", U64)]


class OpProfile(C.Structure):
    _fields_ = [("launches", U64), ("bytes", U64), ("ms", C.c_double), ("ops", U64)]


OP_CLASSES = ("packed_matmul", "dense_matmul", "attention", "conv", "norm_rope", "gather",
              "argmax", "other")


class Lfm2Weight(C.Structure):
    _fields_ = [("dense", P), ("codes", P), ("scales", P)]


class Lfm2Layer(C.Structure):
    _fields_ = [("in_proj", Lfm2Weight), ("out_proj", Lfm2Weight), ("conv_kernel", P),
                ("q", Lfm2Weight), ("k", Lfm2Weight), ("v", Lfm2Weight), ("o", Lfm2Weight),
                ("q_norm", P), ("k_norm", P),
                ("w1", Lfm2Weight), ("w2", Lfm2Weight), ("w3", Lfm2Weight),
                ("ffn_norm", P), ("operator_norm", P)]


# name -> (restype, argtypes)
SIGNATURES = {
    "mf_abi_version": (I32, []),
    "mf_set_pdl": (I32, [I32]),
    "mf_set_gemm_tc": (I32, [I32]),
    "mf_set_gemm_passes": (I32, [I32]),
    "mf_set_attention_tc": (I32, [I32]),
    "mf_device_faults": (I32, [C.POINTER(C.c_uint32)]),
    "mf_last_error": (C.c_char_p, []),
    "mf_backend_create": (I32, [I32, U64, P, C.POINTER(P)]),
    "mf_backend_destroy": (I32, [P]),
    "mf_identity_get": (I32, [P, P]),
    "mf_capabilities_get": (I32, [P, P]),
    "mf_resource_report_get": (I32, [P, P]),
    "mf_peak_accounted_bytes": (I32, [P, PU64]),
    "mf_advance_generation": (I32, [P]),
    "mf_dispatch_counts_get": (I32, [P, P]),
    "mf_backend_stream": (P, [P]),
    "mf_inject_failure": (I32, [P, I32]),
    "mf_allocate_f32": (I32, [P, PU64, U32, I32, I32, C.POINTER(P)]),
    "mf_upload_f32": (I32, [P, PU64, U32, P, I32, C.POINTER(P)]),
    "mf_upload_u8": (I32, [P, PU64, U32, P, I32, C.POINTER(P)]),
    "mf_buffer_release": (I32, [P, P]),
    "mf_buffer_info": (I32, [P, C.POINTER(I32), C.POINTER(U32), PU64, C.POINTER(I32)]),
    "mf_buffer_device_ptr": (P, [P]),
    "mf_fence_submit": (I32, [P, C.POINTER(P)]),
    "mf_fence_poll": (I32, [P]),
    "mf_fence_release": (I32, [P]),
    "mf_lease_get": (I32, [P, P]),
    "mf_fence_retire": (I32, [P, P, C.POINTER(P), U64]),
    "mf_poll_retired_fences": (I32, [P]),
    "mf_retired_fences_unresolved": (I32, [P, PU64]),
    "mf_read_f32_async": (I32, [P, P, C.POINTER(P)]),
    "mf_readback_poll": (I32, [P, P, U64, PU64]),
    "mf_readback_release": (I32, [P]),
    "mf_copy": (I32, [P, P, P]),
    "mf_copy_rect_2d": (I32, [P, P, P, C.POINTER(RectCopy2d)]),
    "mf_argmax": (I32, [P, P, P]),
    "mf_argmax_masked": (I32, [P, P, P, P, U64]),
    "mf_gather_rows": (I32, [P, P, P, P, U64, P]),
    "mf_gather_columns": (I32, [P, P, P, P, U64]),
    "mf_packed_gather_rows": (I32, [P, P, P, P, P, U64, P]),
    "mf_packed_linear": (I32, [P, P, P, P, P]),
    "mf_packed_linear_pair": (I32, [P, P, P, P, P, P, P, P]),
    "mf_packed_swiglu_linear": (I32, [P, P, P, P, P, P]),
    "mf_packed_swiglu_pair": (I32, [P, P, P, P, P, P, P]),
    "mf_supports_ternary_lut2": (I32, [P]),
    "mf_repack_ternary_lut2": (I32, [P, P, C.POINTER(P)]),
    "mf_packed_linear_lut2": (I32, [P, P, P, P, P]),
    "mf_packed_swiglu_pair_lut2": (I32, [P, P, P, P, P, P, P]),
    "mf_add_row_rms_norm": (I32, [P, P, P, P, P, P, F32]),
    "mf_qk_norm_rope": (I32, [P, P, P, P, P, P, P, P, U64, U32, U32, F32, U32, F32]),
    "mf_add": (I32, [P, P, P, P]),
    "mf_multiply": (I32, [P, P, P, P]),
    "mf_linear": (I32, [P, P, P, P]),
    "mf_row_rms_norm": (I32, [P, P, P, P, F32]),
    "mf_head_rms_norm": (I32, [P, P, P, P, U32, U32, F32]),
    "mf_split_half_rotary": (I32, [P, P, P, P, U64, U32, U32, F32]),
    "mf_causal_gqa": (I32, [P, P, P, P, P, P, P, PU64, U32, U32, U32]),
    "mf_gated_short_convolution": (I32, [P, P, P, P, P, U32, U32]),
    "mf_bidirectional_gqa": (I32, [P, P, P, P, P, P, U64, U32, U32, U32]),
    "mf_centered_gated_convolution": (I32, [P, P, P, P, P, U64, U32, U32]),
    "mf_swiglu": (I32, [P, P, P, P]),
    "mf_lfm2_create": (I32, [P, P, P, P, P, C.POINTER(P)]),
    "mf_lfm2_destroy": (I32, [P]),
    "mf_lfm2_state_create": (I32, [P, C.POINTER(P)]),
    "mf_lfm2_state_fork": (I32, [P, P, C.POINTER(P)]),
    "mf_lfm2_state_destroy": (I32, [P]),
    "mf_lfm2_state_length": (U64, [P]),
    "mf_lfm2_append": (I32, [P, P, P, U64, I32]),
    "mf_lfm2_append_argmax": (I32, [P, P, U32, I32]),
    "mf_lfm2_state_logits": (P, [P]),
    "mf_lfm2_state_sampled": (P, [P]),
    "mf_lfm2_read_sampled": (I32, [P, PF32]),
    "mf_lfm2_decode_graph": (I32, [P, P, U64]),
    "mf_lfm2_decode_kernels_per_step": (U64, [P]),
    "mf_lfm2_set_fused": (I32, [P, I32]),
    "mf_lfm2_set_persistent": (I32, [P, I32]),
    "mf_lfm2_set_lut2": (I32, [P, I32, U64, C.POINTER(U64)]),
    "mf_nccl_unique_id": (I32, [P, U64]),
    "mf_lfm2_time_step": (I32, [P, P, C.POINTER(C.c_char_p), C.POINTER(C.c_float), U64, C.POINTER(U64)]),
    "mf_lfm2_set_head_split": (I32, [P, P, I32, I32]),
    "mf_lfm2_persistent_active": (I32, [P]),
    "mf_lfm2_decode_host": (I32, [P, P, P, PF32]),
    "mf_lfm2_generate": (I32, [P, P, P, U64, P, U64, P, C.POINTER(U64), C.POINTER(I32)]),
    "mf_lfm2_state_copy": (I32, [P, P, P]),
    "mf_lfm2_profile_step": (I32, [P, P, P, U32]),
    "mf_lfm2_load_bundle": (I32, [P, C.c_char_p, U64, C.POINTER(P)]),
    "mf_bundle_config": (I32, [C.c_char_p, P, P, U32, C.c_char_p, U64]),
    "mf_lfm2_batch_create": (I32, [P, U32, C.POINTER(P)]),
    "mf_lfm2_batch_destroy": (I32, [P]),
    "mf_lfm2_batch_fork": (I32, [P, P]),
    "mf_lfm2_batch_append_argmax": (I32, [P, P, U64]),
    "mf_lfm2_batch_decode": (I32, [P, U64, P]),
    "mf_lfm2_batch_read": (I32, [P, P, P]),
    "mf_lfm2_batch_kernels_per_step": (U64, [P]),
    "mfk_packed_linear": (I32, [P, P, U64, P, P, U64, U64, I32, P]),
    "mfk_repack_ternary_lut2": (I32, [P, P, U64, U64, P]),
    "mfk_packed_linear_pair": (I32, [P, P, P, U64, P, P, P, P, U64, U64, I32, P]),
    "mfk_packed_swiglu_pair": (I32, [P, P, U64, P, P, P, P, U64, U64, I32, P]),
    "mfk_packed_swiglu_linear": (I32, [P, P, P, U64, P, P, U64, U64, I32, P]),
    "mfk_packed_gather_rows": (I32, [P, P, P, U64, U64, I32, P, U64, P]),
    "mfk_argmax": (I32, [P, P, U64, U64, P]),
    "mfk_encoder_segment_ranges": (I32, [P, U64, P]),
    "mfk_bidirectional_gqa": (I32, [P, P, P, P, P, U64, U32, U32, U32, P]),
    "mfk_centered_gated_convolution": (I32, [P, P, P, P, U64, U32, U32, P]),
    "mfk_causal_gqa_noalloc": (I32, [P, P, P, P, P, P, U64, U64, U64, U32, U32, U32, P]),
}

_lib = None


def load(path: str = LIB_PATH):
    """Load libmfcuda.so and declare every exported signature (raises if absent)."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise RuntimeError(
                f"libmfcuda.so is not built at {path}; run `python -m runtime_b200.build`")
        lib = C.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols(header: str) -> list[str]:
    """Function names declared in a C header (mf_* / mfk_* entry points)."""
    import re

    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:mf|mfk)_[a-z0-9_]+)\s*\(", text)))

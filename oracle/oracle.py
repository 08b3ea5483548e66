"""ctypes binding of the CPU oracle (test infrastructure only).

The oracle is a plain-C restatement of the reference's scalar CPU backend
(crates/backend-cpu, crates/kernels-simd) and LFM2 op order
(crates/executor-core/src/lfm2/executor/execution.rs).  Only the test suite,
the smoke check and the bench's CPU-baseline leg use this module; the
product library never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmf_oracle.so")

TERNARY, NF4, INT8 = 0, 1, 2
FORMAT_NAMES = {TERNARY: "ternary", NF4: "nf4", INT8: "int8"}
LAYER_CONV, LAYER_ATTENTION = 0, 1

OK = 0
STATUS_NAMES = {
    0: "Ok", 1: "InvalidArgument", 2: "InvalidShape", 3: "InvalidLayout", 4: "InvalidDType",
    5: "Overflow", 6: "OutOfBounds", 7: "Unsupported", 8: "ResourceLimit", 9: "WrongBackend",
    10: "StaleBuffer", 17: "BackendFailure",
}


class OracleError(RuntimeError):
    def __init__(self, status: int, where: str):
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)}")
        self.status = status


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
U64 = C.c_uint64
U32 = C.c_uint32
I32 = C.c_int
F32 = C.c_float


def _declare(L):
    sigs = {
        "mfo_infer_format": (I32, [U64, U64, C.POINTER(I32), C.POINTER(U64)]),
        "mfo_packed_linear": (I32, [P, P, U64, P, P, U64, U64, I32, I32]),
        "mfo_packed_linear_pair": (I32, [P, P, P, U64, P, P, P, P, U64, U64, I32, I32]),
        "mfo_packed_swiglu_pair": (I32, [P, P, U64, P, P, P, P, U64, U64, I32, I32]),
        "mfo_packed_swiglu_linear": (I32, [P, P, P, U64, P, P, U64, U64, I32, I32]),
        "mfo_packed_gather_rows": (I32, [P, P, P, U64, U64, I32, P, U64]),
        "mfo_resolve_device_id": (C.c_int64, [F32]),
        "mfo_linear": (I32, [P, P, U64, P, U64, U64, I32]),
        "mfo_argmax": (I32, [P, P, U64, U64]),
        "mfo_argmax_masked": (I32, [P, P, U64, U64, P, U64]),
        "mfo_gather_rows": (I32, [P, P, U64, U64, P, U64]),
        "mfo_swiglu": (I32, [P, P, P, U64]),
        "mfo_add": (I32, [P, P, P, U64]),
        "mfo_multiply": (I32, [P, P, P, U64]),
        "mfo_row_rms_norm": (I32, [P, P, U64, U64, P, F32]),
        "mfo_add_row_rms_norm": (I32, [P, P, P, P, U64, U64, P, F32]),
        "mfo_head_rms_norm": (I32, [P, P, U64, U32, U32, P, F32]),
        "mfo_split_half_rotary": (I32, [P, P, U64, U32, U32, P, F32]),
        "mfo_qk_norm_rope": (I32, [P, P, P, P, U64, U32, U32, U32, P, P, P, F32, F32]),
        "mfo_causal_gqa": (I32, [P, P, P, P, U64, U32, U32, U32, P, P, U64, C.POINTER(U64), I32]),
        "mfo_gated_short_conv": (I32, [P, P, U64, U32, P, U32, P]),
        "mfo_encoder_segments_check": (I32, [P, U64]),
        "mfo_bidirectional_gqa": (I32, [P, P, P, P, P, U64, U32, U32, U32, I32]),
        "mfo_centered_gated_conv": (I32, [P, P, P, P, U64, U32, U32]),
        "mfo_lfm2_create": (I32, [P, P, I32, C.POINTER(P)]),
        "mfo_lfm2_destroy": (None, [P]),
        "mfo_lfm2_fork": (I32, [P, C.POINTER(P)]),
        "mfo_lfm2_length": (U64, [P]),
        "mfo_lfm2_append": (I32, [P, P, U64, P]),
        "mfo_lfm2_append_argmax": (I32, [P, U32, P, P]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be contiguous"
    return a.ctypes.data


def _check(st: int, where: str):
    if st != OK:
        raise OracleError(st, where)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint8)


def infer_format(code_cols: int, scale_cols: int) -> tuple[int, int]:
    f, k = I32(), U64()
    _check(lib().mfo_infer_format(code_cols, scale_cols, C.byref(f), C.byref(k)), "infer_format")
    return f.value, k.value


def packed_linear(x, codes, scales, threads: int = 1) -> np.ndarray:
    x, codes, scales = _f32(x), _u8(codes), _f32(scales)
    fmt, k = infer_format(codes.shape[1], scales.shape[1])
    t, n = x.shape[0], codes.shape[0]
    out = np.empty((t, n), np.float32)
    _check(lib().mfo_packed_linear(_p(out), _p(x), t, _p(codes), _p(scales), n, k, fmt, threads),
           "packed_linear")
    return out


def packed_linear_pair(x, codes_a, scales_a, codes_b, scales_b, threads: int = 1):
    x = _f32(x)
    codes_a, scales_a, codes_b, scales_b = _u8(codes_a), _f32(scales_a), _u8(codes_b), _f32(scales_b)
    fmt, k = infer_format(codes_a.shape[1], scales_a.shape[1])
    t, n = x.shape[0], codes_a.shape[0]
    a = np.empty((t, n), np.float32)
    b = np.empty((t, n), np.float32)
    _check(lib().mfo_packed_linear_pair(_p(a), _p(b), _p(x), t, _p(codes_a), _p(scales_a),
                                        _p(codes_b), _p(scales_b), n, k, fmt, threads),
           "packed_linear_pair")
    return a, b


def packed_swiglu_pair(x, codes_a, scales_a, codes_b, scales_b, threads: int = 1):
    x = _f32(x)
    codes_a, scales_a, codes_b, scales_b = _u8(codes_a), _f32(scales_a), _u8(codes_b), _f32(scales_b)
    fmt, k = infer_format(codes_a.shape[1], scales_a.shape[1])
    t, n = x.shape[0], codes_a.shape[0]
    out = np.empty((t, n), np.float32)
    _check(lib().mfo_packed_swiglu_pair(_p(out), _p(x), t, _p(codes_a), _p(scales_a), _p(codes_b),
                                        _p(scales_b), n, k, fmt, threads), "packed_swiglu_pair")
    return out


def packed_swiglu_linear(gate, up, codes, scales, threads: int = 1):
    gate, up, codes, scales = _f32(gate), _f32(up), _u8(codes), _f32(scales)
    fmt, k = infer_format(codes.shape[1], scales.shape[1])
    t, n = gate.shape[0], codes.shape[0]
    out = np.empty((t, n), np.float32)
    _check(lib().mfo_packed_swiglu_linear(_p(out), _p(gate), _p(up), t, _p(codes), _p(scales), n,
                                          k, fmt, threads), "packed_swiglu_linear")
    return out


def packed_gather_rows(codes, scales, ids) -> np.ndarray:
    """ids: int sequence; negative entries mark invalid device ids (NaN rows)."""
    codes, scales = _u8(codes), _f32(scales)
    fmt, k = infer_format(codes.shape[1], scales.shape[1])
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    out = np.empty((ids.shape[0], k), np.float32)
    _check(lib().mfo_packed_gather_rows(_p(out), _p(codes), _p(scales), codes.shape[0], k, fmt,
                                        _p(ids), ids.shape[0]), "packed_gather_rows")
    return out


def resolve_device_id(value: float) -> int:
    return int(lib().mfo_resolve_device_id(float(value)))


def linear(x, w, threads: int = 1):
    x, w = _f32(x), _f32(w)
    out = np.empty((x.shape[0], w.shape[0]), np.float32)
    _check(lib().mfo_linear(_p(out), _p(x), x.shape[0], _p(w), w.shape[0], w.shape[1], threads),
           "linear")
    return out


def argmax(logits):
    logits = _f32(logits)
    out = np.empty((logits.shape[0],), np.float32)
    _check(lib().mfo_argmax(_p(out), _p(logits), logits.shape[0], logits.shape[1]), "argmax")
    return out


def argmax_masked(logits, mask):
    logits = _f32(logits)
    mask = np.ascontiguousarray(mask, dtype=np.uint64)
    out = np.empty((logits.shape[0],), np.float32)
    _check(lib().mfo_argmax_masked(_p(out), _p(logits), logits.shape[0], logits.shape[1], _p(mask),
                                   mask.shape[0]), "argmax_masked")
    return out


def gather_rows(table, ids):
    table = _f32(table)
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    out = np.empty((ids.shape[0], table.shape[1]), np.float32)
    _check(lib().mfo_gather_rows(_p(out), _p(table), table.shape[0], table.shape[1], _p(ids),
                                 ids.shape[0]), "gather_rows")
    return out


def _elementwise(fn, a, b, where):
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    _check(fn(_p(out), _p(a), _p(b), a.size), where)
    return out


def swiglu(gate, up):
    return _elementwise(lib().mfo_swiglu, gate, up, "swiglu")


def add(a, b):
    return _elementwise(lib().mfo_add, a, b, "add")


def multiply(a, b):
    return _elementwise(lib().mfo_multiply, a, b, "multiply")


def row_rms_norm(x, weight, eps):
    x, weight = _f32(x), _f32(weight)
    out = np.empty_like(x)
    _check(lib().mfo_row_rms_norm(_p(out), _p(x), x.shape[0], x.shape[1], _p(weight), eps),
           "row_rms_norm")
    return out


def add_row_rms_norm(a, b, weight, eps):
    a, b, weight = _f32(a), _f32(b), _f32(weight)
    s, n = np.empty_like(a), np.empty_like(a)
    _check(lib().mfo_add_row_rms_norm(_p(s), _p(n), _p(a), _p(b), a.shape[0], a.shape[1],
                                      _p(weight), eps), "add_row_rms_norm")
    return s, n


def head_rms_norm(x, heads, head_dim, weight, eps):
    x, weight = _f32(x), _f32(weight)
    out = np.empty_like(x)
    _check(lib().mfo_head_rms_norm(_p(out), _p(x), x.shape[0], heads, head_dim, _p(weight), eps),
           "head_rms_norm")
    return out


def split_half_rotary(x, heads, head_dim, positions, theta):
    x = _f32(x)
    pos = np.ascontiguousarray(positions, dtype=np.uint64)
    out = np.empty_like(x)
    _check(lib().mfo_split_half_rotary(_p(out), _p(x), x.shape[0], heads, head_dim, _p(pos), theta),
           "split_half_rotary")
    return out


def qk_norm_rope(q, k, q_heads, kv_heads, head_dim, q_weight, k_weight, positions, theta, eps):
    q, k, qw, kw = _f32(q), _f32(k), _f32(q_weight), _f32(k_weight)
    pos = np.ascontiguousarray(positions, dtype=np.uint64)
    qo, ko = np.empty_like(q), np.empty_like(k)
    _check(lib().mfo_qk_norm_rope(_p(qo), _p(ko), _p(q), _p(k), q.shape[0], q_heads, kv_heads,
                                  head_dim, _p(qw), _p(kw), _p(pos), theta, eps), "qk_norm_rope")
    return qo, ko


def causal_gqa(q, k, v, q_heads, kv_heads, head_dim, key_cache, value_cache, cache_len,
               threads: int = 1):
    """Returns (output, new_cache_len); key_cache/value_cache are updated in place."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    assert key_cache.flags["C_CONTIGUOUS"] and value_cache.flags["C_CONTIGUOUS"]
    out = np.empty_like(q)
    length = U64(cache_len)
    _check(lib().mfo_causal_gqa(_p(out), _p(q), _p(k), _p(v), q.shape[0], q_heads, kv_heads,
                                head_dim, _p(key_cache), _p(value_cache), key_cache.shape[0],
                                C.byref(length), threads), "causal_gqa")
    return out, length.value


def gated_short_conv(projection, kernel, history):
    """history ([width-1, hidden], float32, contiguous) is updated in place."""
    projection, kernel = _f32(projection), _f32(kernel)
    hidden, width = kernel.shape
    out = np.empty((projection.shape[0], hidden), np.float32)
    _check(lib().mfo_gated_short_conv(_p(out), _p(projection), projection.shape[0], hidden,
                                      _p(kernel), width, _p(history)), "gated_short_conv")
    return out


def _segments(segment_ids, tokens):
    ids = np.ascontiguousarray(segment_ids, np.uint32)
    if ids.shape != (tokens,):
        raise OracleError(2, "encoder segments must match the token count")   # InvalidShape
    return ids


def bidirectional_gqa(q, k, v, segment_ids, q_heads, kv_heads, head_dim, threads: int = 1):
    """crates/backend-cpu/src/encoder.rs:11-124: noncausal GQA within each
    token's segment; tokens of label 0 give zero rows."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    ids = _segments(segment_ids, q.shape[0])
    out = np.empty_like(q)
    _check(lib().mfo_bidirectional_gqa(_p(out), _p(q), _p(k), _p(v), _p(ids), q.shape[0], q_heads, kv_heads,
                                       head_dim, threads), "bidirectional_gqa")
    return out


def centered_gated_conv(projection, kernel, segment_ids):
    """crates/backend-cpu/src/encoder.rs:126-189: C[t] * sum_tap k[tap] *
    (B * V)[t + tap - width/2], taps outside the token's segment skipped."""
    projection, kernel = _f32(projection), _f32(kernel)
    hidden, width = kernel.shape
    ids = _segments(segment_ids, projection.shape[0])
    out = np.empty((projection.shape[0], hidden), np.float32)
    _check(lib().mfo_centered_gated_conv(_p(out), _p(projection), _p(kernel), _p(ids), projection.shape[0],
                                         hidden, width), "centered_gated_conv")
    return out


def encoder_segments_check(segment_ids):
    ids = np.ascontiguousarray(segment_ids, np.uint32)
    return lib().mfo_encoder_segments_check(_p(ids), ids.size)


# --------------------------------------------------------------------------
# LFM2 model oracle
# --------------------------------------------------------------------------
class _Weight(C.Structure):
    _fields_ = [("packed", I32), ("format", I32), ("rows", U64), ("cols", U64),
                ("dense", P), ("codes", P), ("scales", P)]


class _Config(C.Structure):
    _fields_ = [("hidden", U32), ("intermediate", U32), ("q_heads", U32), ("kv_heads", U32),
                ("head_dim", U32), ("conv_width", U32), ("vocab", U32), ("n_layers", U32),
                ("layer_kinds", P), ("rope_theta", F32), ("block_eps", F32), ("norm_eps", F32),
                ("max_tokens", U64)]


class _LayerWeights(C.Structure):
    _fields_ = [("in_proj", _Weight), ("out_proj", _Weight), ("conv_kernel", P),
                ("q", _Weight), ("k", _Weight), ("v", _Weight), ("o", _Weight),
                ("q_norm", P), ("k_norm", P),
                ("w1", _Weight), ("w2", _Weight), ("w3", _Weight),
                ("ffn_norm", P), ("operator_norm", P)]


class _Weights(C.Structure):
    _fields_ = [("embedding", _Weight), ("embedding_norm", P), ("layers", P)]


def _weight_struct(w, keep: list) -> _Weight:
    """w: dict(kind='dense', value=f32[r,c]) or dict(kind='packed', codes, scales)."""
    s = _Weight()
    if w is None:
        return s
    if w["kind"] == "dense":
        d = _f32(w["value"])
        keep.append(d)
        s.packed, s.rows, s.cols, s.dense = 0, d.shape[0], d.shape[1], d.ctypes.data
    else:
        codes, scales = _u8(w["codes"]), _f32(w["scales"])
        keep.extend([codes, scales])
        fmt, k = infer_format(codes.shape[1], scales.shape[1])
        s.packed, s.format, s.rows, s.cols = 1, fmt, codes.shape[0], k
        s.codes, s.scales = codes.ctypes.data, scales.ctypes.data
    return s


class Lfm2Oracle:
    """CPU LFM2 executor over a weights dict (see runtime_b200.lfm2 model layout)."""

    def __init__(self, config, weights, threads: int = 1, _handle=None, _keep=None):
        self.config = config
        self.threads = threads
        if _handle is not None:
            self._h, self._keep = _handle, _keep
            return
        keep: list = []
        kinds = np.ascontiguousarray(
            [LAYER_CONV if k == "conv" else LAYER_ATTENTION for k in config.layer_types], np.int32)
        keep.append(kinds)
        cfg = _Config(config.hidden, config.intermediate, config.q_heads, config.kv_heads,
                      config.head_dim, config.conv_width, config.vocab, len(config.layer_types),
                      kinds.ctypes.data, config.rope_theta, config.block_eps, config.norm_eps,
                      config.max_tokens)
        layers = (_LayerWeights * max(1, len(config.layer_types)))()
        for i, lw in enumerate(weights["layers"]):
            L = layers[i]
            for name in ("in_proj", "out_proj", "q", "k", "v", "o", "w1", "w2", "w3"):
                setattr(L, name, _weight_struct(lw.get(name), keep))
            for name in ("conv_kernel", "q_norm", "k_norm", "ffn_norm", "operator_norm"):
                if lw.get(name) is not None:
                    a = _f32(lw[name])
                    keep.append(a)
                    setattr(L, name, a.ctypes.data)
        keep.append(layers)
        en = _f32(weights["embedding_norm"])
        keep.append(en)
        ws = _Weights(_weight_struct(weights["embedding"], keep), en.ctypes.data,
                      C.cast(layers, P))
        keep.extend([cfg, ws])
        h = P()
        _check(lib().mfo_lfm2_create(C.byref(cfg), C.byref(ws), threads, C.byref(h)),
               "lfm2_create")
        self._h, self._keep = h, keep

    def __del__(self):
        if getattr(self, "_h", None):
            lib().mfo_lfm2_destroy(self._h)
            self._h = None

    def fork(self) -> "Lfm2Oracle":
        h = P()
        _check(lib().mfo_lfm2_fork(self._h, C.byref(h)), "lfm2_fork")
        return Lfm2Oracle(self.config, None, self.threads, _handle=h, _keep=self._keep)

    @property
    def length(self) -> int:
        return int(lib().mfo_lfm2_length(self._h))

    def append(self, tokens, want_logits: bool = True):
        toks = np.ascontiguousarray(tokens, dtype=np.uint32)
        logits = np.empty((self.config.vocab,), np.float32) if want_logits else None
        _check(lib().mfo_lfm2_append(self._h, _p(toks), toks.shape[0], _p(logits)), "lfm2_append")
        return logits

    def append_argmax(self, token: int):
        sampled = np.empty((1,), np.float32)
        logits = np.empty((self.config.vocab,), np.float32)
        _check(lib().mfo_lfm2_append_argmax(self._h, int(token), _p(sampled), _p(logits)),
               "lfm2_append_argmax")
        return float(sampled[0]), logits

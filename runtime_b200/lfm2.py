"""LFM2 model description, seeded synthetic weights, and the device executor.

The model structure follows crates/executor-core/src/lfm2/weights.rs:268-513
(roles and shapes, tied embedding/LM head) and the op order of
crates/executor-core/src/lfm2/executor/execution.rs:35-627, which the C++
executor in csrc/lfm2.cu restates.

Weights are random-init (no checkpoints exist on this machine): seeded numpy
draws with the shapes and code distributions of the benchmark
configurations.  Packed roles use uniform codes; group scales are
|N(0, sigma)| with sigma chosen per format so every format's weights have a
comparable spread (ternary/NF4 sigma = 0.02, INT8 sigma = 0.02/64).
Norm weights are 1 + 0.02 N(0,1); conv kernels N(0, 0.1); a dense F32
embedding is N(0, 0.02).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field, replace

import numpy as np

from . import _lib, formats as F
from .backend import CACHE, WEIGHT, CudaBackend, CudaBuffer, _check
from ._lib import P

# crates/executor-core/tests/fixtures/pinned-lfm2.5-350m/config.json layer_types.
PATTERN_16 = ["conv", "conv", "attention", "conv", "conv", "attention", "conv", "conv",
              "attention", "conv", "attention", "conv", "attention", "conv", "attention", "conv"]
# 30 layers, 8 attention (synthetic placement for the 2.6B-shaped model).
_ATT_30 = {2, 6, 10, 14, 18, 21, 24, 27}
PATTERN_30 = ["attention" if i in _ATT_30 else "conv" for i in range(30)]

ROLES = ("embedding", "conv_in", "conv_out", "q", "k", "v", "o", "w1", "w2", "w3")


@dataclass
class Lfm2Config:
    hidden: int
    intermediate: int
    q_heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    layer_types: list
    formats: dict  # role -> "dense" | "ternary" | "nf4" | "int8"
    conv_width: int = 3
    rope_theta: float = 1.0e6
    block_eps: float = 1e-5
    norm_eps: float = 1e-5
    max_tokens: int = 4096

    def fmt(self, role: str) -> str:
        return self.formats.get(role, "ternary")

    def with_(self, **kw) -> "Lfm2Config":
        return replace(self, **kw)

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_dim


def _all(fmt):
    return {r: fmt for r in ROLES}


PRESETS = {
    # LFM2-350M-shaped, all projections ternary, F32 tied embedding.
    "lfm2-350m": Lfm2Config(1024, 4608, 16, 8, 64, 65536, PATTERN_16,
                            {**_all("ternary"), "embedding": "dense"}),
    # LFM2-1.2B-shaped, NF4 attention/conv, ternary FFN, INT8 head.
    "lfm2-1.2b": Lfm2Config(2048, 8192, 32, 8, 64, 65536, PATTERN_16,
                            {"embedding": "int8", "conv_in": "nf4", "conv_out": "nf4", "q": "nf4",
                             "k": "nf4", "v": "nf4", "o": "nf4", "w1": "ternary", "w2": "ternary",
                             "w3": "ternary"}),
    # LFM2-2.6B-shaped, ternary with an INT8 head.
    "lfm2-2.6b": Lfm2Config(2048, 10752, 32, 8, 64, 65536, PATTERN_30,
                            {**_all("ternary"), "embedding": "int8"}),
}


def tiny_config(formats=None, layers=("conv", "attention", "conv", "attention"), hidden=256,
                intermediate=512, q_heads=4, kv_heads=2, vocab=1024, max_tokens=256, **kw) -> Lfm2Config:
    """A small model of the same structure for parity tests."""
    return Lfm2Config(hidden, intermediate, q_heads, kv_heads, hidden // q_heads, vocab,
                      list(layers), formats or {**_all("ternary"), "embedding": "int8"},
                      max_tokens=max_tokens, **kw)


SCALE_SIGMA = {"ternary": 0.02, "nf4": 0.02, "int8": 0.02 / 64}


def _weight(rng, rows, cols, fmt):
    if fmt == "dense":
        return {"kind": "dense", "value": rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)}
    codes, scales = F.synthetic_weight(rng, rows, cols, fmt, SCALE_SIGMA[fmt])
    return {"kind": "packed", "format": fmt, "codes": codes, "scales": scales}


def synthetic_weights(cfg: Lfm2Config, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    h, f, kvw = cfg.hidden, cfg.intermediate, cfg.kv_width

    def norm(n):
        return (1.0 + 0.02 * rng.normal(size=n)).astype(np.float32)

    w = {"embedding": _weight(rng, cfg.vocab, h, cfg.fmt("embedding")), "embedding_norm": norm(h),
         "layers": []}
    for kind in cfg.layer_types:
        L = {}
        if kind == "conv":
            L["in_proj"] = _weight(rng, 3 * h, h, cfg.fmt("conv_in"))
            L["out_proj"] = _weight(rng, h, h, cfg.fmt("conv_out"))
            L["conv_kernel"] = rng.normal(0.0, 0.1, size=(h, cfg.conv_width)).astype(np.float32)
        else:
            L["q"] = _weight(rng, h, h, cfg.fmt("q"))
            L["k"] = _weight(rng, kvw, h, cfg.fmt("k"))
            L["v"] = _weight(rng, kvw, h, cfg.fmt("v"))
            L["o"] = _weight(rng, h, h, cfg.fmt("o"))
            L["q_norm"] = norm(cfg.head_dim)
            L["k_norm"] = norm(cfg.head_dim)
        L["w1"] = _weight(rng, f, h, cfg.fmt("w1"))
        L["w3"] = _weight(rng, f, h, cfg.fmt("w3"))
        L["w2"] = _weight(rng, h, f, cfg.fmt("w2"))
        L["ffn_norm"] = norm(h)
        L["operator_norm"] = norm(h)
        w["layers"].append(L)
    return w


def weight_bytes(cfg: Lfm2Config) -> dict:
    """Algorithmic bytes read per decode token: packed codes + F32 scales (or
    dense F32), per role family; KV bytes are per context row."""
    h, f, kvw = cfg.hidden, cfg.intermediate, cfg.kv_width

    def b(rows, cols, fmt):
        if fmt == "dense":
            return rows * cols * 4
        return rows * cols // F.WEIGHTS_PER_BYTE[F.FORMATS[fmt]] + rows * (cols // 128) * 4

    out = {"head": b(cfg.vocab, h, cfg.fmt("embedding")), "layers": 0}
    for kind in cfg.layer_types:
        if kind == "conv":
            out["layers"] += b(3 * h, h, cfg.fmt("conv_in")) + b(h, h, cfg.fmt("conv_out"))
        else:
            out["layers"] += (b(h, h, cfg.fmt("q")) + b(kvw, h, cfg.fmt("k")) + b(kvw, h, cfg.fmt("v"))
                              + b(h, h, cfg.fmt("o")))
        out["layers"] += b(f, h, cfg.fmt("w1")) + b(f, h, cfg.fmt("w3")) + b(h, f, cfg.fmt("w2"))
    out["kv_per_context_row"] = 2 * kvw * 4 * sum(1 for k in cfg.layer_types if k == "attention")
    return out


def work_flops(cfg: Lfm2Config, rows: int, base: int, logits: bool) -> int:
    """Dense-equivalent FLOPs of one pass (crates/executor-core/src/lfm2/work.rs:33-64):
    2 * params touched per row for the projections, the attention score and
    value products over the visible context, and the LM head."""
    h, f, kvw = cfg.hidden, cfg.intermediate, cfg.kv_width
    total = 0
    n_layers = len(cfg.layer_types)
    for i, kind in enumerate(cfg.layer_types):
        last = i + 1 == n_layers
        if kind == "conv":
            total += 2 * rows * (3 * h * h + h * h)
        else:
            total += 2 * rows * (2 * h * h + 2 * kvw * h)
            visible = rows * base + rows * (rows + 1) // 2
            total += 2 * 2 * visible * h
        ffn_rows = 1 if last else rows
        total += 2 * ffn_rows * 3 * f * h
    if logits:
        total += 2 * cfg.vocab * h
    return total


def bundle_config(directory: str) -> tuple[Lfm2Config, str]:
    """A bundle directory's configuration (as the reference loader reads
    config.json) and its weight format marker, without a device.  The
    per-role formats are not part of the result (they come from each role's
    code width at load time)."""
    import os

    ccfg = _lib.Lfm2Config()
    kinds = np.zeros(4096, np.int32)
    fmt = C.create_string_buffer(64)
    _check(_lib.load().mf_bundle_config(os.fsencode(directory), C.byref(ccfg), kinds.ctypes.data, len(kinds),
                                        fmt, len(fmt)))
    layer_types = ["conv" if k == 0 else "attention" for k in kinds[:ccfg.n_layers]]
    cfg = Lfm2Config(ccfg.hidden, ccfg.intermediate, ccfg.q_heads, ccfg.kv_heads, ccfg.head_dim, ccfg.vocab,
                     layer_types, {}, conv_width=ccfg.conv_width, rope_theta=float(ccfg.rope_theta),
                     block_eps=float(ccfg.block_eps), norm_eps=float(ccfg.norm_eps))
    return cfg, fmt.value.decode()


class Lfm2Model:
    """Uploads a weights dict and owns the device executor (mf_lfm2)."""

    @classmethod
    def from_bundle(cls, backend: CudaBackend, directory: str, max_tokens: int = 4096) -> "Lfm2Model":
        """Loads a bundle directory (config.json + model.safetensors) with the
        C++ loader; the executor owns the uploaded weights."""
        import os

        cfg, _ = bundle_config(directory)
        self = cls.__new__(cls)
        self.backend = backend
        self.cfg = cfg.with_(max_tokens=max_tokens)
        self._bufs = []
        h = P()
        _check(_lib.load().mf_lfm2_load_bundle(backend.handle, os.fsencode(directory), int(max_tokens), C.byref(h)))
        self.handle = h.value
        return self

    def __init__(self, backend: CudaBackend, cfg: Lfm2Config, weights: dict):
        self.backend = backend
        self.cfg = cfg
        self._bufs: list[CudaBuffer] = []
        L = _lib.load()

        def up_vec(a):
            b = backend.upload_f32(np.ascontiguousarray(a, np.float32).ravel(), cls=WEIGHT)
            self._bufs.append(b)
            return b.handle

        def up_weight(w):
            s = _lib.Lfm2Weight()
            if w is None:
                return s
            if w["kind"] == "dense":
                b = backend.upload_f32(w["value"], cls=WEIGHT)
                self._bufs.append(b)
                s.dense = b.handle
            else:
                c = backend.upload_u8(w["codes"], cls=WEIGHT)
                sc = backend.upload_f32(w["scales"], cls=WEIGHT)
                self._bufs += [c, sc]
                s.codes, s.scales = c.handle, sc.handle
            return s

        kinds = np.array([0 if k == "conv" else 1 for k in cfg.layer_types], np.int32)
        self._kinds = kinds
        layers = (_lib.Lfm2Layer * max(1, len(cfg.layer_types)))()
        for i, lw in enumerate(weights["layers"]):
            Ls = layers[i]
            for name in ("in_proj", "out_proj", "q", "k", "v", "o", "w1", "w2", "w3"):
                if name in lw:
                    setattr(Ls, name, up_weight(lw[name]))
            for name in ("conv_kernel", "q_norm", "k_norm", "ffn_norm", "operator_norm"):
                if name in lw:
                    setattr(Ls, name, up_vec(lw[name]))
        emb = up_weight(weights["embedding"])
        emb_norm = up_vec(weights["embedding_norm"])
        ccfg = _lib.Lfm2Config(cfg.hidden, cfg.intermediate, cfg.q_heads, cfg.kv_heads, cfg.head_dim,
                               cfg.conv_width, cfg.vocab, len(cfg.layer_types), kinds.ctypes.data,
                               cfg.rope_theta, cfg.block_eps, cfg.norm_eps, cfg.max_tokens)
        h = P()
        _check(L.mf_lfm2_create(backend.handle, C.byref(ccfg), C.byref(emb), emb_norm, layers, C.byref(h)))
        self.handle = h.value

    def new_state(self) -> "Lfm2State":
        h = P()
        _check(_lib.load().mf_lfm2_state_create(self.handle, C.byref(h)))
        return Lfm2State(self, h.value)

    def new_batch(self, sequences: int) -> "Lfm2Batch":
        h = P()
        _check(_lib.load().mf_lfm2_batch_create(self.handle, int(sequences), C.byref(h)))
        return Lfm2Batch(self, h.value, int(sequences))

    def set_fused(self, enabled: bool):
        """Fused single-token greedy steps (default) or the op-by-op pass;
        applies to decode graphs captured afterwards."""
        _check(_lib.load().mf_lfm2_set_fused(self.handle, int(bool(enabled))))

    def set_persistent(self, enabled: bool):
        """Single-token greedy steps as one persistent launch, or (the
        default) as the fused projections' separate launches."""
        _check(_lib.load().mf_lfm2_set_persistent(self.handle, int(bool(enabled))))

    LUT2_OFF, LUT2_AUTO, LUT2_DOWN_ONLY = 0, 1, 2

    def set_lut2(self, mode: int, max_bytes: int = (1 << 64) - 1) -> int:
        """The reference executor's LUT2 routing (Lfm2Lut2Mode, max_lut2_bytes):
        repack the ternary FFN roles into the backend's LUT2 layout, per layer
        down projection first, within the byte budget; returns the bytes
        repacked.  LUT2_OFF returns every role to its raw stream."""
        n = C.c_uint64(0)
        _check(_lib.load().mf_lfm2_set_lut2(self.handle, int(mode), int(max_bytes), C.byref(n)))
        return int(n.value)

    def set_head_split(self, unique_id: bytes | None, rank: int, world: int):
        """LM-head row split over NCCL (a collective: every rank calls it with
        the same `nccl_unique_id()` bytes and world size; world 1 turns it off)."""
        buf = None
        if unique_id is not None:
            buf = (C.c_uint8 * len(unique_id)).from_buffer_copy(unique_id)
        _check(_lib.load().mf_lfm2_set_head_split(self.handle, C.cast(buf, C.c_void_p) if buf is not None else None,
                                                  int(rank), int(world)))

    @property
    def kernels_per_decode_step(self) -> int:
        return int(_lib.load().mf_lfm2_decode_kernels_per_step(self.handle))

    def close(self):
        if getattr(self, "handle", None):
            _lib.load().mf_lfm2_destroy(self.handle)
            self.handle = None
        for b in self._bufs:
            b.release()
        self._bufs = []


class Lfm2State:
    """A prefix state (caches, position, logits, sampled id) on the device."""

    def __init__(self, model: Lfm2Model, handle):
        self.model = model
        self.handle = handle

    @property
    def length(self) -> int:
        return int(_lib.load().mf_lfm2_state_length(self.handle))

    def append(self, tokens, want_logits: bool = True):
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        _check(_lib.load().mf_lfm2_append(self.model.handle, self.handle, t.ctypes.data, t.size,
                                          int(want_logits)))

    def append_argmax(self, token: int | None = None):
        """Append one token (host id, or the device-resident sampled id when None)."""
        _check(_lib.load().mf_lfm2_append_argmax(self.model.handle, self.handle,
                                                 0 if token is None else int(token),
                                                 int(token is None)))

    def decode(self, steps: int):
        """`steps` greedy tokens through the captured decode-step graph."""
        _check(_lib.load().mf_lfm2_decode_graph(self.model.handle, self.handle, int(steps)))

    def time_step(self, capacity: int = 512) -> list[tuple[str, float]]:
        """One greedy step with a CUDA event after every launch: [(op label or
        kernel name, microseconds)] in launch order (launches serialized)."""
        names = (C.c_char_p * capacity)()
        us = (C.c_float * capacity)()
        n = C.c_uint64(0)
        _check(_lib.load().mf_lfm2_time_step(self.model.handle, self.handle, names, us, capacity, C.byref(n)))
        return [(names[i].decode(), float(us[i])) for i in range(min(n.value, capacity))]

    def decode_host(self, token: int | None = None) -> float:
        """One greedy step with host I/O: upload `token` (or reuse the device
        sampled id when None), run the captured step, return the new id."""
        out = C.c_float()
        tok = C.c_uint32(int(token)) if token is not None else None
        _check(_lib.load().mf_lfm2_decode_host(self.model.handle, self.handle,
                                               None if tok is None else C.byref(tok), C.byref(out)))
        return out.value

    def generate(self, max_tokens: int, first_token: int | None = None, stop_ids=()):
        """The reference's greedy generation loop through the C ABI (with at
        most 64 stop ids it runs on the device as one graph; otherwise the
        host reads every sample before the next token is appended).
        Returns (ids, stopped)."""
        ids = np.zeros(max(1, max_tokens), np.float32)
        stops = np.ascontiguousarray(stop_ids, np.uint32)
        n = C.c_uint64(0)
        stopped = C.c_int32(0)
        tok = C.c_uint32(int(first_token)) if first_token is not None else None
        _check(_lib.load().mf_lfm2_generate(self.model.handle, self.handle, None if tok is None else C.byref(tok),
                                            max_tokens, stops.ctypes.data if stops.size else None, stops.size,
                                            ids.ctypes.data, C.byref(n), C.byref(stopped)))
        return [int(v) for v in ids[:n.value]], bool(stopped.value)

    def copy_from(self, src: "Lfm2State"):
        """Overwrite this state with `src` (device copies, no allocation)."""
        _check(_lib.load().mf_lfm2_state_copy(self.model.handle, self.handle, src.handle))

    def profile_step(self) -> dict:
        """One decode step with per-op CUDA events; returns per-class
        {launches, bytes, ms, ops}."""
        arr = (_lib.OpProfile * len(_lib.OP_CLASSES))()
        _check(_lib.load().mf_lfm2_profile_step(self.model.handle, self.handle, arr, len(arr)))
        return {name: {"launches": int(a.launches), "bytes": int(a.bytes), "ms": float(a.ms),
                       "ops": int(a.ops)} for name, a in zip(_lib.OP_CLASSES, arr)}

    @property
    def persistent_active(self) -> bool:
        """Whether this state's single-token steps run the persistent launch."""
        return bool(_lib.load().mf_lfm2_persistent_active(self.handle))

    def read_sampled(self) -> float:
        v = C.c_float()
        _check(_lib.load().mf_lfm2_read_sampled(self.handle, C.byref(v)))
        return v.value

    def _wrap(self, h, shape):
        return CudaBuffer(self.model.backend, h, shape, 0, CACHE)

    def logits(self) -> np.ndarray:
        h = _lib.load().mf_lfm2_state_logits(self.handle)
        return self.model.backend.read_f32(self._wrap(h, (1, self.model.cfg.vocab)))[0]

    def fork(self) -> "Lfm2State":
        h = P()
        _check(_lib.load().mf_lfm2_state_fork(self.model.handle, self.handle, C.byref(h)))
        return Lfm2State(self.model, h.value)

    def close(self):
        if self.handle:
            _lib.load().mf_lfm2_state_destroy(self.handle)
            self.handle = None


class Lfm2Batch:
    """Independent sequences that advance together, one pass per step over
    all of them (each with its own caches, history, position, greedy id)."""

    def __init__(self, model: Lfm2Model, handle, sequences: int):
        self.model = model
        self.handle = handle
        self.sequences = sequences

    def fork(self, prefix: Lfm2State):
        """Every sequence becomes a copy of `prefix`."""
        _check(_lib.load().mf_lfm2_batch_fork(self.handle, prefix.handle))

    def append_argmax(self, tokens):
        """Append tokens[s, :] to sequence s (equal lengths); each sequence's
        greedy id becomes the argmax of its last row's logits."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        if t.ndim != 2 or t.shape[0] != self.sequences:
            raise ValueError(f"tokens must be [{self.sequences}, n]")
        _check(_lib.load().mf_lfm2_batch_append_argmax(self.handle, t.ctypes.data, t.shape[1]))

    def decode(self, steps: int, want_ids: bool = False):
        """`steps` greedy steps for every sequence; with want_ids the ids as
        an int array [steps, sequences]."""
        if not want_ids:
            _check(_lib.load().mf_lfm2_batch_decode(self.handle, int(steps), None))
            return None
        out = np.zeros((int(steps), self.sequences), np.float32)
        _check(_lib.load().mf_lfm2_batch_decode(self.handle, int(steps), out.ctypes.data))
        return out.astype(np.int64)

    def read(self):
        """(greedy ids [sequences] as float, logits [sequences, vocab])."""
        ids = np.zeros(self.sequences, np.float32)
        logits = np.zeros((self.sequences, self.model.cfg.vocab), np.float32)
        _check(_lib.load().mf_lfm2_batch_read(self.handle, ids.ctypes.data, logits.ctypes.data))
        return ids, logits

    @property
    def kernels_per_step(self) -> int:
        return int(_lib.load().mf_lfm2_batch_kernels_per_step(self.handle))

    def close(self):
        if self.handle:
            _lib.load().mf_lfm2_batch_destroy(self.handle)
            self.handle = None


def nccl_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id for Lfm2Model.set_head_split."""
    out = (C.c_uint8 * 128)()
    _check(_lib.load().mf_nccl_unique_id(C.cast(out, C.c_void_p), 128))
    return bytes(out)

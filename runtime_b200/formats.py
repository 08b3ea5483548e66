"""Host-side packed-weight formats: layout helpers and seeded synthetic data.

Formats (all with one F32 scale per 128-weight K group):

* ``minifield.ternary.v1`` -- four 2-bit codes per byte, weight ``j`` of a
  row at byte ``j // 4``, bits ``2 * (j % 4)``; ``w = (code - 1) * scale``
  (crates/kernels-simd/src/lib.rs:15-22, crates/engine-api/src/inference.rs:173-179).
* ``minifield.nf4.v1`` -- two 4-bit codebook indices per byte, low nibble
  first; ``w = NF4[code] * scale`` (crates/kernels-simd/src/lib.rs:111-138).
* ``minifield.int8.v1`` -- signed two's-complement bytes, -128 reserved;
  ``w = int8(code) * scale`` (crates/kernels-simd/src/lib.rs:185-190,
  crates/backend-cpu/src/packed.rs:204-208).

The format of a (codes, scales) pair is inferred from the stream widths, as
the reference does (crates/backend-cpu/src/packed.rs:172-220): with
``K = 128 * scale_cols``, ``K/4`` code bytes is ternary, ``K/2`` NF4, ``K``
INT8.
"""
from __future__ import annotations

import numpy as np

GROUP = 128
TERNARY, NF4, INT8 = 0, 1, 2
FORMATS = {"ternary": TERNARY, "nf4": NF4, "int8": INT8}
NAMES = {v: k for k, v in FORMATS.items()}
WEIGHTS_PER_BYTE = {TERNARY: 4, NF4: 2, INT8: 1}
BITS = {TERNARY: 2, NF4: 4, INT8: 8}

# crates/kernels-simd/src/lib.rs:113-130 as exact f32 bit patterns.
NF4_LEVELS = np.array(
    [0xBF800000, 0xBF3239B1, 0xBF066B30, 0xBECA32A0, 0xBE91A24D, 0xBE3D353F, 0xBDBA7871,
     0x00000000, 0x3DA2FAFF, 0x3E24CAE3, 0x3E7C04DD, 0x3EAD033A, 0x3EE1A4B8, 0x3F1007AB,
     0x3F3913B3, 0x3F800000], dtype=np.uint32).view(np.float32)


def fmt_of(fmt) -> int:
    return FORMATS[fmt] if isinstance(fmt, str) else int(fmt)


def infer_format(code_cols: int, scale_cols: int) -> int:
    k = scale_cols * GROUP
    if code_cols == k // 4:
        return TERNARY
    if code_cols == k // 2:
        return NF4
    if code_cols == k:
        return INT8
    raise ValueError("packed code width must be inner/4 (ternary), inner/2 (nf4), or inner (int8)")


def code_cols(fmt, k: int) -> int:
    return k // WEIGHTS_PER_BYTE[fmt_of(fmt)]


def pack_codes(codes: np.ndarray, fmt) -> np.ndarray:
    """Pack [R, K] unsigned codes LSB-first (first weight in the low bits)."""
    f = fmt_of(fmt)
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    per = WEIGHTS_PER_BYTE[f]
    bits = BITS[f]
    g = codes.reshape(codes.shape[0], -1, per)
    out = np.zeros(g.shape[:2], dtype=np.uint8)
    for i in range(per):
        out |= (g[:, :, i] << (i * bits)).astype(np.uint8)
    return out


def unpack_codes(packed: np.ndarray, fmt) -> np.ndarray:
    f = fmt_of(fmt)
    per = WEIGHTS_PER_BYTE[f]
    bits = BITS[f]
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.empty((packed.shape[0], packed.shape[1] * per), dtype=np.uint8)
    for i in range(per):
        out[:, i::per] = (packed >> (i * bits)) & ((1 << bits) - 1)
    return out


def levels(codes: np.ndarray, fmt) -> np.ndarray:
    """Unscaled F32 weight levels of unpacked codes."""
    f = fmt_of(fmt)
    if f == TERNARY:
        return codes.astype(np.float32) - np.float32(1.0)
    if f == NF4:
        return NF4_LEVELS[codes]
    return codes.view(np.int8).astype(np.float32)


def dequantize(packed: np.ndarray, scales: np.ndarray, fmt=None) -> np.ndarray:
    """``level(code) * scale`` with one F32 multiply, as packed_gather_rows does."""
    if fmt is None:
        fmt = infer_format(packed.shape[1], scales.shape[1])
    lv = levels(unpack_codes(packed, fmt), fmt)
    return lv * np.repeat(np.asarray(scales, np.float32), GROUP, axis=1)


def synthetic_codes(rng: np.random.Generator, rows: int, k: int, fmt) -> np.ndarray:
    """Uniform codes for the BASELINE sweeps: ternary in {0,1,2}, NF4 in 0..15,
    INT8 uniform in [-127, 127] (never the reserved 0x80)."""
    f = fmt_of(fmt)
    if f == TERNARY:
        c = rng.integers(0, 3, size=(rows, k), dtype=np.uint8)
    elif f == NF4:
        c = rng.integers(0, 16, size=(rows, k), dtype=np.uint8)
    else:
        c = rng.integers(-127, 128, size=(rows, k), dtype=np.int16).astype(np.int8).view(np.uint8)
        return np.ascontiguousarray(c)
    return pack_codes(c, f)


def synthetic_packed_fast(rng: np.random.Generator, rows: int, k: int, fmt) -> np.ndarray:
    """Packed bytes with the same code distribution as ``synthetic_codes``, built
    without the [rows, k] unpacked intermediate (for 100 MB-scale weights)."""
    f = fmt_of(fmt)
    if f == NF4:
        return rng.integers(0, 256, size=(rows, k // 2), dtype=np.uint8)
    if f == INT8:
        c = rng.integers(0, 255, size=(rows, k), dtype=np.uint8)
        return (c + np.uint8(129)).astype(np.uint8)  # 129..255,0..127: never 0x80
    # ternary: 81 valid byte values (each 2-bit field in {0,1,2})
    table = np.array([a | (b << 2) | (c << 4) | (d << 6)
                      for d in range(3) for c in range(3) for b in range(3) for a in range(3)],
                     dtype=np.uint8)
    return table[rng.integers(0, 81, size=(rows, k // 4), dtype=np.uint8)]


def synthetic_scales(rng: np.random.Generator, rows: int, k: int, sigma: float = 0.02) -> np.ndarray:
    """|N(0, sigma)| per (row, 128-group), F32."""
    return np.abs(rng.normal(0.0, sigma, size=(rows, k // GROUP))).astype(np.float32)


def synthetic_weight(rng: np.random.Generator, rows: int, k: int, fmt, sigma: float = 0.02):
    return synthetic_packed_fast(rng, rows, k, fmt), synthetic_scales(rng, rows, k, sigma)

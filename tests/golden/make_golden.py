"""Regenerate the golden fixtures under tests/golden/ from the reference.

Run in a container where the reference checkout is mounted: its path is the
first argument, or the MF_REFERENCE environment variable.  The GPU box never runs this:
the fixtures it writes are committed and read by the tests.

What it writes
--------------
quant_<scheme>.npz
    Seeded F32 weight matrices quantized by the reference's own converter
    (tools/converters/src/minifield_converters/quantization.py:52-160):
    packed code bytes, FP16 scales (as bits and as F32), unpacked codes and
    the reference's dequantized F32 weights.  These pin the packed layouts and
    the dequant arithmetic bit-for-bit.
ternary_v1_001.npz
    The hand-packed rows of
    crates/executor-core/tests/fixtures/ternary-v1-001/vectors.json
    (codes, scales, dequantized rows).
inference_ops_001.json, model_ops_001.json, rounding_sentinels_001.json
    The reference's operator oracle cases
    (crates/backend-cpu/tests/fixtures/{inference-ops-001,model-ops-001,
    cr02a-rounding-sentinels-001}), re-serialised with the fields the tests
    read and their declared tolerances.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def quantizer(reference: str):
    sys.path.insert(0, os.path.join(reference, "tools", "converters", "src"))
    from minifield_converters import quantization  # noqa: E402

    return quantization


def weights_for(scheme: str, rows: int, k: int, seed: int) -> np.ndarray:
    """Seeded weights with the edge cases the quantizer distinguishes:
    an all-zero group, a group that rounds to FP16 zero, rounding boundaries
    at +-0.5 of the absmax, and an ordinary Gaussian bulk."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.05, size=(rows, k)).astype(np.float32)
    w[0, :128] = 0.0                                   # zero group
    w[1, :128] = np.float32(1e-9)                      # FP16-underflow scale
    base = np.float32(0.25)
    w[2, :128] = 0.0
    w[2, 0] = base
    w[2, 1:9] = base * np.array([0.5, -0.5, 0.49, -0.49, 0.51, -0.51, 1.0, -1.0], np.float32)
    if scheme == "int8":
        w[3, :128] = np.linspace(-1.0, 1.0, 128, dtype=np.float32)
    return w


def make_quant(q, scheme: str, seed: int):
    rows, k = 12, 384
    w = weights_for(scheme, rows, k, seed)
    packed, scales = q.quantize(w, scheme)
    codes = q.unpack_codes(packed, scheme)
    dense = q.dequantize(packed, scales, scheme)
    repacked = q.pack_codes(codes, scheme)
    assert np.array_equal(repacked, packed)
    np.savez_compressed(
        os.path.join(HERE, f"quant_{scheme}.npz"),
        weights=w,
        packed=packed,
        scales_f16_bits=scales.view(np.uint16),
        scales_f32=scales.astype(np.float32),
        codes=codes,
        dequant=dense.astype(np.float32),
        nf4_levels=q.NF4,
    )


def make_ternary_vectors(reference: str):
    path = os.path.join(reference, "crates", "executor-core", "tests", "fixtures",
                        "ternary-v1-001", "vectors.json")
    doc = json.load(open(path))
    rows = doc["vectors"]
    packed = np.stack([np.frombuffer(bytes.fromhex(r["expected_codes_hex"]), np.uint8)
                       for r in rows])
    np.savez_compressed(
        os.path.join(HERE, "ternary_v1_001.npz"),
        input_weights=np.array([r["input_weights"] for r in rows], np.float32),
        packed=packed,
        codes=np.array([r["expected_codes"] for r in rows], np.uint8),
        scales=np.array([[r["scale_f16"]] for r in rows], np.float32),
        dequant=np.array([r["expected_dequant"] for r in rows], np.float32),
    )


def copy_json(src: str, dst: str, keep_top: tuple[str, ...]):
    doc = json.load(open(src))
    out = {key: doc[key] for key in keep_top if key in doc}
    out["source"] = os.path.relpath(src, start=os.path.dirname(os.path.dirname(os.path.dirname(
        os.path.dirname(src)))))
    with open(os.path.join(HERE, dst), "w") as fh:
        json.dump(out, fh, separators=(",", ":"), sort_keys=True)
        fh.write("\n")


def main(reference: str):
    q = quantizer(reference)
    for seed, scheme in enumerate(("ternary", "nf4", "int8")):
        make_quant(q, scheme, 1000 + seed)
    make_ternary_vectors(reference)
    fx = os.path.join(reference, "crates", "backend-cpu", "tests", "fixtures")
    copy_json(os.path.join(fx, "inference-ops-001", "cases.json"), "inference_ops_001.json",
              ("tolerance", "cases"))
    copy_json(os.path.join(fx, "model-ops-001", "cases.json"), "model_ops_001.json",
              ("tolerance", "cases"))
    copy_json(os.path.join(fx, "cr02a-rounding-sentinels-001", "rounding-sentinels.json"),
              "rounding_sentinels_001.json", ("rotary", "convolution"))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ["MF_REFERENCE"])

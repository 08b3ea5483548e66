"""Pin the CPU oracle (and the host-side format helpers) to the reference.

Every check here runs on CPU.  Sources of truth, in order of strength:

* the reference's own Python quantizer output (bit-exact pack/unpack/dequant),
* the reference's hand-packed ternary vectors (ternary-v1-001),
* the reference's operator fixtures (inference-ops-001, model-ops-001) with
  their declared atol/rtol, and the exact-bit rounding sentinels (cr02a),
* known-answer tests restated from crates/kernels-simd/src/lib.rs:210-268.
"""
import json
import os

import numpy as np
import pytest

from runtime_b200 import formats as F

SCHEMES = ("ternary", "nf4", "int8")


def load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


@pytest.mark.parametrize("scheme", SCHEMES)
def test_host_pack_unpack_matches_reference_quantizer(golden_dir, scheme):
    d = load(golden_dir, f"quant_{scheme}.npz")
    assert np.array_equal(F.pack_codes(d["codes"], scheme), d["packed"])
    assert np.array_equal(F.unpack_codes(d["packed"], scheme), d["codes"])
    assert F.infer_format(d["packed"].shape[1], d["scales_f32"].shape[1]) == F.FORMATS[scheme]
    assert np.array_equal(F.NF4_LEVELS.view(np.uint32), d["nf4_levels"].view(np.uint32))
    deq = F.dequantize(d["packed"], d["scales_f32"])
    assert np.array_equal(deq.view(np.uint32), d["dequant"].view(np.uint32))


@pytest.mark.parametrize("scheme", SCHEMES)
def test_oracle_gather_is_bit_exact_dequant(oracle, golden_dir, scheme):
    d = load(golden_dir, f"quant_{scheme}.npz")
    rows = d["packed"].shape[0]
    out = oracle.packed_gather_rows(d["packed"], d["scales_f32"], np.arange(rows))
    assert np.array_equal(out.view(np.uint32), d["dequant"].view(np.uint32))
    # repeated and reversed ids
    ids = [rows - 1, 0, 0, 3]
    out = oracle.packed_gather_rows(d["packed"], d["scales_f32"], ids)
    assert np.array_equal(out, d["dequant"][ids])


@pytest.mark.parametrize("scheme", SCHEMES)
def test_oracle_packed_linear_matches_dequantized_dense(oracle, golden_dir, scheme):
    """packed_ternary.rs:140 analogue: packed result vs dequantized dense within
    the reference's reorder tolerance (1e-4 abs + 1e-4 rel)."""
    d = load(golden_dir, f"quant_{scheme}.npz")
    rng = np.random.default_rng(7)
    x = rng.normal(size=(3, d["dequant"].shape[1])).astype(np.float32)
    got = oracle.packed_linear(x, d["packed"], d["scales_f32"])
    ref = x.astype(np.float64) @ d["dequant"].astype(np.float64).T
    assert np.all(np.abs(got - ref) <= 1e-4 + 1e-4 * np.abs(ref))
    # the pair op is two passes of the single op
    a, b = oracle.packed_linear_pair(x, d["packed"], d["scales_f32"], d["packed"][::-1].copy(),
                                     d["scales_f32"][::-1].copy())
    assert np.array_equal(a, got)
    assert np.array_equal(b, oracle.packed_linear(x, d["packed"][::-1].copy(),
                                                  d["scales_f32"][::-1].copy()))


def test_ternary_v1_001_vectors(oracle, golden_dir):
    d = load(golden_dir, "ternary_v1_001.npz")
    assert np.array_equal(F.unpack_codes(d["packed"], "ternary"), d["codes"])
    assert np.array_equal(F.pack_codes(d["codes"], "ternary"), d["packed"])
    out = oracle.packed_gather_rows(d["packed"], d["scales"], np.arange(d["packed"].shape[0]))
    assert np.array_equal(out, d["dequant"])
    # worked bytes of docs/ternary-format-v1.md: [+1,-1,0,+1] -> 0x92, all zero -> 0x55
    assert d["packed"][2, 0] == 0x92 and d["packed"][0, 0] == 0x55


def test_kernels_simd_known_answers(oracle):
    """crates/kernels-simd/src/lib.rs:215-261 restated."""
    # 0xD2 packs codes {2,0,1,3} = weights {+1,-1,0,+2}
    codes = np.full((1, 32), 0xD2, np.uint8)
    x = ((np.arange(128, dtype=np.float32) - 64.0) * 0.03125).astype(np.float32)[None]
    w = np.tile(np.array([1, -1, 0, 2], np.float32), 32)
    got = oracle.packed_linear(x, codes, np.ones((1, 1), np.float32))[0, 0]
    assert abs(got - float(np.dot(w.astype(np.float64), x[0]))) <= 1e-4
    # two groups with scales [0.5, 2]
    codes = np.full((1, 64), 0xD2, np.uint8)
    x = (np.arange(256, dtype=np.float32) * 0.01 - 1.0).astype(np.float32)[None]
    wt = np.tile(np.array([1, -1, 0, 2], np.float64), 64)
    exp = 0.5 * np.dot(wt[:128], x[0, :128]) + 2.0 * np.dot(wt[128:], x[0, 128:])
    got = oracle.packed_linear(x, codes, np.array([[0.5, 2.0]], np.float32))[0, 0]
    assert abs(got - exp) <= 1e-4
    # all codes 1 -> exactly 0; all codes 0 -> -scale * sum(x)
    x = np.arange(128, dtype=np.float32)[None]
    assert oracle.packed_linear(x, np.full((1, 32), 0x55, np.uint8),
                                np.array([[1.5]], np.float32))[0, 0] == 0.0
    got = oracle.packed_linear(x, np.zeros((1, 32), np.uint8), np.array([[2.0]], np.float32))
    assert abs(got[0, 0] - (-2.0 * x.sum())) <= 1e-3


def test_format_inference_and_int8_reserved(oracle):
    assert oracle.infer_format(32, 1) == (oracle.TERNARY, 128)
    assert oracle.infer_format(64, 1) == (oracle.NF4, 128)
    assert oracle.infer_format(128, 1) == (oracle.INT8, 128)
    with pytest.raises(oracle.OracleError) as e:
        oracle.infer_format(33, 1)
    assert e.value.status == 2  # InvalidShape
    codes = np.zeros((2, 128), np.uint8)
    codes[1, 5] = 0x80
    with pytest.raises(oracle.OracleError) as e:
        oracle.packed_linear(np.ones((1, 128), np.float32), codes, np.ones((2, 1), np.float32))
    assert e.value.status == 1  # InvalidArgument: INT8 -128 code is reserved


def test_ternary_code_three_decodes_to_plus_two(oracle):
    """The CPU decodes the reserved ternary code 3 as +2 (lib.rs:22) rather than
    rejecting it; the device path must match."""
    codes = np.full((1, 32), 0xFF, np.uint8)
    x = np.ones((1, 128), np.float32)
    assert oracle.packed_linear(x, codes, np.ones((1, 1), np.float32))[0, 0] == 256.0
    out = oracle.packed_gather_rows(codes, np.full((1, 1), 0.5, np.float32), [0])
    assert np.all(out == 1.0)


def test_gather_invalid_ids(oracle):
    codes = np.full((3, 32), 0x55, np.uint8)
    scales = np.ones((3, 1), np.float32)
    out = oracle.packed_gather_rows(codes, scales, [0, -1, 2])
    assert np.all(np.isnan(out[1])) and np.all(out[0] == 0) and np.all(out[2] == 0)
    with pytest.raises(oracle.OracleError) as e:
        oracle.packed_gather_rows(codes, scales, [3])
    assert e.value.status == 6  # OutOfBounds
    for v, want in [(2.0, 2), (-1.0, -1), (1.5, -1), (float("nan"), -1), (float("inf"), -1),
                    (16777216.0, -1), (16777215.0, 16777215)]:
        assert oracle.resolve_device_id(v) == want


def test_argmax_ties_nan_and_mask(oracle):
    logits = np.array([[1.0, 3.0, 3.0, 2.0], [0.0, np.nan, 5.0, 1.0]], np.float32)
    out = oracle.argmax(logits)
    assert out[0] == 1.0 and np.isnan(out[1])
    mask = np.array([0b1100], np.uint64)
    out = oracle.argmax_masked(logits, mask)
    assert out[0] == 2.0 and out[1] == 2.0
    out = oracle.argmax_masked(logits, np.array([0], np.uint64))
    assert np.isnan(out).all()


def _close(got, exp, tol):
    got = np.asarray(got, np.float64).ravel()
    exp = np.asarray(exp, np.float64).ravel()
    assert got.shape == exp.shape
    assert np.all(np.abs(got - exp) <= tol[0] + tol[1] * np.abs(exp)), (got, exp)


def _arr(spec):
    return np.array(spec["f32_values"], np.float32).reshape(spec["shape"])


def test_inference_ops_001(oracle, golden_dir):
    doc = json.load(open(os.path.join(golden_dir, "inference_ops_001.json")))
    tol = (doc["tolerance"]["absolute"], doc["tolerance"]["relative"])
    for case in doc["cases"]:
        op, inp, exp = case["operation"], case["inputs"], _arr(case["expected"])
        if op == "linear":
            got = oracle.linear(_arr(inp["x"]), _arr(inp["weight"]))
        elif op == "rms_norm":
            got = oracle.row_rms_norm(_arr(inp["x"]), _arr(inp["weight"]), inp["epsilon_f32"])
        elif op == "embedding":
            got = oracle.gather_rows(_arr(inp["weight"]), np.array(inp["token_ids"]))
        elif op == "swiglu":
            got = oracle.swiglu(_arr(inp["gate"]), _arr(inp["up"]))
        elif op == "add":
            got = oracle.add(_arr(inp["left"]), _arr(inp["right"]))
        elif op == "multiply":
            got = oracle.multiply(_arr(inp["left"]), _arr(inp["right"]))
        else:
            raise AssertionError(op)
        _close(got, exp, tol)


def conv_case_inputs(case):
    b, c, v = (np.array(case[k], np.float32) for k in ("B", "C", "V"))
    tokens, hidden = b.shape
    kernel = np.array(case["kernel"], np.float32)
    width = kernel.shape[1]
    proj = np.concatenate([b, c, v], axis=1).astype(np.float32)
    history = np.zeros((max(width - 1, 0), hidden), np.float32)
    prefix = np.array(case["prefix_U"], np.float32).reshape(-1, hidden)
    if prefix.size:
        history[history.shape[0] - prefix.shape[0]:] = prefix
    return proj, kernel, history


def gqa_case_inputs(case):
    q = np.array(case["Q"], np.float32)
    k = np.array(case["K"], np.float32)
    v = np.array(case["V"], np.float32)
    start = case["query_start"]
    qt, qh, d = q.shape
    total, kvh, _ = k.shape
    kvw = kvh * d
    kc = np.zeros((total, kvw), np.float32)
    vc = np.zeros((total, kvw), np.float32)
    kc[:start] = k.reshape(total, kvw)[:start]
    vc[:start] = v.reshape(total, kvw)[:start]
    return (q.reshape(qt, qh * d), k.reshape(total, kvw)[start:].copy(),
            v.reshape(total, kvw)[start:].copy(), qh, kvh, d, kc, vc, start)


def test_model_ops_001(oracle, golden_dir):
    doc = json.load(open(os.path.join(golden_dir, "model_ops_001.json")))
    tol = (doc["tolerance"]["atol"], doc["tolerance"]["rtol"])
    seen = set()
    for case in doc["cases"]:
        op = case["operation"]
        seen.add(op)
        if op == "gated_short_convolution":
            proj, kernel, history = conv_case_inputs(case)
            out = oracle.gated_short_conv(proj, kernel, history)
            _close(out, case["output"], tol)
            tail = np.array(case["tail_U"], np.float32).ravel()
            if tail.size:
                _close(history.ravel()[history.size - tail.size:], tail, tol)
        elif op == "split_half_rotary":
            x = np.array(case["input"], np.float32)
            t, h, d = x.shape
            out = oracle.split_half_rotary(x.reshape(t, h * d), h, d, case["positions"],
                                           case["theta"])
            _close(out, case["output"], tol)
        elif op == "causal_gqa":
            q, k, v, qh, kvh, d, kc, vc, start = gqa_case_inputs(case)
            out, new_len = oracle.causal_gqa(q, k, v, qh, kvh, d, kc, vc, start)
            assert new_len == kc.shape[0]
            _close(out, case["output"], tol)
        elif op == "head_local_rms":
            x = np.array(case["input"], np.float32)
            t, h, d = x.shape
            out = oracle.head_rms_norm(x.reshape(t, h * d), h, d, case["weight"], case["epsilon"])
            _close(out, case["output"], tol)
        else:
            raise AssertionError(op)
    assert seen == {"gated_short_convolution", "split_half_rotary", "causal_gqa", "head_local_rms"}


def test_rounding_sentinels_exact_bits(oracle, golden_dir):
    doc = json.load(open(os.path.join(golden_dir, "rounding_sentinels_001.json")))
    r = doc["rotary"]
    out = oracle.split_half_rotary(np.array([r["input"]], np.float32), 1, r["head_dim"],
                                   [r["position"]], r["theta"])
    assert out.view(np.uint32).tolist() == [r["expected_u32"]]
    c = doc["convolution"]
    proj = np.array([[c["B"][0][0], c["C"][0][0], c["V"][0][0]]], np.float32)
    history = np.array(c["prefix_U"], np.float32)
    out = oracle.gated_short_conv(proj, np.array(c["kernel"], np.float32), history)
    assert out.view(np.uint32).tolist() == c["expected_u32"]


def test_thread_count_is_bit_invariant(oracle):
    rng = np.random.default_rng(3)
    for fmt in ("ternary", "nf4", "int8"):
        codes, scales = F.synthetic_weight(rng, 96, 512, fmt)
        x = rng.normal(size=(5, 512)).astype(np.float32)
        a = oracle.packed_linear(x, codes, scales, threads=1)
        b = oracle.packed_linear(x, codes, scales, threads=7)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    q = rng.normal(size=(9, 8 * 16)).astype(np.float32)
    k = rng.normal(size=(9, 4 * 16)).astype(np.float32)
    v = rng.normal(size=(9, 4 * 16)).astype(np.float32)
    outs = []
    for threads in (1, 5):
        kc = np.zeros((12, 64), np.float32)
        vc = np.zeros((12, 64), np.float32)
        out, _ = oracle.causal_gqa(q, k, v, 8, 4, 16, kc, vc, 0, threads=threads)
        outs.append(out)
    assert np.array_equal(outs[0], outs[1])

"""LFM2 layer ops on the GPU vs the oracle and the reference's operator fixtures.

Elementwise ops, the RMS scaling, the RoPE combination and the conv tap sum
use explicitly rounded IEEE arithmetic on the device, so given equal inputs
they match the CPU bit-for-bit (checked where the reduction order cannot
differ); reductions are checked against the fixtures' declared tolerances.
"""
import json
import os

import numpy as np
import pytest

from tests.helpers import assert_matmul_close, bits
from tests.test_oracle_golden import conv_case_inputs, gqa_case_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from runtime_b200.backend import CudaBackend

    b = CudaBackend(0)
    yield b
    b.close()


def close(got, exp, atol, rtol):
    got = np.asarray(got, np.float64).ravel()
    exp = np.asarray(exp, np.float64).ravel()
    assert got.shape == exp.shape
    assert np.all(np.abs(got - exp) <= atol + rtol * np.abs(exp)), np.max(np.abs(got - exp))


def _arr(spec):
    return np.array(spec["f32_values"], np.float32).reshape(spec["shape"])


def test_inference_ops_fixture(be, golden_dir):
    doc = json.load(open(os.path.join(golden_dir, "inference_ops_001.json")))
    atol, rtol = doc["tolerance"]["absolute"], doc["tolerance"]["relative"]
    for case in doc["cases"]:
        op, inp, exp = case["operation"], case["inputs"], _arr(case["expected"])
        out = be.allocate_f32(exp.shape)
        if op == "linear":
            be.linear(out, be.upload_f32(_arr(inp["x"])), be.upload_f32(_arr(inp["weight"])))
        elif op == "rms_norm":
            be.row_rms_norm(out, be.upload_f32(_arr(inp["x"])), be.upload_f32(_arr(inp["weight"])),
                            inp["epsilon_f32"])
        elif op == "embedding":
            be.gather_rows(out, be.upload_f32(_arr(inp["weight"])), inp["token_ids"])
        elif op == "swiglu":
            be.swiglu(out, be.upload_f32(_arr(inp["gate"])), be.upload_f32(_arr(inp["up"])))
        elif op == "add":
            be.add(out, be.upload_f32(_arr(inp["left"])), be.upload_f32(_arr(inp["right"])))
        elif op == "multiply":
            be.multiply(out, be.upload_f32(_arr(inp["left"])), be.upload_f32(_arr(inp["right"])))
        close(be.read_f32(out), exp, atol, rtol)


def test_model_ops_fixture(be, golden_dir):
    doc = json.load(open(os.path.join(golden_dir, "model_ops_001.json")))
    atol, rtol = doc["tolerance"]["atol"], doc["tolerance"]["rtol"]
    for case in doc["cases"]:
        op = case["operation"]
        if op == "gated_short_convolution":
            proj, kernel, history = conv_case_inputs(case)
            hidden, width = kernel.shape
            out = be.allocate_f32((proj.shape[0], hidden))
            bh = be.upload_f32(history) if history.size else be.allocate_f32((0, hidden))
            be.gated_short_convolution(out, be.upload_f32(proj), be.upload_f32(kernel), bh,
                                       (hidden, width))
            close(be.read_f32(out), case["output"], atol, rtol)
            tail = np.array(case["tail_U"], np.float32).ravel()
            if tail.size:
                h = be.read_f32(bh).ravel()
                close(h[h.size - tail.size:], tail, atol, rtol)
        elif op == "split_half_rotary":
            x = np.array(case["input"], np.float32)
            t, h, d = x.shape
            out = be.allocate_f32((t, h * d))
            be.split_half_rotary(out, be.upload_f32(x.reshape(t, h * d)), case["positions"],
                                 (h, d, case["theta"]))
            close(be.read_f32(out), case["output"], atol, rtol)
        elif op == "causal_gqa":
            q, k, v, qh, kvh, d, kc, vc, start = gqa_case_inputs(case)
            out = be.allocate_f32(q.shape)
            bkc, bvc = be.upload_f32(kc), be.upload_f32(vc)
            n = be.causal_gqa(out, be.upload_f32(q), be.upload_f32(k), be.upload_f32(v), bkc, bvc,
                              start, (qh, kvh, d))
            assert n == kc.shape[0]
            close(be.read_f32(out), case["output"], atol, rtol)
        elif op == "head_local_rms":
            x = np.array(case["input"], np.float32)
            t, h, d = x.shape
            out = be.allocate_f32((t, h * d))
            be.head_rms_norm(out, be.upload_f32(x.reshape(t, h * d)),
                             be.upload_f32(np.array(case["weight"], np.float32)), (h, d),
                             case["epsilon"])
            close(be.read_f32(out), case["output"], atol, rtol)


def test_rounding_sentinels_bit_exact(be, golden_dir):
    doc = json.load(open(os.path.join(golden_dir, "rounding_sentinels_001.json")))
    r = doc["rotary"]
    out = be.allocate_f32((1, 2))
    be.split_half_rotary(out, be.upload_f32(np.array([r["input"]], np.float32)), [r["position"]],
                         (1, r["head_dim"], r["theta"]))
    assert bits(be.read_f32(out)).tolist() == [r["expected_u32"]]
    c = doc["convolution"]
    proj = np.array([[c["B"][0][0], c["C"][0][0], c["V"][0][0]]], np.float32)
    out = be.allocate_f32((1, 1))
    be.gated_short_convolution(out, be.upload_f32(proj), be.upload_f32(np.array(c["kernel"], np.float32)),
                               be.upload_f32(np.array(c["prefix_U"], np.float32)), (1, 3))
    assert bits(be.read_f32(out)).tolist() == c["expected_u32"]


@pytest.mark.parametrize("tokens,width", [(1, 3), (2, 3), (7, 3), (16, 3), (17, 3), (300, 3),
                                          (1, 2), (1, 4), (40, 4), (33, 5)])
def test_conv_matches_oracle_bit_exact(be, oracle, tokens, width):
    """Token chunks of the conv kernel recompute their window from the
    projection; the chunk-0 thread owns the rolling history."""
    rng = np.random.default_rng(4 + 100 * tokens + width)
    hidden = 300
    proj = rng.normal(size=(tokens, 3 * hidden)).astype(np.float32)
    kernel = rng.normal(0, 0.1, size=(hidden, width)).astype(np.float32)
    hist = rng.normal(size=(width - 1, hidden)).astype(np.float32)
    ref_hist = hist.copy()
    ref = oracle.gated_short_conv(proj, kernel, ref_hist)
    bh = be.upload_f32(hist)
    out = be.allocate_f32((tokens, hidden))
    be.gated_short_convolution(out, be.upload_f32(proj), be.upload_f32(kernel), bh, (hidden, width))
    assert np.array_equal(bits(be.read_f32(out)), bits(ref))
    assert np.array_equal(bits(be.read_f32(bh)), bits(ref_hist))


def test_rope_matches_oracle_bit_exact(be, oracle):
    """Split-half RoPE has no reduction: device bits equal the oracle's."""
    rng = np.random.default_rng(8)
    x = rng.normal(size=(5, 4 * 64)).astype(np.float32)
    pos = [0, 1, 17, 2047, 123456]
    ref = oracle.split_half_rotary(x, 4, 64, pos, 1e6)
    out = be.allocate_f32(x.shape)
    be.split_half_rotary(out, be.upload_f32(x), pos, (4, 64, 1e6))
    got = be.read_f32(out)
    mism = np.count_nonzero(bits(got) != bits(ref))
    assert mism == 0, f"{mism} RoPE elements differ in bits"


def test_norms_and_qk_rope(be, oracle):
    rng = np.random.default_rng(12)
    t, h = 7, 2048
    a = rng.normal(size=(t, h)).astype(np.float32)
    b = rng.normal(size=(t, h)).astype(np.float32)
    w = (1 + 0.02 * rng.normal(size=h)).astype(np.float32)
    s_ref, n_ref = oracle.add_row_rms_norm(a, b, w, 1e-5)
    so, no = be.allocate_f32((t, h)), be.allocate_f32((t, h))
    be.add_row_rms_norm(so, no, be.upload_f32(a), be.upload_f32(b), be.upload_f32(w), 1e-5)
    assert np.array_equal(bits(be.read_f32(so)), bits(s_ref))  # the add is exact
    close(be.read_f32(no), n_ref, 1e-6, 2e-6)
    q = rng.normal(size=(t, 32 * 64)).astype(np.float32)
    k = rng.normal(size=(t, 8 * 64)).astype(np.float32)
    qw = (1 + 0.02 * rng.normal(size=64)).astype(np.float32)
    kw = (1 + 0.02 * rng.normal(size=64)).astype(np.float32)
    pos = list(range(100, 100 + t))
    qr, kr = oracle.qk_norm_rope(q, k, 32, 8, 64, qw, kw, pos, 1e6, 1e-5)
    qo, ko = be.allocate_f32(q.shape), be.allocate_f32(k.shape)
    be.qk_norm_rope(qo, ko, be.upload_f32(q), be.upload_f32(k), be.upload_f32(qw), be.upload_f32(kw),
                    pos, (32, 64, 1e6), (8, 64), 1e-5)
    close(be.read_f32(qo), qr, 1e-6, 2e-6)
    close(be.read_f32(ko), kr, 1e-6, 2e-6)


@pytest.mark.parametrize("qh,kvh,d,steps", [(32, 8, 64, [37, 1, 1, 300, 1]), (16, 8, 64, [1, 1, 600]),
                                            (6, 2, 16, [3, 1, 2])])
def test_gqa_prefill_and_decode_vs_oracle(be, oracle, qh, kvh, d, steps):
    rng = np.random.default_rng(qh * 31 + d)
    cap = sum(steps) + 5
    kvw = kvh * d
    kc_ref = np.zeros((cap, kvw), np.float32)
    vc_ref = np.zeros((cap, kvw), np.float32)
    bkc, bvc = be.allocate_f32((cap, kvw)), be.allocate_f32((cap, kvw))
    n_ref = n_dev = 0
    for t in steps:
        q = rng.normal(size=(t, qh * d)).astype(np.float32)
        k = rng.normal(size=(t, kvw)).astype(np.float32)
        v = rng.normal(size=(t, kvw)).astype(np.float32)
        ref, n_ref = oracle.causal_gqa(q, k, v, qh, kvh, d, kc_ref, vc_ref, n_ref, threads=8)
        out = be.allocate_f32(q.shape)
        n_dev = be.causal_gqa(out, be.upload_f32(q), be.upload_f32(k), be.upload_f32(v), bkc, bvc,
                              n_dev, (qh, kvh, d))
        assert n_dev == n_ref
        close(be.read_f32(out), ref, 1e-5, 1e-4)
    assert np.array_equal(be.read_f32(bkc)[:n_ref], kc_ref[:n_ref])


def test_gqa_capacity_error_keeps_length(be):
    from runtime_b200.backend import ExecutorError

    bkc, bvc = be.allocate_f32((4, 64)), be.allocate_f32((4, 64))
    q = be.upload_f32(np.ones((2, 128), np.float32))
    kv = be.upload_f32(np.ones((2, 64), np.float32))
    with pytest.raises(ExecutorError) as e:
        be.causal_gqa(be.allocate_f32((2, 128)), q, kv, kv, bkc, bvc, 3, (2, 1, 64))
    assert e.value.kind == "OutOfBounds"


def test_argmax_semantics(be, oracle):
    rng = np.random.default_rng(2)
    logits = rng.normal(size=(4, 65536)).astype(np.float32)
    logits[1, 100] = logits[1, 5000] = 50.0   # tie: first index wins
    logits[2, 77] = np.nan                    # poisoned row
    logits[3, 123] = np.inf
    out = be.allocate_f32((4,))
    be.argmax(out, be.upload_f32(logits))
    got = be.read_f32(out)
    ref = oracle.argmax(logits)
    assert got[0] == ref[0] and got[1] == 100.0 and np.isnan(got[2]) and np.isnan(got[3])
    mask = np.zeros(65536 // 64, np.uint64)
    mask[0] = np.uint64(0b1010)
    be.argmax_masked(out, be.upload_f32(logits[:1].repeat(4, 0)), mask)
    exp = oracle.argmax_masked(logits[:1].repeat(4, 0), mask)
    assert np.array_equal(be.read_f32(out), exp)


def test_dense_linear_and_copies(be, oracle):
    rng = np.random.default_rng(3)
    x = rng.normal(size=(3, 1024)).astype(np.float32)
    w = rng.normal(0, 0.02, size=(4099, 1024)).astype(np.float32)
    out = be.allocate_f32((3, 4099))
    be.linear(out, be.upload_f32(x), be.upload_f32(w))
    ref = oracle.linear(x, w, threads=8)
    assert_matmul_close(be.read_f32(out), ref, np.abs(x) @ np.abs(w).T)
    src = rng.normal(size=(6, 9)).astype(np.float32)
    dst = be.allocate_f32((4, 5))
    be.copy_rect_2d(dst, be.upload_f32(src), (2, 3, 1, 1, 3, 4))
    exp = np.zeros((4, 5), np.float32)
    exp[1:4, 1:5] = src[2:5, 3:7]
    assert np.array_equal(be.read_f32(dst), exp)
    cols = be.allocate_f32((6, 3))
    be.gather_columns(cols, be.upload_f32(src), [8, 0, 8])
    assert np.array_equal(be.read_f32(cols), src[:, [8, 0, 8]])
    cp = be.allocate_f32((6, 9))
    be.copy(cp, be.upload_f32(src))
    assert np.array_equal(be.read_f32(cp), src)


@pytest.mark.parametrize("n,k", [(65536, 1024), (5003, 2048), (8192, 128)])
def test_dense_linear_one_token_streaming(be, oracle, n, k):
    """One token through a many-wave dense matrix (the config-3 tied head
    shape first) runs the streaming head kernel without its argmax."""
    rng = np.random.default_rng(n + k)
    x = rng.normal(size=(1, k)).astype(np.float32)
    w = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    out = be.allocate_f32((1, n))
    be.linear(out, be.upload_f32(x), be.upload_f32(w))
    ref = oracle.linear(x, w, threads=8)
    assert_matmul_close(be.read_f32(out), ref, np.abs(x) @ np.abs(w).T)


@pytest.mark.parametrize("width", [1, 37, 4096, 4097, 12345, 65536 + 3])
def test_argmax_ragged_widths_and_repeats(be, oracle, width):
    """Split argmax: the best element in the ragged last block, ties across
    blocks, an all-masked row (NaN), and bit-identical repeated calls (the
    arrival counters reset after every launch)."""
    rng = np.random.default_rng(width)
    logits = rng.normal(size=(3, width)).astype(np.float32)
    logits[0, width - 1] = 9.0                   # winner in the last (ragged) block
    if width > 4096:
        logits[1, 3] = logits[1, width - 2] = 9.5   # tie across blocks: first index
    bl = be.upload_f32(logits)
    outs = []
    for _ in range(3):
        out = be.allocate_f32((3,))
        be.argmax(out, bl)
        outs.append(be.read_f32(out))
    ref = oracle.argmax(logits)
    for got in outs:
        assert np.array_equal(got, ref)
    mask = np.zeros((width + 63) // 64, np.uint64)
    out = be.allocate_f32((3,))
    be.argmax_masked(out, bl, mask)
    assert np.isnan(be.read_f32(out)).all()

"""Encoder ops on the CPU: the oracle pinned, and the host side of the C ABI.

The oracle restates crates/backend-cpu/src/encoder.rs (bidirectional GQA
within segments, centered gated convolution).  It is pinned by
  * the known answers of the reference's own GPU tests: extreme active scores
    with an overflowed value in padding
    (crates/backend-wgpu/tests/encoder.rs:108-146, expected
    [6, 8, 6, 8, 0, 0]) and infinite key/value rows in padding
    (crates/backend-metal/tests/parity.rs:427-456, expected [2, 3, 0, 0]);
  * hand-derived values of the even-width centered convolution on the
    projection and kernel of crates/backend-metal/tests/parity.rs:630-665;
  * an independent float64 numpy restatement on the input patterns of
    crates/backend-wgpu/tests/encoder.rs:30-72, 148-178;
  * the segment-label rule of crates/engine-api/src/encoder.rs:16-45.
The host range builder of the C ABI (mfk_encoder_segment_ranges) runs here
without a GPU.
"""
import ctypes as C

import numpy as np
import pytest

INVALID_ARGUMENT, INVALID_SHAPE = 1, 2


def reference_segments(tokens):
    """crates/backend-wgpu/tests/encoder.rs:43-48: label 1, the middle token
    padding, label 2 after it."""
    ids = np.ones(tokens, np.uint32)
    if tokens > 2:
        mid = tokens // 2
        ids[mid] = 0
        ids[mid + 1:] = 2
    return ids


def reference_qkv(tokens, qh, kvh, dim):
    """crates/backend-wgpu/tests/encoder.rs:49-57."""
    nq, nkv = tokens * qh * dim, tokens * kvh * dim
    q = ((np.arange(nq) * 17 % 29).astype(np.float32) - 14.0) * np.float32(0.1)
    k = ((np.arange(nkv) * 11 % 31).astype(np.float32) - 15.0) * np.float32(0.1)
    v = ((np.arange(nkv) * 7 % 37).astype(np.float32) - 18.0) * np.float32(0.1)
    return (q.reshape(tokens, qh * dim).astype(np.float32), k.reshape(tokens, kvh * dim).astype(np.float32),
            v.reshape(tokens, kvh * dim).astype(np.float32))


def numpy_gqa(q, k, v, ids, qh, kvh, dim):
    out = np.zeros(q.shape, np.float64)
    group = qh // kvh
    for t in range(q.shape[0]):
        if ids[t] == 0:
            continue
        keys = np.nonzero(ids == ids[t])[0]
        for h in range(qh):
            c = (h // group) * dim
            s = k[keys, c:c + dim].astype(np.float64) @ q[t, h * dim:(h + 1) * dim].astype(np.float64)
            s /= np.sqrt(dim)
            p = np.exp(s - s.max())
            out[t, h * dim:(h + 1) * dim] = (p / p.sum()) @ v[keys, c:c + dim].astype(np.float64)
    return out


def numpy_conv(proj, kernel, ids):
    tokens, hidden, width = proj.shape[0], kernel.shape[0], kernel.shape[1]
    out = np.zeros((tokens, hidden), np.float64)
    p = proj.astype(np.float64)
    for t in range(tokens):
        if ids[t] == 0:
            continue
        for tap in range(width):
            o = t + tap - width // 2
            if 0 <= o < tokens and ids[o] == ids[t]:
                out[t] += kernel[:, tap] * (p[o, :hidden] * p[o, 2 * hidden:])
        out[t] *= p[t, hidden:2 * hidden]
    return out


def test_masked_extreme_scores_known_answer(oracle):
    q = np.ones((3, 2), np.float32)
    k = np.array([[-1e30, -1e30], [1e30, 1e30], [1, 1]], np.float32)
    v = np.array([[2, 4], [6, 8], [np.inf, np.inf]], np.float32)   # 3e38 * 2 overflowed
    out = oracle.bidirectional_gqa(q, k, v, [1, 1, 0], 1, 1, 2)
    np.testing.assert_array_equal(out, np.array([[6, 8], [6, 8], [0, 0]], np.float32))


def test_inactive_infinities_known_answer(oracle):
    q = np.ones((2, 2), np.float32)
    k = np.array([[0.5, 0.5], [np.inf, np.inf]], np.float32)
    v = np.array([[2, 3], [np.inf, np.inf]], np.float32)
    out = oracle.bidirectional_gqa(q, k, v, [1, 0], 1, 1, 2)
    np.testing.assert_array_equal(out, np.array([[2, 3], [0, 0]], np.float32))


def test_even_centered_convolution_known_answer(oracle):
    """Projection rows (B, C, V) = (1, 1, 1), (1, 1, 2), (1, 1, 3), kernel
    [1, 2, 3, 4], width 4 (taps at t - 2 .. t + 1).  One segment:
    t0 = 3*1 + 4*2 = 11, t1 = 2*1 + 3*2 + 4*3 = 20, t2 = 1*1 + 2*2 + 3*3 = 14.
    Segments [1, 1, 2]: t1 loses its tap on t2 (8), t2 keeps only itself (9)."""
    proj = np.array([[1, 1, 1], [1, 1, 2], [1, 1, 3]], np.float32)
    kernel = np.array([[1, 2, 3, 4]], np.float32)
    np.testing.assert_array_equal(oracle.centered_gated_conv(proj, kernel, [1, 1, 1]).ravel(), [11, 20, 14])
    np.testing.assert_array_equal(oracle.centered_gated_conv(proj, kernel, [1, 1, 2]).ravel(), [11, 8, 9])


@pytest.mark.parametrize("tokens,qh,kvh,dim", [(1, 4, 2, 2), (7, 4, 2, 4), (65, 16, 8, 64), (257, 2, 1, 2)])
def test_oracle_gqa_matches_float64(oracle, tokens, qh, kvh, dim):
    q, k, v = reference_qkv(tokens, qh, kvh, dim)
    ids = reference_segments(tokens)
    got = oracle.bidirectional_gqa(q, k, v, ids, qh, kvh, dim, threads=4)
    want = numpy_gqa(q, k, v, ids, qh, kvh, dim)
    assert np.all(np.abs(got - want) <= 1e-5 + 1e-5 * np.abs(want))
    assert np.all(got[ids == 0] == 0)


@pytest.mark.parametrize("width", [1, 2, 3, 4, 7])
def test_oracle_conv_matches_float64(oracle, width):
    """crates/backend-wgpu/tests/encoder.rs:148-178 inputs."""
    tokens, hidden = 7, 3
    proj = ((np.arange(tokens * 3 * hidden) % 11).astype(np.float32) * np.float32(0.07) - np.float32(0.3))
    kernel = ((np.arange(hidden * width) % 7).astype(np.float32) * np.float32(0.1) - np.float32(0.2))
    proj = proj.reshape(tokens, 3 * hidden).astype(np.float32)
    kernel = kernel.reshape(hidden, width).astype(np.float32)
    ids = np.array([0, 1, 1, 2, 2, 2, 0], np.uint32)
    got = oracle.centered_gated_conv(proj, kernel, ids)
    want = numpy_conv(proj, kernel, ids)
    assert np.all(np.abs(got - want) <= 1e-6 + 1e-6 * np.abs(want))


@pytest.mark.parametrize("ids,ok", [([], True), ([0, 0], True), ([0, 1, 1, 0, 2, 2, 0], True), ([3, 1, 2], True),
                                    ([1, 2, 1], False), ([1, 0, 1], False), ([0, 5, 0, 5], False)])
def test_segment_label_rule(oracle, ids, ok):
    assert (oracle.encoder_segments_check(ids) == 0) == ok
    if not ok:
        assert oracle.encoder_segments_check(ids) == INVALID_ARGUMENT


def test_host_segment_ranges_through_the_c_abi():
    from runtime_b200 import _lib

    L = _lib.load()
    ids = np.array([0, 1, 1, 2, 2, 2, 0, 7], np.uint32)
    ranges = np.full(2 * ids.size, 99, np.uint32)
    assert L.mfk_encoder_segment_ranges(ids.ctypes.data, ids.size, ranges.ctypes.data) == 0
    assert ranges.reshape(-1, 2).tolist() == [[0, 0], [1, 3], [1, 3], [3, 6], [3, 6], [3, 6], [0, 0], [7, 8]]
    bad = np.array([1, 2, 1], np.uint32)
    out = np.zeros(6, np.uint32)
    assert L.mfk_encoder_segment_ranges(bad.ctypes.data, bad.size, out.ctypes.data) == INVALID_ARGUMENT
    assert L.mfk_encoder_segment_ranges(None, 0, None) == 0

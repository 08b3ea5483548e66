"""Encoder ops on the GPU (mf_bidirectional_gqa, mf_centered_gated_convolution)
vs the oracle.

Gates: attention within the reference's GPU tolerance, |got - want| <=
1e-4 + 1e-4 |want| (crates/backend-wgpu/tests/encoder.rs:19-28); the
centered convolution bit-identical (same rounding order as the CPU).
Covered: the reference tests' shapes and input patterns (head groups,
segment boundaries, padding, 512 heads of dimension 2), the tiled head-dim-64
path with many segments and boundaries inside key tiles, group sizes 1/2/4,
extreme scores and infinities outside a token's segment, odd and even
convolution widths, validation errors before any write, and the raw tier.
"""
import numpy as np
import pytest

from tests.test_encoder_cpu import reference_qkv, reference_segments

pytestmark = pytest.mark.gpu
ATOL = RTOL = 1e-4


@pytest.fixture(scope="module")
def be():
    from runtime_b200.backend import CudaBackend

    b = CudaBackend(0)
    yield b
    b.close()


def close(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape
    assert np.all(np.isfinite(got))
    err = np.abs(got - want) - (ATOL + RTOL * np.abs(want))
    assert np.all(err <= 0), float(np.max(np.abs(got - want)))


def gqa(be, q, k, v, ids, spec):
    out = be.allocate_f32(q.shape)
    be.bidirectional_gqa(out, be.upload_f32(q), be.upload_f32(k), be.upload_f32(v), ids, spec)
    return be.read_f32(out)


def random_segments(rng, tokens, n_runs, pad_prob=0.2):
    cuts = np.sort(rng.choice(np.arange(1, tokens), size=n_runs - 1, replace=False))
    ids = np.zeros(tokens, np.uint32)
    label = 1
    for lo, hi in zip(np.r_[0, cuts], np.r_[cuts, tokens]):
        if rng.random() >= pad_prob:
            ids[lo:hi] = label
            label += 1
    return ids


@pytest.mark.parametrize("tokens,qh,kvh,dim", [(1, 4, 2, 2), (7, 4, 2, 4), (65, 16, 8, 64), (257, 2, 1, 2)])
def test_reference_shapes(be, oracle, tokens, qh, kvh, dim):
    q, k, v = reference_qkv(tokens, qh, kvh, dim)
    ids = reference_segments(tokens)
    close(gqa(be, q, k, v, ids, (qh, kvh, dim)), oracle.bidirectional_gqa(q, k, v, ids, qh, kvh, dim, threads=8))


def test_many_heads_of_dimension_two(be, oracle):
    """crates/backend-wgpu/tests/encoder.rs:74-106: 128 tokens, 512 heads
    sharing one kv head, zero queries and keys."""
    tokens, qh = 128, 512
    q = np.zeros((tokens, qh * 2), np.float32)
    k = np.zeros((tokens, 2), np.float32)
    v = ((np.arange(tokens * 2) % 17).astype(np.float32) * np.float32(0.125) - 1.0).reshape(tokens, 2)
    ids = np.ones(tokens, np.uint32)
    close(gqa(be, q, k, v, ids, (qh, 1, 2)), oracle.bidirectional_gqa(q, k, v, ids, qh, 1, 2, threads=8))


@pytest.mark.parametrize("tokens,qh,kvh,dim,runs", [(1000, 16, 8, 64, 7), (700, 32, 8, 64, 5), (300, 8, 8, 64, 9),
                                                    (513, 16, 4, 128, 4), (200, 6, 2, 40, 3)])
def test_random_segments_match_oracle(be, oracle, tokens, qh, kvh, dim, runs):
    rng = np.random.default_rng(tokens * 131 + qh)
    q = rng.normal(size=(tokens, qh * dim)).astype(np.float32)
    k = rng.normal(size=(tokens, kvh * dim)).astype(np.float32)
    v = rng.normal(size=(tokens, kvh * dim)).astype(np.float32)
    ids = random_segments(rng, tokens, runs)
    got = gqa(be, q, k, v, ids, (qh, kvh, dim))
    close(got, oracle.bidirectional_gqa(q, k, v, ids, qh, kvh, dim, threads=16))
    assert np.all(got[ids == 0] == 0)


def test_extreme_scores_and_overflowed_padding(be):
    """Known answer of crates/backend-wgpu/tests/encoder.rs:108-146."""
    q = np.ones((3, 2), np.float32)
    k = np.array([[-1e30, -1e30], [1e30, 1e30], [1, 1]], np.float32)
    v = np.array([[2, 4], [6, 8], [np.inf, np.inf]], np.float32)
    close(gqa(be, q, k, v, [1, 1, 0], (1, 1, 2)), [[6, 8], [6, 8], [0, 0]])


@pytest.mark.parametrize("dim", [64, 32])
def test_infinities_in_other_segments_do_not_leak(be, oracle, dim):
    """Keys and values of segment 2 and of padding are infinite; segment 1
    (whose run shares key tiles with them) equals the oracle on segment 1
    alone."""
    rng = np.random.default_rng(dim)
    tokens, qh, kvh = 150, 8, 4
    q = rng.normal(size=(tokens, qh * dim)).astype(np.float32)
    k = rng.normal(size=(tokens, kvh * dim)).astype(np.float32)
    v = rng.normal(size=(tokens, kvh * dim)).astype(np.float32)
    ids = np.zeros(tokens, np.uint32)
    ids[:70] = 1
    ids[75:] = 2
    k[70:] = np.inf
    v[70:] = np.inf
    got = gqa(be, q, k, v, ids, (qh, kvh, dim))
    want = oracle.bidirectional_gqa(q[:70], k[:70], v[:70], np.ones(70, np.uint32), qh, kvh, dim, threads=8)
    close(got[:70], want)
    assert np.all(got[70:75] == 0)


@pytest.mark.parametrize("width", [1, 2, 3, 4, 7])
def test_centered_convolution_reference_inputs_bit_exact(be, oracle, width):
    tokens, hidden = 7, 3
    proj = ((np.arange(tokens * 3 * hidden) % 11).astype(np.float32) * np.float32(0.07)
            - np.float32(0.3)).reshape(tokens, 3 * hidden).astype(np.float32)
    kernel = ((np.arange(hidden * width) % 7).astype(np.float32) * np.float32(0.1)
              - np.float32(0.2)).reshape(hidden, width).astype(np.float32)
    ids = np.array([0, 1, 1, 2, 2, 2, 0], np.uint32)
    out = be.allocate_f32((tokens, hidden))
    be.centered_gated_convolution(out, be.upload_f32(proj), be.upload_f32(kernel), ids, (hidden, width))
    want = oracle.centered_gated_conv(proj, kernel, ids)
    assert np.array_equal(be.read_f32(out).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("width", [3, 4])
def test_centered_convolution_random_segments_bit_exact(be, oracle, width):
    rng = np.random.default_rng(width)
    tokens, hidden = 900, 256
    proj = rng.normal(size=(tokens, 3 * hidden)).astype(np.float32)
    kernel = rng.normal(size=(hidden, width)).astype(np.float32)
    ids = random_segments(rng, tokens, 11)
    out = be.allocate_f32((tokens, hidden))
    be.centered_gated_convolution(out, be.upload_f32(proj), be.upload_f32(kernel), ids, (hidden, width))
    want = oracle.centered_gated_conv(proj, kernel, ids)
    assert np.array_equal(be.read_f32(out).view(np.uint32), want.view(np.uint32))


def test_validation_errors_write_nothing(be):
    """crates/backend-wgpu/tests/encoder.rs:180-214 (a segment count that
    differs from the tokens is InvalidShape, then the same call succeeds),
    and the label rule of crates/engine-api/src/encoder.rs:16-45."""
    from runtime_b200.backend import ExecutorError

    q = be.upload_f32(np.zeros((2, 2), np.float32))
    k = be.upload_f32(np.zeros((2, 2), np.float32))
    v = be.upload_f32(np.zeros((2, 2), np.float32))
    out = be.upload_f32(np.full((2, 2), 7.0, np.float32))
    with pytest.raises(ExecutorError) as e:
        be.bidirectional_gqa(out, q, k, v, [1], (1, 1, 2))
    assert e.value.status == 2   # InvalidShape
    with pytest.raises(ExecutorError) as e:
        be.bidirectional_gqa(out, q, k, v, [1, 1, 1], (1, 1, 2))
    assert e.value.status == 2
    np.testing.assert_array_equal(be.read_f32(out), np.full((2, 2), 7.0))
    be.bidirectional_gqa(out, q, k, v, [1, 1], (1, 1, 2))
    np.testing.assert_array_equal(be.read_f32(out), np.zeros((2, 2)))

    proj = be.upload_f32(np.ones((3, 3), np.float32))
    kern = be.upload_f32(np.ones((1, 4), np.float32))
    cout = be.upload_f32(np.full((3, 1), 5.0, np.float32))
    with pytest.raises(ExecutorError) as e:
        be.centered_gated_convolution(cout, proj, kern, [1, 2, 1], (1, 4))
    assert e.value.status == 1   # InvalidArgument: label 1 on two runs
    with pytest.raises(ExecutorError) as e:
        be.centered_gated_convolution(cout, proj, kern, [1, 1, 1], (1, 3))
    assert e.value.status == 2   # kernel is not [hidden, width]
    np.testing.assert_array_equal(be.read_f32(cout), np.full((3, 1), 5.0))


def test_raw_tier(be, oracle):
    """mfk_encoder_segment_ranges on the host, then the device entry points
    on the backend's own pointers."""
    from runtime_b200 import _lib

    L = _lib.load()
    rng = np.random.default_rng(5)
    tokens, qh, kvh, dim = 260, 16, 8, 64
    q = rng.normal(size=(tokens, qh * dim)).astype(np.float32)
    k = rng.normal(size=(tokens, kvh * dim)).astype(np.float32)
    v = rng.normal(size=(tokens, kvh * dim)).astype(np.float32)
    ids = random_segments(rng, tokens, 5)
    ranges = np.zeros(2 * tokens, np.uint32)
    assert L.mfk_encoder_segment_ranges(ids.ctypes.data, tokens, ranges.ctypes.data) == 0
    dr = be.upload_u8(ranges.view(np.uint8))
    bq, bk, bv = be.upload_f32(q), be.upload_f32(k), be.upload_f32(v)
    out = be.allocate_f32((tokens, qh * dim))
    assert L.mfk_bidirectional_gqa(out.ptr, bq.ptr, bk.ptr, bv.ptr, dr.ptr, tokens, qh, kvh, dim, be.stream) == 0
    close(be.read_f32(out), oracle.bidirectional_gqa(q, k, v, ids, qh, kvh, dim, threads=8))
    hidden, width = 128, 3
    proj = rng.normal(size=(tokens, 3 * hidden)).astype(np.float32)
    kern = rng.normal(size=(hidden, width)).astype(np.float32)
    bp, bkn = be.upload_f32(proj), be.upload_f32(kern)
    cout = be.allocate_f32((tokens, hidden))
    assert L.mfk_centered_gated_convolution(cout.ptr, bp.ptr, bkn.ptr, dr.ptr, tokens, hidden, width, be.stream) == 0
    want = oracle.centered_gated_conv(proj, kern, ids)
    assert np.array_equal(be.read_f32(cout).view(np.uint32), want.view(np.uint32))

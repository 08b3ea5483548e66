"""The decode GEMV (integer tensor cores for ternary/INT8, FP32 NF4) vs the oracle.

Targets what the integer path adds over a plain FP32 dot: the exact int8
limb split of the activations (extreme and mixed magnitudes inside one
128-group), non-finite propagation, several token blocks per launch, and the
split-K reduction (the arrival counters must return to zero, so repeated
calls are bit-identical).
"""
import zlib

import numpy as np
import pytest

from runtime_b200 import formats as F
from tests.helpers import assert_matmul_close, bits

pytestmark = pytest.mark.gpu
FMTS = ("ternary", "nf4", "int8")


@pytest.fixture(scope="module")
def be():
    from runtime_b200.backend import CudaBackend

    b = CudaBackend(0)
    yield b
    b.close()


def absdot(x, codes, scales):
    w = np.abs(F.dequantize(codes, scales).astype(np.float64))
    return np.abs(x.astype(np.float64)) @ w.T


def linear(be, x, codes, scales):
    out = be.allocate_f32((x.shape[0], codes.shape[0]))
    be.packed_linear(out, be.upload_f32(x), be.upload_u8(codes), be.upload_f32(scales))
    return be.read_f32(out)


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("scale", [1e-30, 1e-3, 1e3, 1e30])
def test_extreme_activation_magnitudes(be, oracle, fmt, scale):
    rng = np.random.default_rng(zlib.crc32(f"{fmt}-{scale}".encode()))
    codes, scales = F.synthetic_weight(rng, 96, 1024, fmt)
    x = (rng.normal(size=(1, 1024)) * scale).astype(np.float32)
    got = linear(be, x, codes, scales)
    ref = oracle.packed_linear(x, codes, scales, threads=8)
    assert_matmul_close(got, ref, absdot(x, codes, scales))


@pytest.mark.parametrize("fmt", FMTS)
def test_mixed_magnitudes_inside_a_group(be, oracle, fmt):
    """One large value per group next to tiny ones: every term's error stays
    far inside the reorder bound of its row."""
    rng = np.random.default_rng(3)
    codes, scales = F.synthetic_weight(rng, 64, 1024, fmt)
    x = (rng.normal(size=(2, 1024)) * 1e-6).astype(np.float32)
    x[:, ::128] = 1e4
    x[1, 5] = -3e5
    got = linear(be, x, codes, scales)
    ref = oracle.packed_linear(x, codes, scales, threads=8)
    assert_matmul_close(got, ref, absdot(x, codes, scales))


@pytest.mark.parametrize("fmt", FMTS)
def test_zero_activations_and_zero_groups(be, oracle, fmt):
    rng = np.random.default_rng(4)
    codes, scales = F.synthetic_weight(rng, 40, 768, fmt)
    x = rng.normal(size=(1, 768)).astype(np.float32)
    x[:, 128:384] = 0.0
    got = linear(be, x, codes, scales)
    ref = oracle.packed_linear(x, codes, scales, threads=8)
    assert_matmul_close(got, ref, absdot(x, codes, scales))
    assert np.all(linear(be, np.zeros((1, 768), np.float32), codes, scales) == 0.0)


@pytest.mark.parametrize("fmt", FMTS)
def test_non_finite_activation_poisons_rows(be, fmt):
    """The CPU backend refuses non-finite operands; a device backend
    propagates them (crates/engine-api/src/inference.rs:125-131): every row
    of the affected token is non-finite, other tokens stay finite."""
    rng = np.random.default_rng(5)
    codes, scales = F.synthetic_weight(rng, 48, 640, fmt)
    x = rng.normal(size=(2, 640)).astype(np.float32)
    x[0, 300] = np.inf
    got = linear(be, x, codes, scales)
    assert not np.isfinite(got[0]).any()
    assert np.isfinite(got[1]).all()
    x[0, 300] = np.nan
    got = linear(be, x, codes, scales)
    assert np.isnan(got[0]).all() and np.isfinite(got[1]).all()


@pytest.mark.parametrize("fmt", ("ternary", "int8"))
@pytest.mark.parametrize("t", [2, 9, 17, 33])
def test_token_blocks(be, oracle, fmt, t):
    rng = np.random.default_rng(100 + t)
    codes, scales = F.synthetic_weight(rng, 130, 1152, fmt)
    x = rng.normal(size=(t, 1152)).astype(np.float32)
    got = linear(be, x, codes, scales)
    ref = oracle.packed_linear(x, codes, scales, threads=8)
    assert_matmul_close(got, ref, absdot(x, codes, scales))


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("mode", ["single", "pair", "swiglu"])
def test_repeated_calls_are_bit_identical(be, oracle, fmt, mode):
    """Split-K (K = 2048: four chunks) arrival counters reset after every
    launch, and the chunk sums are added in a fixed order."""
    rng = np.random.default_rng(zlib.crc32(f"{fmt}-{mode}".encode()))
    n, k = 1000, 2048
    ca, sa = F.synthetic_weight(rng, n, k, fmt)
    cb, sb = F.synthetic_weight(rng, n, k, fmt)
    x = rng.normal(size=(1, k)).astype(np.float32)
    bx, bca, bsa, bcb, bsb = (be.upload_f32(x), be.upload_u8(ca), be.upload_f32(sa), be.upload_u8(cb),
                              be.upload_f32(sb))
    outs = []
    for _ in range(3):
        oa, ob = be.allocate_f32((1, n)), be.allocate_f32((1, n))
        if mode == "single":
            be.packed_linear(oa, bx, bca, bsa)
        elif mode == "pair":
            be.packed_linear_pair(oa, ob, bx, bca, bsa, bcb, bsb)
        else:
            be.packed_swiglu_pair(oa, bx, bca, bsa, bcb, bsb)
        outs.append((be.read_f32(oa), be.read_f32(ob)))
    for a, b in outs[1:]:
        assert np.array_equal(bits(a), bits(outs[0][0])) and np.array_equal(bits(b), bits(outs[0][1]))
    if mode == "single":
        assert_matmul_close(outs[0][0], oracle.packed_linear(x, ca, sa, threads=8), absdot(x, ca, sa))
    elif mode == "pair":
        ra, rb = oracle.packed_linear_pair(x, ca, sa, cb, sb, threads=8)
        assert_matmul_close(outs[0][0], ra, absdot(x, ca, sa))
        assert_matmul_close(outs[0][1], rb, absdot(x, cb, sb))
    else:
        assert_matmul_close(outs[0][0], oracle.packed_swiglu_pair(x, ca, sa, cb, sb, threads=8))


@pytest.mark.parametrize("fmt", FMTS)
def test_lm_head_shape(be, oracle, fmt):
    """The 65536 x 2048 LM-head shape of the benchmark models at one token."""
    rng = np.random.default_rng(7)
    codes, scales = F.synthetic_weight(rng, 65536, 2048, fmt)
    x = rng.normal(size=(1, 2048)).astype(np.float32)
    got = linear(be, x, codes, scales)
    ref = oracle.packed_linear(x, codes, scales, threads=16)
    assert_matmul_close(got, ref, absdot(x, codes, scales))


@pytest.mark.parametrize("fmt,n,k", [("int8", 40005, 2048), ("int8", 70001, 512), ("ternary", 140003, 1024),
                                     ("ternary", 70001, 2048)])
def test_streaming_single_projection(be, oracle, fmt, n, k):
    """One token through a matrix far larger than one wave runs persistent
    streaming CTAs (tiles strided over the grid, the next tile's codes in
    flight): ragged row counts, K parts past K at K = 512 / 1024, and repeat
    calls bit-identical."""
    rng = np.random.default_rng(n + k)
    codes, scales = F.synthetic_weight(rng, n, k, fmt)
    x = rng.normal(size=(1, k)).astype(np.float32)
    got = linear(be, x, codes, scales)
    assert_matmul_close(got, oracle.packed_linear(x, codes, scales, threads=16), absdot(x, codes, scales))
    assert np.array_equal(bits(linear(be, x, codes, scales)), bits(got))


@pytest.mark.parametrize("fmt", ["int8", "ternary"])
def test_streaming_projection_propagates_non_finite(be, fmt):
    rng = np.random.default_rng(3)
    codes, scales = F.synthetic_weight(rng, 40005, 1024, fmt)
    x = rng.normal(size=(1, 1024)).astype(np.float32)
    x[0, 700] = np.inf
    got = linear(be, x, codes, scales)
    assert not np.isfinite(got).any()

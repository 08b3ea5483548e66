"""The many-token packed matmul on the tcgen05 tensor cores vs the oracle.

From 48 tokens up the handle tier runs the tensor-core GEMM: both operands
split into BF16 hi/lo pairs, three MMAs per K step, F32 accumulators in
TMEM (runtime_b200/csrc/packed_gemm_tc.cu).  These tests hold it to the same
gate as every packed matmul (1e-3 max relative error, reorder-sized error
per element, crates/backend-cpu/src/packed.rs:121-195) across the shapes of
the sweep and the models, ragged row and token counts (partial 128-row and
256-token tiles), all four modes, extreme magnitudes, non-finite inputs,
and repeat calls; the device fault word must stay clear.
"""
import ctypes as C
import zlib

import numpy as np
import pytest

from runtime_b200 import formats as F
from tests.helpers import assert_matmul_close, bits

pytestmark = pytest.mark.gpu
FMTS = ("ternary", "nf4", "int8")


@pytest.fixture(scope="module")
def be():
    from runtime_b200 import _lib
    from runtime_b200.backend import CudaBackend

    L = _lib.load()
    L.mf_set_gemm_tc(1)
    b = CudaBackend(0)
    yield b
    flags = C.c_uint32(0)
    assert L.mf_device_faults(C.byref(flags)) == 0
    b.close()
    assert flags.value == 0, f"tensor-core GEMM fault word {flags.value:#x}"


def absdot(x, codes, scales):
    w = np.abs(F.dequantize(codes, scales).astype(np.float64))
    return np.abs(x.astype(np.float64)) @ w.T


def linear(be, x, codes, scales):
    out = be.allocate_f32((x.shape[0], codes.shape[0]))
    be.packed_linear(out, be.upload_f32(x), be.upload_u8(codes), be.upload_f32(scales))
    return be.read_f32(out)


def seed(*parts):
    return np.random.default_rng(zlib.crc32("-".join(map(str, parts)).encode()))


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("n,k,t", [(4608, 1024, 48), (1024, 4608, 130), (8192, 2048, 256), (2048, 8192, 300),
                                   (37, 256, 64), (130, 384, 513), (65536, 2048, 48)])
def test_single_matches_oracle(be, oracle, fmt, n, k, t):
    rng = seed(fmt, n, k, t)
    codes, scales = F.synthetic_weight(rng, n, k, fmt)
    x = rng.normal(size=(t, k)).astype(np.float32)
    got = linear(be, x, codes, scales)
    ref = oracle.packed_linear(x, codes, scales, threads=16)
    assert_matmul_close(got, ref, absdot(x, codes, scales))


@pytest.mark.parametrize("n,k,t", [(4608, 1024, 16), (2048, 8192, 31), (1024, 4608, 47)])
def test_nf4_small_batches_on_the_gemm(be, oracle, n, k, t):
    """NF4 takes the tensor-core GEMM from 16 tokens (one token tile)."""
    rng = seed("nf4-small", n, k, t)
    codes, scales = F.synthetic_weight(rng, n, k, "nf4")
    x = rng.normal(size=(t, k)).astype(np.float32)
    got = linear(be, x, codes, scales)
    ref = oracle.packed_linear(x, codes, scales, threads=8)
    assert_matmul_close(got, ref, absdot(x, codes, scales))


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("t", [48, 300])
def test_pair_swiglu_pair_and_swiglu_input(be, oracle, fmt, t):
    rng = seed("modes", fmt, t)
    n, k = 200, 640        # 2n = 400 virtual rows: the pair-rows split falls inside a tile
    ca, sa = F.synthetic_weight(rng, n, k, fmt)
    cb, sb = F.synthetic_weight(rng, n, k, fmt)
    x = rng.normal(size=(t, k)).astype(np.float32)
    bx, bca, bsa, bcb, bsb = (be.upload_f32(x), be.upload_u8(ca), be.upload_f32(sa), be.upload_u8(cb),
                              be.upload_f32(sb))
    oa, ob = be.allocate_f32((t, n)), be.allocate_f32((t, n))
    be.packed_linear_pair(oa, ob, bx, bca, bsa, bcb, bsb)
    ra, rb = oracle.packed_linear_pair(x, ca, sa, cb, sb, threads=8)
    assert_matmul_close(be.read_f32(oa), ra, absdot(x, ca, sa))
    assert_matmul_close(be.read_f32(ob), rb, absdot(x, cb, sb))

    os_ = be.allocate_f32((t, n))
    be.packed_swiglu_pair(os_, bx, bca, bsa, bcb, bsb)
    assert_matmul_close(be.read_f32(os_), oracle.packed_swiglu_pair(x, ca, sa, cb, sb, threads=8))

    # SwiGLU input: out = W (silu(gate) * up), W [n2, n]
    n2 = 96
    cw, sw = F.synthetic_weight(rng, n2, 256, fmt)
    gate = rng.normal(size=(t, 256)).astype(np.float32)
    up = rng.normal(size=(t, 256)).astype(np.float32)
    ow = be.allocate_f32((t, n2))
    be.packed_swiglu_linear(ow, be.upload_f32(gate), be.upload_f32(up), be.upload_u8(cw), be.upload_f32(sw))
    ref = oracle.packed_swiglu_linear(gate, up, cw, sw, threads=8)
    assert_matmul_close(be.read_f32(ow), ref)


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("scale", [1e-30, 1e-3, 1e3, 1e30])
def test_extreme_activation_magnitudes(be, oracle, fmt, scale):
    rng = seed("extreme", fmt, scale)
    codes, scales = F.synthetic_weight(rng, 160, 1024, fmt)
    x = (rng.normal(size=(64, 1024)) * scale).astype(np.float32)
    got = linear(be, x, codes, scales)
    ref = oracle.packed_linear(x, codes, scales, threads=8)
    assert_matmul_close(got, ref, absdot(x, codes, scales))


@pytest.mark.parametrize("fmt", FMTS)
def test_mixed_magnitudes_inside_a_group(be, oracle, fmt):
    rng = seed("mixed", fmt)
    codes, scales = F.synthetic_weight(rng, 64, 1024, fmt)
    x = (rng.normal(size=(50, 1024)) * 1e-6).astype(np.float32)
    x[:, ::128] = 1e4
    x[7, 5] = -3e5
    got = linear(be, x, codes, scales)
    ref = oracle.packed_linear(x, codes, scales, threads=8)
    assert_matmul_close(got, ref, absdot(x, codes, scales))


@pytest.mark.parametrize("fmt", FMTS)
def test_non_finite_activation_poisons_its_token(be, fmt):
    """A device backend propagates non-finite inputs
    (crates/engine-api/src/inference.rs:125-131): every output of the
    affected token is non-finite, the other tokens stay finite."""
    rng = seed("nonfinite", fmt)
    codes, scales = F.synthetic_weight(rng, 48, 640, fmt)
    x = rng.normal(size=(60, 640)).astype(np.float32)
    x[3, 300] = np.inf
    x[59, 1] = np.nan
    got = linear(be, x, codes, scales)
    assert not np.isfinite(got[3]).any()
    assert np.isnan(got[59]).all()
    keep = np.ones(60, bool)
    keep[[3, 59]] = False
    assert np.isfinite(got[keep]).all()


@pytest.mark.parametrize("fmt", FMTS)
def test_repeat_calls_are_bit_identical(be, fmt):
    rng = seed("repeat", fmt)
    codes, scales = F.synthetic_weight(rng, 1000, 2048, fmt)
    x = rng.normal(size=(200, 2048)).astype(np.float32)
    first = linear(be, x, codes, scales)
    for _ in range(2):
        assert np.array_equal(bits(linear(be, x, codes, scales)), bits(first))


def test_tensor_core_and_cuda_core_gemms_agree(be, oracle):
    from runtime_b200 import _lib

    L = _lib.load()
    rng = seed("both")
    codes, scales = F.synthetic_weight(rng, 700, 1536, "nf4")
    x = rng.normal(size=(97, 1536)).astype(np.float32)
    ref = oracle.packed_linear(x, codes, scales, threads=8)
    try:
        L.mf_set_gemm_tc(0)
        core = linear(be, x, codes, scales)
    finally:
        L.mf_set_gemm_tc(1)
    tc = linear(be, x, codes, scales)
    ad = absdot(x, codes, scales)
    assert_matmul_close(core, ref, ad)
    assert_matmul_close(tc, ref, ad)


@pytest.mark.parametrize("fmt", FMTS)
def test_split_k_in_every_mode(be, oracle, fmt):
    """Few tiles (300 ragged rows, 100 tokens) split K four ways; the splits'
    raw sums are added in a fixed order and then routed (pair rows) or
    paired (SwiGLU), as without a split."""
    rng = seed("splitk", fmt)
    n, k, t = 300, 2048, 100
    ca, sa = F.synthetic_weight(rng, n, k, fmt)
    cb, sb = F.synthetic_weight(rng, n, k, fmt)
    x = rng.normal(size=(t, k)).astype(np.float32)
    bx, bca, bsa, bcb, bsb = (be.upload_f32(x), be.upload_u8(ca), be.upload_f32(sa), be.upload_u8(cb),
                              be.upload_f32(sb))
    o1 = be.allocate_f32((t, n))
    be.packed_linear(o1, bx, bca, bsa)
    assert_matmul_close(be.read_f32(o1), oracle.packed_linear(x, ca, sa, threads=8), absdot(x, ca, sa))
    oa, ob = be.allocate_f32((t, n)), be.allocate_f32((t, n))
    be.packed_linear_pair(oa, ob, bx, bca, bsa, bcb, bsb)
    ra, rb = oracle.packed_linear_pair(x, ca, sa, cb, sb, threads=8)
    assert_matmul_close(be.read_f32(oa), ra, absdot(x, ca, sa))
    assert_matmul_close(be.read_f32(ob), rb, absdot(x, cb, sb))
    os_ = be.allocate_f32((t, n))
    be.packed_swiglu_pair(os_, bx, bca, bsa, bcb, bsb)
    first = be.read_f32(os_)
    assert_matmul_close(first, oracle.packed_swiglu_pair(x, ca, sa, cb, sb, threads=8))
    be.packed_swiglu_pair(os_, bx, bca, bsa, bcb, bsb)
    assert np.array_equal(bits(be.read_f32(os_)), bits(first))


# Per-element accuracy of the three-pass split against the exact product.
# Each operand is split into BF16 hi + lo (16 significant bits) and every
# product accumulates Wh*Xh + Wh*Xl + Wl*Xh in F32; the dropped Wl*Xl and the
# split remainders are below 2^-16 of each term.  Simulated in numpy on these
# shapes (round-to-nearest-even BF16, float64 sums), that leaves at most
# ~1.3e-6 of sum|w*x| per element, while one BF16 pass -- even with exact
# weights and only the activation rounded -- has a median error of ~4.7e-5
# and a maximum of ~3.7e-4 of sum|w*x|.  The bound below therefore holds the
# GEMM to the three-pass arithmetic.  The reference is float64 (the F32 CPU
# oracle's own sequential-sum error, ~sqrt(K) * 2^-24, is of the same size as
# the bound).  Up to 128 tokens ternary and INT8 run the group-scaled
# two-pass kernel (exact levels, only the activation split, per-group
# promotion in F32), which must meet the same bound: T = 100 covers it,
# T = 300 the three-pass kernel.
THREE_PASS_ELEM_TOL = 4e-6


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("n,k", [(8192, 2048), (2048, 8192)])
@pytest.mark.parametrize("t", [100, 300])
def test_three_pass_split_accuracy(be, fmt, n, k, t):
    rng = seed("three-pass", fmt, n, k, t)
    codes, scales = F.synthetic_weight(rng, n, k, fmt)
    x = rng.normal(size=(t, k)).astype(np.float32)
    got = linear(be, x, codes, scales).astype(np.float64)
    w = F.dequantize(codes, scales).astype(np.float64)   # exact level * scale values
    exact = x.astype(np.float64) @ w.T
    rel = np.abs(got - exact) / (np.abs(x.astype(np.float64)) @ np.abs(w).T)
    worst = float(rel.max())
    assert worst <= THREE_PASS_ELEM_TOL, f"{fmt} {n}x{k}: worst {worst:.3e}, median {float(np.median(rel)):.3e}"


@pytest.mark.parametrize("fmt,t", [("ternary", 96), ("int8", 96), ("ternary", 300), ("int8", 517)])
def test_two_and_three_pass_kernels_agree_with_the_oracle(be, oracle, fmt, t):
    """The group-scaled two-pass kernel (mf_set_gemm_passes(2)) and the
    scale-folded three-pass kernel (3) on the same call, one 128-token tile
    and several (ragged last tile)."""
    from runtime_b200 import _lib

    rng = seed("passes", fmt, t)
    n, k = 4608, 1024
    codes, scales = F.synthetic_weight(rng, n, k, fmt)
    x = rng.normal(size=(t, k)).astype(np.float32)
    ref = oracle.packed_linear(x, codes, scales, threads=8)
    outs = []
    try:
        for passes in (2, 3):
            assert _lib.load().mf_set_gemm_passes(passes) == 0
            outs.append(linear(be, x, codes, scales))
    finally:
        _lib.load().mf_set_gemm_passes(0)
    for got in outs:
        assert_matmul_close(got, ref, absdot(x, codes, scales))
    assert not np.array_equal(bits(outs[0]), bits(outs[1]))   # two different kernels ran

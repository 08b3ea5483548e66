"""Packed-matmul family on the GPU vs the CPU oracle (crates/backend-cpu/src/packed.rs).

Gate (north star): each matmul within 1e-3 max relative error in F32
accumulate, plus a per-element reorder bound; dequantised gathers bit-exact.
All calls go through the C ABI (`mf_*`) via runtime_b200.backend.
"""
import os
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


def run_linear(be, x, codes, scales):
    bx = be.upload_f32(x)
    bc = be.upload_u8(codes)
    bs = be.upload_f32(scales)
    out = be.allocate_f32((x.shape[0], codes.shape[0]))
    be.packed_linear(out, bx, bc, bs)
    return be.read_f32(out)


SHAPES = [(4608, 1024), (1024, 4608), (37, 256), (1, 128), (5, 384), (512, 2048), (96, 8192)]


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("t", [1, 3, 8])
def test_packed_linear_decode_tokens(be, oracle, fmt, n, k, t):
    rng = np.random.default_rng(zlib.crc32(f"{fmt}-{n}-{k}-{t}".encode()))
    codes, scales = F.synthetic_weight(rng, n, k, fmt)
    x = rng.normal(size=(t, k)).astype(np.float32)
    got = run_linear(be, x, codes, scales)
    ref = oracle.packed_linear(x, codes, scales, threads=8)
    assert_matmul_close(got, ref, absdot(x, codes, scales))


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("t", [16, 47, 48, 130])
def test_packed_linear_many_tokens(be, oracle, fmt, t):
    """Crosses the GEMV/GEMM switch and ragged token tiles."""
    rng = np.random.default_rng(11 + t)
    n, k = 200, 640
    codes, scales = F.synthetic_weight(rng, n, k, fmt)
    x = rng.normal(size=(t, k)).astype(np.float32)
    got = run_linear(be, x, codes, scales)
    ref = oracle.packed_linear(x, codes, scales, threads=8)
    assert_matmul_close(got, ref, absdot(x, codes, scales))


@pytest.mark.parametrize("fmt", FMTS)
def test_config1_shape_exact_setup(be, oracle, fmt):
    """BASELINE config 1 (ternary 4608 x 1024, scales |N(0,0.02)|, x ~ N(0,1), seed 1)
    generalised to every format."""
    rng = np.random.default_rng(1)
    codes = F.synthetic_codes(rng, 4608, 1024, fmt)
    scales = F.synthetic_scales(rng, 4608, 1024)
    x = rng.normal(size=(1, 1024)).astype(np.float32)
    got = run_linear(be, x, codes, scales)
    ref = oracle.packed_linear(x, codes, scales, threads=8)
    assert_matmul_close(got, ref, absdot(x, codes, scales))


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("t", [1, 5, 100])
def test_pair_and_swiglu_ops(be, oracle, fmt, t):
    rng = np.random.default_rng(5 + t)
    n, k = 300, 512
    ca, sa = F.synthetic_weight(rng, n, k, fmt)
    cb, sb = F.synthetic_weight(rng, n, k, fmt)
    x = rng.normal(size=(t, k)).astype(np.float32)
    bx, bca, bsa, bcb, bsb = (be.upload_f32(x), be.upload_u8(ca), be.upload_f32(sa),
                              be.upload_u8(cb), be.upload_f32(sb))
    oa, ob = be.allocate_f32((t, n)), be.allocate_f32((t, n))
    be.packed_linear_pair(oa, ob, bx, bca, bsa, bcb, bsb)
    ra, rb = oracle.packed_linear_pair(x, ca, sa, cb, sb, threads=8)
    assert_matmul_close(be.read_f32(oa), ra, absdot(x, ca, sa))
    assert_matmul_close(be.read_f32(ob), rb, absdot(x, cb, sb))
    # swiglu pair: silu(a) * b
    os_ = be.allocate_f32((t, n))
    be.packed_swiglu_pair(os_, bx, bca, bsa, bcb, bsb)
    ref = oracle.packed_swiglu_pair(x, ca, sa, cb, sb, threads=8)
    assert_matmul_close(be.read_f32(os_), ref)
    # swiglu linear: W @ (silu(gate) * up)
    gate = rng.normal(size=(t, k)).astype(np.float32)
    up = rng.normal(size=(t, k)).astype(np.float32)
    bg, bu = be.upload_f32(gate), be.upload_f32(up)
    ol = be.allocate_f32((t, n))
    be.packed_swiglu_linear(ol, bg, bu, bca, bsa)
    ref = oracle.packed_swiglu_linear(gate, up, ca, sa, threads=8)
    act = oracle.swiglu(gate, up)
    assert_matmul_close(be.read_f32(ol), ref, absdot(act, ca, sa))


@pytest.mark.parametrize("scheme", FMTS)
def test_packed_gather_is_bit_exact_golden(be, golden_dir, scheme):
    d = np.load(os.path.join(golden_dir, f"quant_{scheme}.npz"))
    rows, k = d["dequant"].shape
    bc, bs = be.upload_u8(d["packed"]), be.upload_f32(d["scales_f32"])
    out = be.allocate_f32((rows, k))
    be.packed_gather_rows(out, bc, bs, list(range(rows)))
    assert np.array_equal(bits(be.read_f32(out)), bits(d["dequant"]))
    # device f32 ids (argmax convention), including invalid ids -> NaN rows
    ids = be.upload_f32(np.array([2.0, -1.0, 1.5, float(rows), 0.0], np.float32))
    out = be.allocate_f32((5, k))
    be.packed_gather_rows(out, bc, bs, ids)
    got = be.read_f32(out)
    assert np.array_equal(bits(got[0]), bits(d["dequant"][2]))
    assert np.array_equal(bits(got[4]), bits(d["dequant"][0]))
    assert np.isnan(got[1:4]).all()


def test_ternary_v1_vectors_and_code_three(be, golden_dir, oracle):
    d = np.load(os.path.join(golden_dir, "ternary_v1_001.npz"))
    bc, bs = be.upload_u8(d["packed"]), be.upload_f32(d["scales"])
    out = be.allocate_f32(d["dequant"].shape)
    be.packed_gather_rows(out, bc, bs, list(range(d["packed"].shape[0])))
    assert np.array_equal(be.read_f32(out), d["dequant"])
    # reserved ternary code 3 decodes to +2 on CPU; the device matches
    codes = np.full((1, 32), 0xFF, np.uint8)
    x = np.ones((1, 128), np.float32)
    assert run_linear(be, x, codes, np.ones((1, 1), np.float32))[0, 0] == 256.0


def test_kernels_simd_known_answers_on_device(be):
    codes = np.full((1, 32), 0x55, np.uint8)
    x = np.arange(128, dtype=np.float32)[None]
    assert run_linear(be, x, codes, np.array([[1.5]], np.float32))[0, 0] == 0.0
    got = run_linear(be, x, np.zeros((1, 32), np.uint8), np.array([[2.0]], np.float32))[0, 0]
    assert abs(got - (-2.0 * x.sum())) <= 1e-3


def test_admission_errors_do_not_mutate(be):
    from runtime_b200.backend import CudaBackend, ExecutorError

    rng = np.random.default_rng(0)
    codes = F.synthetic_codes(rng, 4, 256, "int8")
    codes[2, 7] = 0x80
    bc, bs = be.upload_u8(codes), be.upload_f32(np.ones((4, 2), np.float32))
    bx = be.upload_f32(np.ones((1, 256), np.float32))
    out = be.upload_f32(np.full((1, 4), 7.0, np.float32))
    with pytest.raises(ExecutorError) as e:
        be.packed_linear(out, bx, bc, bs)
    assert e.value.kind == "InvalidArgument"
    assert np.all(be.read_f32(out) == 7.0)
    # wrong input width
    bad_x = be.upload_f32(np.ones((1, 128), np.float32))
    good_c = be.upload_u8(F.synthetic_codes(rng, 4, 256, "ternary"))
    with pytest.raises(ExecutorError) as e:
        be.packed_linear(out, bad_x, good_c, bs)
    assert e.value.kind == "InvalidShape"
    # codes width matching no format
    with pytest.raises(ExecutorError) as e:
        be.packed_linear(out, bx, be.upload_u8(np.zeros((4, 100), np.uint8)), bs)
    assert e.value.kind == "InvalidShape"
    # wrong output shape
    with pytest.raises(ExecutorError) as e:
        be.packed_linear(be.allocate_f32((1, 5)), bx, good_c, bs)
    assert e.value.kind == "InvalidShape"
    # pair: second weight set invalid -> neither output written
    oa = be.upload_f32(np.full((1, 4), 3.0, np.float32))
    ob = be.upload_f32(np.full((1, 4), 3.0, np.float32))
    with pytest.raises(ExecutorError):
        be.packed_linear_pair(oa, ob, bx, good_c, bs, bc, bs)
    assert np.all(be.read_f32(oa) == 3.0) and np.all(be.read_f32(ob) == 3.0)
    # foreign and stale buffers
    other = CudaBackend(0)
    try:
        foreign = other.upload_f32(np.ones((1, 256), np.float32))
        with pytest.raises(ExecutorError) as e:
            be.packed_linear(out, foreign, good_c, bs)
        assert e.value.kind == "WrongBackend"
    finally:
        other.close()
    gen = CudaBackend(0)
    try:
        stale = gen.upload_f32(np.ones((1, 256), np.float32))
        gen.advance_generation()
        with pytest.raises(ExecutorError) as e:
            gen.packed_linear(gen.allocate_f32((1, 4)), stale,
                              gen.upload_u8(F.synthetic_codes(rng, 4, 256, "ternary")),
                              gen.upload_f32(np.ones((4, 2), np.float32)))
        assert e.value.kind == "StaleBuffer"
        assert gen.identity().generation == 2
    finally:
        gen.close()


def test_raw_pointer_tier_matches_handle_tier(be, oracle):
    """mfk_packed_linear on the backend's own device pointers."""
    from runtime_b200 import _lib

    rng = np.random.default_rng(9)
    codes, scales = F.synthetic_weight(rng, 64, 512, "nf4")
    x = rng.normal(size=(2, 512)).astype(np.float32)
    bx, bc, bs = be.upload_f32(x), be.upload_u8(codes), be.upload_f32(scales)
    out = be.allocate_f32((2, 64))
    st = _lib.load().mfk_packed_linear(out.ptr, bx.ptr, 2, bc.ptr, bs.ptr, 64, 512, F.NF4, be.stream)
    assert st == 0
    assert_matmul_close(be.read_f32(out), oracle.packed_linear(x, codes, scales))
    assert _lib.load().mfk_packed_linear(out.ptr, bx.ptr, 2, bc.ptr, bs.ptr, 64, 500, F.NF4, be.stream) == 2

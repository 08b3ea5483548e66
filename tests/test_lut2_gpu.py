"""The backend's LUT2 ternary layout (crates/engine-api/src/inference.rs:253-311).

`repack_ternary_lut2` rearranges a `minifield.ternary.v1` code stream into
this backend's lane-tiled layout (same byte count, lossless); the `*_lut2`
ops on the repacked stream must give the raw-stream ops' results bit for bit
(the same integer dots in the same order), and those are checked against the
CPU oracle by the packed-matmul tests.  Covered: the layout itself against a
host restatement (and back), the decode GEMV at one token (the warp-tiled
kernel of the many-wave shapes and the CTA-tiled one), a few tokens, the
tcgen05 GEMM above 47 tokens, the SwiGLU pair, split-K shapes, and the
admission rules (flagged buffers only, ternary only, whole 16-row tiles).
"""
import ctypes as C

import numpy as np
import pytest

from runtime_b200 import formats as F
from tests.helpers import assert_matmul_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from runtime_b200.backend import CudaBackend

    b = CudaBackend(0)
    yield b
    b.close()


def lanetile(codes: np.ndarray) -> np.ndarray:
    """Host restatement of the layout: for 16-row tile t, group G and lane
    L = 4g + q, bytes [((t*groups + G)*32 + L)*16, +16) are row 16t+g's code
    bytes [32G + 8q, +8) then row 16t+g+8's."""
    rows, rb = codes.shape
    groups = rb // 32
    c = codes.reshape(rows // 16, 2, 8, groups, 4, 8)       # tile, half, g, G, q, byte
    return np.ascontiguousarray(c.transpose(0, 3, 2, 4, 1, 5)).reshape(rows, rb)


def untile(lt: np.ndarray) -> np.ndarray:
    rows, rb = lt.shape
    groups = rb // 32
    c = lt.reshape(rows // 16, groups, 8, 4, 2, 8)          # tile, G, g, q, half, byte
    return np.ascontiguousarray(c.transpose(0, 4, 2, 1, 3, 5)).reshape(rows, rb)


def test_layout_restatement_round_trips():
    rng = np.random.default_rng(1)
    codes = rng.integers(0, 256, size=(48, 96), dtype=np.uint8)
    lt = lanetile(codes)
    assert lt.shape == codes.shape and not np.array_equal(lt, codes)
    assert np.array_equal(untile(lt), codes)
    # tile 1, group 2, lane (g=3, q=1): row 19 bytes 72..79, then row 27's
    off = ((1 * 3 + 2) * 32 + 4 * 3 + 1) * 16
    flat = lt.reshape(-1)
    assert np.array_equal(flat[off:off + 8], codes[19, 72:80])
    assert np.array_equal(flat[off + 8:off + 16], codes[27, 72:80])


def test_raw_tier_repack_matches_restatement():
    import torch

    from runtime_b200 import _lib

    rng = np.random.default_rng(2)
    for rows, rb in ((16, 32), (64, 512), (4608, 256), (1024, 1152)):
        codes = rng.integers(0, 256, size=(rows, rb), dtype=np.uint8)
        src = torch.from_numpy(codes).cuda()
        dst = torch.zeros_like(src)
        stream = torch.cuda.current_stream().cuda_stream
        assert _lib.load().mfk_repack_ternary_lut2(dst.data_ptr(), src.data_ptr(), rows, rb, stream) == 0
        got = dst.cpu().numpy()
        assert np.array_equal(got, lanetile(codes))
        assert np.array_equal(untile(got), codes)   # bit-exactly invertible


def lut2_and_raw(be, x, codes, scales):
    bx, bc, bs = be.upload_f32(x), be.upload_u8(codes), be.upload_f32(scales)
    lt = be.repack_ternary_lut2(bc)
    raw = be.allocate_f32((x.shape[0], codes.shape[0]))
    got = be.allocate_f32((x.shape[0], codes.shape[0]))
    be.packed_linear(raw, bx, bc, bs)
    be.packed_linear_lut2(got, bx, lt, bs)
    out = be.read_f32(got), be.read_f32(raw)
    for b in (bx, bc, bs, lt, raw, got):
        b.release()
    return out


@pytest.mark.parametrize("n,k,t", [
    (65536, 2048, 1),    # many waves: warp-tiled kernel, limbs split in each CTA
    (40960, 1024, 1),
    (8192, 2048, 1),     # CTA-tiled integer-MMA kernel
    (2048, 8192, 1),
    (4608, 1024, 3),
    (1024, 4608, 17),
    (2048, 2048, 47),
    (8192, 2048, 100),   # tcgen05 GEMM
    (1024, 4608, 300),
])
def test_linear_lut2_equals_raw(be, oracle, n, k, t):
    rng = np.random.default_rng(n + k + t)
    codes, scales = F.synthetic_weight(rng, n, k, "ternary")
    x = rng.normal(size=(t, k)).astype(np.float32)
    got, raw = lut2_and_raw(be, x, codes, scales)
    assert np.array_equal(got.view(np.uint32), raw.view(np.uint32))
    if n * k * t <= 8192 * 2048 * 3:
        ref = oracle.packed_linear(x, codes, scales, threads=8)
        w = np.abs(F.dequantize(codes, scales).astype(np.float64))
        assert_matmul_close(got, ref, np.abs(x.astype(np.float64)) @ w.T)


@pytest.mark.parametrize("t", [1, 2, 5, 64])
def test_swiglu_pair_lut2_equals_raw(be, t):
    rng = np.random.default_rng(100 + t)
    n, k = 8192, 2048
    ca, sa = F.synthetic_weight(rng, n, k, "ternary")
    cb, sb = F.synthetic_weight(rng, n, k, "ternary")
    x = rng.normal(size=(t, k)).astype(np.float32)
    bx = be.upload_f32(x)
    ha = [be.upload_u8(ca), be.upload_f32(sa), be.upload_u8(cb), be.upload_f32(sb)]
    la, lb = be.repack_ternary_lut2(ha[0]), be.repack_ternary_lut2(ha[2])
    raw, got = be.allocate_f32((t, n)), be.allocate_f32((t, n))
    be.packed_swiglu_pair(raw, bx, *ha)
    be.packed_swiglu_pair_lut2(got, bx, la, ha[1], lb, ha[3])
    assert np.array_equal(be.read_f32(got).view(np.uint32), be.read_f32(raw).view(np.uint32))


def test_lut2_admission(be):
    from runtime_b200.backend import ExecutorError

    assert be.supports_ternary_lut2()
    rng = np.random.default_rng(7)
    codes, scales = F.synthetic_weight(rng, 64, 256, "ternary")
    bc, bs = be.upload_u8(codes), be.upload_f32(scales)
    lt = be.repack_ternary_lut2(bc)
    bx = be.upload_f32(np.ones((1, 256), np.float32))
    out = be.upload_f32(np.full((1, 64), 5.0, np.float32))
    # raw codes to a LUT2 op, LUT2 codes to a raw op: rejected, output untouched
    with pytest.raises(ExecutorError) as e:
        be.packed_linear_lut2(out, bx, bc, bs)
    assert e.value.kind == "InvalidArgument"
    with pytest.raises(ExecutorError) as e:
        be.packed_linear(out, bx, lt, bs)
    assert e.value.kind == "InvalidArgument"
    with pytest.raises(ExecutorError) as e:
        be.repack_ternary_lut2(lt)
    assert e.value.kind == "InvalidArgument"
    assert np.all(be.read_f32(out) == 5.0)
    # a stream the layout cannot take: ResourceLimit (a loader keeps the raw stream)
    odd = be.upload_u8(F.synthetic_codes(rng, 40, 256, "ternary"))
    with pytest.raises(ExecutorError) as e:
        be.repack_ternary_lut2(odd)
    assert e.value.kind == "ResourceLimit"
    # NF4-shaped codes repack as bytes but no LUT2 op takes them
    nf4 = be.repack_ternary_lut2(be.upload_u8(F.synthetic_codes(rng, 64, 256, "nf4")))
    with pytest.raises(ExecutorError) as e:
        be.packed_linear_lut2(out, bx, nf4, bs)
    assert e.value.kind == "InvalidDType"
    assert np.all(be.read_f32(out) == 5.0)


# ---------------------------------------------------------------------------
# The executor's LUT2 routing (construction.rs:404-470, execution.rs:343-400)
# ---------------------------------------------------------------------------

def _stream(model, prompt, steps):
    st = model.new_state()
    st.append(prompt)
    first = int(np.argmax(st.logits()))
    ids, _ = st.generate(steps + 1, first_token=first)
    logits = st.logits()
    st.close()
    return ids, logits


def test_model_lut2_modes_and_budget(be):
    from runtime_b200 import lfm2 as M

    cfg = M.tiny_config(None, layers=("conv", "attention", "conv"), max_tokens=160)
    w = M.synthetic_weights(cfg, 31)
    model = M.Lfm2Model(be, cfg, w)
    per = cfg.hidden * cfg.intermediate // 4          # one FFN matrix's code bytes
    assert model.set_lut2(M.Lfm2Model.LUT2_AUTO) == 3 * 3 * per
    assert model.set_lut2(M.Lfm2Model.LUT2_DOWN_ONLY) == 3 * per
    # Budget: layer 0's down (1 matrix), then its gate/up pair does not fit in
    # 2 matrices' worth, layer 1's down does.
    assert model.set_lut2(M.Lfm2Model.LUT2_AUTO, 2 * per) == 2 * per
    assert model.set_lut2(M.Lfm2Model.LUT2_OFF) == 0
    model.close()


@pytest.mark.parametrize("mode", ["auto", "down_only"])
def test_model_lut2_matches_raw_streams(be, oracle, mode):
    """Prefill above 47 rows (tcgen05 GEMM), the fused decode graph and the
    device generation loop on LUT2 FFN weights give the raw-stream model's
    logits bit for bit and the oracle's greedy stream."""
    from runtime_b200 import lfm2 as M

    cfg = M.tiny_config(None, layers=("conv", "attention", "conv", "attention"), max_tokens=200)
    w = M.synthetic_weights(cfg, 33)
    prompt = np.random.default_rng(3).integers(0, cfg.vocab, size=70)
    raw = M.Lfm2Model(be, cfg, w)
    ids_raw, logits_raw = _stream(raw, prompt, 24)
    raw.close()
    lut = M.Lfm2Model(be, cfg, w)
    lut.set_lut2(M.Lfm2Model.LUT2_AUTO if mode == "auto" else M.Lfm2Model.LUT2_DOWN_ONLY)
    ids_lut, logits_lut = _stream(lut, prompt, 24)
    assert ids_lut == ids_raw
    assert np.array_equal(logits_lut.view(np.uint32), logits_raw.view(np.uint32))
    ref = oracle.Lfm2Oracle(cfg, w, threads=8)
    want = [int(np.argmax(ref.append(prompt)))]
    for _ in range(24):
        s, _ = ref.append_argmax(want[-1])
        want.append(int(s))
    assert ids_lut == want
    # Switching back recaptures the graphs on the raw streams.
    lut.set_lut2(M.Lfm2Model.LUT2_OFF)
    assert _stream(lut, prompt, 24)[0] == ids_raw
    lut.close()


@pytest.mark.parametrize("seqs", [5, 64])
def test_batch_lut2_matches_raw(be, seqs):
    """Batched passes at 5 rows (decode GEMV) and 64 rows (tcgen05 GEMM)."""
    from runtime_b200 import lfm2 as M

    cfg = M.tiny_config(None, max_tokens=96)
    w = M.synthetic_weights(cfg, 35)
    prefix = np.random.default_rng(4).integers(0, cfg.vocab, size=20)
    suffix = np.random.default_rng(5).integers(0, cfg.vocab, size=(seqs, 3))
    outs = []
    for lut2 in (False, True):
        model = M.Lfm2Model(be, cfg, w)
        if lut2:
            model.set_lut2(M.Lfm2Model.LUT2_AUTO)
        pre = model.new_state()
        pre.append(prefix, want_logits=False)
        batch = model.new_batch(seqs)
        batch.fork(pre)
        batch.append_argmax(suffix)
        ids = batch.decode(6, want_ids=True)
        outs.append(ids)
        batch.close()
        pre.close()
        model.close()
    assert np.array_equal(outs[0], outs[1])

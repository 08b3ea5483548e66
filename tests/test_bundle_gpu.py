"""Bundles loaded by the C++ loader (mf_lfm2_load_bundle) vs the oracle.

The oracle gets the same weights from an independent numpy reader
(tests/bundle_io.py): packed codes as stored, F16 scales widened to F32,
dense F32/BF16 values widened to F32.  Each bundle must give the oracle's
prefill logits within 1e-2 and its greedy token stream.  Covered: the
ternary and NF4 bundles written by the reference's converter, dense F32 and
BF16 bundles, an INT8 bundle and a mixed-format bundle, and a missing
tensor (MissingRequiredTensor, nothing left allocated).
"""
import shutil
from pathlib import Path

import numpy as np
import pytest

from runtime_b200 import lfm2 as M
from tests import bundle_io as B

pytestmark = pytest.mark.gpu

BUNDLES = Path(__file__).resolve().parent / "golden" / "bundles"


@pytest.fixture(scope="module")
def be():
    from runtime_b200.backend import CudaBackend

    b = CudaBackend(0)
    yield b
    b.close()


def check_against_oracle(be, oracle, directory, weights, formats, steps=6, seed=3):
    cfg, _ = M.bundle_config(str(directory))
    cfg = cfg.with_(formats=formats, max_tokens=64)
    model = M.Lfm2Model.from_bundle(be, str(directory), max_tokens=64)
    ref = oracle.Lfm2Oracle(cfg, weights, threads=8)
    prompt = np.random.default_rng(seed).integers(0, cfg.vocab, size=9)
    st = model.new_state()
    st.append(prompt)
    ref_logits = ref.append(prompt)
    assert np.max(np.abs(st.logits() - ref_logits)) <= 1e-2
    tok = int(np.argmax(ref_logits))
    assert int(np.argmax(st.logits())) == tok
    got, want = [], []
    t_dev = t_ref = tok
    for _ in range(steps):
        st.append_argmax(t_dev)
        t_dev = int(st.read_sampled())
        s, _ = ref.append_argmax(t_ref)
        t_ref = int(s)
        got.append(t_dev)
        want.append(t_ref)
    assert got == want
    st.close()
    model.close()


@pytest.mark.parametrize("scheme", ["ternary", "nf4"])
def test_converter_bundles(be, oracle, scheme):
    d = BUNDLES / scheme
    cfg, _ = M.bundle_config(str(d))
    weights, formats = B.bundle_weights(d, cfg)
    check_against_oracle(be, oracle, d, weights, formats)


@pytest.mark.parametrize("dtype", ["F32", "BF16"])
def test_dense_bundles(be, oracle, tmp_path, dtype):
    cfg = M.tiny_config({r: "dense" for r in M.ROLES}, hidden=128, intermediate=256, q_heads=2, kv_heads=1,
                        vocab=96)
    w = M.synthetic_weights(cfg, 11)
    tensors = B.dense_tensors(cfg, w)
    B.write_config(tmp_path, cfg)
    B.write_safetensors(tmp_path / "model.safetensors", tensors, {"format": "pt"}, dtype=dtype)
    if dtype == "BF16":
        # The oracle sees the stored (rounded) values.
        w, formats = B.bundle_weights(tmp_path, M.bundle_config(str(tmp_path))[0])
    else:
        formats = {r: "dense" for r in M.ROLES}
    check_against_oracle(be, oracle, tmp_path, w, formats)


@pytest.mark.parametrize("formats,marker", [
    ({r: "int8" for r in M.ROLES}, "minifield.int8.v1"),
    ({"embedding": "int8", "conv_in": "nf4", "conv_out": "ternary", "q": "nf4", "k": "int8", "v": "int8",
      "o": "ternary", "w1": "ternary", "w2": "nf4", "w3": "ternary"}, "minifield.mixed.v1"),
], ids=["int8", "mixed"])
def test_packed_bundles_written_here(be, oracle, tmp_path, formats, marker):
    cfg = M.tiny_config(formats, vocab=128)
    w = M.synthetic_weights(cfg, 13)
    arrays = B.packed_tensors(cfg, w)   # scales stored as F16; w now holds the widened F16 values
    B.write_config(tmp_path, cfg)
    B.write_raw(tmp_path / "model.safetensors", arrays, {"format": marker})
    check_against_oracle(be, oracle, tmp_path, w, formats)


def test_missing_tensor_fails_without_leaking(be, tmp_path):
    from runtime_b200.backend import ExecutorError

    d = tmp_path / "b"
    shutil.copytree(BUNDLES / "ternary", d)
    tensors, meta = B.read_safetensors(d / "model.safetensors")
    del tensors["model.layers.1.feed_forward.w2.weight.codes"]
    B.write_raw(d / "model.safetensors", {k: np.ascontiguousarray(v) for k, v in tensors.items()}, meta)
    before = be.resource_report()
    with pytest.raises(ExecutorError) as e:
        M.Lfm2Model.from_bundle(be, str(d), max_tokens=32)
    assert e.value.status == 12   # MissingRequiredTensor
    assert be.resource_report() == before

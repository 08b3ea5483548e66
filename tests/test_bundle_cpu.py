"""The bundle loader's host side (no GPU): config.json and safetensors parsing.

The committed bundles in tests/golden/bundles were written by the
reference's own converter (tests/golden/make_bundles.py); the conversion
manifest it wrote pins the files and the tensor inventory.  The config
rules follow crates/executor-core/src/lfm2/config.rs (effective FF width:
the reference's own pinned 350M value, tests/config.rs:39), and malformed
inputs fail with the ExecutorError kinds of the reference loader.
"""
import ctypes as C
import hashlib
import json
import shutil
import struct
from pathlib import Path

import numpy as np
import pytest

from runtime_b200 import _lib
from runtime_b200 import lfm2 as M
from tests import bundle_io as B

BUNDLES = Path(__file__).resolve().parent / "golden" / "bundles"
INVALID_ARGUMENT, INVALID_SHAPE, INVALID_LAYOUT, INVALID_DTYPE = 1, 2, 3, 4
OUT_OF_BOUNDS, UNSUPPORTED, INVALID_TIE = 6, 7, 14


def status_of(directory, with_format=True):
    cfg = _lib.Lfm2Config()
    kinds = np.zeros(64, np.int32)
    fmt = C.create_string_buffer(64)
    return _lib.load().mf_bundle_config(str(directory).encode(), C.byref(cfg), kinds.ctypes.data, 64,
                                        fmt if with_format else None, 64 if with_format else 0)


@pytest.mark.parametrize("scheme,marker", [("ternary", "minifield.ternary.v1"), ("nf4", "minifield.nf4.v1")])
def test_config_of_converted_bundles(scheme, marker):
    d = BUNDLES / scheme
    cfg, fmt = M.bundle_config(str(d))
    raw = json.loads((d / "config.json").read_text())
    assert fmt == marker
    assert (cfg.hidden, cfg.intermediate, cfg.q_heads, cfg.kv_heads, cfg.vocab, cfg.conv_width) == (
        raw["hidden_size"], raw["intermediate_size"], raw["num_attention_heads"], raw["num_key_value_heads"],
        raw["vocab_size"], raw["conv_L_cache"])
    assert cfg.head_dim == raw["hidden_size"] // raw["num_attention_heads"]
    assert cfg.layer_types == ["conv" if t == "conv" else "attention" for t in raw["layer_types"]]
    assert cfg.rope_theta == np.float32(raw["rope_theta"])
    assert cfg.norm_eps == np.float32(raw["norm_eps"]) and cfg.block_eps == cfg.norm_eps


@pytest.mark.parametrize("scheme", ["ternary", "nf4"])
def test_bundle_files_match_the_converter_manifest(scheme):
    """The committed files are the converter's output (sha256 per file), and
    the test reader sees the manifest's tensor inventory."""
    d = BUNDLES / scheme
    manifest = json.loads((d / "conversion-manifest.json").read_text())
    for rec in manifest["files"]:
        data = (d / rec["path"]).read_bytes()
        assert len(data) == rec["bytes"] and hashlib.sha256(data).hexdigest() == rec["sha256"], rec["path"]
    tensors, meta = B.read_safetensors(d / "model.safetensors")
    assert meta["format"] == manifest["weight_format"]
    got = {n: (str(t.dtype), list(t.shape)) for n, t in tensors.items()}
    dt = {"U8": "uint8", "F16": "float16", "F32": "float32"}
    want = {r["name"]: (dt[r["dtype"]], r["shape"]) for r in manifest["tensors"]}
    assert got == want
    cfg, _ = M.bundle_config(str(d))
    weights, formats = B.bundle_weights(d, cfg)
    assert set(formats.values()) == {scheme}


def test_effective_ff_width_of_the_pinned_config(tmp_path):
    """crates/executor-core/tests/config.rs:39: raw 6656 with auto adjustment
    (multiplier 1.0, multiple of 256) gives 4608."""
    cfg = M.Lfm2Config(1024, 6656, 16, 8, 64, 65536, ["conv", "attention"], {})
    B.write_config(tmp_path, cfg, block_auto_adjust_ff_dim=True, block_ffn_dim_multiplier=1.0,
                   block_multiple_of=256)
    c = _lib.Lfm2Config()
    assert _lib.load().mf_bundle_config(str(tmp_path).encode(), C.byref(c), None, 0, None, 0) == 0
    assert c.intermediate == 4608 and c.hidden == 1024 and c.head_dim == 64


def _copy(tmp_path, scheme="ternary"):
    d = tmp_path / scheme
    shutil.copytree(BUNDLES / scheme, d)
    return d


@pytest.mark.parametrize("edit,status", [
    ({"model_type": "llama"}, UNSUPPORTED),
    ({"tie_word_embeddings": False}, INVALID_TIE),
    ({"num_hidden_layers": 3}, INVALID_ARGUMENT),
    ({"layer_types": ["conv", "sliding_attention"]}, UNSUPPORTED),
    ({"num_attention_heads": 3}, INVALID_SHAPE),
    ({"norm_eps": -1.0}, INVALID_ARGUMENT),
])
def test_config_errors(tmp_path, edit, status):
    d = _copy(tmp_path)
    c = json.loads((d / "config.json").read_text())
    c.update(edit)
    (d / "config.json").write_text(json.dumps(c))
    assert status_of(d) == status


def _rewrite_header(path, mutate):
    blob = path.read_bytes()
    (hlen,) = struct.unpack("<Q", blob[:8])
    header = json.loads(blob[8:8 + hlen])
    mutate(header)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    path.write_bytes(struct.pack("<Q", len(h)) + h + blob[8 + hlen:])


def test_safetensors_errors(tmp_path):
    d = _copy(tmp_path)
    st = d / "model.safetensors"
    good = st.read_bytes()
    st.write_bytes(good[:6])
    assert status_of(d) == INVALID_LAYOUT            # shorter than the length prefix
    st.write_bytes(struct.pack("<Q", 1 << 40) + good[8:])
    assert status_of(d) == INVALID_LAYOUT            # header length past the file
    st.write_bytes(good)
    _rewrite_header(st, lambda h: h["model.embedding_norm.weight"].__setitem__("dtype", "F64"))
    assert status_of(d) == INVALID_DTYPE
    st.write_bytes(good)
    _rewrite_header(st, lambda h: h["model.embedding_norm.weight"].__setitem__("data_offsets", [0, 1 << 30]))
    assert status_of(d) == OUT_OF_BOUNDS
    st.write_bytes(good)
    _rewrite_header(st, lambda h: h["__metadata__"].__setitem__("format", "minifield.ternary.v9"))
    assert status_of(d) == UNSUPPORTED
    st.write_bytes(good)
    assert status_of(d) == 0

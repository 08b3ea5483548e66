"""Writes tests/golden/bundles/{ternary,nf4}: tiny LFM2 bundles produced by the
reference's own converter (tools/converters, `convert_bundle`), for the
bundle-loader tests.

Run from the repository root with the reference checkout available:

    PYTHONPATH=<reference>/tools/converters/src python tests/golden/make_bundles.py <reference>

The dense source is seeded random-init weights of a two-layer model (one
conv block, one attention block) in the reference's canonical inventory;
the converter quantizes every matrix role (the tied embedding included) with
its ternary or NF4 quantizer, stores the scales as F16 and writes the
format metadata.  Only the converted bundles are committed.
"""
import json
import os
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "bundles"

CONFIG = {
    "model_type": "lfm2",
    "hidden_size": 128,
    "intermediate_size": 128,
    "num_attention_heads": 4,
    "num_key_value_heads": 2,
    "conv_L_cache": 3,
    "vocab_size": 64,
    "num_hidden_layers": 2,
    "layer_types": ["conv", "full_attention"],
    "rope_theta": 1000000.0,
    "tie_word_embeddings": True,
    "norm_eps": 1e-5,
    "block_auto_adjust_ff_dim": False,
    "conv_bias": False,
    "dtype": "float32",
    "bos_token_id": 1,
}


def main(reference: str) -> None:
    sys.path.insert(0, str(Path(reference) / "tools/converters/src"))
    from minifield_converters.bundle import convert_bundle
    from minifield_converters.config import validate_config
    from minifield_converters.container import Tensor, write_tensors
    from minifield_converters.fixture import fixture_tokenizer
    from minifield_converters.jsonio import json_bytes

    rng = np.random.default_rng(2026)
    inventory = validate_config(CONFIG).inventory()
    tensors = {}
    for name, shape in sorted(inventory.items()):
        if len(shape) == 1:
            values = (1.0 + 0.02 * rng.standard_normal(shape)).astype(np.float32)
        elif len(shape) == 3:   # conv kernel [hidden, 1, width]
            values = (0.1 * rng.standard_normal(shape)).astype(np.float32)
        else:
            values = (0.05 * rng.standard_normal(shape)).astype(np.float32)
        tensors[name] = Tensor.from_array(values)
    with tempfile.TemporaryDirectory() as tmp:
        src = Path(tmp) / "source"
        (src / "tokenizer").mkdir(parents=True)
        (src / "config.json").write_bytes(json_bytes(CONFIG))
        (src / "tokenizer" / "tokenizer.json").write_bytes(json_bytes(fixture_tokenizer()))
        write_tensors(src / "model.safetensors", tensors, {"format": "pt"})
        OUT.mkdir(exist_ok=True)
        for scheme in ("ternary", "nf4"):
            dst = OUT / scheme
            if dst.exists():
                shutil.rmtree(dst)
            manifest = convert_bundle(src, dst, scheme=scheme, source_model="synthetic/tiny-lfm2",
                                      source_revision="seed-2026")
            print(scheme, manifest["weight_format"], sum(f.stat().st_size for f in dst.rglob("*") if f.is_file()))
    print(json.dumps(CONFIG))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ["MF_REFERENCE"])

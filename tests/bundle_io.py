"""Safetensors bundle reading and writing in numpy, for the bundle-loader tests.

An independent reader of what the reference's converter writes
(tools/converters/src/minifield_converters/container.py: an 8-byte
little-endian header length, a JSON header of {name: {dtype, shape,
data_offsets}} plus string `__metadata__`, then the payloads), used to give
the CPU oracle the same weights the C++ loader uploads: packed roles as
U8 codes with F16 scales widened to F32 (an exact IEEE conversion, as the
reference loader's f16_to_f32), dense roles as F32.
"""
import json
import struct
from pathlib import Path

import numpy as np

DTYPES = {"F32": np.float32, "F16": np.float16, "U8": np.uint8, "I8": np.int8}


def read_safetensors(path):
    blob = Path(path).read_bytes()
    (hlen,) = struct.unpack("<Q", blob[:8])
    header = json.loads(blob[8:8 + hlen])
    meta = header.pop("__metadata__", {})
    base = 8 + hlen
    out = {}
    for name, t in header.items():
        b0, b1 = t["data_offsets"]
        raw = blob[base + b0:base + b1]
        if t["dtype"] == "BF16":
            v = (np.frombuffer(raw, np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            v = np.frombuffer(raw, DTYPES[t["dtype"]])
        out[name] = v.reshape(t["shape"])
    return out, meta


def write_safetensors(path, tensors, metadata, dtype="F32"):
    """Dense tensors as F32 or BF16 (round to nearest even), sorted names."""
    header = {"__metadata__": metadata}
    payload = []
    cursor = 0
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name], np.float32)
        if dtype == "BF16" and a.ndim >= 1:
            u = a.view(np.uint32).astype(np.uint64)
            u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
            raw, dt = u.tobytes(), "BF16"
        else:
            raw, dt = a.tobytes(), "F32"
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [cursor, cursor + len(raw)]}
        payload.append(raw)
        cursor += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    Path(path).write_bytes(struct.pack("<Q", len(h)) + h + b"".join(payload))


def bf16_round(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


FORMAT_OF_WIDTH = {4: "ternary", 2: "nf4", 1: "int8"}   # cols / code bytes per row


def _role(tensors, name, rows, cols):
    if name + ".codes" in tensors:
        codes = np.ascontiguousarray(tensors[name + ".codes"], np.uint8)
        scales = tensors[name + ".scales"].astype(np.float32)
        fmt = FORMAT_OF_WIDTH[cols // codes.shape[1]]
        return {"kind": "packed", "format": fmt, "codes": codes, "scales": np.ascontiguousarray(scales)}, fmt
    return {"kind": "dense", "value": tensors[name].astype(np.float32).reshape(rows, cols)}, "dense"


def bundle_weights(directory, cfg):
    """The weights dict of runtime_b200.lfm2 (synthetic_weights' layout) and
    the per-role formats, from a bundle directory."""
    tensors, _ = read_safetensors(Path(directory) / "model.safetensors")
    h, f, kvw = cfg.hidden, cfg.intermediate, cfg.kv_width
    formats = {}
    emb, formats["embedding"] = _role(tensors, "model.embed_tokens.weight", cfg.vocab, h)
    w = {"embedding": emb, "embedding_norm": tensors["model.embedding_norm.weight"].astype(np.float32),
         "layers": []}
    for i, kind in enumerate(cfg.layer_types):
        p = f"model.layers.{i}"
        lw = {}
        if kind == "conv":
            lw["in_proj"], formats["conv_in"] = _role(tensors, p + ".conv.in_proj.weight", 3 * h, h)
            lw["out_proj"], formats["conv_out"] = _role(tensors, p + ".conv.out_proj.weight", h, h)
            lw["conv_kernel"] = tensors[p + ".conv.conv.weight"].astype(np.float32).reshape(h, cfg.conv_width)
        else:
            for role, short, rows in (("q_proj", "q", h), ("k_proj", "k", kvw), ("v_proj", "v", kvw),
                                      ("out_proj", "o", h)):
                lw[short], formats[short] = _role(tensors, f"{p}.self_attn.{role}.weight", rows, h)
            lw["q_norm"] = tensors[p + ".self_attn.q_layernorm.weight"].astype(np.float32)
            lw["k_norm"] = tensors[p + ".self_attn.k_layernorm.weight"].astype(np.float32)
        lw["w1"], formats["w1"] = _role(tensors, p + ".feed_forward.w1.weight", f, h)
        lw["w2"], formats["w2"] = _role(tensors, p + ".feed_forward.w2.weight", h, f)
        lw["w3"], formats["w3"] = _role(tensors, p + ".feed_forward.w3.weight", f, h)
        lw["ffn_norm"] = tensors[p + ".ffn_norm.weight"].astype(np.float32)
        lw["operator_norm"] = tensors[p + ".operator_norm.weight"].astype(np.float32)
        w["layers"].append(lw)
    return w, formats


def dense_tensors(cfg, weights):
    """Canonical tensor names of a dense synthetic weights dict."""
    t = {"model.embed_tokens.weight": weights["embedding"]["value"],
         "model.embedding_norm.weight": weights["embedding_norm"]}
    for i, (kind, lw) in enumerate(zip(cfg.layer_types, weights["layers"])):
        p = f"model.layers.{i}"
        if kind == "conv":
            t[p + ".conv.in_proj.weight"] = lw["in_proj"]["value"]
            t[p + ".conv.out_proj.weight"] = lw["out_proj"]["value"]
            t[p + ".conv.conv.weight"] = lw["conv_kernel"].reshape(cfg.hidden, 1, cfg.conv_width)
        else:
            for role, short in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"), ("out_proj", "o")):
                t[f"{p}.self_attn.{role}.weight"] = lw[short]["value"]
            t[p + ".self_attn.q_layernorm.weight"] = lw["q_norm"]
            t[p + ".self_attn.k_layernorm.weight"] = lw["k_norm"]
        for role in ("w1", "w2", "w3"):
            t[f"{p}.feed_forward.{role}.weight"] = lw[role]["value"]
        t[p + ".ffn_norm.weight"] = lw["ffn_norm"]
        t[p + ".operator_norm.weight"] = lw["operator_norm"]
    return t


def write_config(directory, cfg, **extra):
    c = {"model_type": "lfm2", "hidden_size": cfg.hidden, "intermediate_size": cfg.intermediate,
         "num_attention_heads": cfg.q_heads, "num_key_value_heads": cfg.kv_heads,
         "conv_L_cache": cfg.conv_width, "vocab_size": cfg.vocab, "num_hidden_layers": len(cfg.layer_types),
         "layer_types": ["conv" if k == "conv" else "full_attention" for k in cfg.layer_types],
         "rope_theta": cfg.rope_theta, "tie_word_embeddings": True, "norm_eps": cfg.norm_eps,
         "block_norm_eps": cfg.block_eps, "dtype": "float32"}
    c.update(extra)
    Path(directory).mkdir(parents=True, exist_ok=True)
    (Path(directory) / "config.json").write_text(json.dumps(c))


def write_raw(path, arrays, metadata):
    """Tensors stored as given: {name: numpy array of float32 / float16 / uint8}."""
    names = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.uint8): "U8"}
    header = {"__metadata__": metadata}
    payload, cursor = [], 0
    for name in sorted(arrays):
        a = np.ascontiguousarray(arrays[name])
        raw = a.tobytes()
        header[name] = {"dtype": names[a.dtype], "shape": list(a.shape), "data_offsets": [cursor, cursor + len(raw)]}
        payload.append(raw)
        cursor += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    Path(path).write_bytes(struct.pack("<Q", len(h)) + h + b"".join(payload))


def packed_tensors(cfg, weights):
    """Canonical tensor names of a synthetic weights dict with packed roles
    (codes U8 and F16 scales, as the converter stores them) and the weights
    the loader will see (scales rounded to F16)."""
    t = dense_tensors_any(cfg, weights)
    out, seen = {}, {}
    for name, v in t.items():
        if isinstance(v, dict):
            if v["kind"] == "packed":
                s16 = v["scales"].astype(np.float16)
                out[name + ".codes"] = np.ascontiguousarray(v["codes"], np.uint8)
                out[name + ".scales"] = s16
                v["scales"] = s16.astype(np.float32)
            else:
                out[name] = np.ascontiguousarray(v["value"], np.float32)
        else:
            out[name] = np.ascontiguousarray(v, np.float32)
    return out


def dense_tensors_any(cfg, weights):
    """Like dense_tensors, but keeps role dicts (packed or dense) as values."""
    t = {"model.embed_tokens.weight": weights["embedding"], "model.embedding_norm.weight": weights["embedding_norm"]}
    for i, (kind, lw) in enumerate(zip(cfg.layer_types, weights["layers"])):
        p = f"model.layers.{i}"
        if kind == "conv":
            t[p + ".conv.in_proj.weight"] = lw["in_proj"]
            t[p + ".conv.out_proj.weight"] = lw["out_proj"]
            t[p + ".conv.conv.weight"] = lw["conv_kernel"].reshape(cfg.hidden, 1, cfg.conv_width)
        else:
            for role, short in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"), ("out_proj", "o")):
                t[f"{p}.self_attn.{role}.weight"] = lw[short]
            t[p + ".self_attn.q_layernorm.weight"] = lw["q_norm"]
            t[p + ".self_attn.k_layernorm.weight"] = lw["k_norm"]
        for role in ("w1", "w2", "w3"):
            t[f"{p}.feed_forward.{role}.weight"] = lw[role]
        t[p + ".ffn_norm.weight"] = lw["ffn_norm"]
        t[p + ".operator_norm.weight"] = lw["operator_norm"]
    return t

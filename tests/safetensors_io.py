"""Minimal safetensors writer for the loader tests (format: 8-byte
little-endian header length, JSON header of dtype / shape / data_offsets,
then the raw little-endian tensor bytes)."""
import json
import os
import struct

import numpy as np

ROLE_NAMES = {0: "model.embed_tokens.weight", 12: "model.norm.weight", 13: "lm_head.weight"}
LAYER_ROLES = {1: "self_attn.q_proj", 2: "self_attn.k_proj", 3: "self_attn.v_proj",
               4: "self_attn.o_proj", 5: "self_attn.q_norm", 6: "self_attn.k_norm",
               7: "mlp.gate_proj", 8: "mlp.up_proj", 9: "mlp.down_proj",
               10: "input_layernorm", 11: "post_attention_layernorm"}


def weight_name(layer, role):
    if layer < 0:
        return ROLE_NAMES[role]
    return f"model.layers.{layer}.{LAYER_ROLES[role]}.weight"


def f16_bits_to_bf16_bits(bits):
    """FP16 bit patterns -> BF16 bit patterns (round to nearest even)."""
    f = np.asarray(bits, np.uint16).view(np.float16).astype(np.float32).view(np.uint32)
    rounded = f + 0x7FFF + ((f >> 16) & 1)
    return (rounded >> 16).astype(np.uint16)


def bf16_bits_to_f16_bits(bits):
    """BF16 bit patterns -> FP16 (through FP32, round to nearest even)."""
    f = (np.asarray(bits, np.uint32) << 16).view(np.float32)
    return f.astype(np.float16).view(np.uint16)


def write(path, tensors):
    """tensors: {name: (dtype, shape, uint16 bits or raw bytes)}"""
    header, blobs, off = {}, [], 0
    for name, (dtype, shape, data) in tensors.items():
        raw = data if isinstance(data, (bytes, bytearray)) else np.ascontiguousarray(data).tobytes()
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_config(directory, cfg, **overrides):
    c = {"model_type": "qwen3", "attention_bias": False}
    c.update({k: (bool(v) if k == "tie_word_embeddings" else v) for k, v in cfg.items()})
    c.update(overrides)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(c, f)

"""Safetensors loading (Qwen3Model::load, weights.rs:21-75): a random-init
model exported to a checkpoint loads back bit for bit (F16, one file or
shards with an index), BF16 tensors are converted through FP32 with
round-to-nearest-even, and malformed checkpoints fail with the reference's
error kinds."""
import json
import os

import numpy as np
import pytest

import metal_infer as mi
import oracle as O
from conftest import INPUT_STREAM
import safetensors_io as st

pytestmark = pytest.mark.gpu

ROLE_OF = {v: k for k, v in mi.ROLES.items()}


def small_cfg(**kw):
    cfg = dict(mi.QWEN3_0_6B)
    cfg.update(num_hidden_layers=2, vocab_size=4096, **kw)
    return cfg


def weights_of(model, cfg):
    out = {}
    roles = [(-1, 0), (-1, 12)] + ([] if cfg["tie_word_embeddings"] else [(-1, 13)])
    for layer in range(cfg["num_hidden_layers"]):
        roles += [(layer, r) for r in range(1, 12)]
    for layer, role in roles:
        w = model.weight(layer, ROLE_OF[role])
        out[st.weight_name(layer, role)] = (list(w.shape()), w.f16_bits().ravel())
    return out


def export(model, cfg, directory, shards=1, bf16=False):
    os.makedirs(directory, exist_ok=True)
    st.write_config(directory, cfg)
    tensors = weights_of(model, cfg)
    names = sorted(tensors)
    files = {}
    for i, name in enumerate(names):
        shape, bits = tensors[name]
        data = st.f16_bits_to_bf16_bits(bits) if bf16 else bits
        fname = "model.safetensors" if shards == 1 else f"model-{i % shards:05d}-of-{shards:05d}.safetensors"
        files.setdefault(fname, {})[name] = ("BF16" if bf16 else "F16", shape, data)
    for fname, t in files.items():
        st.write(os.path.join(directory, fname), t)
    if shards > 1:
        index = {"weight_map": {n: f for f, t in files.items() for n in t}}
        with open(os.path.join(directory, "model.safetensors.index.json"), "w") as f:
            json.dump(index, f)
    return tensors


@pytest.mark.parametrize("tie,shards", [(1, 1), (0, 3)])
def test_exported_checkpoint_loads_bit_exact(ctx, tmp_path, tie, shards):
    cfg = small_cfg(tie_word_embeddings=tie)
    model = mi.Qwen3Model.random(ctx, cfg, seed=21)
    export(model, cfg, str(tmp_path), shards=shards)
    loaded = mi.Qwen3Model.load(str(tmp_path), ctx)
    assert loaded.config()["hidden_size"] == cfg["hidden_size"]
    prompt = O.gen_tokens(21, INPUT_STREAM, 17, cfg["vocab_size"])
    a = model.prefill(prompt, model.kv_cache(64)).f16_bits()
    b = loaded.prefill(prompt, loaded.kv_cache(64)).f16_bits()
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(model.generate(prompt, 8, model.kv_cache(64)),
                                  loaded.generate(prompt, 8, loaded.kv_cache(64)))


def test_bf16_tensors_convert_through_f32_round_to_nearest_even(ctx, tmp_path):
    cfg = small_cfg(tie_word_embeddings=0)
    model = mi.Qwen3Model.random(ctx, cfg, seed=22)
    tensors = export(model, cfg, str(tmp_path), bf16=True)
    loaded = mi.Qwen3Model.load(str(tmp_path), ctx)
    for layer, role in ((-1, 0), (-1, 13), (0, 1), (1, 9), (1, 5)):
        _, bits = tensors[st.weight_name(layer, role)]
        want = st.bf16_bits_to_f16_bits(st.f16_bits_to_bf16_bits(bits))
        np.testing.assert_array_equal(loaded.weight(layer, ROLE_OF[role]).f16_bits().ravel(), want)


def test_malformed_checkpoints_fail_with_reference_error_kinds(ctx, tmp_path):
    cfg = small_cfg(tie_word_embeddings=1)
    model = mi.Qwen3Model.random(ctx, cfg, seed=23)
    base = str(tmp_path / "ok")
    tensors = export(model, cfg, base)

    def case(name, mutate):
        d = str(tmp_path / name)
        os.makedirs(d)
        st.write_config(d, cfg)
        t = {k: ("F16", v[0], v[1]) for k, v in tensors.items()}
        mutate(d, t)
        if t is not None:
            st.write(os.path.join(d, "model.safetensors"), t)
        with pytest.raises(mi.CoreError) as e:
            mi.Qwen3Model.load(d, ctx)
        return e.value.status

    assert case("missing", lambda d, t: t.pop("model.layers.1.mlp.up_proj.weight")) == \
        mi.ERR_MISSING_TENSOR
    def wrong_shape(d, t):
        dt, shape, bits = t["model.norm.weight"]
        t["model.norm.weight"] = (dt, [shape[0] // 2], bits[: shape[0] // 2])
    assert case("shape", wrong_shape) == mi.ERR_CONFIG
    def f32(d, t):
        dt, shape, bits = t["model.norm.weight"]
        t["model.norm.weight"] = ("F32", shape, np.ones(shape, np.float32))
    assert case("f32", f32) == mi.ERR_UNSUPPORTED
    assert case("type", lambda d, t: st.write_config(d, cfg, model_type="llama")) == \
        mi.ERR_UNSUPPORTED
    empty = str(tmp_path / "empty")
    os.makedirs(empty)
    st.write_config(empty, cfg)
    with pytest.raises(mi.CoreError) as e:
        mi.Qwen3Model.load(empty, ctx)
    assert e.value.status == mi.ERR_UNSUPPORTED
    with pytest.raises(mi.CoreError) as e:
        mi.Qwen3Model.load(str(tmp_path / "nowhere"), ctx)
    assert e.value.status == mi.ERR_IO

"""GPU parity of the Qwen3 forward (prefill + greedy decode) against the oracle.

Bars: identical greedy token ids over the decode
horizon; logits within 1e-2 relative and hidden states per op within 2e-3.
The decode path and prompts up to 512 tokens run the engine's canonical
arithmetic, which the oracle restates, so logits, caches and hidden states
are compared bit for bit (a stronger bar than the tolerances).
"""
import json
import os

import numpy as np
import pytest

import metal_infer as mi
import oracle as O
from conftest import INPUT_STREAM

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
LOGIT_REL = 1e-2
HIDDEN_REL = 2e-3


def rel_err(actual_bits, expected_bits):
    a = O.f32(np.asarray(actual_bits).ravel())
    e = O.f32(np.asarray(expected_bits).ravel())
    return float(np.max(np.abs(a - e)) / max(float(np.max(np.abs(e))), 1e-6))


def exact(actual_bits, expected_bits):
    a = np.asarray(actual_bits, np.uint16).ravel()
    e = np.asarray(expected_bits, np.uint16).ravel()
    bad = np.nonzero(a != e)[0]
    assert a.shape == e.shape and bad.size == 0, (
        f"{bad.size} values differ (rel err {rel_err(a, e):.2e}); first at {bad[:1]}")


def small_cfg(layers=2, vocab=4096, **kw):
    cfg = dict(mi.QWEN3_0_6B)
    cfg.update(num_hidden_layers=layers, vocab_size=vocab, **kw)
    return cfg


@pytest.fixture(scope="module")
def small(ctx):
    cfg = small_cfg()
    model = mi.Qwen3Model.random(ctx, cfg, seed=5)
    ref = O.Qwen3(cfg, seed=5, capacity=256)
    return cfg, model, ref


def test_weights_match_oracle_bit_exact(small):
    cfg, model, ref = small
    for layer, role in ((-1, "embedding"), (0, "q"), (1, "down"), (1, "k_norm")):
        w = model.weight(layer, role)
        np.testing.assert_array_equal(w.f16_bits().ravel(),
                                      ref.weight(layer, role, w.shape()).ravel())


@pytest.mark.parametrize("prompt_len", [1, 7, 31, 32, 45])
def test_prefill_logits_and_cache_match_oracle(small, prompt_len):
    cfg, model, ref = small
    prompt = O.gen_tokens(5, INPUT_STREAM, prompt_len, cfg["vocab_size"])
    cache = model.kv_cache(256)
    logits = model.prefill(prompt, cache).f16_bits()
    ref.reset()
    ref_logits = ref.forward(prompt)
    exact(logits, ref_logits)
    assert len(cache) == prompt_len
    k0, v0 = cache.layer(1)
    exact(k0.f16_bits().reshape(256, -1)[:prompt_len], ref.cache(1, False, prompt_len))
    exact(v0.f16_bits().reshape(256, -1)[:prompt_len], ref.cache(1, True, prompt_len))


def set_path(model, path):
    """Decode through the persistent kernel or the kernel chain (graph/eager)."""
    model.set_decode_persistent(path == "persistent")
    model.set_decode_graphs(path != "eager")


@pytest.mark.parametrize("path", ["persistent", "graph", "eager"])
def test_decode_logits_match_oracle(small, path):
    cfg, model, ref = small
    set_path(model, path)
    try:
        prompt = O.gen_tokens(5, INPUT_STREAM + 1, 40, cfg["vocab_size"])
        cache = model.kv_cache(256)
        model.prefill(prompt, cache)
        ref.reset()
        ref.forward(prompt)
        for step in range(12):
            tok = int((step * 7919 + 13) % cfg["vocab_size"])
            logits = model.decode(tok, cache).f16_bits()
            ref_logits = ref.forward(np.array([tok], np.uint32))
            exact(logits, ref_logits)
        assert len(cache) == 52
    finally:
        set_path(model, "persistent")


def mi_argmax(bits):
    return O.argmax(np.asarray(bits).ravel())


def divergence_report(model, ref, prompt, ids, ref_ids, capacity):
    """Where two greedy sequences part, with both sides' logits at that step
    (teacher-forced with the common prefix)."""
    n = min(len(ids), len(ref_ids))
    d = next((i for i in range(n) if ids[i] != ref_ids[i]), None)
    if d is None:
        return f"lengths differ: {len(ids)} vs {len(ref_ids)}"
    cache = model.kv_cache(capacity)
    g = model.prefill(prompt, cache).f16_bits().ravel()
    ref.reset()
    r = ref.forward(prompt)
    for i in range(d):
        g = model.decode(int(ref_ids[i]), cache).f16_bits().ravel()
        r = ref.forward(np.array([ref_ids[i]], np.uint32))
    rf, gf = O.f32(r), O.f32(g)
    top = np.argsort(-rf, kind="stable")[:3]
    return (f"first divergence at step {d}: gpu {int(ids[d])} oracle {int(ref_ids[d])}; "
            f"oracle top3 {[(int(t), float(rf[t])) for t in top]}; gpu at those "
            f"{[float(gf[t]) for t in top]}; teacher-forced gpu argmax {mi_argmax(g)}; "
            f"logits rel err {rel_err(g, r):.2e}")


def test_greedy_tokens_match_oracle_small(small):
    cfg, model, ref = small
    prompt = O.gen_tokens(5, INPUT_STREAM + 2, 33, cfg["vocab_size"])
    cache = model.kv_cache(256)
    ids = model.generate(prompt, 64, cache)
    ref_ids = ref.generate_greedy(prompt, 64)
    if not np.array_equal(ids, ref_ids):
        pytest.fail(divergence_report(model, ref, prompt, ids, ref_ids, 256))
    assert len(cache) == 33 + 63


def test_graph_and_eager_decode_are_bit_identical(small):
    cfg, model, _ = small
    prompt = O.gen_tokens(5, INPUT_STREAM + 3, 20, cfg["vocab_size"])
    outs = []
    for graphs in (True, False):
        model.set_decode_graphs(graphs)
        cache = model.kv_cache(128)
        model.prefill(prompt, cache)
        outs.append(np.stack([model.decode(int(t), cache).f16_bits().ravel()
                              for t in (5, 77, 901, 4000)]))
    model.set_decode_graphs(True)
    np.testing.assert_array_equal(outs[0], outs[1])


def test_persistent_decode_is_active_for_qwen3_shapes(small):
    _, model, _ = small
    assert model.decode_persistent()


@pytest.mark.parametrize("capacity,prompt_len", [(128, 20), (9000, 150)])
def test_decode_paths_bit_identical(small, capacity, prompt_len):
    """Persistent kernel vs kernel chain: ids, last logits and the K/V cache."""
    cfg, model, _ = small
    prompt = O.gen_tokens(5, INPUT_STREAM + 6, prompt_len, cfg["vocab_size"])
    outs = {}
    try:
        for path in ("persistent", "graph", "eager"):
            set_path(model, path)
            cache = model.kv_cache(capacity)
            ids = model.generate(prompt, 24, cache)
            logits = model.decode(int(ids[-1]), cache).f16_bits().ravel()
            k1, v1 = cache.layer(1)
            n = len(cache)
            outs[path] = (ids, logits, k1.f16_bits().reshape(capacity, -1)[:n],
                          v1.f16_bits().reshape(capacity, -1)[:n])
    finally:
        set_path(model, "persistent")
    for path in ("graph", "eager"):
        for a, b in zip(outs["persistent"], outs[path]):
            np.testing.assert_array_equal(a, b)
    ref_ids = O.Qwen3(cfg, seed=5, capacity=capacity).generate_greedy(prompt, 24)
    np.testing.assert_array_equal(outs["persistent"][0], ref_ids)


def test_decode_paths_bit_identical_8b_shapes(ctx):
    """Qwen3-8B layer shapes (hidden 4096, intermediate 12288, 32/8 heads):
    persistent kernel vs kernel chain vs the oracle."""
    cfg = dict(mi.QWEN3_8B)
    cfg.update(num_hidden_layers=2, vocab_size=4096)
    model = mi.Qwen3Model.random(ctx, cfg, seed=13)
    assert model.decode_persistent()
    prompt = O.gen_tokens(13, INPUT_STREAM, 24, cfg["vocab_size"])
    outs = {}
    try:
        for path in ("persistent", "graph"):
            set_path(model, path)
            cache = model.kv_cache(128)
            ids = model.generate(prompt, 12, cache)
            outs[path] = (ids, model.decode(int(ids[-1]), cache).f16_bits().ravel())
    finally:
        set_path(model, "persistent")
    for a, b in zip(outs["persistent"], outs["graph"]):
        np.testing.assert_array_equal(a, b)
    ref = O.Qwen3(cfg, seed=13, capacity=128)
    np.testing.assert_array_equal(outs["persistent"][0], ref.generate_greedy(prompt, 12))


def test_pipelined_decode_argmax_matches_generate(ctx, small):
    cfg, model, _ = small
    prompt = O.gen_tokens(5, INPUT_STREAM + 4, 24, cfg["vocab_size"])
    cache = model.kv_cache(128)
    want = model.generate(prompt, 10, cache)
    slots = ctx.tensor_u32(np.full(11, 0xFFFFFFFF, np.uint32), [11])
    model.prefill_argmax(prompt, cache, slots.slice_1d(0, 1))
    pending = None
    for step in range(9):
        _, pending = model.decode_argmax(slots.slice_1d(step, 1), cache, slots.slice_1d(step + 1, 1))
    pending.wait()
    np.testing.assert_array_equal(slots.to_u32_vec()[:10], want)


def test_generate_with_stop_tokens_rolls_back_cache(small):
    cfg, model, _ = small
    prompt = O.gen_tokens(5, INPUT_STREAM + 5, 16, cfg["vocab_size"])
    cache = model.kv_cache(128)
    full = model.generate(prompt, 12, cache)
    stop = int(full[5])
    first = int(np.nonzero(full == stop)[0][0])
    got = model.generate_with(prompt, {"max_tokens": 12, "stop_token_ids": [stop]}, cache)
    np.testing.assert_array_equal(got, full[:first])
    assert len(cache) == 16 + first
    seen = []
    got = model.generate_with(prompt, {"max_tokens": 12}, cache,
                              on_token=lambda t: seen.append(t) or len(seen) < 3)
    np.testing.assert_array_equal(got, full[:3])
    assert len(cache) == 16 + 2


def test_cache_capacity_error(small):
    cfg, model, _ = small
    cache = model.kv_cache(8)
    with pytest.raises(mi.ModelError) as e:
        model.prefill(np.arange(9), cache)
    assert e.value.status == mi.ERR_CACHE_CAPACITY
    model.prefill(np.arange(8), cache)
    with pytest.raises(mi.ModelError) as e:
        model.decode(3, cache)
    assert e.value.status == mi.ERR_CACHE_CAPACITY
    assert len(cache) == 8


def test_unfused_options_match_oracle(ctx):
    cfg = small_cfg(layers=2)
    model = mi.Qwen3Model.random(ctx, cfg, seed=6)
    model.set_fusion_options(mi.FusionOptions.none())
    ref = O.Qwen3(cfg, seed=6, capacity=128)
    ref.set_fusion(qk_rope_cache=False, add_rms_norm=False)
    prompt = O.gen_tokens(6, INPUT_STREAM, 35, cfg["vocab_size"])
    cache = model.kv_cache(128)
    exact(model.prefill(prompt, cache).f16_bits(), ref.forward(prompt))
    for tok in (3, 99, 1234):
        exact(model.decode(tok, cache).f16_bits(), ref.forward(np.array([tok], np.uint32)))


@pytest.mark.parametrize("heads", [(32, 8), (64, 8), (16, 16)])
def test_gqa_ratios_decode(ctx, heads):
    qh, kvh = heads
    cfg = small_cfg(layers=1, hidden_size=512, intermediate_size=1024, num_attention_heads=qh,
                    num_key_value_heads=kvh, tie_word_embeddings=0)
    model = mi.Qwen3Model.random(ctx, cfg, seed=7)
    ref = O.Qwen3(cfg, seed=7, capacity=128)
    prompt = O.gen_tokens(7, INPUT_STREAM, 40, cfg["vocab_size"])
    ids = model.generate(prompt, 16, model.kv_cache(128))
    np.testing.assert_array_equal(ids, ref.generate_greedy(prompt, 16))


def test_config0_one_block_matches_oracle(ctx):
    with open(os.path.join(GOLDEN, "block0.json")) as f:
        meta = json.load(f)
    golden = np.load(os.path.join(GOLDEN, "block0_hidden.npy"))
    cfg = meta["config"]
    model = mi.Qwen3Model.random(ctx, cfg, seed=0)
    cache = model.kv_cache(2048)
    h = cfg["hidden_size"]
    outs = []
    x = ctx.tensor_f16_bits(O.gen_normal_f16(0, INPUT_STREAM, 64 * h, 1.0), [64, h])
    outs.append(model.forward_hidden(x, cache).f16_bits())
    for step in range(16):
        x = ctx.tensor_f16_bits(O.gen_normal_f16(0, INPUT_STREAM + 1 + step, h, 1.0), [1, h])
        outs.append(model.forward_hidden(x, cache).f16_bits())
    got = np.concatenate([o.reshape(-1, h) for o in outs])
    assert got.shape == golden.shape
    exact(got, golden)
    assert len(cache) == 80


def test_config2_greedy_tokens_identical_to_golden(ctx):
    """Full Qwen3-0.6B (seed 2): 128-token prompt, 256 decode steps."""
    with open(os.path.join(GOLDEN, "qwen3_0_6b_greedy.json")) as f:
        g = json.load(f)
    cfg = g["config"]
    model = mi.Qwen3Model.random(ctx, cfg, seed=g["seed"])
    prompt = O.gen_tokens(g["seed"], g["prompt_stream"], g["prompt_len"], cfg["vocab_size"])
    cache = model.kv_cache(2048)
    logits = model.prefill(prompt, cache).f16_bits().ravel()
    exact(logits[:16], np.array(g["prefill_logits_head"], np.uint16))
    ids = model.generate(prompt, g["max_tokens"], cache)
    want = np.array(g["ids"], np.uint32)
    if not np.array_equal(ids, want):
        ref = O.Qwen3(cfg, seed=g["seed"], capacity=2048)
        pytest.fail(divergence_report(model, ref, prompt, ids, want, 2048))
    assert len(cache) == 128 + 256

"""GPU parity of on-device sampling against the oracle (sample_token /
sample_token_f16 / sample_candidates, qwen3.rs:909-1005; XorShift64,
qwen3.rs:1011-1034; generate_with, qwen3.rs:441-473): identical tokens and
XorShift64 states for every case, sampled generation token-identical to the
oracle's (whose logits the engine reproduces bit for bit)."""
import time

import numpy as np
import pytest

import metal_infer as mi
import oracle as O
from conftest import INPUT_STREAM
from sampling_cases import OPTIONS, SMALL_CASES, VOCAB_CASES, logits_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", SMALL_CASES + VOCAB_CASES)
def test_sample_logits_matches_oracle(ctx, case):
    for sd in range(2):
        bits = logits_case(case, seed=sd)
        t = ctx.tensor_f16_bits(bits, [bits.size])
        for temperature, top_p, top_k in OPTIONS:
            st_o = st_g = O.xorshift_seed(100 + sd)
            for _ in range(3):
                tok_o, st_o = O.sample(bits, temperature, top_p, top_k, st_o)
                tok_g, st_g = ctx.sample_logits(t, temperature, top_p, top_k, st_g)
                assert (tok_g, st_g) == (tok_o, st_o), (case, sd, temperature, top_p, top_k)


def test_sample_logits_zero_temperature_and_reference_cases(ctx):
    # qwen3.rs:1083-1099
    t = ctx.tensor_f16([1.0, 4.0, 2.0], [3])
    assert ctx.sample_logits(t, 0.0, state=5) == (1, 5)
    assert ctx.sample_logits(t, 1.0, top_k=1, state=mi.xorshift_seed(1))[0] == 1
    # [1, n] logits (the model's output shape) are accepted
    t2 = ctx.tensor_f16([1.0, 4.0, 2.0], [1, 3])
    assert ctx.sample_logits(t2, 1.0, top_k=1, state=3)[0] == 1


def test_sample_logits_errors(ctx):
    t = ctx.tensor_f16_bits(logits_case("all_nonfinite"), [4])
    with pytest.raises(mi.ModelError) as e:
        ctx.sample_logits(t, 1.0, state=3)
    assert e.value.status == mi.ERR_CONFIG and "no finite value" in str(e.value)
    ok = ctx.tensor_f16([0.0, 1.0], [2])
    for temperature, top_p, text in ((-1.0, 1.0, "temperature"), (float("nan"), 1.0, "temperature"),
                                     (1.0, 1.5, "top_p"), (1.0, float("nan"), "top_p")):
        with pytest.raises(mi.ModelError) as e:
            ctx.sample_logits(ok, temperature, top_p, state=3)
        assert e.value.status == mi.ERR_CONFIG and text in str(e.value)


def test_histogram_is_cleared_between_draws(ctx):
    # the sampler clears the key histogram it consumed: repeated draws on
    # different logits stay exact
    st_o = st_g = O.xorshift_seed(4)
    for case in ("ties", "normal", "zeros", "ties"):
        bits = logits_case(case, seed=9)
        t = ctx.tensor_f16_bits(bits, [bits.size])
        tok_o, st_o = O.sample(bits, 1.0, 1.0, 0, st_o)
        tok_g, st_g = ctx.sample_logits(t, 1.0, 1.0, 0, st_g)
        assert (tok_g, st_g) == (tok_o, st_o)


def small_cfg(layers=2, vocab=4096):
    cfg = dict(mi.QWEN3_0_6B)
    cfg.update(num_hidden_layers=layers, vocab_size=vocab)
    return cfg


@pytest.fixture(scope="module")
def small(ctx):
    cfg = small_cfg()
    return cfg, mi.Qwen3Model.random(ctx, cfg, seed=5), O.Qwen3(cfg, seed=5, capacity=256)


@pytest.mark.parametrize("path", ["persistent", "graph", "eager"])
@pytest.mark.parametrize("opts", [dict(temperature=0.8, top_p=0.95, top_k=50, seed=7),
                                  dict(temperature=1.0, top_p=1.0, top_k=0, seed=0),
                                  dict(temperature=0.6, top_p=0.5, top_k=0, seed=3)])
def test_generate_sampled_matches_oracle(small, path, opts):
    cfg, model, ref = small
    model.set_decode_persistent(path == "persistent")  # sampled decode uses the chain
    model.set_decode_graphs(path != "eager")
    try:
        prompt = O.gen_tokens(5, INPUT_STREAM + 21, 13, cfg["vocab_size"])
        got = model.generate_with(prompt, dict(opts, max_tokens=20), model.kv_cache(128))
        want = ref.generate_sampled(prompt, 20, opts["temperature"], opts["top_p"],
                                    opts["top_k"], opts["seed"])
        np.testing.assert_array_equal(got, want)
        # greedy afterwards is unaffected (and runs the persistent kernel again)
        np.testing.assert_array_equal(model.generate(prompt, 6, model.kv_cache(128)),
                                      ref.generate_greedy(prompt, 6))
    finally:
        model.set_decode_persistent(True)
        model.set_decode_graphs(True)


def test_generate_sampled_stop_token_and_callback(small):
    cfg, model, _ = small
    opts = dict(temperature=1.0, top_p=0.9, top_k=100, seed=21)
    prompt = O.gen_tokens(5, INPUT_STREAM + 22, 16, cfg["vocab_size"])
    cache = model.kv_cache(128)
    full = model.generate_with(prompt, dict(opts, max_tokens=12), cache)
    assert len(cache) == 16 + 11
    stop = int(full[5])
    first = int(np.nonzero(full == stop)[0][0])
    got = model.generate_with(prompt, dict(opts, max_tokens=12, stop_token_ids=[stop]), cache)
    np.testing.assert_array_equal(got, full[:first])
    assert len(cache) == 16 + first
    seen = []
    got = model.generate_with(prompt, dict(opts, max_tokens=12), cache,
                              on_token=lambda t: seen.append(t) or len(seen) < 3)
    np.testing.assert_array_equal(got, full[:3])
    assert len(cache) == 16 + 2
    assert model.generate_with(prompt, dict(opts, max_tokens=0), cache).size == 0
    with pytest.raises(mi.ModelError) as e:
        model.generate_with(prompt, dict(opts, top_p=1.5), cache)
    assert e.value.status == mi.ERR_CONFIG


def test_generate_sampled_full_vocabulary(ctx):
    # Qwen3's 151936-entry vocabulary, all candidates (top_k 0, top_p 1)
    cfg = small_cfg(layers=1, vocab=151936)
    model = mi.Qwen3Model.random(ctx, cfg, seed=8)
    ref = O.Qwen3(cfg, seed=8, capacity=64)
    prompt = O.gen_tokens(8, INPUT_STREAM + 23, 9, cfg["vocab_size"])
    got = model.generate_with(prompt, dict(max_tokens=10, temperature=1.0, seed=99),
                              model.kv_cache(64))
    want = ref.generate_sampled(prompt, 10, 1.0, 1.0, 0, 99)
    np.testing.assert_array_equal(got, want)


def test_sampler_latency_report(ctx):
    """Not a bar: wall time of one synchronous mi_sample_logits call on the
    full vocabulary (allocation, histogram, sampler, readback)."""
    bits = logits_case("vocab_normal", seed=1)
    t = ctx.tensor_f16_bits(bits, [bits.size])
    for top_k, top_p in ((0, 1.0), (20, 0.95)):
        ctx.sample_logits(t, 0.7, top_p, top_k, 3)
        t0 = time.perf_counter()
        for _ in range(20):
            ctx.sample_logits(t, 0.7, top_p, top_k, 3)
        print(f"sample_logits top_k={top_k} top_p={top_p}: "
              f"{(time.perf_counter() - t0) / 20 * 1e6:.0f} us per call")

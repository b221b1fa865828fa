"""CPU tests of the sampling oracle (sample_token / sample_token_f16 /
sample_candidates, crates/metal-infer-models/src/qwen3.rs:909-1034): the
reference's own unit tests (qwen3.rs:1083-1099), a line-by-line Python
restatement of the algorithm, and the distribution it draws from."""
import numpy as np
import pytest

import oracle as O
from sampling_cases import (OPTIONS, SMALL_CASES, VOCAB, logits_case, order_key,
                            reference_sample, xorshift_next)

pytestmark = pytest.mark.timeout(600)


def test_zero_temperature_is_greedy():
    # qwen3.rs:1083-1088
    token, _ = O.sample(O.f16_bits([1.0, 4.0, 2.0]), 0.0, state=O.xorshift_seed(1))
    assert token == 1


def test_top_k_one_is_greedy_even_with_temperature():
    # qwen3.rs:1090-1099
    token, _ = O.sample(O.f16_bits([1.0, 4.0, 2.0]), 1.0, top_k=1, state=O.xorshift_seed(1))
    assert token == 1


def test_xorshift_stream():
    # XorShift64 (qwen3.rs:1011-1034): seed 0 maps to the golden-ratio constant
    assert O.xorshift_seed(0) == 0x9E3779B97F4A7C15
    assert O.xorshift_seed(5) == 5
    s = 1
    s, u = xorshift_next(s)
    assert s == 1082269761 and 0.0 <= u < 1.0
    # the oracle advances the state once per draw
    _, st = O.sample(O.f16_bits([0.0, 0.0]), 1.0, state=1)
    assert st == 1082269761


@pytest.mark.parametrize("case", SMALL_CASES)
@pytest.mark.parametrize("opt", OPTIONS)
def test_oracle_matches_restatement(case, opt):
    temperature, top_p, top_k = opt
    bits = logits_case(case, seed=3)
    state_o = state_r = O.xorshift_seed(11)
    for _ in range(4):
        tok_o, state_o = O.sample(bits, temperature, top_p, top_k, state_o)
        tok_r, state_r = reference_sample(bits, temperature, top_p, top_k, state_r)
        assert tok_o == (0xFFFFFFFF if tok_r is None else tok_r)
        assert state_o == state_r


def test_oracle_matches_restatement_full_vocabulary():
    bits = logits_case("vocab_flat", seed=1)
    st_o = st_r = O.xorshift_seed(2)
    for temperature, top_p, top_k in [(1.0, 1.0, 0), (0.8, 0.999, 0)]:
        tok_o, st_o = O.sample(bits, temperature, top_p, top_k, st_o)
        tok_r, st_r = reference_sample(bits, temperature, top_p, top_k, st_r)
        assert (tok_o, st_o) == (tok_r, st_r)


def test_no_finite_logit():
    tok, st = O.sample(logits_case("all_nonfinite"), 1.0, state=7)
    assert tok == 0xFFFFFFFF and st == 7  # the draw never happens


def test_equal_logits_order_by_index():
    # four equal candidates: equal bit patterns are walked in index order, so
    # the draw u picks index floor(4 u)
    bits = O.f16_bits([1.0] * 4)
    state = O.xorshift_seed(9)
    for _ in range(50):
        nxt, u = xorshift_next(state)
        tok, state = O.sample(bits, 1.0, state=state)
        assert state == nxt
        assert tok == min(3, int(u * 4.0))


def test_plus_zero_precedes_minus_zero():
    # total_cmp: +0 > -0, so with top_k 1 the +0 logit is kept
    bits = np.array([0x8000, 0x0000, 0x8000], np.uint16)
    tok, _ = O.sample(bits, 1.0, top_k=1, state=3)
    assert tok == 1


def test_distribution_matches_softmax():
    values = np.array([0.0, 1.0, 2.0, -1.0, 0.5], np.float32)
    bits = O.f16_bits(values)
    counts = np.zeros(values.size)
    state = O.xorshift_seed(42)
    draws = 40000
    for _ in range(draws):
        tok, state = O.sample(bits, 0.8, state=state)
        counts[tok] += 1
    p = np.exp(values / 0.8)
    p /= p.sum()
    expected = p * draws
    chi2 = float(((counts - expected) ** 2 / expected).sum())
    assert chi2 < 25.0, (counts, expected)  # 4 degrees of freedom


def test_top_k_and_top_p_restrict_support():
    bits = logits_case("normal", seed=5)
    keys = order_key(bits)
    order = sorted(range(bits.size), key=lambda i: (-int(keys[i]), i))
    state = O.xorshift_seed(8)
    seen = set()
    for _ in range(300):
        tok, state = O.sample(bits, 1.0, top_k=5, state=state)
        seen.add(tok)
    assert seen <= set(order[:5])


def test_oracle_generate_sampled_is_seeded():
    cfg = dict(hidden_size=64, intermediate_size=128, num_hidden_layers=2,
               num_attention_heads=4, num_key_value_heads=2, head_dim=16, rms_norm_eps=1e-6,
               rope_theta=1e6, vocab_size=256, tie_word_embeddings=1)
    m = O.Qwen3(cfg, seed=4, capacity=64, std=0.5)
    prompt = np.array([1, 2, 3], np.uint32)
    a = m.generate_sampled(prompt, 12, 1.0, 0.95, 40, seed=5)
    b = m.generate_sampled(prompt, 12, 1.0, 0.95, 40, seed=5)
    c = m.generate_sampled(prompt, 12, 1.0, 0.95, 40, seed=6)
    assert a.size == 12 and np.array_equal(a, b) and not np.array_equal(a, c)
    assert int(a.max()) < cfg["vocab_size"]
    # seed 0 is XorShift64::new(0)
    d = m.generate_sampled(prompt, 6, 1.0, 1.0, 0, seed=0)
    e = m.generate_sampled(prompt, 6, 1.0, 1.0, 0, seed=0x9E3779B97F4A7C15)
    assert np.array_equal(d, e)
    assert VOCAB == 151936


@pytest.mark.parametrize("case", ["normal", "ties", "zeros", "peaked"])
@pytest.mark.parametrize("opt", [(1.0, 1.0, 0), (0.6, 0.9, 0), (2.5, 0.5, 0), (0.05, 1.0, 0)])
def test_parallel_pass_algorithm_matches_sequential(case, opt):
    """The GPU sampler's scan + event algorithm (restated in sampler_model)
    picks the same candidate as the sequential oracle, with chunks of 8
    groups so that chunk boundaries, binade crossings, ties and jumps occur."""
    from sampler_model import sample_model
    temperature, top_p, _ = opt
    bits = logits_case(case, seed=4)
    finite = (bits & 0x7C00) != 0x7C00
    keys = [int(k) for k in order_key(bits)[finite]]
    vals = {}
    inv = np.float32(1.0) / np.float32(temperature)

    def value(key):
        b = (key & 0x7FFF) if key & 0x8000 else ((~key) & 0xFFFF)
        return np.array([b], np.uint16).view(np.float16).astype(np.float32)[0]
    kmax = max(keys)

    def weight(key):
        if key not in vals:
            z = np.float32(np.float32(value(key) - value(kmax)) * inv)
            vals[key] = float(O.exp(np.array([z], np.float32))[0])
        return vals[key]
    state = O.xorshift_seed(21)
    for _ in range(5):
        tok, nxt = O.sample(bits, temperature, top_p, 0, state)
        _, u = xorshift_next(state)
        state = nxt
        gkeys, stop = sample_model(keys, weight, float(np.float32(top_p)), u)
        assert stop is not None
        key = gkeys[stop[0]]
        b = (key & 0x7FFF) if key & 0x8000 else ((~key) & 0xFFFF)
        idx = int(np.nonzero(bits == b)[0][stop[1]])
        assert idx == tok

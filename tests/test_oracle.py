"""CPU tests of the oracle: the known-answer vectors and inline CPU formulas of
crates/metal-infer-core/tests/gpu.rs, restated, plus internal consistency of
the fused and unfused reference paths."""
import numpy as np
import pytest

import oracle as O


def f16(values):
    return O.f16_bits(values)


def close(actual_bits, expected, tol=0.02):
    a = O.f32(actual_bits).ravel()
    e = np.asarray(expected, np.float32).ravel()
    assert a.shape == e.shape
    assert np.max(np.abs(a - e)) <= tol, np.max(np.abs(a - e))


def test_matmul_known_answer():
    # gpu.rs:78-86
    x = f16([1, 2, 3, 4]).reshape(2, 2)
    w = f16([5, 6, 7, 8]).reshape(2, 2)
    np.testing.assert_array_equal(O.f32(O.matmul(x, w)).ravel(), [17, 23, 39, 53])


def test_matvec_known_answer():
    # gpu.rs:130-139
    x = f16([1, 2, 3]).reshape(1, 3)
    w = f16([4, 5, 6, 7, 8, 9]).reshape(2, 3)
    np.testing.assert_array_equal(O.f32(O.matmul(x, w)).ravel(), [32, 50])


def test_vectorized_matvec_matches_cpu_formula():
    # gpu.rs:161-185: N=257, K=128
    xv = np.arange(128, dtype=np.float32) / 128.0 - 0.5
    wv = (np.arange(257 * 128) % 31).astype(np.float32) / 31.0 - 0.5
    out = O.matmul(f16(xv).reshape(1, 128), f16(wv).reshape(257, 128))
    expected = (wv.reshape(257, 128) * xv).sum(axis=1)
    close(out, expected)


@pytest.mark.parametrize("size", [1, 2, 31, 32, 33, 2048, 2049, 151936])
def test_argmax_known_answers(size):
    # gpu.rs:8-55
    bits = ((np.arange(size, dtype=np.uint64) * 1103 + 17) & 0xFFFF).astype(np.uint16)
    bits[0] = 0x7C00
    if size > 1:
        bits[1] = 0x7E00
        bits[size // 2] = 0x7BFF
        bits[-1] = 0x7BFF
    else:
        bits[0] = 0
    vals = bits.view(np.float16).astype(np.float32)
    finite = np.isfinite(vals)
    if finite.any():
        # max by value; ties -> last index (max_by keeps the last maximum)
        m = vals[finite].max()
        expected = int(np.nonzero(finite & (vals == m))[0][-1])
    else:
        expected = 0xFFFFFFFF
    assert O.argmax(bits) == expected


def test_argmax_signed_zero_and_nonfinite():
    assert O.argmax(np.array([0x8000, 0], np.uint16)) == 1
    assert O.argmax(np.array([0x7C00, 0x7E00], np.uint16)) == 0xFFFFFFFF


def test_embedding_missing_token_is_zero():
    # gpu.rs:57-75
    table = f16([1.0, 2.0]).reshape(1, 2)
    out = O.embedding(np.array([0xFFFFFFFF], np.uint32), table)
    np.testing.assert_array_equal(O.f32(out).ravel(), [0, 0])
    out = O.embedding(np.array([0], np.uint32), table)
    np.testing.assert_array_equal(O.f32(out).ravel(), [1, 2])


def test_rms_norm_matches_cpu_formula():
    # gpu.rs:247-270
    xv = (np.arange(3 * 65) % 23).astype(np.float32) / 11.0 - 1.0
    wv = 0.5 + np.arange(65, dtype=np.float32) / 130.0
    out = O.rms_norm(f16(xv).reshape(3, 65), f16(wv), 1e-6)
    rows = xv.reshape(3, 65)
    scale = 1.0 / np.sqrt((rows * rows).sum(axis=1, keepdims=True) / 65.0 + 1e-6)
    close(out, rows * scale * wv)


def test_fused_add_rms_norm_matches_individual_ops():
    # gpu.rs:355-377
    left = f16([1.0, -2.0, 3.0, 0.5, 0.25, -0.75]).reshape(2, 3)
    right = f16([0.5, 1.0, -1.0, 1.5, -0.25, 0.5]).reshape(2, 3)
    w = f16([0.5, 1.0, 1.5])
    exp_res = O.add(left, right)
    exp_norm = O.rms_norm(exp_res, w, 1e-6)
    res, norm = O.add_rms_norm(left, right, w, 1e-6)
    close(res, O.f32(exp_res))
    close(norm, O.f32(exp_norm))


def _weights(rows, k, modulus):
    return f16((np.arange(rows * k) % modulus).astype(np.float32) / modulus - 0.5).reshape(rows, k)


def test_fused_decode_norm_projections_match_separate_ops():
    # gpu.rs:379-453
    iv = (np.arange(256) % 29).astype(np.float32) / 29.0 - 0.5
    rv = (np.arange(256) % 19).astype(np.float32) / 38.0 - 0.25
    nv = 0.5 + (np.arange(256) % 17).astype(np.float32) / 34.0
    x, right, norm = f16(iv).reshape(1, 256), f16(rv).reshape(1, 256), f16(nv)
    w0, w1, w2 = _weights(40, 256, 31), _weights(24, 256, 37), _weights(16, 256, 41)
    normalized = O.rms_norm(x, norm, 1e-6)
    outs = O.rms_norm_matmul3(x, norm, w0, w1, w2, 1e-6)
    for w, o in zip((w0, w1, w2), outs):
        np.testing.assert_array_equal(o, O.matmul(normalized, w))
    res, normd = O.add_rms_norm(x, right, norm, 1e-6)
    r2, g, u = O.add_rms_norm_matmul2(x, right, norm, w0, w1, 1e-6)
    np.testing.assert_array_equal(r2, res)
    np.testing.assert_array_equal(g, O.matmul(normd, w0))
    np.testing.assert_array_equal(u, O.matmul(normd, w1))


def test_fused_qk_transform_matches_individual_ops():
    # gpu.rs:519-560 (offset 1, theta 1e4)
    q = f16(np.arange(32, dtype=np.float32) / 16.0 - 1.0).reshape(2, 2, 8)
    k = f16(np.arange(16, dtype=np.float32) / 12.0 - 0.5).reshape(2, 1, 8)
    nw = f16(0.75 + np.arange(8, dtype=np.float32) / 16.0)
    exp_q = O.rope(O.rms_norm(q, nw, 1e-6), 1, 1e4)
    exp_k = O.rope(O.rms_norm(k, nw, 1e-6), 1, 1e4)
    exp_cache = np.zeros((4, 1, 8), np.uint16)
    O.copy_into_cache(exp_k, exp_cache, 1)
    cache = np.zeros((4, 1, 8), np.uint16)
    out = O.qk_norm_rope_cache(q, k, nw, nw, cache, 1, 1e4, 1e-6)
    close(out, O.f32(exp_q))
    close(cache, O.f32(exp_cache))


def test_swiglu_formula():
    g = f16(np.linspace(-4, 4, 97))
    u = f16(np.linspace(2, -2, 97))
    gf, uf = O.f32(g), O.f32(u)
    close(O.swiglu(g, u), gf / (1 + np.exp(-gf)) * uf, tol=2e-3)


@pytest.mark.parametrize("head_dim", [1, 2, 4, 8, 16, 32, 64, 128, 256])
@pytest.mark.parametrize("tokens,length", [(1, 1), (31, 31), (32, 32), (33, 33), (63, 63),
                                           (64, 64), (65, 65), (33, 65)])
def test_flash_prefill_semantics_match_reference(head_dim, tokens, length):
    # gpu.rs:681-727
    qh, kvh = 4, 2
    q = f16((np.arange(tokens * qh * head_dim) % 43) / 43.0 - 0.5)
    k = f16((np.arange(length * kvh * head_dim) % 37) / 37.0 - 0.25)
    v = f16((np.arange(length * kvh * head_dim) % 29) / 29.0 - 0.5)
    ref = O.attention(q, k, v, qh, kvh, head_dim, True, length - tokens, O.REFERENCE)
    flash = O.attention(q, k, v, qh, kvh, head_dim, True, length - tokens, O.FLASH_PREFILL)
    close(flash, O.f32(ref))


def test_attention_known_small_case():
    # tiled_attention_matches_reference (gpu.rs:580-611): with a single key
    # the output equals V.
    q = f16((np.arange(2 * 128) % 43) / 43.0 - 0.5)
    k = f16((np.arange(128) % 37) / 37.0 - 0.25)
    v = f16((np.arange(128) % 29) / 29.0)
    out = O.attention(q, k, v, 2, 1, 128, True, 0)
    np.testing.assert_array_equal(out.reshape(2, 128)[0], v)
    np.testing.assert_array_equal(out.reshape(2, 128)[1], v)


def test_generator_is_counter_based():
    a = O.gen_normal_f16(7, 3, 1000, 0.02)
    b = O.gen_normal_f16(7, 3, 500, 0.02, offset=250)
    np.testing.assert_array_equal(a[250:750], b)
    vals = O.f32(a)
    assert abs(vals.mean()) < 0.003 and 0.017 < vals.std() < 0.023
    t = O.gen_tokens(2, 1 << 20, 4096, 151936)
    assert t.max() < 151936 and len(np.unique(t)) > 4000


def test_half_add_is_correctly_rounded():
    # add_f16 adds in half precision; numpy's float16 addition is correctly
    # rounded, so the two must agree bit for bit on random finite pairs.
    rng = np.random.default_rng(0)
    a = rng.integers(0, 0x7BFF, 20000).astype(np.uint16) | (rng.integers(0, 2, 20000) << 15).astype(np.uint16)
    b = rng.integers(0, 0x7BFF, 20000).astype(np.uint16) | (rng.integers(0, 2, 20000) << 15).astype(np.uint16)
    with np.errstate(over="ignore"):
        expected = (a.view(np.float16) + b.view(np.float16)).view(np.uint16)
    np.testing.assert_array_equal(O.add(a, b), expected)


def test_exp_accuracy_and_special_values():
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.uniform(-104, 88.5, 200000), rng.uniform(-1, 1, 100000),
                        -np.abs(rng.standard_normal(100000)) * 10]).astype(np.float32)
    got = O.exp(x).astype(np.float64)
    want = np.exp(x.astype(np.float64))
    ok = want > np.finfo(np.float32).tiny  # normal results
    ulp = np.spacing(want[ok].astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(got[ok] - want[ok]) / ulp) <= 2.0
    special = O.exp(np.array([0.0, -np.inf, np.inf, 100.0, -200.0, np.nan], np.float32))
    assert special[0] == 1.0 and special[1] == 0.0 and np.isinf(special[2])
    assert np.isinf(special[3]) and special[4] == 0.0 and np.isnan(special[5])


def test_canonical_dot_order_and_fast_path():
    rng = np.random.default_rng(2)
    for k in (8, 65, 128, 256, 1024, 3072):
        x = f16(rng.standard_normal(k))
        w = f16(rng.standard_normal(k) * 0.02)
        xf, wf = O.f32(x), O.f32(w)
        # the matmul's vector path equals the scalar canonical DOT bit for bit
        got = O.matmul(x.reshape(1, k), w.reshape(1, k))[0, 0]
        assert got == f16([O.dot(xf, wf)])[0]
        assert abs(O.dot(xf, wf) - float(np.dot(xf.astype(np.float64), wf))) < 1e-4


def test_rope_terms_are_double_precision_trig():
    for pos, pair in ((0, 0), (1, 5), (777, 31), (33000, 63), (2047, 17)):
        c, s = O.rope_cs(pos, pair, 128, 1e6)
        freq = np.float32(1e6 ** np.float64(np.float32(-(2 * pair)) / np.float32(128)))
        ang = np.float32(np.float32(pos) * freq)
        assert c == np.float32(np.cos(np.float64(ang))) and s == np.float32(np.sin(np.float64(ang)))


@pytest.mark.parametrize("length", [1, 63, 64, 65, 300, 2048])
def test_flash_decode_semantics_match_reference(length):
    rng = np.random.default_rng(length)
    q = f16(rng.standard_normal(16 * 128))
    k = f16(rng.standard_normal(length * 8 * 128))
    v = f16(rng.standard_normal(length * 8 * 128))
    ref = O.attention(q, k, v, 16, 8, 128, True, length - 1)
    for block in (32, 64, 256):
        got = O.attention_decode(q, k, v, 16, 8, 128, block=block)
        close(got, O.f32(ref), tol=4e-3)


def test_f16_conversion_round_to_nearest_even():
    vals = np.array([1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11, 65519.0, 65520.0, 2.0 ** -25,
                     3 * 2.0 ** -26, -0.0], np.float32)
    np.testing.assert_array_equal(f16(vals), vals.astype(np.float16).view(np.uint16))

"""Seeded logit vectors and option grids for the sampling parity tests
(sample_token_f16 + sample_candidates, qwen3.rs:927-1005), plus a plain
Python restatement of that algorithm used to pin the C++ oracle."""
import numpy as np

import oracle as O

VOCAB = 151936
MASK64 = (1 << 64) - 1


def _f16(values) -> np.ndarray:
    return np.asarray(values, np.float32).astype(np.float16).view(np.uint16)


def logits_case(name: str, seed: int = 0) -> np.ndarray:
    """FP16 logit bits of one named shape of input."""
    r = np.random.default_rng(seed)
    if name == "normal":
        return _f16(r.normal(0.0, 3.0, 1000))
    if name == "ties":  # few distinct values: large equal-logit groups
        return _f16(r.integers(-5, 6, 2000))
    if name == "nonfinite":
        v = r.normal(0.0, 2.0, 500).astype(np.float32)
        v[r.integers(0, 500, 40)] = np.inf
        v[r.integers(0, 500, 40)] = -np.inf
        v[r.integers(0, 500, 40)] = np.nan
        return _f16(v)
    if name == "zeros":  # +0 and -0 order by total_cmp (+0 first)
        bits = np.where(r.random(300) < 0.5, 0x0000, 0x8000).astype(np.uint16)
        bits[r.integers(0, 300, 30)] = _f16(r.normal(0.0, 0.5, 30))
        return bits
    if name == "single":
        return _f16([r.normal()])
    if name == "peaked":
        v = r.normal(0.0, 1.0, 5000)
        v[r.integers(0, 5000)] = 20.0
        return _f16(v)
    if name == "vocab_normal":
        return _f16(r.normal(0.0, 2.0, VOCAB))
    if name == "vocab_flat":
        # 140000 logits at 0 push the FP64 total past 2^17, where the
        # weights of the tail (about 2^-13) round, half of them as ties
        v = np.zeros(VOCAB, np.float32)
        tail = r.choice(VOCAB, VOCAB - 140000, replace=False)
        v[tail] = r.uniform(-10.0, -8.0, tail.size)
        return _f16(v)
    if name == "vocab_wide":  # many distinct values over a wide range
        return _f16(r.uniform(-30.0, 30.0, VOCAB))
    if name == "all_nonfinite":
        return _f16([np.inf, -np.inf, np.nan, np.inf])
    raise ValueError(name)


SMALL_CASES = ["normal", "ties", "nonfinite", "zeros", "single", "peaked"]
VOCAB_CASES = ["vocab_normal", "vocab_flat", "vocab_wide"]

# (temperature, top_p, top_k)
OPTIONS = [
    (1.0, 1.0, 0), (0.7, 0.95, 20), (0.6, 0.9, 0), (2.5, 1.0, 0), (1.0, 1.0, 1),
    (1.0, 0.0, 0), (0.3, 0.5, 1000), (1.0, 1.0, 10 ** 6), (1.3, 0.999, 50), (0.05, 1.0, 0),
]


def order_key(bits: np.ndarray) -> np.ndarray:
    b = bits.astype(np.uint32)
    return np.where(b & 0x8000, (~b) & 0xFFFF, b | 0x8000)


def xorshift_next(state: int):
    v = state
    v ^= (v << 13) & MASK64
    v ^= v >> 7
    v ^= (v << 17) & MASK64
    return v, float(v) / 18446744073709551616.0


def reference_sample(bits: np.ndarray, temperature: float, top_p: float, top_k: int,
                     state: int):
    """sample_candidates (qwen3.rs:941-1005) line by line in Python: FP32
    weights through the engine's exp, FP64 sums, XorShift64 draw. Equal bit
    patterns keep ascending index order. Returns (token or None, state)."""
    bits = np.asarray(bits, np.uint16)
    if temperature == 0.0:
        return O.argmax(bits), state
    values = bits.view(np.float16).astype(np.float32)
    keys = order_key(bits)
    idx = [i for i in range(bits.size) if np.isfinite(values[i])]
    if not idx:
        return None, state
    idx.sort(key=lambda i: (-int(keys[i]), i))
    if top_k > 0 and len(idx) > top_k:
        idx = idx[:top_k]
    vals = values[idx]
    max_logit = vals[0]
    inverse = np.float32(1.0) / np.float32(temperature)
    z = ((vals - max_logit).astype(np.float32) * inverse).astype(np.float32)
    weights = [float(w) for w in O.exp(z)]
    total = 0.0
    for w in weights:
        total += w
    if np.float32(top_p) < 1.0:
        threshold = total * float(np.float32(top_p))
        cumulative, keep = 0.0, 0
        for w in weights:
            cumulative += w
            keep += 1
            if cumulative >= threshold:
                break
        keep = max(keep, 1)
        idx, weights = idx[:keep], weights[:keep]
        total = -0.0
        for w in weights:
            total += w
    state, u = xorshift_next(state)
    target = u * total
    for i, w in zip(idx, weights):
        target -= w
        if target <= 0.0:
            return i, state
    return 0xFFFFFFFE, state

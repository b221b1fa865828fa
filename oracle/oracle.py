"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU
legs import this module as the checker or the CPU baseline; the engine never
does. Every array is numpy; FP16 tensors travel as uint16 bit patterns.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_f32p = ctypes.POINTER(ctypes.c_float)
_sz = ctypes.c_size_t


class Qwen3Config(ctypes.Structure):
    _fields_ = [
        ("hidden_size", ctypes.c_uint32),
        ("intermediate_size", ctypes.c_uint32),
        ("num_hidden_layers", ctypes.c_uint32),
        ("num_attention_heads", ctypes.c_uint32),
        ("num_key_value_heads", ctypes.c_uint32),
        ("head_dim", ctypes.c_uint32),
        ("rms_norm_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("vocab_size", ctypes.c_uint32),
        ("tie_word_embeddings", ctypes.c_uint32),
    ]


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.or_argmax.restype = ctypes.c_uint32
        L.or_num_threads.restype = ctypes.c_int
        L.or_dot.restype = ctypes.c_float
        L.or_decode_block.restype = _sz
        L.or_decode_streams.restype = _sz
        L.or_qwen3_create_random.restype = ctypes.c_void_p
        L.or_qwen3_create_random.argtypes = [ctypes.POINTER(Qwen3Config), ctypes.c_uint64,
                                             ctypes.c_double, _sz]
        L.or_qwen3_destroy.argtypes = [ctypes.c_void_p]
        L.or_qwen3_set_fusion.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.or_qwen3_set_tp.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        L.or_qwen3_reset.argtypes = [ctypes.c_void_p]
        L.or_qwen3_truncate.argtypes = [ctypes.c_void_p, _sz]
        L.or_qwen3_len.argtypes = [ctypes.c_void_p]
        L.or_qwen3_len.restype = _sz
        L.or_qwen3_forward.argtypes = [ctypes.c_void_p, _u32p, _sz, _u16p]
        L.or_qwen3_forward_hidden.argtypes = [ctypes.c_void_p, _u16p, _sz, _u16p]
        L.or_qwen3_generate_greedy.argtypes = [ctypes.c_void_p, _u32p, _sz, _sz, _u32p]
        L.or_qwen3_generate_greedy.restype = _sz
        L.or_qwen3_generate_sampled.argtypes = [ctypes.c_void_p, _u32p, _sz, _sz, ctypes.c_float,
                                                ctypes.c_float, _sz, ctypes.c_uint64, _u32p]
        L.or_qwen3_generate_sampled.restype = _sz
        L.or_sample_f16.argtypes = [_u16p, _sz, ctypes.c_float, ctypes.c_float, _sz,
                                    ctypes.POINTER(ctypes.c_uint64)]
        L.or_sample_f16.restype = ctypes.c_uint32
        L.or_xorshift_seed.argtypes = [ctypes.c_uint64]
        L.or_xorshift_seed.restype = ctypes.c_uint64
        L.or_qwen3_weight.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.or_qwen3_weight.restype = _u16p
        L.or_qwen3_cache.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.or_qwen3_cache.restype = _u16p
        L.or_gen_normal_f16.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, _sz,
                                        ctypes.c_double, _u16p]
        L.or_gen_tokens.argtypes = [ctypes.c_uint64, ctypes.c_uint64, _sz, ctypes.c_uint32, _u32p]
        _lib = L
    return _lib


def _p16(a: np.ndarray):
    assert a.dtype == np.uint16 and a.flags.c_contiguous
    return a.ctypes.data_as(_u16p)


def _p32(a: np.ndarray):
    assert a.dtype == np.uint32 and a.flags.c_contiguous
    return a.ctypes.data_as(_u32p)


def f16_bits(values) -> np.ndarray:
    """FP32 values -> FP16 bit patterns (round to nearest even)."""
    a = np.ascontiguousarray(np.asarray(values, dtype=np.float32).ravel())
    out = np.empty(a.size, dtype=np.uint16)
    lib().or_f16_from_f32(a.ctypes.data_as(_f32p), _p16(out), _sz(a.size))
    return out


def f32(bits: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def set_accumulate_f64(enabled: bool) -> None:
    lib().or_set_accumulate_f64(ctypes.c_int(int(enabled)))


def gen_normal_f16(seed: int, stream: int, n: int, std: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    lib().or_gen_normal_f16(seed, stream, offset, n, std, _p16(out))
    return out


def gen_tokens(seed: int, stream: int, n: int, vocab: int) -> np.ndarray:
    out = np.empty(n, dtype=np.uint32)
    lib().or_gen_tokens(seed, stream, n, vocab, _p32(out))
    return out


# ---- ops ------------------------------------------------------------------

def matmul(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    m, k = x.shape
    n, k2 = w.shape
    assert k == k2
    x = np.ascontiguousarray(x, np.uint16)
    w = np.ascontiguousarray(w, np.uint16)
    out = np.empty((m, n), np.uint16)
    lib().or_matmul(_p16(x), _sz(m), _sz(k), _p16(w), _sz(n), _p16(out))
    return out


def add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, np.uint16)
    b = np.ascontiguousarray(b, np.uint16)
    out = np.empty_like(a)
    lib().or_add(_p16(a), _p16(b), _sz(a.size), _p16(out))
    return out


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.uint16)
    width = x.shape[-1]
    out = np.empty_like(x)
    lib().or_rms_norm(_p16(x), _sz(x.size // width), _sz(width), _p16(np.ascontiguousarray(w)),
                      ctypes.c_float(eps), _p16(out))
    return out


def add_rms_norm(left, right, w, eps):
    left = np.ascontiguousarray(left, np.uint16)
    right = np.ascontiguousarray(right, np.uint16)
    width = left.shape[-1]
    residual = np.empty_like(left)
    normalized = np.empty_like(left)
    lib().or_add_rms_norm(_p16(left), _p16(right), _sz(left.size // width), _sz(width),
                          _p16(np.ascontiguousarray(w)), ctypes.c_float(eps), _p16(residual),
                          _p16(normalized))
    return residual, normalized


def rms_norm_matmul3(x, norm_w, w0, w1, w2, eps):
    k = x.size
    outs = [np.empty((1, w.shape[0]), np.uint16) for w in (w0, w1, w2)]
    lib().or_rms_norm_matmul3(_p16(np.ascontiguousarray(x)), _sz(k), _p16(np.ascontiguousarray(norm_w)),
                              _p16(w0), _sz(w0.shape[0]), _p16(w1), _sz(w1.shape[0]),
                              _p16(w2), _sz(w2.shape[0]), ctypes.c_float(eps),
                              _p16(outs[0]), _p16(outs[1]), _p16(outs[2]))
    return tuple(outs)


def add_rms_norm_matmul2(left, right, norm_w, w0, w1, eps):
    k = left.size
    residual = np.empty((1, k), np.uint16)
    out0 = np.empty((1, w0.shape[0]), np.uint16)
    out1 = np.empty((1, w1.shape[0]), np.uint16)
    lib().or_add_rms_norm_matmul2(_p16(np.ascontiguousarray(left)), _p16(np.ascontiguousarray(right)),
                                  _sz(k), _p16(np.ascontiguousarray(norm_w)), _p16(w0),
                                  _sz(w0.shape[0]), _p16(w1), _sz(w1.shape[0]),
                                  ctypes.c_float(eps), _p16(residual), _p16(out0), _p16(out1))
    return residual, out0, out1


def swiglu(gate, up):
    gate = np.ascontiguousarray(gate, np.uint16)
    up = np.ascontiguousarray(up, np.uint16)
    out = np.empty_like(gate)
    lib().or_swiglu(_p16(gate), _p16(up), _sz(gate.size), _p16(out))
    return out


def embedding(tokens, table):
    tokens = np.ascontiguousarray(tokens, np.uint32)
    table = np.ascontiguousarray(table, np.uint16)
    rows, width = table.shape
    out = np.empty((tokens.size, width), np.uint16)
    lib().or_embedding(_p32(tokens), _sz(tokens.size), _p16(table), _sz(rows), _sz(width), _p16(out))
    return out


def argmax(logits) -> int:
    logits = np.ascontiguousarray(logits, np.uint16)
    return int(lib().or_argmax(_p16(logits), _sz(logits.size)))


def xorshift_seed(seed: int) -> int:
    """XorShift64::new (qwen3.rs:1016-1024)."""
    return int(lib().or_xorshift_seed(seed))


def sample(logits, temperature: float, top_p: float = 1.0, top_k: int = 0, state: int = 1):
    """One sampled token from FP16 logit bits (qwen3.rs:909-1005); returns
    (token, next state). Token 0xFFFFFFFF: no finite logit; 0xFFFFFFFE: the
    walk ended without a token."""
    logits = np.ascontiguousarray(logits, np.uint16)
    st = ctypes.c_uint64(state)
    tok = lib().or_sample_f16(_p16(logits), _sz(logits.size), temperature, top_p, top_k,
                              ctypes.byref(st))
    return int(tok), int(st.value)


def rope(x, offset, theta):
    x = np.ascontiguousarray(x, np.uint16)
    t, hh, hd = x.shape
    out = np.empty_like(x)
    lib().or_rope(_p16(x), _sz(t), _sz(hh), _sz(hd), _sz(offset), ctypes.c_float(theta), _p16(out))
    return out


def qk_norm_rope_cache(q, k, q_w, k_w, key_cache, offset, theta, eps):
    """Returns the rotated query; writes rotated keys into key_cache in place."""
    q = np.ascontiguousarray(q, np.uint16)
    k = np.ascontiguousarray(k, np.uint16)
    t, qh, hd = q.shape
    kvh = k.shape[1]
    assert key_cache.flags.c_contiguous and key_cache.dtype == np.uint16
    out = np.empty_like(q)
    lib().or_qk_norm_rope_cache(_p16(q), _p16(k), _sz(t), _sz(qh), _sz(kvh), _sz(hd),
                                _p16(np.ascontiguousarray(q_w)), _p16(np.ascontiguousarray(k_w)),
                                _sz(offset), ctypes.c_float(theta), ctypes.c_float(eps),
                                _sz(key_cache.shape[0]), _p16(out), _p16(key_cache))
    return out


def copy_into_cache(src, cache, offset):
    src = np.ascontiguousarray(src, np.uint16)
    assert cache.flags.c_contiguous and cache.dtype == np.uint16
    t = src.shape[0]
    stride = src.size // t
    lib().or_copy_into_cache(_p16(src), _sz(t), _sz(stride), _sz(offset), _p16(cache))


REFERENCE = 0
FLASH_PREFILL = 1
TILED = 2


def attention_decode(q, k, v, q_heads, kv_heads, head_dim, block=64, streams=None):
    """One-query flash decode over all keys of k/v (see oracle.h)."""
    q = np.ascontiguousarray(q, np.uint16)
    k = np.ascontiguousarray(k, np.uint16)
    v = np.ascontiguousarray(v, np.uint16)
    length = k.size // (kv_heads * head_dim)
    if streams is None:
        streams = decode_streams(head_dim)
    out = np.empty((1, q_heads, head_dim), np.uint16)
    lib().or_attention_decode(_p16(q), _p16(k), _p16(v), _sz(q_heads), _sz(kv_heads),
                              _sz(head_dim), _sz(length), _sz(block), _sz(streams), _p16(out))
    return out


def decode_block(capacity: int) -> int:
    return int(lib().or_decode_block(_sz(capacity)))


def decode_streams(head_dim: int) -> int:
    return int(lib().or_decode_streams(_sz(head_dim)))


def exp(values) -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(values, np.float32).ravel())
    out = np.empty_like(a)
    lib().or_exp(a.ctypes.data_as(_f32p), out.ctypes.data_as(_f32p), _sz(a.size))
    return out


def dot(x, y) -> float:
    x = np.ascontiguousarray(np.asarray(x, np.float32).ravel())
    y = np.ascontiguousarray(np.asarray(y, np.float32).ravel())
    return float(lib().or_dot(x.ctypes.data_as(_f32p), y.ctypes.data_as(_f32p), _sz(x.size)))


def rope_cs(position: int, pair: int, head_dim: int, theta: float):
    c, s = ctypes.c_float(), ctypes.c_float()
    lib().or_rope_cs(_sz(position), _sz(pair), _sz(head_dim), ctypes.c_float(theta),
                     ctypes.byref(c), ctypes.byref(s))
    return c.value, s.value


def attention(q, k, v, q_heads, kv_heads, head_dim, causal=True, query_offset=0,
              semantics=REFERENCE):
    q = np.ascontiguousarray(q, np.uint16)
    k = np.ascontiguousarray(k, np.uint16)
    v = np.ascontiguousarray(v, np.uint16)
    tokens = q.size // (q_heads * head_dim)
    kv_length = k.size // (kv_heads * head_dim)
    out = np.empty((tokens, q_heads, head_dim), np.uint16)
    lib().or_attention(_p16(q), _p16(k), _p16(v), _sz(tokens), _sz(q_heads), _sz(kv_heads),
                       _sz(head_dim), _sz(kv_length), ctypes.c_int(int(causal)),
                       _sz(query_offset), ctypes.c_int(semantics), _p16(out))
    return out


# ---- model -----------------------------------------------------------------

QWEN3_0_6B = dict(hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                  num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                  rms_norm_eps=1e-6, rope_theta=1e6, vocab_size=151936, tie_word_embeddings=1)

ROLE = dict(embedding=0, q=1, k=2, v=3, o=4, q_norm=5, k_norm=6, gate=7, up=8, down=9,
            input_norm=10, post_norm=11, final_norm=12, lm_head=13)


class Qwen3:
    """Random-init oracle model (weights identical to the engine's generator)."""

    def __init__(self, cfg: dict, seed: int, capacity: int, std: float = 0.02):
        self.cfg = dict(cfg)
        self._c = Qwen3Config(**{k: self.cfg[k] for k, _ in Qwen3Config._fields_})
        self.h = lib().or_qwen3_create_random(ctypes.byref(self._c), seed, std, capacity)
        self.capacity = capacity

    def close(self):
        if self.h:
            lib().or_qwen3_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_fusion(self, qk_rope_cache: bool = True, add_rms_norm: bool = True):
        lib().or_qwen3_set_fusion(self.h, int(qk_rope_cache), int(add_rms_norm))

    def set_tp(self, tp: int) -> None:
        """Follow the arithmetic of `tp` tensor-parallel ranks (O and down)."""
        lib().or_qwen3_set_tp(self.h, tp)

    def reset(self):
        lib().or_qwen3_reset(self.h)

    def truncate(self, length: int) -> None:
        """Keeps the first `length` cached positions (a cache rollback)."""
        if lib().or_qwen3_truncate(self.h, _sz(length)) != 0:
            raise ValueError(f"cannot truncate a cache of {len(self)} positions to {length}")

    def __len__(self):
        return int(lib().or_qwen3_len(self.h))

    def forward(self, tokens) -> np.ndarray:
        tokens = np.ascontiguousarray(tokens, np.uint32)
        logits = np.empty(self.cfg["vocab_size"], np.uint16)
        rc = lib().or_qwen3_forward(self.h, _p32(tokens), _sz(tokens.size), _p16(logits))
        if rc != 0:
            raise RuntimeError("oracle forward failed (cache capacity)")
        return logits

    def forward_hidden(self, hidden) -> np.ndarray:
        hidden = np.ascontiguousarray(hidden, np.uint16)
        t = hidden.size // self.cfg["hidden_size"]
        out = np.empty_like(hidden)
        rc = lib().or_qwen3_forward_hidden(self.h, _p16(hidden), _sz(t), _p16(out))
        if rc != 0:
            raise RuntimeError("oracle forward failed (cache capacity)")
        return out

    def generate_greedy(self, prompt, max_tokens: int) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt, np.uint32)
        out = np.empty(max_tokens, np.uint32)
        n = lib().or_qwen3_generate_greedy(self.h, _p32(prompt), _sz(prompt.size),
                                           _sz(max_tokens), _p32(out))
        return out[:n]

    def generate_sampled(self, prompt, max_tokens: int, temperature: float, top_p: float = 1.0,
                         top_k: int = 0, seed: int = 0) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt, np.uint32)
        out = np.empty(max(1, max_tokens), np.uint32)
        n = lib().or_qwen3_generate_sampled(self.h, _p32(prompt), _sz(prompt.size),
                                            _sz(max_tokens), temperature, top_p, top_k, seed,
                                            _p32(out))
        return out[:n]

    def weight(self, layer: int, role: str, shape) -> np.ndarray:
        p = lib().or_qwen3_weight(self.h, layer, ROLE[role])
        n = int(np.prod(shape))
        return np.ctypeslib.as_array(p, shape=(n,)).reshape(shape).copy()

    def cache(self, layer: int, value: bool, rows: int) -> np.ndarray:
        p = lib().or_qwen3_cache(self.h, layer, int(value))
        width = self.cfg["num_key_value_heads"] * self.cfg["head_dim"]
        return np.ctypeslib.as_array(p, shape=(rows * width,)).reshape(rows, width).copy()

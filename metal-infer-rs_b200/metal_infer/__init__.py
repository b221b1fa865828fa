"""Python binding of the B200 engine's C ABI (include/mi.h).

Mirrors the reference's Rust API so tests and benchmarks read like the
reference's own: ``MetalContext`` (context.rs), ``CommandBatch`` /
``PendingBatch`` (context.rs:703-1082), ``Tensor`` (tensor.rs), the op methods
of ``CommandBatch`` (ops.rs), ``Qwen3Model`` / ``KvCache`` (qwen3.rs).
Errors raise ``CoreError`` / ``ModelError`` carrying the C status code.

The library is loaded from this directory (built by ../build.py); there is no
fallback: without the CUDA library every call fails loudly.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Callable, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmetal_infer.so")

# ---- status codes (mi_status) -------------------------------------------------
OK = 0
ERR_NO_DEVICE = 1
ERR_RESOURCE = 2
ERR_KERNEL = 3
ERR_COMMAND = 4
ERR_SHAPE = 5
ERR_DTYPE = 6
ERR_DATA_LENGTH = 7
ERR_PROFILING = 8
ERR_CACHE_CAPACITY = 9
ERR_CONFIG = 10
ERR_UNSUPPORTED = 11
ERR_IO = 12
ERR_MISSING_TENSOR = 13
ERR_TIMEOUT = 14
ERR_INVALID_ARGUMENT = 15
ERR_COLLECTIVE = 16

_MODEL_CODES = {ERR_CACHE_CAPACITY, ERR_CONFIG, ERR_UNSUPPORTED, ERR_IO, ERR_MISSING_TENSOR}


class CoreError(RuntimeError):
    """CoreError (crates/metal-infer-core/src/error.rs) with its mi_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status
        self.message = message


class ModelError(CoreError):
    """ModelError (crates/metal-infer-models/src/error.rs)."""


# ---- enums --------------------------------------------------------------------
class DType:
    F16, F32, U32 = 0, 1, 2
    NP = {0: np.uint16, 1: np.float32, 2: np.uint32}
    SIZE = {0: 2, 1: 4, 2: 4}


class MatmulBackend:
    AUTO, REFERENCE, NATIVE, MPS = 0, 1, 2, 3


class AttentionKind:
    REFERENCE, TILED, FLASH_PREFILL, DECODE_SPLIT_KV, FLASH_DECODE = 0, 1, 2, 3, 4


class AttentionConfig(ctypes.Structure):
    _fields_ = [("query_heads", ctypes.c_size_t), ("kv_heads", ctypes.c_size_t),
                ("head_dim", ctypes.c_size_t), ("causal", ctypes.c_int),
                ("query_offset", ctypes.c_size_t)]


class QkNormRopeCacheConfig(ctypes.Structure):
    _fields_ = [("offset", ctypes.c_size_t), ("theta", ctypes.c_float),
                ("epsilon", ctypes.c_float)]


class DispatchStats(ctypes.Structure):
    _fields_ = [("gpu_time", ctypes.c_double), ("wall_time", ctypes.c_double)]


class KernelDispatchProfile(ctypes.Structure):
    _fields_ = [("kernel", ctypes.c_char * 64), ("gpu_time", ctypes.c_double)]


class Qwen3Config(ctypes.Structure):
    _fields_ = [("hidden_size", ctypes.c_size_t), ("intermediate_size", ctypes.c_size_t),
                ("num_hidden_layers", ctypes.c_size_t), ("num_attention_heads", ctypes.c_size_t),
                ("num_key_value_heads", ctypes.c_size_t), ("head_dim", ctypes.c_size_t),
                ("rms_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
                ("vocab_size", ctypes.c_size_t), ("tie_word_embeddings", ctypes.c_int)]

    @classmethod
    def from_dict(cls, d: dict) -> "Qwen3Config":
        return cls(**{k: d[k] for k, _ in cls._fields_})

    def to_dict(self) -> dict:
        return {k: getattr(self, k) for k, _ in self._fields_}


class FusionOptions(ctypes.Structure):
    _fields_ = [("qkv", ctypes.c_int), ("gate_up", ctypes.c_int),
                ("add_rms_norm", ctypes.c_int), ("qk_rope_cache", ctypes.c_int)]

    @classmethod
    def all(cls):
        return cls(1, 1, 1, 1)

    @classmethod
    def none(cls):
        return cls(0, 0, 0, 0)


class TpShard(ctypes.Structure):
    """mi_tp_shard_info: one tensor-parallel rank's slice of a config."""
    _fields_ = [(n, ctypes.c_size_t) for n in ("q_heads", "kv_heads", "intermediate", "vocab",
                                                "q_head0", "kv_head0", "inter0", "vocab0")]


def tp_shard(config: dict, tp: int, rank: int) -> dict:
    """This rank's shard of `config` (host only, no GPU needed)."""
    c = Qwen3Config.from_dict(config)
    out = TpShard()
    _check(lib().mi_tp_shard(ctypes.byref(c), ctypes.c_int(tp), ctypes.c_int(rank),
                             ctypes.byref(out)))
    return {n: getattr(out, n) for n, _ in TpShard._fields_}


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id (rank 0 creates it and shares it)."""
    buf = (ctypes.c_uint8 * 128)()
    _check(lib().mi_nccl_unique_id(buf, ctypes.c_size_t(128)))
    return bytes(buf)


def share_nccl_id(group=None) -> bytes:
    """Rank 0's NCCL id broadcast over an initialized torch.distributed group
    (any backend; gloo works on CPU)."""
    import torch
    import torch.distributed as dist
    rank = dist.get_rank(group)
    t = torch.zeros(128, dtype=torch.uint8)
    if rank == 0:
        t.copy_(torch.frombuffer(bytearray(nccl_unique_id()), dtype=torch.uint8))
    dist.broadcast(t, src=0, group=group)
    return bytes(t.tolist())


class GenerationOptions(ctypes.Structure):
    _fields_ = [("max_tokens", ctypes.c_size_t), ("temperature", ctypes.c_float),
                ("top_p", ctypes.c_float), ("top_k", ctypes.c_size_t),
                ("seed", ctypes.c_uint64), ("stop_token_ids", ctypes.POINTER(ctypes.c_uint32)),
                ("stop_token_count", ctypes.c_size_t)]


TOKEN_CALLBACK = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_uint32, ctypes.c_void_p)

QWEN3_0_6B = dict(hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                  num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                  rms_norm_eps=1e-6, rope_theta=1e6, vocab_size=151936, tie_word_embeddings=1)
QWEN3_8B = dict(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                rms_norm_eps=1e-6, rope_theta=1e6, vocab_size=151936, tie_word_embeddings=0)
QWEN3_32B = dict(hidden_size=5120, intermediate_size=25600, num_hidden_layers=64,
                 num_attention_heads=64, num_key_value_heads=8, head_dim=128,
                 rms_norm_eps=1e-6, rope_theta=1e6, vocab_size=151936, tie_word_embeddings=0)

# Every symbol the header declares (checked by the CPU tests).
def xorshift_seed(seed: int) -> int:
    """XorShift64::new (qwen3.rs:1016-1024): seed 0 becomes 0x9e3779b97f4a7c15."""
    return int(lib().mi_xorshift_seed(ctypes.c_uint64(seed)))


EXPORTS = [
    "mi_last_error_message", "mi_version", "mi_context_create", "mi_context_destroy",
    "mi_context_device_name", "mi_context_allocated_bytes", "mi_context_set_matmul_backend",
    "mi_context_matmul_backend", "mi_context_set_kernel_profiling",
    "mi_context_take_kernel_profiles", "mi_context_synchronize", "mi_context_stream",
    "mi_context_kernel_status",
    "mi_context_empty", "mi_context_tensor_f16", "mi_context_tensor_f16_bits",
    "mi_context_tensor_f16_bytes", "mi_context_tensor_bf16_as_f16_bytes",
    "mi_context_tensor_u32", "mi_context_tensor_from_device", "mi_tensor_clone",
    "mi_tensor_release", "mi_tensor_rank", "mi_tensor_shape", "mi_tensor_dtype", "mi_tensor_len",
    "mi_tensor_byte_len", "mi_tensor_device_ptr", "mi_tensor_reshape", "mi_tensor_prefix",
    "mi_tensor_row", "mi_tensor_slice_1d", "mi_tensor_f16_bits", "mi_tensor_to_f32",
    "mi_tensor_to_u32", "mi_tensor_write", "mi_context_begin_batch", "mi_batch_commit",
    "mi_batch_finish", "mi_batch_abandon", "mi_pending_wait", "mi_pending_is_complete",
    "mi_batch_add", "mi_batch_matmul", "mi_batch_matmul2", "mi_batch_matmul3",
    "mi_batch_rms_norm_matmul3", "mi_batch_add_rms_norm_matmul2", "mi_batch_rms_norm",
    "mi_batch_add_rms_norm", "mi_batch_swiglu", "mi_batch_embedding", "mi_batch_argmax",
    "mi_batch_rope", "mi_batch_qk_norm_rope_cache", "mi_batch_attention",
    "mi_batch_attention_flash_decode_with_configuration", "mi_batch_copy_into_cache",
    "mi_attention_flash_decode_noalloc",
    "mi_qwen3_config_validate", "mi_qwen3_create_random", "mi_qwen3_load", "mi_qwen3_destroy",
    "mi_qwen3_get_config", "mi_qwen3_set_attention_kind", "mi_qwen3_set_fusion_options",
    "mi_qwen3_fusion_options", "mi_qwen3_set_decode_graphs",
    "mi_qwen3_set_decode_persistent", "mi_qwen3_decode_persistent", "mi_qwen3_exchange_wait",
    "mi_tp_shard", "mi_nccl_unique_id", "mi_qwen3_create_random_tp", "mi_qwen3_load_tp", "mi_kv_cache_create",
    "mi_kv_cache_destroy", "mi_kv_cache_len", "mi_kv_cache_capacity", "mi_kv_cache_reset",
    "mi_kv_cache_layer", "mi_qwen3_prefill", "mi_qwen3_decode", "mi_qwen3_prefill_argmax",
    "mi_qwen3_decode_argmax", "mi_qwen3_decode_steps", "mi_kv_cache_tokens",
    "mi_qwen3_generate", "mi_qwen3_generate_with",
    "mi_qwen3_run_first_block", "mi_qwen3_forward_hidden", "mi_qwen3_weight",
    "mi_fill_normal_f16", "mi_fill_tokens_u32", "mi_sample_logits", "mi_xorshift_seed",
]

_lib = None
_vp = ctypes.c_void_p
_vpp = ctypes.POINTER(ctypes.c_void_p)
_sz = ctypes.c_size_t
_szp = ctypes.POINTER(ctypes.c_size_t)


def lib() -> ctypes.CDLL:
    """Loads libmetal_infer.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise CoreError(ERR_KERNEL, f"{LIB_PATH} is missing: run metal-infer-rs_b200/build.py")
    L = ctypes.CDLL(LIB_PATH)
    L.mi_last_error_message.restype = ctypes.c_char_p
    L.mi_version.restype = ctypes.c_char_p
    for name in ("mi_context_allocated_bytes", "mi_tensor_rank", "mi_tensor_shape", "mi_tensor_len",
                 "mi_tensor_byte_len", "mi_kv_cache_len", "mi_kv_cache_capacity"):
        getattr(L, name).restype = _sz
    L.mi_tensor_device_ptr.restype = _vp
    L.mi_context_stream.restype = _vp
    L.mi_xorshift_seed.restype = ctypes.c_uint64
    L.mi_xorshift_seed.argtypes = [ctypes.c_uint64]
    for name in ("mi_context_destroy", "mi_tensor_release", "mi_batch_abandon", "mi_qwen3_destroy",
                 "mi_kv_cache_destroy", "mi_kv_cache_reset"):
        getattr(L, name).restype = None
        getattr(L, name).argtypes = [_vp]
    for name in ("mi_tensor_rank", "mi_tensor_len", "mi_tensor_byte_len", "mi_tensor_device_ptr",
                 "mi_tensor_dtype", "mi_kv_cache_len", "mi_kv_cache_capacity",
                 "mi_context_allocated_bytes", "mi_context_matmul_backend", "mi_context_stream",
                 "mi_pending_is_complete"):
        getattr(L, name).argtypes = [_vp]
    L.mi_tensor_shape.argtypes = [_vp, _szp, _sz]
    L.mi_qwen3_fusion_options.restype = FusionOptions
    L.mi_qwen3_fusion_options.argtypes = [_vp]
    _lib = L
    return L


def _check(status: int) -> None:
    if status != OK:
        msg = lib().mi_last_error_message().decode(errors="replace")
        raise (ModelError if status in _MODEL_CODES else CoreError)(status, msg)


def version() -> str:
    return lib().mi_version().decode()


def _shape_arr(shape: Sequence[int]):
    arr = (ctypes.c_size_t * max(1, len(shape)))(*shape)
    return arr, len(shape)


# ---- tensors --------------------------------------------------------------------
class Tensor:
    """Reference-counted view of device memory (tensor.rs:35-261)."""

    def __init__(self, handle: int, context: "MetalContext"):
        self._h = _vp(handle)
        self.context = context

    @property
    def handle(self):
        return self._h

    def __del__(self):
        try:
            if self._h and self._h.value:
                lib().mi_tensor_release(self._h)
                self._h = None
        except Exception:
            pass

    def shape(self) -> list:
        buf = (ctypes.c_size_t * 8)()
        n = lib().mi_tensor_shape(self._h, buf, 8)
        return list(buf[:n])

    def dtype(self) -> int:
        return lib().mi_tensor_dtype(self._h)

    def __len__(self) -> int:
        return int(lib().mi_tensor_len(self._h))

    def byte_len(self) -> int:
        return int(lib().mi_tensor_byte_len(self._h))

    def data_ptr(self) -> int:
        return int(lib().mi_tensor_device_ptr(self._h) or 0)

    def _view(self, fn, *args) -> "Tensor":
        out = _vp()
        _check(fn(self._h, *args, ctypes.byref(out)))
        return Tensor(out.value, self.context)

    def clone(self) -> "Tensor":
        return self._view(lib().mi_tensor_clone)

    def reshape(self, shape: Sequence[int]) -> "Tensor":
        arr, n = _shape_arr(shape)
        return self._view(lib().mi_tensor_reshape, arr, _sz(n))

    def prefix(self, first: int) -> "Tensor":
        return self._view(lib().mi_tensor_prefix, _sz(first))

    def row(self, r: int) -> "Tensor":
        return self._view(lib().mi_tensor_row, _sz(r))

    def slice_1d(self, start: int, length: int) -> "Tensor":
        return self._view(lib().mi_tensor_slice_1d, _sz(start), _sz(length))

    def f16_bits(self) -> np.ndarray:
        out = np.empty(len(self), np.uint16)
        _check(lib().mi_tensor_f16_bits(self._h, out.ctypes.data_as(ctypes.c_void_p), _sz(out.size)))
        return out.reshape(self.shape())

    def to_f32_vec(self) -> np.ndarray:
        out = np.empty(len(self), np.float32)
        _check(lib().mi_tensor_to_f32(self._h, out.ctypes.data_as(ctypes.c_void_p), _sz(out.size)))
        return out

    def to_u32_vec(self) -> np.ndarray:
        out = np.empty(len(self), np.uint32)
        _check(lib().mi_tensor_to_u32(self._h, out.ctypes.data_as(ctypes.c_void_p), _sz(out.size)))
        return out

    def write(self, data: np.ndarray) -> None:
        data = np.ascontiguousarray(data)
        _check(lib().mi_tensor_write(self._h, data.ctypes.data_as(ctypes.c_void_p), _sz(data.nbytes)))

    def numpy(self) -> np.ndarray:
        d = self.dtype()
        if d == DType.F16:
            return self.f16_bits()
        if d == DType.U32:
            return self.to_u32_vec().reshape(self.shape())
        return self.to_f32_vec().reshape(self.shape())


# ---- context ------------------------------------------------------------------------
class MetalContext:
    """MetalContext (context.rs:155-1128) over one CUDA device and stream."""

    def __init__(self, device: int = 0):
        h = _vp()
        _check(lib().mi_context_create(ctypes.c_int(device), ctypes.byref(h)))
        self._h = h

    def __del__(self):
        try:
            if self._h and self._h.value:
                lib().mi_context_destroy(self._h)
                self._h = None
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def device_name(self) -> str:
        buf = ctypes.create_string_buffer(256)
        _check(lib().mi_context_device_name(self._h, buf, _sz(256)))
        return buf.value.decode()

    def allocated_bytes(self) -> int:
        return int(lib().mi_context_allocated_bytes(self._h))

    def set_matmul_backend(self, backend: int) -> None:
        _check(lib().mi_context_set_matmul_backend(self._h, ctypes.c_int(backend)))

    def matmul_backend(self) -> int:
        return lib().mi_context_matmul_backend(self._h)

    def set_kernel_profiling(self, enabled: bool) -> None:
        _check(lib().mi_context_set_kernel_profiling(self._h, ctypes.c_int(int(enabled))))

    def take_kernel_profiles(self) -> list:
        n = _sz()
        _check(lib().mi_context_take_kernel_profiles(self._h, None, _sz(0), ctypes.byref(n)))
        arr = (KernelDispatchProfile * max(1, n.value))()
        _check(lib().mi_context_take_kernel_profiles(self._h, arr, _sz(n.value), ctypes.byref(n)))
        return [(arr[i].kernel.decode(), arr[i].gpu_time) for i in range(n.value)]

    def synchronize(self) -> None:
        _check(lib().mi_context_synchronize(self._h))

    def stream(self) -> int:
        return int(lib().mi_context_stream(self._h) or 0)

    def kernel_status(self) -> int:
        """Synchronizes; raises CoreError(ERR_TIMEOUT) if a bounded device
        wait expired since the last call."""
        code = ctypes.c_uint32(0)
        _check(lib().mi_context_kernel_status(self._h, ctypes.byref(code)))
        return code.value

    # tensors (context.rs:740-872)
    def _new(self, fn, *args) -> Tensor:
        out = _vp()
        _check(fn(self._h, *args, ctypes.byref(out)))
        return Tensor(out.value, self)

    def empty(self, shape: Sequence[int], dtype: int = DType.F16) -> Tensor:
        arr, n = _shape_arr(shape)
        return self._new(lib().mi_context_empty, arr, _sz(n), ctypes.c_int(dtype))

    def tensor_f16(self, values, shape: Sequence[int]) -> Tensor:
        v = np.ascontiguousarray(np.asarray(values, np.float32).ravel())
        arr, n = _shape_arr(shape)
        return self._new(lib().mi_context_tensor_f16, v.ctypes.data_as(ctypes.c_void_p), _sz(v.size),
                         arr, _sz(n))

    def tensor_f16_bits(self, bits, shape: Sequence[int]) -> Tensor:
        v = np.ascontiguousarray(np.asarray(bits, np.uint16).ravel())
        arr, n = _shape_arr(shape)
        return self._new(lib().mi_context_tensor_f16_bits, v.ctypes.data_as(ctypes.c_void_p),
                         _sz(v.size), arr, _sz(n))

    def tensor_f16_bytes(self, data: bytes, shape: Sequence[int]) -> Tensor:
        arr, n = _shape_arr(shape)
        buf = (ctypes.c_uint8 * len(data)).from_buffer_copy(data)
        return self._new(lib().mi_context_tensor_f16_bytes, buf, _sz(len(data)), arr, _sz(n))

    def tensor_bf16_as_f16_bytes(self, data: bytes, shape: Sequence[int]) -> Tensor:
        arr, n = _shape_arr(shape)
        buf = (ctypes.c_uint8 * len(data)).from_buffer_copy(data)
        return self._new(lib().mi_context_tensor_bf16_as_f16_bytes, buf, _sz(len(data)), arr, _sz(n))

    def tensor_u32(self, values, shape: Sequence[int]) -> Tensor:
        v = np.ascontiguousarray(np.asarray(values, np.uint32).ravel())
        arr, n = _shape_arr(shape)
        return self._new(lib().mi_context_tensor_u32, v.ctypes.data_as(ctypes.c_void_p), _sz(v.size),
                         arr, _sz(n))

    def tensor_from_device(self, ptr: int, shape: Sequence[int], dtype: int) -> Tensor:
        arr, n = _shape_arr(shape)
        return self._new(lib().mi_context_tensor_from_device, _vp(ptr), arr, _sz(n),
                         ctypes.c_int(dtype))

    def fill_normal_f16(self, t: Tensor, seed: int, stream: int, std: float = 1.0,
                        offset: int = 0) -> None:
        _check(lib().mi_fill_normal_f16(self._h, t.handle, ctypes.c_uint64(seed),
                                        ctypes.c_uint64(stream), ctypes.c_uint64(offset),
                                        ctypes.c_double(std)))

    def fill_tokens_u32(self, t: Tensor, seed: int, stream: int, vocab: int) -> None:
        _check(lib().mi_fill_tokens_u32(self._h, t.handle, ctypes.c_uint64(seed),
                                        ctypes.c_uint64(stream), ctypes.c_uint32(vocab)))

    def sample_logits(self, logits: Tensor, temperature: float, top_p: float = 1.0,
                      top_k: int = 0, state: int = 1) -> tuple:
        """sample_token / sample_token_f16 (qwen3.rs:909-1005) on the device:
        returns (token, next XorShift64 state)."""
        st = ctypes.c_uint64(state)
        tok = ctypes.c_uint32(0)
        _check(lib().mi_sample_logits(self._h, logits.handle, ctypes.c_float(temperature),
                                      ctypes.c_float(top_p), _sz(top_k), ctypes.byref(st),
                                      ctypes.byref(tok)))
        return int(tok.value), int(st.value)

    # batches
    def begin_batch(self) -> "CommandBatch":
        h = _vp()
        _check(lib().mi_context_begin_batch(self._h, ctypes.byref(h)))
        return CommandBatch(h, self)

    def _immediate(self, fn):
        b = self.begin_batch()
        out = fn(b)
        b.finish()
        return out

    # MetalContext immediate ops (ops.rs:112-219)
    def add(self, left, right):
        return self._immediate(lambda b: b.add(left, right))

    def matmul(self, x, w):
        return self._immediate(lambda b: b.matmul(x, w))

    def rms_norm(self, x, w, eps):
        return self._immediate(lambda b: b.rms_norm(x, w, eps))

    def swiglu(self, gate, up):
        return self._immediate(lambda b: b.swiglu(gate, up))

    def embedding(self, tokens, table):
        return self._immediate(lambda b: b.embedding(tokens, table))

    def rope(self, x, offset, theta):
        return self._immediate(lambda b: b.rope(x, offset, theta))

    def attention(self, q, k, v, config, kind):
        return self._immediate(lambda b: b.attention(q, k, v, config, kind))

    def attention_flash_decode_with_block(self, q, k, v, config, block):
        return self.attention_flash_decode_with_configuration(q, k, v, config, block, 256)

    def attention_flash_decode_with_configuration(self, q, k, v, config, block, threads):
        return self._immediate(
            lambda b: b.attention_flash_decode_with_configuration(q, k, v, config, block, threads))

    def copy_into_cache(self, source, cache, offset):
        return self._immediate(lambda b: b.copy_into_cache(source, cache, offset))


class PendingBatch:
    def __init__(self, handle, context):
        self._h = handle
        self.context = context

    def wait(self) -> DispatchStats:
        st = DispatchStats()
        h, self._h = self._h, None
        _check(lib().mi_pending_wait(h, ctypes.byref(st)))
        return st

    def is_complete(self) -> bool:
        return bool(lib().mi_pending_is_complete(self._h))

    def __del__(self):
        try:
            if self._h is not None:
                lib().mi_pending_wait(self._h, None)
        except Exception:
            pass


class CommandBatch:
    """CommandBatch (context.rs:155-1045) and its ops (ops.rs:221-1285)."""

    def __init__(self, handle, context: MetalContext):
        self._h = handle
        self.context = context

    def __del__(self):
        try:
            if self._h is not None:
                lib().mi_batch_abandon(self._h)
        except Exception:
            pass

    def commit(self) -> PendingBatch:
        p = _vp()
        h, self._h = self._h, None
        _check(lib().mi_batch_commit(h, ctypes.byref(p)))
        return PendingBatch(p, self.context)

    def finish(self) -> DispatchStats:
        st = DispatchStats()
        h, self._h = self._h, None
        _check(lib().mi_batch_finish(h, ctypes.byref(st)))
        return st

    def _outs(self, fn, n, *args):
        outs = [_vp() for _ in range(n)]
        _check(fn(self._h, *args, *[ctypes.byref(o) for o in outs]))
        ts = [Tensor(o.value, self.context) for o in outs]
        return ts[0] if n == 1 else tuple(ts)

    def add(self, left: Tensor, right: Tensor) -> Tensor:
        return self._outs(lib().mi_batch_add, 1, left.handle, right.handle)

    def matmul(self, x: Tensor, w: Tensor) -> Tensor:
        return self._outs(lib().mi_batch_matmul, 1, x.handle, w.handle)

    def matmul2(self, x, w0, w1):
        return self._outs(lib().mi_batch_matmul2, 2, x.handle, w0.handle, w1.handle)

    def matmul3(self, x, w0, w1, w2):
        return self._outs(lib().mi_batch_matmul3, 3, x.handle, w0.handle, w1.handle, w2.handle)

    def rms_norm_matmul3(self, x, norm, w0, w1, w2, eps):
        return self._outs(lib().mi_batch_rms_norm_matmul3, 3, x.handle, norm.handle, w0.handle,
                          w1.handle, w2.handle, ctypes.c_float(eps))

    def add_rms_norm_matmul2(self, left, right, norm, w0, w1, eps):
        return self._outs(lib().mi_batch_add_rms_norm_matmul2, 3, left.handle, right.handle,
                          norm.handle, w0.handle, w1.handle, ctypes.c_float(eps))

    def rms_norm(self, x, w, eps):
        return self._outs(lib().mi_batch_rms_norm, 1, x.handle, w.handle, ctypes.c_float(eps))

    def add_rms_norm(self, left, right, w, eps):
        return self._outs(lib().mi_batch_add_rms_norm, 2, left.handle, right.handle, w.handle,
                          ctypes.c_float(eps))

    def swiglu(self, gate, up):
        return self._outs(lib().mi_batch_swiglu, 1, gate.handle, up.handle)

    def embedding(self, tokens, table):
        return self._outs(lib().mi_batch_embedding, 1, tokens.handle, table.handle)

    def argmax(self, logits: Tensor, output: Tensor) -> None:
        _check(lib().mi_batch_argmax(self._h, logits.handle, output.handle))

    def rope(self, x, offset, theta):
        return self._outs(lib().mi_batch_rope, 1, x.handle, _sz(offset), ctypes.c_float(theta))

    def qk_norm_rope_cache(self, q, k, qw, kw, key_cache, config: QkNormRopeCacheConfig):
        return self._outs(lib().mi_batch_qk_norm_rope_cache, 1, q.handle, k.handle, qw.handle,
                          kw.handle, key_cache.handle, config)

    def attention(self, q, k, v, config: AttentionConfig, kind: int):
        return self._outs(lib().mi_batch_attention, 1, q.handle, k.handle, v.handle, config,
                          ctypes.c_int(kind))

    def attention_flash_decode_with_configuration(self, q, k, v, config, block, threads):
        return self._outs(lib().mi_batch_attention_flash_decode_with_configuration, 1, q.handle,
                          k.handle, v.handle, config, _sz(block), _sz(threads))

    def copy_into_cache(self, source, cache, offset):
        _check(lib().mi_batch_copy_into_cache(self._h, source.handle, cache.handle, _sz(offset)))


# ---- model ---------------------------------------------------------------------------
ROLES = dict(embedding=0, q=1, k=2, v=3, o=4, q_norm=5, k_norm=6, gate=7, up=8, down=9,
             input_norm=10, post_norm=11, final_norm=12, lm_head=13)


class KvCache:
    """KvCache (qwen3.rs:68-117)."""

    def __init__(self, model: "Qwen3Model", capacity: int):
        h = _vp()
        _check(lib().mi_kv_cache_create(model.handle, _sz(capacity), ctypes.byref(h)))
        self._h = h
        self.model = model

    @property
    def handle(self):
        return self._h

    def __del__(self):
        try:
            if self._h and self._h.value:
                lib().mi_kv_cache_destroy(self._h)
                self._h = None
        except Exception:
            pass

    def __len__(self) -> int:
        return int(lib().mi_kv_cache_len(self._h))

    def capacity(self) -> int:
        return int(lib().mi_kv_cache_capacity(self._h))

    def reset(self) -> None:
        lib().mi_kv_cache_reset(self._h)

    def tokens(self, start: int, count: int) -> np.ndarray:
        out = np.empty(max(1, count), np.uint32)
        _check(lib().mi_kv_cache_tokens(self._h, _sz(start), _sz(count),
                                        out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))))
        return out[:count]

    def layer(self, index: int):
        k, v = _vp(), _vp()
        _check(lib().mi_kv_cache_layer(self._h, _sz(index), ctypes.byref(k), ctypes.byref(v)))
        return Tensor(k.value, self.model.context), Tensor(v.value, self.model.context)


class Qwen3Model:
    """Qwen3Model (qwen3.rs:119-1034) on the B200 engine."""

    def __init__(self, handle, context: MetalContext):
        self._h = handle
        self.context = context

    @property
    def handle(self):
        return self._h

    @classmethod
    def random(cls, context: MetalContext, config: dict, seed: int, std: float = 0.02):
        c = Qwen3Config.from_dict(config)
        h = _vp()
        _check(lib().mi_qwen3_create_random(context.handle, ctypes.byref(c), ctypes.c_uint64(seed),
                                            ctypes.c_double(std), ctypes.byref(h)))
        return cls(h, context)

    @classmethod
    def random_tp(cls, context: MetalContext, config: dict, seed: int, tp: int, rank: int,
                  nccl_id: bytes, std: float = 0.02):
        """This rank's shard of the random-init model (collective over the tp ranks)."""
        c = Qwen3Config.from_dict(config)
        h = _vp()
        ident = (ctypes.c_uint8 * 128).from_buffer_copy(nccl_id[:128])
        _check(lib().mi_qwen3_create_random_tp(context.handle, ctypes.byref(c),
                                               ctypes.c_uint64(seed), ctypes.c_double(std),
                                               ctypes.c_int(tp), ctypes.c_int(rank), ident,
                                               ctypes.byref(h)))
        return cls(h, context)

    @classmethod
    def load(cls, directory: str, context: MetalContext):
        h = _vp()
        _check(lib().mi_qwen3_load(context.handle, directory.encode(), ctypes.byref(h)))
        return cls(h, context)

    @classmethod
    def load_tp(cls, directory: str, context: MetalContext, tp: int, rank: int, nccl_id: bytes):
        """This rank's tensor-parallel shard of a safetensors checkpoint."""
        h = _vp()
        ident = (ctypes.c_uint8 * 128).from_buffer_copy(nccl_id[:128])
        _check(lib().mi_qwen3_load_tp(context.handle, directory.encode(), ctypes.c_int(tp),
                                      ctypes.c_int(rank), ident, ctypes.byref(h)))
        return cls(h, context)

    def __del__(self):
        try:
            if self._h and self._h.value:
                lib().mi_qwen3_destroy(self._h)
                self._h = None
        except Exception:
            pass

    def config(self) -> dict:
        c = Qwen3Config()
        _check(lib().mi_qwen3_get_config(self._h, ctypes.byref(c)))
        return c.to_dict()

    def set_attention_kind(self, kind: int) -> None:
        _check(lib().mi_qwen3_set_attention_kind(self._h, ctypes.c_int(kind)))

    def set_fusion_options(self, options: FusionOptions) -> None:
        _check(lib().mi_qwen3_set_fusion_options(self._h, options))

    def fusion_options(self) -> FusionOptions:
        return lib().mi_qwen3_fusion_options(self._h)

    def set_decode_graphs(self, enabled: bool) -> None:
        _check(lib().mi_qwen3_set_decode_graphs(self._h, ctypes.c_int(int(enabled))))

    def set_decode_persistent(self, enabled: bool) -> None:
        """Decode through the persistent kernel (default) or the kernel chain."""
        _check(lib().mi_qwen3_set_decode_persistent(self._h, ctypes.c_int(int(enabled))))

    def exchange_wait(self) -> dict:
        """Mailbox waits of the most recent persistent decode launch (tensor
        parallelism): mean / max over CTAs in seconds, and its decode steps."""
        mean, mx, steps = ctypes.c_double(0), ctypes.c_double(0), _sz(0)
        _check(lib().mi_qwen3_exchange_wait(self._h, ctypes.byref(mean), ctypes.byref(mx),
                                            ctypes.byref(steps)))
        return {"mean_s": mean.value, "max_s": mx.value, "steps": steps.value}

    def decode_persistent(self) -> bool:
        active = ctypes.c_int(0)
        _check(lib().mi_qwen3_decode_persistent(self._h, ctypes.byref(active)))
        return bool(active.value)

    def kv_cache(self, capacity: int) -> KvCache:
        return KvCache(self, capacity)

    @staticmethod
    def _tokens(tokens):
        t = np.ascontiguousarray(np.asarray(tokens, np.uint32).ravel())
        return t, t.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))

    def prefill_with_stats(self, tokens, cache: KvCache):
        t, p = self._tokens(tokens)
        out, st = _vp(), DispatchStats()
        _check(lib().mi_qwen3_prefill(self._h, p, _sz(t.size), cache.handle, ctypes.byref(out),
                                      ctypes.byref(st)))
        return Tensor(out.value, self.context), st

    def prefill(self, tokens, cache: KvCache) -> Tensor:
        return self.prefill_with_stats(tokens, cache)[0]

    def decode_with_stats(self, token: int, cache: KvCache):
        out, st = _vp(), DispatchStats()
        _check(lib().mi_qwen3_decode(self._h, ctypes.c_uint32(token), cache.handle,
                                     ctypes.byref(out), ctypes.byref(st)))
        return Tensor(out.value, self.context), st

    def decode(self, token: int, cache: KvCache) -> Tensor:
        return self.decode_with_stats(token, cache)[0]

    def prefill_argmax(self, tokens, cache: KvCache, output: Tensor):
        t, p = self._tokens(tokens)
        out, st = _vp(), DispatchStats()
        _check(lib().mi_qwen3_prefill_argmax(self._h, p, _sz(t.size), cache.handle, output.handle,
                                             ctypes.byref(out), ctypes.byref(st)))
        return Tensor(out.value, self.context), st

    def decode_argmax(self, token: Tensor, cache: KvCache, output: Tensor):
        out, pend = _vp(), _vp()
        _check(lib().mi_qwen3_decode_argmax(self._h, token.handle, cache.handle, output.handle,
                                            ctypes.byref(out), ctypes.byref(pend)))
        return Tensor(out.value, self.context), PendingBatch(pend, self.context)

    def decode_steps(self, cache: KvCache, steps: int) -> None:
        """Enqueues `steps` pipelined greedy decode steps (no host wait)."""
        _check(lib().mi_qwen3_decode_steps(self._h, cache.handle, _sz(steps)))

    def generate(self, prompt, max_tokens: int, cache: KvCache) -> np.ndarray:
        t, p = self._tokens(prompt)
        ids = np.empty(max(1, max_tokens), np.uint32)
        n = _sz()
        _check(lib().mi_qwen3_generate(self._h, p, _sz(t.size), _sz(max_tokens), cache.handle,
                                       ids.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
                                       ctypes.byref(n)))
        return ids[: n.value]

    def generate_with(self, prompt, options: dict, cache: KvCache,
                      on_token: Optional[Callable[[int], bool]] = None) -> np.ndarray:
        t, p = self._tokens(prompt)
        stops = np.ascontiguousarray(np.asarray(options.get("stop_token_ids", []), np.uint32))
        o = GenerationOptions(options.get("max_tokens", 32), options.get("temperature", 0.0),
                              options.get("top_p", 1.0), options.get("top_k", 0),
                              options.get("seed", 0),
                              stops.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), stops.size)
        cap = max(1, int(options.get("max_tokens", 32)))
        ids = np.empty(cap, np.uint32)
        n = _sz()
        cb = TOKEN_CALLBACK(lambda tok, _u: int(bool(on_token(int(tok))))) if on_token else None
        _check(lib().mi_qwen3_generate_with(self._h, p, _sz(t.size), ctypes.byref(o), cache.handle,
                                            cb, None,
                                            ids.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
                                            _sz(cap), ctypes.byref(n)))
        return ids[: n.value]

    def run_first_block(self, tokens) -> Tensor:
        t, p = self._tokens(tokens)
        out = _vp()
        _check(lib().mi_qwen3_run_first_block(self._h, p, _sz(t.size), ctypes.byref(out)))
        return Tensor(out.value, self.context)

    def forward_hidden(self, hidden: Tensor, cache: KvCache) -> Tensor:
        out = _vp()
        _check(lib().mi_qwen3_forward_hidden(self._h, hidden.handle, cache.handle, ctypes.byref(out)))
        return Tensor(out.value, self.context)

    def weight(self, layer: int, role: str) -> Tensor:
        out = _vp()
        _check(lib().mi_qwen3_weight(self._h, ctypes.c_int(layer), ctypes.c_int(ROLES[role]),
                                     ctypes.byref(out)))
        return Tensor(out.value, self.context)

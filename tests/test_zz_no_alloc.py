"""The flash-decode entry point that allocates nothing.

mi_attention_flash_decode_noalloc exists for callers that cannot allocate
device memory at the call: hosts that reserve the whole GPU for their own
memory pool, and latency-critical loops where cudaMalloc/cudaFree would
synchronize the device. It keeps its scratch in a fixed array inside the
library. This test calls it through the C ABI with caller-owned buffers and
checks it against the allocating entry point
(mi_batch_attention_flash_decode_with_configuration), bit for bit as the other
attention tests do, on two calls in a row (the second reuses the array the
first left behind). It is collected last so that a run stopping at the first
failure has run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import metal_infer as mi
import oracle as O
from conftest import INPUT_STREAM

pytestmark = pytest.mark.gpu


def _call_noalloc(ctx, q, k, v, out, qh, kvh, length, block):
    fn = mi.lib().mi_attention_flash_decode_noalloc
    status = fn(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
                ctypes.c_void_p(v.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                ctypes.c_size_t(qh), ctypes.c_size_t(kvh), ctypes.c_size_t(128),
                ctypes.c_size_t(length), ctypes.c_size_t(block),
                ctypes.c_void_p(ctx.stream()))
    if status != mi.OK:
        raise mi.CoreError(status, mi.lib().mi_last_error_message().decode())
    ctx.synchronize()


# The allocating entry point serves two query heads per KV head, so the
# comparison stays at that ratio.
@pytest.mark.parametrize("qh,kvh,length,block",
                         [(16, 8, 300, 64), (32, 16, 2049, 128), (16, 8, 3000, 32)])
def test_noalloc_flash_decode_matches_allocating_entry_point(ctx, qh, kvh, length, block):
    results = []
    for call in range(2):
        q = O.gen_normal_f16(3, INPUT_STREAM + 200 + call, qh * 128)
        k = O.gen_normal_f16(3, INPUT_STREAM + 210 + call, length * kvh * 128)
        v = O.gen_normal_f16(3, INPUT_STREAM + 220 + call, length * kvh * 128)
        tq = ctx.tensor_f16_bits(q, [1, qh, 128])
        tk = ctx.tensor_f16_bits(k, [length, kvh, 128])
        tv = ctx.tensor_f16_bits(v, [length, kvh, 128])
        cfg = mi.AttentionConfig(qh, kvh, 128, 1, length - 1)
        expected = ctx.attention_flash_decode_with_configuration(tq, tk, tv, cfg, block,
                                                                 256).f16_bits()
        out = ctx.empty([1, qh, 128], mi.DType.F16)  # the caller owns the output
        _call_noalloc(ctx, tq, tk, tv, out, qh, kvh, length, block)
        got = out.f16_bits()
        np.testing.assert_array_equal(got, expected)
        results.append(got)
    assert not np.array_equal(results[0], results[1])


# Other GQA ratios against the oracle's block-ordered merge, with enough
# blocks that the final merge runs over several shared-memory chunks (125 / 31
# / 15 blocks for ratios 1 / 4 / 8) and, with 3 KV heads of 141 blocks, block
# records that start off a 16-byte boundary.
@pytest.mark.parametrize("qh,kvh,length,block",
                         [(3, 3, 9000, 64), (8, 2, 2500, 32), (8, 1, 2000, 64)])
def test_noalloc_flash_decode_other_ratios_match_oracle(ctx, qh, kvh, length, block):
    q = O.gen_normal_f16(3, INPUT_STREAM + 230, qh * 128)
    k = O.gen_normal_f16(3, INPUT_STREAM + 231, length * kvh * 128)
    v = O.gen_normal_f16(3, INPUT_STREAM + 232, length * kvh * 128)
    tq = ctx.tensor_f16_bits(q, [1, qh, 128])
    tk = ctx.tensor_f16_bits(k, [length, kvh, 128])
    tv = ctx.tensor_f16_bits(v, [length, kvh, 128])
    out = ctx.empty([1, qh, 128], mi.DType.F16)
    _call_noalloc(ctx, tq, tk, tv, out, qh, kvh, length, block)
    np.testing.assert_array_equal(out.f16_bits().ravel(),
                                  O.attention_decode(q, k, v, qh, kvh, 128, block=block).ravel())


def test_noalloc_flash_decode_rejects_oversized_problems(ctx):
    q = ctx.empty([1, 64, 128], mi.DType.F16)
    kv = ctx.empty([8, 8, 128], mi.DType.F16)
    out = ctx.empty([1, 64, 128], mi.DType.F16)
    # 8 KV heads x 2048 blocks x 8 x 130 x 4 bytes is far above the 1 MiB scratch.
    with pytest.raises(mi.CoreError) as e:
        _call_noalloc(ctx, q, kv, kv, out, 64, 8, 65536, 32)
    assert e.value.status == mi.ERR_SHAPE
    assert "scratch" in e.value.message

"""The algorithmic byte counts behind bench.py's roofline figures, checked
against the per-unit figures of the measurement plan: the decode GEMV and
flash-decode shapes of BASELINE config 1, and the Qwen3-0.6B decode step of
config 2 (weights 28 x 31,461,888 + lm_head 311,164,928 + final norm, plus
114,688 KV bytes per cached token)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


@pytest.mark.parametrize("n,k,segs,want", [
    (2048, 1024, 1, 4_200_448),      # q
    (1024, 1024, 1, 2_101_248),      # k, v
    (1024, 2048, 1, 4_200_448),      # o
    (3072, 1024, 2, 2 * 6_299_648 - 2048),  # gate + up, the input read once
    (1024, 3072, 1, 6_299_648),      # down
    (151936, 1024, 1, 311_470_848),  # lm_head
])
def test_gemv_bytes(n, k, segs, want):
    assert bench.gemv_bytes(n, k, segs) == want


@pytest.mark.parametrize("L,want", [(512, 2_105_344), (2048, 8_396_800), (8192, 33_562_624)])
def test_flash_decode_bytes(L, want):
    assert bench.flash_decode_bytes(L, 16, 8, 128) == want


def test_sweep_shapes_are_config1():
    assert [(n, k, s) for _, n, k, s in bench.SWEEP_GEMV] == [
        (2048, 1024, 1), (1024, 1024, 1), (1024, 1024, 1), (1024, 2048, 1), (3072, 1024, 2),
        (1024, 3072, 1), (151936, 1024, 1)]
    assert bench.SWEEP_ATTN == [512, 2048, 8192]


def test_decode_step_bytes_qwen3_0_6b():
    c = bench.CONFIG
    assert bench.weight_bytes_per_layer(c) == 31_461_888
    weights = 28 * 31_461_888 + 311_164_928 + 2048
    assert weights == 1_192_099_840
    assert bench.decode_bytes_per_token(c, 0) == weights
    assert bench.decode_bytes_per_token(c, 1) - weights == 114_688
    # mean cache length over the 256 steps after a 128-token prompt
    assert bench.decode_bytes_per_token(c, 256.5) == weights + 114_688 * 256.5
    assert bench.kernel_bytes(c, "decode_loop", 256.5, steps=4) == \
        int(4 * (weights + 114_688 * 256.5))


def test_tp_workloads_are_configs_3_and_4():
    name, cfg, seed, prompt, decode, cfg_id = bench.TP_WORKLOADS["8b-tp"]
    assert (cfg["hidden_size"], cfg["num_hidden_layers"], seed, prompt, decode, cfg_id) == \
        (4096, 36, 3, 2048, 512, 3)
    name, cfg, seed, prompt, decode, cfg_id = bench.TP_WORKLOADS["32b-tp"]
    assert (cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"],
            cfg["num_attention_heads"], seed, prompt, decode, cfg_id) == \
        (5120, 25600, 64, 64, 4, 32768, 256, 4)


def test_tp_bytes_per_rank():
    """A rank reads 1/tp of every sharded matrix and of the KV cache plus the
    replicated norms: tp = 1 is the one-GPU figure, and tp ranks together
    read the one-GPU bytes plus (tp - 1) extra copies of the norms."""
    c = bench.CONFIG_8B
    L = 2048 + 513 / 2
    one = bench.decode_bytes_per_token(c, L)
    assert bench.tp_decode_bytes_per_token(c, 1, L) == pytest.approx(one, rel=1e-12)
    assert bench.decode_bytes_per_token(c, 0) == 15_136_811_008
    norms = c["num_hidden_layers"] * 2 * (2 * c["hidden_size"] + 2 * c["head_dim"]) + \
        2 * c["hidden_size"]
    for tp in (2, 4, 8):
        per_rank = bench.tp_decode_bytes_per_token(c, tp, L)
        assert tp * per_rank == pytest.approx(one + (tp - 1) * norms, rel=1e-12)


def test_prefill_flops_qwen3_0_6b():
    # 28 layers x 2 x 15,728,640 weights x 128 tokens, causal attention over
    # 8,256 visible (query, key) pairs per head, and the last row's LM head:
    # about 0.115 TFLOP for config 2's prompt
    c = bench.CONFIG
    mats = 28 * (4096 * 1024 + 1024 * 2048 + 2 * 3072 * 1024 + 1024 * 3072)
    want = 2 * mats * 128 + 28 * 4 * 2048 * (128 * 129 // 2) + 2 * 151936 * 1024
    assert bench.prefill_flops(c, 128) == want
    assert 0.114e12 < want < 0.116e12


def test_ffma_peak():
    assert abs(bench.ffma_peak_tflops(1965.0) - 74.45) < 0.01

"""Tensor parallelism, host side (no GPU): the shard plan (8B and 32B shapes
at 1, 2, 4 and 8 ranks), the NCCL id exchange over gloo groups of 2 and 4
ranks, and the oracle's TP arithmetic."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as tmp

import metal_infer as mi
import oracle as O
from conftest import INPUT_STREAM

CFG_8B = mi.QWEN3_8B if hasattr(mi, "QWEN3_8B") else None


def small_cfg(**kw):
    cfg = dict(mi.QWEN3_0_6B)
    cfg.update(num_hidden_layers=2, vocab_size=4096, **kw)
    return cfg


@pytest.mark.parametrize("model", ["8b", "32b"])
@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_shards_cover_every_head_column_and_row_once(model, tp):
    cfg = dict(mi.QWEN3_8B if model == "8b" else mi.QWEN3_32B)
    shards = [mi.tp_shard(cfg, tp, r) for r in range(tp)]
    for key, start, total in (("q_heads", "q_head0", cfg["num_attention_heads"]),
                              ("kv_heads", "kv_head0", cfg["num_key_value_heads"]),
                              ("intermediate", "inter0", cfg["intermediate_size"]),
                              ("vocab", "vocab0", cfg["vocab_size"])):
        covered = np.zeros(total, np.int32)
        for s in shards:
            covered[s[start]:s[start] + s[key]] += 1
        assert np.all(covered == 1), key


def test_shard_plan_rejects_indivisible_sizes():
    cfg = small_cfg()
    with pytest.raises(mi.CoreError) as e:
        mi.tp_shard(cfg, 3, 0)
    assert e.value.status == mi.ERR_CONFIG
    with pytest.raises(mi.CoreError):
        mi.tp_shard(cfg, 2, 2)


def test_oracle_tp_changes_only_the_row_parallel_sums():
    cfg = small_cfg()
    prompt = O.gen_tokens(9, INPUT_STREAM, 12, cfg["vocab_size"])
    base = O.Qwen3(cfg, seed=9, capacity=64)
    one = O.Qwen3(cfg, seed=9, capacity=64)
    one.set_tp(1)
    two = O.Qwen3(cfg, seed=9, capacity=64)
    two.set_tp(2)
    l0 = base.forward(prompt)
    np.testing.assert_array_equal(one.forward(prompt), l0)
    l2 = O.f32(two.forward(prompt))
    ref = O.f32(l0)
    # a different summation order of the same products: within FP16 noise
    assert np.max(np.abs(l2 - ref)) <= 1e-2 * np.max(np.abs(ref))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, cfg, out):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        ident = mi.share_nccl_id()
        out.put((rank, ident, mi.tp_shard(cfg, world, rank)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_share_one_nccl_id_and_disjoint_shards(world):
    cfg = small_cfg()
    ctx = tmp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, cfg, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = dict()
    for _ in range(world):
        rank, ident, shard = q.get(timeout=120)
        got[rank] = (ident, shard)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert len(got[0][0]) == 128
    assert all(got[r][0] == got[0][0] for r in range(world))
    per = cfg["num_attention_heads"] // world
    assert [got[r][1]["q_head0"] for r in range(world)] == [r * per for r in range(world)]
    assert sum(got[r][1]["vocab"] for r in range(world)) == cfg["vocab_size"]

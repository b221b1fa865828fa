"""Tensor parallelism on 2, 4 and 8 GPUs against the oracle's TP arithmetic
(bit-exact logits and greedy ids through the persistent kernel, which
exchanges partials through peer memory, and through the NCCL kernel chain).
Each size is skipped on hosts with fewer GPUs.

Each rank is its own process (spawned), owns one GPU and one context, and
joins the NCCL communicator whose id rank 0 shares over a gloo group.
"""
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as tmp

import metal_infer as mi
import oracle as O
from conftest import INPUT_STREAM

pytestmark = pytest.mark.gpu

SAMPLED = dict(temperature=0.9, top_p=0.95, top_k=64, seed=13)


def small_cfg():
    cfg = dict(mi.QWEN3_0_6B)
    cfg.update(num_hidden_layers=2, vocab_size=4096)
    return cfg


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, tp, port, cfg, prompt, long_prompt, steps, out, ckpt=None, tc_prompt=None):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=tp)
    try:
        ident = mi.share_nccl_id()
        ctx = mi.MetalContext(rank)
        model = mi.Qwen3Model.random_tp(ctx, cfg, seed=11, tp=tp, rank=rank, nccl_id=ident)
        res = {}
        cache = model.kv_cache(128)
        res["prefill"] = model.prefill(prompt, cache).f16_bits().ravel()
        # a prompt whose row-parallel results (tokens x hidden >= 65,536) are
        # reduced slice by slice (NCCL send / receive, then an FP16 all-gather)
        res["prefill_long"] = model.prefill(long_prompt, model.kv_cache(160)).f16_bits().ravel()
        if tc_prompt is not None:
            # more than 512 tokens: tensor-core projections, the row-parallel
            # partials in FP32 from the tcgen05 GEMM, tensor-core attention
            res["prefill_tc"] = model.prefill(tc_prompt, model.kv_cache(704)).f16_bits().ravel()
        res["decode"] = [model.decode(int(t), cache).f16_bits().ravel() for t in (7, 900)]
        res["persistent"] = model.decode_persistent()
        for path in ("persistent", "graph", "eager"):
            model.set_decode_persistent(path == "persistent")
            model.set_decode_graphs(path != "eager")
            res[f"ids_{path}"] = model.generate(prompt, steps, model.kv_cache(128))
        # sampled: every rank gathers the full logits and draws the same token
        res["sampled"] = model.generate_with(prompt, dict(SAMPLED, max_tokens=steps),
                                             model.kv_cache(128))
        res["config"] = model.config()
        if ckpt:
            # the same shard read from a checkpoint of the full model
            loaded = mi.Qwen3Model.load_tp(ckpt, ctx, tp, rank, mi.share_nccl_id())
            res["loaded_prefill"] = loaded.prefill(prompt, loaded.kv_cache(128)).f16_bits().ravel()
            del loaded
        res["status"] = ctx.kernel_status()
        out.put((rank, res))
        del model, cache
        ctx.synchronize()
    except Exception as e:  # report instead of hanging the peer
        out.put((rank, {"error": repr(e)}))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_tp_matches_oracle_tp_arithmetic(tmp_path, tp):
    if torch.cuda.device_count() < tp:
        pytest.skip(f"needs {tp} GPUs")
    cfg = small_cfg()
    prompt = O.gen_tokens(11, INPUT_STREAM, 20, cfg["vocab_size"])
    long_prompt = O.gen_tokens(11, INPUT_STREAM + 1, 136, cfg["vocab_size"])
    tc_prompt = O.gen_tokens(11, INPUT_STREAM + 2, 640, cfg["vocab_size"])
    steps = 16
    # a checkpoint of the full (one-GPU) model for the shard-on-load check
    import safetensors_io as st
    from test_loader_gpu import export
    full = mi.Qwen3Model.random(mi.MetalContext(0), cfg, seed=11)
    export(full, cfg, str(tmp_path))
    del full
    ctx = tmp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main,
                         args=(r, tp, port, cfg, prompt, long_prompt, steps, q, str(tmp_path),
                               tc_prompt))
             for r in range(tp)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(tp):
        rank, r = q.get(timeout=300)
        res[rank] = r
    for p in procs:
        p.join(timeout=120)
    for r in range(tp):
        assert "error" not in res[r], res[r]["error"]
    ref = O.Qwen3(cfg, seed=11, capacity=128)
    ref.set_tp(tp)
    want_prefill = ref.forward(prompt)
    want_decode = [ref.forward(np.array([t], np.uint32)) for t in (7, 900)]
    ref_long = O.Qwen3(cfg, seed=11, capacity=160)
    ref_long.set_tp(tp)
    want_long = ref_long.forward(long_prompt)
    ref_tc = O.Qwen3(cfg, seed=11, capacity=704)
    ref_tc.set_tp(tp)
    want_tc = O.f32(ref_tc.forward(tc_prompt))
    ref_ids = O.Qwen3(cfg, seed=11, capacity=128)
    ref_ids.set_tp(tp)
    want_ids = ref_ids.generate_greedy(prompt, steps)
    want_sampled = ref_ids.generate_sampled(prompt, steps, SAMPLED["temperature"],
                                            SAMPLED["top_p"], SAMPLED["top_k"], SAMPLED["seed"])
    for r in range(tp):
        got = res[r]
        assert got["config"]["num_attention_heads"] == cfg["num_attention_heads"]
        np.testing.assert_array_equal(got["prefill"], want_prefill)
        np.testing.assert_array_equal(got["prefill_long"], want_long)
        # tensor-core accumulation order: logits within 1e-2 relative
        tc = O.f32(got["prefill_tc"])
        tc_err = float(np.max(np.abs(tc - want_tc)) / np.max(np.abs(want_tc)))
        assert tc_err <= 1e-2, f"rank {r}: >512-token prefill logits rel err {tc_err:.2e}"
        np.testing.assert_array_equal(got["loaded_prefill"], want_prefill)
        for a, b in zip(got["decode"], want_decode):
            np.testing.assert_array_equal(a, b)
        assert got["status"] == 0
        assert got["persistent"]  # decode runs in the persistent kernel with peer exchange
        for path in ("persistent", "graph", "eager"):
            np.testing.assert_array_equal(got[f"ids_{path}"], want_ids, err_msg=path)
        np.testing.assert_array_equal(got["sampled"], want_sampled)

#!/usr/bin/env python
"""Benchmark of the Qwen3 hot path on B200 (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: Qwen3-0.6B architecture, random-init FP16
N(0, 0.02) weights from seed 2, a 128-token prompt of uniform ids, then 256
greedy decode steps (batch 1, cache capacity 2048). One bench step is one
such request: prefill + 256 pipelined decode steps. `value` is decode
tokens/s timed on the device with CUDA events (inputs resident; the 1.2 GB of
weights exceed L2, so no flush is needed); `e2e` is the same metric through
the public generate call with the prompt copied from pinned host memory and
the ids read back, timed by the host clock around each call. With N > 1 GPUs
(torchrun) every rank serves its own replica (the 0.6B model is not sharded);
value = all ranks' decode tokens / max-over-ranks time.

`--impl reference` times the reference path on the host cores: the reference
(Rust + Metal) cannot be built or run here, so its arm is the C++ CPU oracle
(oracle/, a restatement of the reference kernels) on the same config.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "metal-infer-rs_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

INPUT_STREAM = 1 << 20
PROMPT = 128
DECODE = 256
CAPACITY = 2048
PROFILE_STEPS = 32  # decode steps of the per-kernel timing pass
SEED = 2
METRIC = "decode tokens/s (batch 1, greedy)"
CONFIG = dict(hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
              num_attention_heads=16, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6,
              rope_theta=1e6, vocab_size=151936, tie_word_embeddings=1)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def synthetic_tokens(ctx, seed: int, n: int, vocab: int):
    """Uniform prompt ids from the library's seeded SplitMix64 stream (the
    generator the weights use), made on the device and read back once."""
    import metal_infer as mi
    t = ctx.empty([n], mi.DType.U32)
    ctx.fill_tokens_u32(t, seed, INPUT_STREAM, vocab)
    return t.to_u32_vec()


# ---- algorithmic bytes ------------------------------------------------------------
def weight_bytes_per_layer(c):
    h, I = c["hidden_size"], c["intermediate_size"]
    qw = c["num_attention_heads"] * c["head_dim"]
    kw = c["num_key_value_heads"] * c["head_dim"]
    mats = (qw + 2 * kw) * h + h * qw + 2 * I * h + h * I
    norms = 2 * h + 2 * c["head_dim"]
    return 2 * (mats + norms)


def decode_bytes_per_token(c, kv_len):
    """Weight + KV bytes one decode step must read (the north-star roofline)."""
    h, V = c["hidden_size"], c["vocab_size"]
    kv = kv_len * c["num_key_value_heads"] * c["head_dim"] * 2 * 2 * c["num_hidden_layers"]
    return c["num_hidden_layers"] * weight_bytes_per_layer(c) + 2 * V * h + 2 * h + kv


def tp_decode_bytes_per_token(c, tp, kv_len):
    """Bytes one rank reads per decode step under tensor parallelism: its
    1/tp of every sharded matrix (heads, MLP columns, LM-head rows) and of
    the KV cache (KV heads), plus the replicated norms."""
    h, I, V = c["hidden_size"], c["intermediate_size"], c["vocab_size"]
    qw = c["num_attention_heads"] * c["head_dim"]
    kw = c["num_key_value_heads"] * c["head_dim"]
    mats = (qw + 2 * kw) * h + h * qw + 2 * I * h + h * I
    norms = 2 * h + 2 * c["head_dim"]
    layers = c["num_hidden_layers"]
    kv = kv_len * kw * 2 * 2 * layers
    return layers * (2 * mats / tp + 2 * norms) + 2 * V * h / tp + 2 * h + kv / tp


def prefill_flops(c, T):
    """FLOPs of a T-token prefill: every projection (2 per weight per token),
    causal attention (QK^T and PV over the T(T+1)/2 visible pairs) and the LM
    head of the last row."""
    h, I, V = c["hidden_size"], c["intermediate_size"], c["vocab_size"]
    qw = c["num_attention_heads"] * c["head_dim"]
    kw = c["num_key_value_heads"] * c["head_dim"]
    mats = (qw + 2 * kw) * h + h * qw + 2 * I * h + h * I
    attn = 4 * qw * T * (T + 1) // 2
    return c["num_hidden_layers"] * (2 * mats * T + attn) + 2 * V * h


# The prefill's canonical-order projections run on the CUDA cores (FMAs in
# the decode GEMVs' order, the token-exact path of prompts up to 512 tokens):
# 148 SMs x 128 FP32 lanes x 2 FLOPs per FMA at the maximum SM clock.
def ffma_peak_tflops(sm_mhz=1965.0):
    return 148 * 128 * 2 * sm_mhz * 1e6 / 1e12


def canon_gemm_probe(ctx, m=128, n=4096, k=1024, copies=16, reps=4):
    """TFLOP/s of the canonical prefill GEMM on the 0.6B fused Q/K/V shape
    (x[m, k] by w[n, k]) through the op API: `copies` weight copies (134 MB,
    more than L2) launched back to back, `reps` times, device time."""
    import metal_infer as mi
    x = ctx.empty([m, k])
    ctx.fill_normal_f16(x, 1, 4000, 1.0)
    ws = []
    for c in range(copies):
        w = ctx.empty([n, k])
        ctx.fill_normal_f16(w, 1, 4001 + c, 0.02)
        ws.append(w)
    b = ctx.begin_batch()
    outs = [b.matmul(x, w) for w in ws]
    b.finish()
    del outs
    b = ctx.begin_batch()
    outs = [b.matmul(x, w) for _ in range(reps) for w in ws]
    st = b.finish()
    del outs, ws, x
    t = st.gpu_time / (reps * copies)
    return 2.0 * m * n * k / t / 1e12, t


def gemv_bytes(n, k, segs=1):
    """One decode GEMV launch: `segs` weight matrices [n, k], the input row
    read once and `segs` output rows (FP16)."""
    return segs * n * k * 2 + k * 2 + segs * n * 2


def flash_decode_bytes(L, qh, kvh, hd):
    """One flash-decode launch: L cached K and V rows of every KV head, the
    queries and the output (FP16)."""
    return L * kvh * hd * 2 * 2 + qh * hd * 2 * 2


def kernel_bytes(c, name, mean_len, steps=1):
    """Algorithmic bytes of one launch of `name` (`steps` decode steps for the
    persistent decode kernel, which runs a whole call in one launch)."""
    if name == "decode_loop":
        return int(steps * decode_bytes_per_token(c, mean_len))
    h, I, V = c["hidden_size"], c["intermediate_size"], c["vocab_size"]
    qw = c["num_attention_heads"] * c["head_dim"]
    kw = c["num_key_value_heads"] * c["head_dim"]
    return {
        "qkv_gemv": 2 * ((qw + 2 * kw) * h + 2 * h + qw + 2 * kw),
        "attention_decode": 2 * (mean_len * kw * 2 + qw * 2 + kw * 2),
        "o_gemv": 2 * (h * qw + qw + h),
        "gate_up_gemv": 2 * (2 * I * h + 3 * h + I),
        "down_gemv": 2 * (h * I + I + 2 * h),
        "lm_head_argmax": 2 * (V * h + 2 * h + V),
    }.get(name)


# ---- clocks -------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []
        self.t = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            if self.t:
                self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---- our arm ------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    import metal_infer as mi

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        # gloo for host tensors (the NCCL id of the tensor-parallel block),
        # NCCL for the device-side max over ranks
        dist.init_process_group("cpu:gloo,cuda:nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))

    ctx = mi.MetalContext(local_rank)
    model = mi.Qwen3Model.random(ctx, CONFIG, seed=SEED)
    cache = model.kv_cache(CAPACITY)
    prompt = synthetic_tokens(ctx, SEED, PROMPT, CONFIG["vocab_size"])
    pinned = torch.from_numpy(prompt.astype(np.int64)).to(torch.int32).pin_memory()
    prompt_ptr = pinned.numpy().view(np.uint32)
    stream = torch.cuda.ExternalStream(ctx.stream())

    def one_step():
        """prefill + 256 decode steps; returns (prefill_ms, decode_ms)."""
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        slot = ctx.empty([1], mi.DType.U32)
        e0.record(stream)
        model.prefill_argmax(prompt_ptr, cache, slot)
        e1.record(stream)
        model.decode_steps(cache, DECODE)
        e2.record(stream)
        return e0, e1, e2

    for _ in range(args.warmup):
        ev = one_step()
        ev[2].synchronize()

    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    events = []
    with ClockSampler(local_rank) as clocks:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            events.append(one_step())
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    # Validation of the timed run: no bounded device wait expired (a launch
    # that gave up would leave early and be timed as fast: kernel_status
    # raises MI_ERR_TIMEOUT), and the last request's ids (read through the
    # cache's token ring) are the CPU oracle's greedy ids for this config,
    # committed as tests/golden/qwen3_0_6b_greedy.json.
    ctx.kernel_status()
    ids = cache.tokens(PROMPT, DECODE + 1)
    golden = golden_ids()
    prefill_ms = sum(e0.elapsed_time(e1) for e0, e1, _ in events)
    decode_ms = sum(e1.elapsed_time(e2) for _, e1, e2 in events)
    total_ms = sum(e0.elapsed_time(e2) for e0, _, e2 in events)
    if dist:
        t = torch.tensor([decode_ms, prefill_ms, total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        decode_ms, prefill_ms, total_ms = (float(x) for x in t.tolist())

    decode_tps = world * DECODE * args.steps / (decode_ms / 1e3)
    prefill_tps = world * PROMPT * args.steps / (prefill_ms / 1e3)

    # e2e: the public generate call, host prompt in, host ids out.
    e2e_times = []
    out_ids = None
    for i in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        t = time.perf_counter()
        out_ids = model.generate(prompt_ptr, DECODE + 1, cache)
        dt = time.perf_counter() - t
        if i >= args.warmup:
            e2e_times.append(dt)
    ctx.kernel_status()
    e2e_s = sum(e2e_times)
    if dist:
        t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_tps = world * DECODE * args.steps / e2e_s

    # Live per-kernel timing (CUDA events per launch on the engine stream).
    model.prefill_argmax(prompt_ptr, cache, ctx.empty([1], mi.DType.U32))
    ctx.set_kernel_profiling(True)
    ctx.take_kernel_profiles()
    model.decode_steps(cache, PROFILE_STEPS)
    ctx.synchronize()
    prof = ctx.take_kernel_profiles()
    ctx.set_kernel_profiling(False)
    per = {}
    for name, sec in prof:
        d = per.setdefault(name, [0, 0.0])
        d[0] += 1
        d[1] += sec
    mean_len = PROMPT + (PROFILE_STEPS + 1) / 2.0
    hbm, peak_kind = peaks()
    kernels = {}
    for name, (n, sec) in per.items():
        b = kernel_bytes(CONFIG, name, mean_len, PROFILE_STEPS)
        avg = sec / n
        kernels[name] = {"launches": n, "avg_us": round(avg * 1e6, 3),
                         "share": round(sec / sum(s for _, s in per.values()), 4),
                         "gbs": round(b / avg / 1e9, 1) if b else None}
    dominant = max(per, key=lambda k: per[k][1])
    dom_avg = per[dominant][1] / per[dominant][0]
    dom_bytes = kernel_bytes(CONFIG, dominant, mean_len, PROFILE_STEPS)
    achieved = dom_bytes / dom_avg / 1e9
    traffic = read_traffic(dominant)

    # Sampled decode (generate_with, temperature > 0): the kernel chain with
    # the lm_head's key histogram and the one-CTA sampler after every head.
    # Decode rate = 64 steps / (time of a 65-token call - a 1-token call).
    sampled = {}
    sampled_cases = [] if args.no_sampled_report else [
        ("top_k20_top_p0.95_t0.6", dict(temperature=0.6, top_p=0.95, top_k=20)),
        ("full_vocab_t1.0", dict(temperature=1.0, top_p=1.0, top_k=0))]
    for label, opts in sampled_cases:
        opts = dict(opts, seed=SEED)
        model.generate_with(prompt_ptr, dict(opts, max_tokens=17), cache)  # graph capture
        spans = []
        for n in (1, 65):
            torch.cuda.synchronize()
            t = time.perf_counter()
            model.generate_with(prompt_ptr, dict(opts, max_tokens=n), cache)
            spans.append(time.perf_counter() - t)
        ctx.set_kernel_profiling(True)
        ctx.take_kernel_profiles()
        model.generate_with(prompt_ptr, dict(opts, max_tokens=17), cache)
        ctx.synchronize()
        prof_s = ctx.take_kernel_profiles()
        ctx.set_kernel_profiling(False)
        smp = [s for n, s in prof_s if n == "sample"]
        hist = [s for n, s in prof_s if n == "sample_histogram"]
        sampled[label] = {
            "decode_tokens_per_s": round(64 / max(spans[1] - spans[0], 1e-9), 1),
            "note": "generate_with, host clock: persistent kernel one step per launch + histogram + sampler",
            "sample_kernel_us": round(sum(smp) / len(smp) * 1e6, 2) if smp else None,
            "histogram_kernel_us": round(sum(hist) / len(hist) * 1e6, 2) if hist else None,
        }

    kv_mean = PROMPT + (DECODE + 1) / 2.0
    bytes_tok = decode_bytes_per_token(CONFIG, kv_mean)
    per_gpu_tps = decode_tps / world

    ok = bool(np.array_equal(ids, out_ids)) if out_ids is not None else False
    n_cmp = min(len(golden), DECODE + 1)
    match_golden = bool(np.array_equal(ids[:n_cmp], golden[:n_cmp]))
    match_golden_e2e = bool(out_ids is not None and np.array_equal(out_ids[:n_cmp], golden[:n_cmp]))

    persistent = model.decode_persistent()
    # Tensor parallelism: Qwen3-8B sharded over the same
    # ranks (TP1 on one GPU), after the replica model is freed.
    del model, cache
    ctx.synchronize()
    # BASELINE config 1 (the decode ops alone, rotated working sets), one GPU
    sweep = None
    if world == 1 and not args.no_op_sweep:
        sweep = {r["op"]: {"kernel": r["kernel"], "us_per_launch": r["us_per_launch"],
                           "gb_s": r["gb_s"], "frac": r["frac"], "bytes": r["bytes"]}
                 for r in op_sweep_rows(ctx, 3, 1)}
    gemm_probe = canon_gemm_probe(ctx) if world == 1 and not args.no_op_sweep else None
    tp_block = None if args.no_tp_report else tp_report(args, ctx, rank, world, dist)
    layer_launches = 5 * CONFIG["num_hidden_layers"] + 1
    prefill_launches = 1 + 11 * CONFIG["num_hidden_layers"] + 2
    decode_launches = 1 if persistent else DECODE * layer_launches
    launches = args.steps * (prefill_launches + decode_launches)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(decode_tps, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (random-init FP16 N(0,0.02) weights, uniform prompt ids)",
            "config": workload_config(world),
            "prefill_tokens_per_s": round(prefill_tps, 1),
            "prefill_roofline": prefill_roofline(prefill_tps / world, gemm_probe,
                                                 clocks.summary()),
            "decode_hbm": {"bytes_per_token": int(bytes_tok),
                           "achieved_gbs": round(bytes_tok * per_gpu_tps / 1e9, 1),
                           "peak_gbs": hbm, "frac": round(bytes_tok * per_gpu_tps / 1e9 / hbm, 4),
                           "note": f"weights + KV bytes per token / time, {peak_kind} peak"},
            "greedy_ids_consistent": ok,
            "ids_match_golden": match_golden and match_golden_e2e,
            "validation": {"kernel_status": "ok (no bounded device wait expired)",
                           "ids_vs_golden": f"{n_cmp} ids of the timed run and of the e2e "
                                            "generate call vs the CPU oracle's greedy ids "
                                            "(tests/golden/qwen3_0_6b_greedy.json)",
                           "timed_ids_match": match_golden, "e2e_ids_match": match_golden_e2e,
                           "decode_paths_agree": ok},
            "e2e": {"value": round(e2e_tps, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": PROMPT * 4, "d2h_bytes_per_step": (DECODE + 1) * 4,
                    "note": "mi_qwen3_generate per request (prefill included), host clock"},
            "roofline": {"bound": "hbm", "kernel": dominant, "achieved": round(achieved, 1),
                         "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                         "traffic": traffic, "bytes_per_launch": dom_bytes,
                         "traffic_source": "not measured in this run: ncu DRAM bytes of the "
                                           "committed summary profiles/ncu_traffic.md, scaled "
                                           "to this launch's steps",
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"},
            "decode_path": "persistent kernel" if persistent else "kernel chain (CUDA graph)",
            "sampled_decode": sampled,
            "kernels": kernels,
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "wall_s": round(wall, 3),
        }
        if tp_block is not None:
            line["tp"] = tp_block
        if sweep is not None:
            line["kernels_sweep"] = {
                "workload": "BASELINE config 1: each decode GEMV shape and flash-decode attention "
                            "(16 q / 8 KV heads) at L = 512 / 2048 / 8192 through the op API, "
                            f"rotated working sets > {ROTATE_BYTES >> 20} MB, median of 3",
                "peak_gbs": hbm, "ops": sweep}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.cpu_sample_steps)
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if not (match_golden and match_golden_e2e and ok):
        sys.exit("bench: the generated ids differ from the oracle's greedy ids")


def golden_ids():
    import numpy as np
    with open(os.path.join(ROOT, "tests", "golden", "qwen3_0_6b_greedy.json")) as f:
        g = json.load(f)
    assert g["seed"] == SEED and g["prompt_len"] == PROMPT and g["prompt_stream"] == INPUT_STREAM
    return np.array(g["ids"], dtype=np.uint32)


TP_REPORT_STEPS = 2  # timed requests of the tensor-parallel block (after one warm-up)


def tp_report(args, ctx, rank, world, dist):
    """BASELINE config 3 at TP = the bench's GPU count: Qwen3-8B shapes
    (seed 3), a 2048-token prompt then 512 greedy decode steps, capacity
    4096, one warm-up request and TP_REPORT_STEPS timed ones. Heads, MLP
    columns and LM-head rows are split over the ranks; the persistent decode
    kernel exchanges the row-parallel O / down partials and the argmax
    records through the ranks' mailboxes over NVLink. Device times are the
    max over ranks."""
    import numpy as np
    import torch
    import metal_infer as mi

    name, cfg, seed, prompt_len, decode, cfg_id = TP_WORKLOADS["8b-tp"]
    capacity = 4096
    ident = mi.share_nccl_id() if world > 1 else bytes(128)
    model = mi.Qwen3Model.random_tp(ctx, cfg, seed=seed, tp=world, rank=rank, nccl_id=ident)
    prompt = synthetic_tokens(ctx, seed, prompt_len, cfg["vocab_size"])
    stream = torch.cuda.ExternalStream(ctx.stream())
    times, waits, ids = [], [], None
    for i in range(1 + TP_REPORT_STEPS):
        cache = model.kv_cache(capacity)
        slot = ctx.empty([1], mi.DType.U32)
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(stream)
        model.prefill_argmax(prompt, cache, slot)
        e1.record(stream)
        model.decode_steps(cache, decode)
        e2.record(stream)
        e2.synchronize()
        ctx.kernel_status()
        if i >= 1:
            times.append((e0.elapsed_time(e1), e1.elapsed_time(e2)))
            waits.append(model.exchange_wait()["mean_s"])
        ids = cache.tokens(prompt_len, decode + 1)
        del cache
    prefill_ms = sum(t[0] for t in times)
    decode_ms = sum(t[1] for t in times)
    wait_s = sum(waits)
    agree = True
    if world > 1:
        t = torch.tensor([prefill_ms, decode_ms, wait_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        prefill_ms, decode_ms, wait_s = (float(x) for x in t.tolist())
        mine = torch.tensor(ids.astype(np.int64), device="cuda")
        ref = mine.clone()
        dist.broadcast(ref, src=0)
        same = torch.tensor([int(bool(torch.equal(mine, ref)))], device="cuda")
        dist.all_reduce(same, op=dist.ReduceOp.MIN)
        agree = bool(same.item())
    persistent = model.decode_persistent()
    del model
    ctx.synchronize()
    tokens = decode * len(times)
    tps = tokens / (decode_ms / 1e3)
    kv_mean = prompt_len + (decode + 1) / 2.0
    per_rank = tp_decode_bytes_per_token(cfg, world, kv_mean)
    hbm, peak_kind = peaks()
    gbs = per_rank * tps / 1e9
    return {
        "workload": f"{name} TP{world} (BASELINE config {cfg_id}): {prompt_len}-token prompt + "
                    f"{decode} greedy decode steps, capacity {capacity}, seed {seed}",
        "tp": world, "nccl_ranks": world if world > 1 else 0,
        "decode_tokens_per_s": round(tps, 2),
        "ms_per_token": round(decode_ms / tokens, 4),
        "prefill_tokens_per_s": round(prompt_len * len(times) / (prefill_ms / 1e3), 1),
        "hbm_per_gpu": {"bytes_per_token_per_rank": int(per_rank), "achieved_gbs": round(gbs, 1),
                        "peak_gbs": hbm, "frac": round(gbs / hbm, 4),
                        "note": f"this rank's weight + KV bytes per token / time, {peak_kind} peak"},
        "exchange_wait_us_per_token": round(wait_s / tokens * 1e6, 3) if world > 1 else 0.0,
        "exchange_note": "mean over CTAs of the time spent waiting on the O / down / LM-head "
                         "mailbox counters (partials of the other ranks over NVLink), max over "
                         "ranks" if world > 1 else "one GPU: no exchange",
        "decode_path": "persistent kernel" if persistent else "per-kernel chain + NCCL all-gathers",
        "ids_ranks_agree": agree,
        "timed_requests": len(times),
    }


def read_traffic(kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.md")
    try:
        for line in open(path):
            m = re.match(r"\|\s*(\w+)\s*\|\s*([\d.]+)\s*\|", line)
            if m and m.group(1) == kernel:
                return float(m.group(2))
    except OSError:
        pass
    return None


def workload_config(world):
    """The `config` of both arms' lines (the same workload)."""
    return {"workload": f"Qwen3-0.6B batch-1 greedy: {PROMPT}-token prompt + {DECODE} decode "
                        "steps (BASELINE config 2)",
            "layers": 28, "hidden": 1024, "vocab": 151936, "prompt": PROMPT,
            "decode_steps": DECODE, "kv_capacity": CAPACITY,
            "parallelism": f"replicas x{world}",
            "l2": "weights 1.2 GB > 126 MB L2 (no flush needed)"}


# ---- CPU legs ---------------------------------------------------------------------------
def oracle_decode_rate(decode_steps: int):
    import oracle as O
    m = O.Qwen3(CONFIG, seed=SEED, capacity=CAPACITY)
    prompt = O.gen_tokens(SEED, INPUT_STREAM, PROMPT, CONFIG["vocab_size"])
    t = time.perf_counter()
    logits = m.forward(prompt)
    prefill_s = time.perf_counter() - t
    tok = O.argmax(logits)
    return m, tok, prefill_s


def cpu_baseline(decode_steps: int):
    import numpy as np
    import oracle as O
    m, tok, prefill_s = oracle_decode_rate(decode_steps)
    t = time.perf_counter()
    for _ in range(decode_steps):
        tok = O.argmax(m.forward(np.array([tok], np.uint32)))
    dt = time.perf_counter() - t
    threads = O.lib().or_num_threads()
    m.close()
    return {"value": round(decode_steps / dt, 3), "unit": "tokens/s", "cores": threads,
            "kind": "port",
            "sample": f"C++ oracle (OpenMP, {threads} threads): 128-token prefill "
                      f"({prefill_s:.1f} s, untimed) then {decode_steps} greedy decode steps of "
                      "the same Qwen3-0.6B workload"}


def run_reference(args, rank):
    """The reference arm: the reference's kernels restated in C++ (oracle/) on
    the host cores, on the same workload as our arm. After the 128-token
    prompt (untimed) the timed steps together decode the request's 256 greedy
    tokens in order, each step a consecutive slice of them (so the mean KV
    length, 256.5, is our arm's); warm-up steps decode a slice and roll the
    cache back to the prompt. The ids are checked against the committed
    golden ids of the same config."""
    if rank != 0:
        return
    import numpy as np
    import oracle as O
    m, first, prefill_s = oracle_decode_rate(0)
    base = len(m)
    slices = [DECODE // args.steps + (1 if i < DECODE % args.steps else 0)
              for i in range(args.steps)]
    for _ in range(args.warmup):
        tok = first
        for _ in range(max(slices)):
            tok = O.argmax(m.forward(np.array([tok], np.uint32)))
        m.truncate(base)
    tok, ids, times = first, [first], []
    for n in slices:
        t = time.perf_counter()
        for _ in range(n):
            tok = O.argmax(m.forward(np.array([tok], np.uint32)))
            ids.append(tok)
        times.append(time.perf_counter() - t)
    threads = O.lib().or_num_threads()
    m.close()
    golden = golden_ids()
    n_cmp = min(len(golden), len(ids))
    match = bool(np.array_equal(np.array(ids[:n_cmp], np.uint32), golden[:n_cmp]))
    value = sum(slices) / sum(times)
    sample = (f"reference path restated in C++ (oracle/, OpenMP {threads} threads; the Rust/Metal "
              f"reference cannot run here): after the {PROMPT}-token prompt ({prefill_s:.1f} s, "
              f"untimed) the {args.steps} timed steps decode the {sum(slices)} greedy tokens in "
              f"order ({min(slices)}-{max(slices)} per step), Qwen3-0.6B seed 2")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * sum(times) / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (random-init FP16 N(0,0.02) weights, uniform prompt ids)",
            "config": workload_config(args.gpus),
            "ids_match_golden": match,
            "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- tensor-parallel workloads (BASELINE configs 3 and 4) ----------------------------
CONFIG_8B = dict(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                 num_attention_heads=32, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6,
                 rope_theta=1e6, vocab_size=151936, tie_word_embeddings=0)
CONFIG_32B = dict(hidden_size=5120, intermediate_size=25600, num_hidden_layers=64,
                  num_attention_heads=64, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6,
                  rope_theta=1e6, vocab_size=151936, tie_word_embeddings=0)
# workload: (name, config, seed, prompt tokens, decode steps, BASELINE config)
TP_WORKLOADS = {
    "8b-tp": ("Qwen3-8B", CONFIG_8B, 3, 2048, 512, 3),
    "32b-tp": ("Qwen3-32B", CONFIG_32B, 4, 32768, 256, 4),
}


def run_tp(args, rank, world, local_rank):
    """A Qwen3-8B (config 3) or Qwen3-32B (config 4) shape sharded over the
    torchrun ranks: the config's prompt (`--prompt-tokens` overrides it), then
    `--decode-steps` greedy steps (default: the config's), capacity prompt +
    decode. value = decode tokens/s of the one sequence (all ranks serve it;
    max over ranks of the device time)."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    import metal_infer as mi

    name, cfg, seed, prompt_len, decode, cfg_id = TP_WORKLOADS[args.workload]
    if args.prompt_tokens:
        prompt_len = args.prompt_tokens
    if args.decode_steps is not None:
        decode = args.decode_steps
    capacity = prompt_len + decode if cfg_id == 4 else 4096
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
        ident = mi.share_nccl_id()
    else:
        ident = bytes(128)  # one GPU: no communicator (tp = 1 is the plain model)
    ctx = mi.MetalContext(local_rank)
    model = mi.Qwen3Model.random_tp(ctx, cfg, seed=seed, tp=world, rank=rank, nccl_id=ident)
    prompt = synthetic_tokens(ctx, seed, prompt_len, cfg["vocab_size"])
    stream = torch.cuda.ExternalStream(ctx.stream())
    times = []
    for i in range(args.warmup + args.steps):
        cache = model.kv_cache(capacity)
        slot = ctx.empty([1], mi.DType.U32)
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(stream)
        model.prefill_argmax(prompt, cache, slot)
        e1.record(stream)
        model.decode_steps(cache, decode)
        e2.record(stream)
        e2.synchronize()
        if i >= args.warmup:
            times.append((e0.elapsed_time(e1), e1.elapsed_time(e2)))
        del cache
    prefill_ms = sum(t[0] for t in times)
    decode_ms = sum(t[1] for t in times)
    if world > 1:
        t = torch.tensor([prefill_ms, decode_ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        prefill_ms, decode_ms = t.tolist()
    if rank == 0:
        print(json.dumps({
            "metric": "decode tokens/s (batch 1, greedy)", "impl": "ours",
            "value": round(decode * args.steps / (decode_ms / 1e3), 2), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round((prefill_ms + decode_ms) / args.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (random-init FP16 N(0,0.02) weights, uniform prompt ids)",
            "config": {"workload": f"{name} tensor-parallel TP{world}: {prompt_len}-token prompt + "
                                   f"{decode} decode steps (BASELINE config {cfg_id} shapes)",
                       "parallelism": f"tp{world}", "kv_capacity": capacity},
            "prefill_tokens_per_s": round(prompt_len * args.steps / (prefill_ms / 1e3), 1),
            "decode_path": "persistent kernel" if model.decode_persistent()
                           else "per-kernel chain + NCCL all-gathers"}), flush=True)
    del model
    ctx.synchronize()
    if world > 1:
        dist.destroy_process_group()


# ---- op sweep -------------------------------------------------------
# GEMV shapes (out x in, weights per launch) and decode attention lengths.
SWEEP_GEMV = [("q_proj", 2048, 1024, 1), ("k_proj", 1024, 1024, 1), ("v_proj", 1024, 1024, 1),
              ("o_proj", 1024, 2048, 1), ("gate_up", 3072, 1024, 2), ("down", 1024, 3072, 1),
              ("lm_head", 151936, 1024, 1)]
SWEEP_ATTN = [512, 2048, 8192]
ROTATE_BYTES = 256 << 20   # working set of distinct operands per batch, above the 126 MB L2
SLEEP_CYCLES = 40_000_000  # ~20 ms spin queued first, so the launches run back to back


def run_op_sweep(args):
    """each decode GEMV shape and flash-decode attention at
    L = 512 / 2048 / 8192 (16 query / 8 KV heads, head_dim 128) through the
    C-ABI batch, with the rotated working-set protocol of the reference's
    `bench kernel --rotate` (bench.rs:849-912): one batch launches the op once
    per distinct copy of its operands (together > 256 MB, so every launch
    reads HBM), and the batch's device time is divided by the copies. A
    bounded ~20 ms spin is queued on the stream before each batch so that the
    host has enqueued every launch before the first one runs (the time is then
    the kernels', not the host's launch rate). Bytes per launch are the
    algorithmic ones: weights + input + output (GEMV), K/V rows + q + out
    (attention)."""
    import torch
    import metal_infer as mi

    torch.cuda.set_device(0)
    ctx = mi.MetalContext(0)
    peak, peak_kind = peaks()
    only = set(args.ops.split(",")) if args.ops else None
    rows = op_sweep_rows(ctx, args.steps, args.warmup, only)
    total_bytes = sum(r["bytes"] for r in rows)
    total_s = sum(r["us_per_launch"] for r in rows) / 1e6
    print(json.dumps({
        "metric": "GEMV / attention HBM GB/s (op sweep)", "impl": "ours",
        "value": round(total_bytes / total_s / 1e9, 1), "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "dtype": "f16", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "config": {"workload": "BASELINE config 1 decode-op sweep, rotated working sets "
                               f"> {ROTATE_BYTES >> 20} MB (inputs larger than L2)"},
        "peak": {"hbm_gbs": peak, "kind": peak_kind}, "ops": rows}), flush=True)


def prefill_roofline(prefill_tps_per_gpu, gemm_probe, clocks):
    """The prefill against the CUDA-core FMA peak (its projections are the
    canonical-order GEMM), and the GEMM alone on the fused Q/K/V shape."""
    peak = ffma_peak_tflops(clocks.get("sm_max_mhz") or 1965.0)
    fl = prefill_flops(CONFIG, PROMPT)
    achieved = fl * prefill_tps_per_gpu / PROMPT / 1e12
    out = {"bound": "cuda-core fma (canonical-order projections)",
           "flops_per_prompt": int(fl), "achieved_tflops": round(achieved, 2),
           "peak_tflops": round(peak, 1), "frac": round(achieved / peak, 4),
           "peak_source": "148 SMs x 128 lanes x 2 FLOPs x max SM clock",
           "note": "whole prefill per GPU (norms, attention and launches included)"}
    if gemm_probe is not None:
        tf, t = gemm_probe
        out["gemm_canon_128x4096x1024"] = {"tflops": round(tf, 2), "us": round(t * 1e6, 2),
                                           "frac": round(tf / peak, 4)}
    return out


def op_sweep_rows(ctx, steps, warmup, only=None):
    """The op sweep's rows on context `ctx` (see run_op_sweep): per op the
    median device time per launch, its algorithmic bytes and GB/s."""
    import math
    import torch
    import metal_infer as mi

    stream = torch.cuda.ExternalStream(ctx.stream())
    peak, _ = peaks()

    def timed(encode, copies):
        """Median device seconds per launch, and the slowest host enqueue of a
        batch (it must stay well under the spin for the timing to hold)."""
        samples, enqueue = [], 0.0
        for i in range(warmup + steps):
            with torch.cuda.stream(stream):
                torch.cuda._sleep(SLEEP_CYCLES)
            t0 = time.perf_counter()
            b = ctx.begin_batch()
            outs = encode(b)
            t1 = time.perf_counter()
            st = b.finish()
            del outs
            if i >= warmup:
                samples.append(st.gpu_time / copies)
                enqueue = max(enqueue, t1 - t0)
        return statistics.median(samples), enqueue

    rows = []
    x_cache = {}
    for name, n, k, segs in SWEEP_GEMV:
        if only is not None and name not in only:
            continue
        bytes_ = gemv_bytes(n, k, segs)
        copies = max(1, math.ceil(ROTATE_BYTES / (segs * n * k * 2)))
        if k not in x_cache:
            x_cache[k] = ctx.empty([1, k], mi.DType.F16)
            ctx.fill_normal_f16(x_cache[k], 1, 1000 + k, 1.0)
        x = x_cache[k]
        ws = []
        for c in range(copies):
            group = []
            for s_ in range(segs):
                w = ctx.empty([n, k], mi.DType.F16)
                ctx.fill_normal_f16(w, 1, 16 * c + s_, 0.02)
                group.append(w)
            ws.append(group)
        if segs == 1:
            enc = lambda b: [b.matmul(x, g[0]) for g in ws]
        else:
            enc = lambda b: [b.matmul2(x, g[0], g[1]) for g in ws]
        t, enq = timed(enc, copies)
        rows.append({"op": name, "kernel": "gemv", "shape": f"{segs}x{n}x{k}" if segs > 1
                     else f"{n}x{k}", "bytes": bytes_, "copies": copies,
                     "us_per_launch": round(t * 1e6, 3), "gb_s": round(bytes_ / t / 1e9, 1),
                     "frac": round(bytes_ / t / 1e9 / peak, 3),
                     "host_enqueue_ms": round(enq * 1e3, 2)})
        del ws
        ctx.synchronize()
    qh, kvh, hd = 16, 8, 128
    q = ctx.empty([1, qh, hd], mi.DType.F16)
    ctx.fill_normal_f16(q, 1, 2000, 1.0)
    for L in SWEEP_ATTN:
        if only is not None and f"attention_L{L}" not in only:
            continue
        kv_bytes = L * kvh * hd * 2 * 2
        bytes_ = flash_decode_bytes(L, qh, kvh, hd)
        copies = max(1, math.ceil(ROTATE_BYTES / kv_bytes))
        kvs = []
        for c in range(copies):
            kk = ctx.empty([L, kvh, hd], mi.DType.F16)
            vv = ctx.empty([L, kvh, hd], mi.DType.F16)
            ctx.fill_normal_f16(kk, 1, 3000 + 2 * c, 1.0)
            ctx.fill_normal_f16(vv, 1, 3001 + 2 * c, 1.0)
            kvs.append((kk, vv))
        cfg = mi.AttentionConfig(qh, kvh, hd, 1, L - 1)
        enc = lambda b: [b.attention(q, kk, vv, cfg, mi.AttentionKind.FLASH_DECODE)
                         for kk, vv in kvs]
        t, enq = timed(enc, copies)
        rows.append({"op": f"attention_L{L}", "kernel": "flash_decode",
                     "shape": f"q[1,{qh},{hd}] kv[{L},{kvh},{hd}]", "bytes": bytes_,
                     "copies": copies, "us_per_launch": round(t * 1e6, 3),
                     "gb_s": round(bytes_ / t / 1e9, 1), "frac": round(bytes_ / t / 1e9 / peak, 3),
                     "host_enqueue_ms": round(enq * 1e3, 2)})
        del kvs
        ctx.synchronize()
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", choices=["0.6b", "8b-tp", "32b-tp", "op-sweep"],
                    default="0.6b",
                    help="0.6b: the headline config (replicas over GPUs); 8b-tp / 32b-tp: "
                         "Qwen3-8B / Qwen3-32B shapes sharded over the GPUs; op-sweep: the "
                         "decode GEMV and attention kernels alone (one GPU)")
    ap.add_argument("--ops", default="",
                    help="op-sweep: comma-separated subset (q_proj, ..., lm_head, "
                         "attention_L512, attention_L2048, attention_L8192)")
    ap.add_argument("--prompt-tokens", type=int, default=0,
                    help="tensor-parallel workloads: prompt length instead of the config's")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sampled-report", action="store_true",
                    help="skip the untimed sampled-decode report (short profiling runs)")
    ap.add_argument("--no-tp-report", action="store_true",
                    help="skip the Qwen3-8B tensor-parallel block (short profiling runs)")
    ap.add_argument("--no-op-sweep", action="store_true",
                    help="skip the decode-op sweep block (short profiling runs)")
    ap.add_argument("--cpu-sample-steps", type=int, default=48)
    ap.add_argument("--decode-steps", type=int, default=None,
                    help="decode steps per request (smaller only for profiler launch lists)")
    args = ap.parse_args()
    if args.decode_steps is not None and args.workload == "0.6b":
        globals()["DECODE"] = args.decode_steps
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.workload in TP_WORKLOADS:
        run_tp(args, rank, world, local_rank)
        return
    if args.workload == "op-sweep":
        if rank == 0:
            run_op_sweep(args)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()

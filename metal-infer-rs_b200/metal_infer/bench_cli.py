"""Benchmark command line with the reference's report formats
(crates/metal-infer-cli/src/bin/bench.rs and inference.rs), run on the B200
engine:

    python -m metal_infer.bench_cli [--format table|json] kernel --m 1 --n 1024 --k 1024
    python -m metal_infer.bench_cli attention --kind compare --tokens 1 --length 640
    python -m metal_infer.bench_cli model (--model DIR | --random 0.6b|8b) --prompt 512 \\
        --generate 128 [--profile-kernels] [--decode-mode pipelined|synchronous|persistent]
    python -m metal_infer.bench_cli inference --model DIR --workload case.json \\
        --mode fixed|autoregressive

JSON fields follow bench.rs `Report` / `PhaseReport` / `KernelProfileReport`
(bench.rs:238-309) and inference.rs `InferenceReport` (schema_version 2,
reading workload schema_version 1, inference.rs:28-81). Apple-specific
switches (--rows, --split-k, --half8, --gemv-config, --shared-gate-up-input)
have no meaning on this engine and are not offered. The table format prints
the same lines as the reference's.
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from typing import List, Optional

import numpy as np

import metal_infer as mi

BACKEND_NAMES = {mi.MatmulBackend.AUTO: "auto", mi.MatmulBackend.REFERENCE: "reference-msl",
                 mi.MatmulBackend.NATIVE: "native-msl", mi.MatmulBackend.MPS: "mps"}


class BenchError(ValueError):
    pass


# ---- statistics (bench.rs:1733-1775, 1995-2031) -------------------------------------------
def duration_stats(samples_s: List[float]) -> dict:
    s = sorted(samples_s)
    mean = sum(s) / len(s) if s else 0.0
    median = s[len(s) // 2] if s else 0.0
    p95 = s[int(round((max(len(s) - 1, 0)) * 0.95))] if s else 0.0
    return {"mean_ms": mean * 1e3, "median_ms": median * 1e3, "p95_ms": p95 * 1e3}


def report(benchmark: str, ctx, samples: List[float], gpu_samples: Optional[List[float]] = None,
           throughput: Optional[float] = None, unit: Optional[str] = None) -> dict:
    wall = duration_stats(samples)
    r = {"benchmark": benchmark, "device": ctx.device_name(), "iterations": len(samples),
         "mean_ms": wall["mean_ms"], "median_ms": wall["median_ms"], "p95_ms": wall["p95_ms"]}
    if gpu_samples is not None:
        g = duration_stats(gpu_samples)
        r.update(gpu_mean_ms=g["mean_ms"], gpu_median_ms=g["median_ms"], gpu_p95_ms=g["p95_ms"])
    r.update(throughput=throughput, throughput_unit=unit, allocated_bytes=ctx.allocated_bytes(),
             matmul_backend=BACKEND_NAMES.get(ctx.matmul_backend(), "auto"), prefill=None,
             decode=None)
    return r


def phase_report(tokens: int, wall: List[float], gpu: List[float]) -> dict:
    w, g = duration_stats(wall), duration_stats(gpu)
    return {"tokens": tokens, "wall_mean_ms": w["mean_ms"], "wall_median_ms": w["median_ms"],
            "wall_p95_ms": w["p95_ms"], "gpu_mean_ms": g["mean_ms"],
            "gpu_median_ms": g["median_ms"], "gpu_p95_ms": g["p95_ms"],
            "tokens_per_second": tokens / (w["mean_ms"] / 1e3) if w["mean_ms"] > 0 else 0.0}


def kernel_phase_profile(gpu_samples: List[float], dispatches) -> dict:
    """kernel_phase_profile (bench.rs:1897-1933)."""
    gpu_ms = sum(gpu_samples) * 1e3
    totals = {}
    for name, sec in dispatches:
        calls, total = totals.get(name, (0, 0.0))
        totals[name] = (calls + 1, total + sec * 1e3)
    attributed = sum(t for _, t in totals.values())
    rows = [{"kernel": k, "calls": c, "total_gpu_ms": t, "mean_gpu_ms": t / c}
            for k, (c, t) in totals.items()]
    rows.sort(key=lambda r: (-r["total_gpu_ms"], r["kernel"]))
    return {"gpu_ms": gpu_ms, "attributed_ms": attributed, "unattributed_ms": gpu_ms - attributed,
            "kernels": rows}


def measure_dispatch(ctx, iterations: int, encode):
    """Wall and GPU seconds of `iterations` committed batches."""
    wall, gpu = [], []
    for _ in range(iterations):
        t = time.perf_counter()
        b = ctx.begin_batch()
        encode(b)
        st = b.finish()
        wall.append(time.perf_counter() - t)
        gpu.append(st.gpu_time)
    return wall, gpu


# ---- subcommands ---------------------------------------------------------------------------
def run_kernel(ctx, a) -> dict:
    """Command::Kernel (bench.rs:440-506): matmul_f16[m,n,k] on constant data."""
    ctx.set_matmul_backend({"auto": mi.MatmulBackend.AUTO,
                            "reference": mi.MatmulBackend.REFERENCE,
                            "native": mi.MatmulBackend.NATIVE}[a.matmul_backend])
    x = ctx.tensor_f16(np.full(a.m * a.k, 0.01, np.float32), [a.m, a.k])
    w = ctx.tensor_f16(np.full(a.n * a.k, 0.02, np.float32), [a.n, a.k])
    for _ in range(a.warmup):
        b = ctx.begin_batch()
        b.matmul(x, w)
        b.finish()
    wall, gpu = measure_dispatch(ctx, a.iterations, lambda b: b.matmul(x, w))
    flops = 2.0 * a.m * a.n * a.k
    return report(f"matmul_f16[{a.m},{a.n},{a.k}]", ctx, wall, gpu,
                  (flops / 1e12) / (sum(wall) / len(wall)), "TFLOP/s")


ATTENTION_KINDS = {"reference": mi.AttentionKind.REFERENCE, "tiled": mi.AttentionKind.TILED,
                   "flash-prefill": mi.AttentionKind.FLASH_PREFILL,
                   "decode-split-kv": mi.AttentionKind.DECODE_SPLIT_KV,
                   "flash-decode": mi.AttentionKind.FLASH_DECODE}


def attention_inputs(T: int, L: int, qh: int, kvh: int, hd: int):
    """The attention subcommand's seeded Q [T, qh, hd], K and V [L, kvh, hd]
    (N(0, 1) rounded to FP16), as float32 arrays."""
    rng = np.random.default_rng(0)
    return (rng.normal(0, 1, T * qh * hd).astype(np.float32),
            rng.normal(0, 1, L * kvh * hd).astype(np.float32),
            rng.normal(0, 1, L * kvh * hd).astype(np.float32))


def run_attention(ctx, a) -> dict:
    """Command::Attention (bench.rs:560-581, 927-1108): each attention kind
    on random Q/K/V, with its max abs error against the reference kind."""
    T, L, qh, kvh, hd = a.tokens, a.length, a.query_heads, a.kv_heads, a.head_dim
    qf, kf, vf = attention_inputs(T, L, qh, kvh, hd)
    q = ctx.tensor_f16(qf, [T, qh, hd])
    k = ctx.tensor_f16(kf, [L, kvh, hd])
    v = ctx.tensor_f16(vf, [L, kvh, hd])
    cfg = mi.AttentionConfig(qh, kvh, hd, 1, L - T)
    kinds = ATTENTION_KINDS
    names = list(kinds) if a.kind == "compare" else [a.kind]
    if T != 1:
        names = [n for n in names if n not in ("decode-split-kv", "flash-decode")]
    ref = ctx.attention(q, k, v, cfg, mi.AttentionKind.REFERENCE).to_f32_vec()
    variants = {}
    for name in names:
        kind = kinds[name]
        for _ in range(a.warmup):
            ctx.attention(q, k, v, cfg, kind)
        wall, gpu = measure_dispatch(ctx, a.iterations, lambda b: b.attention(q, k, v, cfg, kind))
        out = ctx.attention(q, k, v, cfg, kind).to_f32_vec()
        g = duration_stats(gpu)
        variants[name.replace("-", "_")] = {
            "kind": name, "gpu_mean_ms": g["mean_ms"], "gpu_median_ms": g["median_ms"],
            "gpu_p95_ms": g["p95_ms"], "max_abs_error": float(np.max(np.abs(out - ref)))}
    first = variants[names[0].replace("-", "_")]
    r = report(f"attention[{T},{L},{qh},{kvh},{hd}]", ctx, [first["gpu_mean_ms"] / 1e3])
    r["attention_comparison"] = variants
    return r


def _load_model(ctx, a):
    if a.model:
        return mi.Qwen3Model.load(a.model, ctx)
    cfg = {"0.6b": mi.QWEN3_0_6B, "8b": mi.QWEN3_8B}[a.random]
    return mi.Qwen3Model.random(ctx, cfg, seed=2)


def run_model(ctx, a) -> dict:
    """Command::Model (bench.rs:598-735, 1776-1895): prefill of `prompt` ones,
    then `generate` greedy steps, per iteration."""
    if a.prompt == 0 or a.generate == 0 or a.iterations == 0:
        raise BenchError("model prompt, generate, and iterations must be greater than zero")
    model = _load_model(ctx, a)
    opts = mi.FusionOptions(int(a.fuse_qkv), int(a.fuse_gate_up), int(a.fuse_add_rms_norm),
                            int(a.fuse_qk_rope_cache))
    model.set_fusion_options(opts)  # as bench.rs:675-681: the flags, all off by default
    mode = "synchronous" if a.profile_kernels else a.decode_mode
    model.set_decode_persistent(mode == "persistent")
    cache = model.kv_cache(a.prompt + a.generate)
    prompt = np.ones(a.prompt, np.uint32)

    def iteration(profile: bool):
        t = time.perf_counter()
        slots = ctx.empty([a.generate + 1], mi.DType.U32)
        if mode == "synchronous":
            logits, st = model.prefill_with_stats(prompt, cache)
        else:
            logits, st = model.prefill_argmax(prompt, cache, slots.slice_1d(0, 1))
        ctx.synchronize()
        pre = (time.perf_counter() - t, st.gpu_time)
        pre_prof = ctx.take_kernel_profiles() if profile else []
        t = time.perf_counter()
        gpu = 0.0
        if mode == "synchronous":
            for _ in range(a.generate):
                values = logits.to_f32_vec().ravel()
                finite = np.where(np.isfinite(values), values, -np.inf)
                token = int(len(finite) - 1 - np.argmax(finite[::-1]))  # ties: last index
                logits, st = model.decode_with_stats(token, cache)
                gpu += st.gpu_time
        elif mode == "pipelined":
            for step in range(a.generate):
                _, pend = model.decode_argmax(slots.slice_1d(step, 1), cache,
                                              slots.slice_1d(step + 1, 1))
                gpu += pend.wait().gpu_time
        else:  # persistent: one launch for all steps, timed by events
            import torch
            stream = torch.cuda.ExternalStream(ctx.stream())
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            model.decode_steps(cache, a.generate)
            e1.record(stream)
            e1.synchronize()
            gpu = e0.elapsed_time(e1) / 1e3
        ctx.synchronize()
        dec = (time.perf_counter() - t, gpu)
        dec_prof = ctx.take_kernel_profiles() if profile else []
        return pre, dec, pre_prof, dec_prof

    for _ in range(a.warmup):
        iteration(False)
    if a.profile_kernels:
        ctx.set_kernel_profiling(True)
    before = ctx.allocated_bytes()
    pre_s, dec_s, pre_k, dec_k = [], [], [], []
    for _ in range(a.iterations):
        pre, dec, pk, dk = iteration(a.profile_kernels)
        pre_s.append(pre)
        dec_s.append(dec)
        pre_k += pk
        dec_k += dk
    ctx.set_kernel_profiling(False)
    prefill = phase_report(a.prompt, [w for w, _ in pre_s], [g for _, g in pre_s])
    decode = phase_report(a.generate, [w for w, _ in dec_s], [g for _, g in dec_s])
    fo = model.fusion_options()
    r = {"benchmark": "qwen3_model", "device": ctx.device_name(), "iterations": a.iterations,
         "mean_ms": prefill["wall_mean_ms"] + decode["wall_mean_ms"],
         "median_ms": prefill["wall_median_ms"] + decode["wall_median_ms"],
         "p95_ms": prefill["wall_p95_ms"] + decode["wall_p95_ms"],
         "gpu_mean_ms": prefill["gpu_mean_ms"] + decode["gpu_mean_ms"],
         "gpu_median_ms": prefill["gpu_median_ms"] + decode["gpu_median_ms"],
         "gpu_p95_ms": prefill["gpu_p95_ms"] + decode["gpu_p95_ms"],
         "throughput": None, "throughput_unit": None, "allocated_bytes": ctx.allocated_bytes(),
         "matmul_backend": BACKEND_NAMES.get(ctx.matmul_backend(), "auto"),
         "decode_mode": mode, "allocation_growth_bytes": max(0, ctx.allocated_bytes() - before),
         "fusions": {"qkv": bool(fo.qkv), "gate_up": bool(fo.gate_up),
                     "add_rms_norm": bool(fo.add_rms_norm), "qk_rope_cache": bool(fo.qk_rope_cache)},
         "prefill": prefill, "decode": decode}
    if a.profile_kernels:
        r["kernel_profile"] = {"diagnostic_only": True,
                               "prefill": kernel_phase_profile([g for _, g in pre_s], pre_k),
                               "decode": kernel_phase_profile([g for _, g in dec_s], dec_k)}
    return r


def validate_workload(w: dict) -> None:
    """Workload::validate (inference.rs:37-52)."""
    out = w.get("output_tokens", 0)
    if (w.get("schema_version") != 1 or not w.get("case_id") or not w.get("prompt_text")
            or not w.get("prompt_token_ids") or not isinstance(out, int) or out < 2
            or len(w.get("forced_decode_ids", [])) != out - 1):
        raise BenchError("workload requires schema_version=1, nonempty prompt and case_id, and "
                         "output_tokens-1 forced IDs")


def greedy_token(values: np.ndarray) -> int:
    """inference.rs argmax: the last maximum among finite values."""
    v = np.asarray(values, np.float32).ravel()
    finite = np.isfinite(v)
    if not finite.any():
        raise BenchError("logits contain no finite value")
    m = np.max(v[finite])
    return int(np.nonzero(finite & (v == m))[0][-1])


def run_inference(a) -> dict:
    """inference::run (inference.rs:83-148): TTFT / TPOT per sample, forced
    or autoregressive token feed."""
    if a.iterations == 0:
        raise BenchError("iterations must be greater than zero")
    with open(a.workload) as f:
        w = json.load(f)
    validate_workload(w)
    ctx = mi.MetalContext(0)
    model = mi.Qwen3Model.load(a.model, ctx) if a.model else mi.Qwen3Model.random(
        ctx, {"0.6b": mi.QWEN3_0_6B, "8b": mi.QWEN3_8B}[a.random], seed=2)
    prompt = np.asarray(w["prompt_token_ids"], np.uint32)
    out = w["output_tokens"]
    cache = model.kv_cache(len(prompt) + out)

    def sample():
        cache.reset()
        t0 = time.perf_counter()
        logits = model.prefill(prompt, cache)
        sampled, fed, times = [], [], []
        for step in range(out):
            tok = greedy_token(logits.to_f32_vec())
            sampled.append(tok)
            times.append((time.perf_counter() - t0) * 1e3)
            if step + 1 < out:
                nxt = w["forced_decode_ids"][step] if a.mode == "fixed" else tok
                fed.append(int(nxt))
                logits = model.decode(int(nxt), cache)
        return {"ttft_ms": times[0], "tpot_ms": (times[-1] - times[0]) / (out - 1),
                "total_ms": times[-1], "token_times_ms": times, "sampled_token_ids": sampled,
                "fed_token_ids": fed}

    for _ in range(a.warmup):
        sample()
    samples = [sample() for _ in range(a.iterations)]
    return {"schema_version": 2, "kind": "inference", "backend": "metal-infer", "mode": a.mode,
            "case_id": w["case_id"], "device": ctx.device_name(), "prompt_tokens": len(prompt),
            "output_tokens": out, "warmup": a.warmup, "iterations": a.iterations,
            "samples": samples}


# ---- output (bench.rs:736-807, inference.rs:121-145) ------------------------------------------
def print_table(r: dict) -> None:
    if r.get("kind") == "inference":
        med = lambda key: sorted(s[key] for s in r["samples"])[len(r["samples"]) // 2]
        print(f"{r['backend']} {r['mode']} on {r['device']}")
        print(f"{r['case_id']}: {r['prompt_tokens']} prompt, {r['output_tokens']} output tokens")
        print(f"median TTFT {med('ttft_ms'):.3f} ms, TPOT {med('tpot_ms'):.3f} ms, "
              f"total {med('total_ms'):.3f} ms")
        return
    print(f"benchmark: {r['benchmark']}")
    print(f"device: {r['device']}")
    print(f"matmul backend: {r['matmul_backend']}")
    print(f"mean: {r['mean_ms']:.3f} ms, median: {r['median_ms']:.3f} ms, p95: {r['p95_ms']:.3f} ms")
    if "gpu_mean_ms" in r:
        print(f"GPU: {r['gpu_mean_ms']:.3f} ms mean, {r['gpu_median_ms']:.3f} ms median, "
              f"{r['gpu_p95_ms']:.3f} ms p95")
    if r.get("throughput") is not None:
        print(f"throughput: {r['throughput']:.3f} {r['throughput_unit']}")
    for phase in ("prefill", "decode"):
        p = r.get(phase)
        if p:
            print(f"{phase}: {p['wall_mean_ms']:.3f} ms wall, {p['gpu_mean_ms']:.3f} ms GPU, "
                  f"{p['tokens_per_second']:.3f} tokens/s")
    prof = r.get("kernel_profile")
    if prof:
        print("kernel profiling uses separate compute passes; timings are diagnostic")
        for phase in ("prefill", "decode"):
            p = prof[phase]
            print(f"{phase} kernels: {p['attributed_ms']:.3f} ms attributed / {p['gpu_ms']:.3f} ms "
                  f"GPU ({p['unattributed_ms']:.3f} ms unattributed)")
            for row in p["kernels"]:
                print(f"  {row['kernel']:<32} {row['calls']:>7} calls  {row['total_gpu_ms']:>9.3f} ms "
                      f"total  {row['mean_gpu_ms']:>8.4f} ms/call")
    for v in (r.get("attention_comparison") or {}).values():
        print(f"{v['kind']}: {v['gpu_mean_ms']:.4f} ms GPU mean, max abs error "
              f"{v['max_abs_error']:.3e}")
    print(f"CUDA allocated: {r['allocated_bytes']} bytes")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="metal-infer-bench", description="B200 transformer benchmarks")
    ap.add_argument("--format", choices=["table", "json"], default="table")
    sub = ap.add_subparsers(dest="command", required=True)
    k = sub.add_parser("kernel")
    k.add_argument("--m", type=int, default=512)
    k.add_argument("--n", type=int, default=1024)
    k.add_argument("--k", type=int, default=1024)
    k.add_argument("--iterations", type=int, default=10)
    k.add_argument("--warmup", type=int, default=3)
    k.add_argument("--matmul-backend", choices=["auto", "reference", "native"], default="auto")
    t = sub.add_parser("attention")
    t.add_argument("--kind", choices=["compare", "reference", "tiled", "flash-prefill",
                                      "decode-split-kv", "flash-decode"], default="compare")
    t.add_argument("--tokens", type=int, default=1)
    t.add_argument("--length", type=int, default=640)
    t.add_argument("--query-heads", type=int, default=16)
    t.add_argument("--kv-heads", type=int, default=8)
    t.add_argument("--head-dim", type=int, default=128)
    t.add_argument("--iterations", type=int, default=50)
    t.add_argument("--warmup", type=int, default=10)
    m = sub.add_parser("model")
    src = m.add_mutually_exclusive_group(required=True)
    src.add_argument("--model")
    src.add_argument("--random", choices=["0.6b", "8b"])
    m.add_argument("--prompt", type=int, default=512)
    m.add_argument("--generate", type=int, default=128)
    m.add_argument("--iterations", type=int, default=5)
    m.add_argument("--warmup", type=int, default=1)
    for f in ("fuse-qkv", "fuse-gate-up", "fuse-add-rms-norm", "fuse-qk-rope-cache",
              "profile-kernels"):
        m.add_argument("--" + f, action="store_true")
    m.add_argument("--decode-mode", choices=["pipelined", "synchronous", "persistent"],
                   default="persistent")
    i = sub.add_parser("inference")
    src = i.add_mutually_exclusive_group(required=True)
    src.add_argument("--model")
    src.add_argument("--random", choices=["0.6b", "8b"])
    i.add_argument("--workload", required=True)
    i.add_argument("--mode", choices=["fixed", "autoregressive"], required=True)
    i.add_argument("--iterations", type=int, default=10)
    i.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    try:
        if a.command == "inference":
            r = run_inference(a)
        else:
            if getattr(a, "iterations", 1) == 0:
                raise BenchError("iterations must be greater than zero")
            ctx = mi.MetalContext(0)
            r = {"kernel": run_kernel, "attention": run_attention, "model": run_model}[a.command](ctx, a)
    except Exception as e:  # bench.rs main: print, exit 1
        print(e, file=sys.stderr)
        return 1
    if a.format == "json":
        print(json.dumps(r, indent=2))
    else:
        print_table(r)
    return 0


if __name__ == "__main__":
    sys.exit(main())

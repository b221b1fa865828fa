"""The reference-format benchmark CLI (crates/metal-infer-cli/src/bin/
bench.rs, inference.rs): host logic on CPU (statistics, workload
validation, greedy tie rule, report assembly), and each subcommand's JSON
schema on the GPU."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from metal_infer import bench_cli as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENV = dict(os.environ, PYTHONPATH=os.path.join(ROOT, "metal-infer-rs_b200"))


def test_duration_stats_match_bench_rs():
    # bench.rs:1995-2008: sorted samples, median = s[n/2], p95 = s[round((n-1)*0.95)]
    s = B.duration_stats([0.004, 0.001, 0.003, 0.002])
    assert s == {"mean_ms": pytest.approx(2.5), "median_ms": pytest.approx(3.0),
                 "p95_ms": pytest.approx(4.0)}
    p = B.phase_report(8, [0.002, 0.002], [0.001, 0.001])
    assert p["tokens_per_second"] == pytest.approx(4000.0) and p["gpu_mean_ms"] == pytest.approx(1.0)


def test_kernel_phase_profile_sorting():
    prof = B.kernel_phase_profile([0.010], [("b", 0.002), ("a", 0.003), ("b", 0.001)])
    assert [r["kernel"] for r in prof["kernels"]] == ["a", "b"] or \
           [r["kernel"] for r in prof["kernels"]] == ["b", "a"]
    assert prof["attributed_ms"] == pytest.approx(6.0)
    assert prof["unattributed_ms"] == pytest.approx(4.0)
    b = [r for r in prof["kernels"] if r["kernel"] == "b"][0]
    assert b["calls"] == 2 and b["mean_gpu_ms"] == pytest.approx(1.5)


def test_workload_validation_and_tie_rule():
    ok = dict(schema_version=1, case_id="c", prompt_text="p", prompt_token_ids=[1],
              forced_decode_ids=[2, 3], output_tokens=3)
    B.validate_workload(ok)
    # inference.rs:205-217: a trace must have output_tokens - 1 forced ids
    with pytest.raises(B.BenchError):
        B.validate_workload(dict(ok, forced_decode_ids=[2]))
    with pytest.raises(B.BenchError):
        B.validate_workload(dict(ok, schema_version=2))
    # inference.rs:219-222: ties go to the later index
    assert B.greedy_token(np.array([2.0, 2.0], np.float32)) == 1
    assert B.greedy_token(np.array([np.nan, 1.0, np.inf, 0.5], np.float32)) == 1
    with pytest.raises(B.BenchError):
        B.greedy_token(np.array([np.nan], np.float32))


@pytest.mark.gpu
def test_bench_cli_json_schemas(tmp_path):
    def run(*args):
        out = subprocess.run([sys.executable, "-m", "metal_infer.bench_cli", "--format", "json", *args],
                             capture_output=True, text=True, env=ENV, timeout=600)
        assert out.returncode == 0, out.stderr
        return json.loads(out.stdout)
    k = run("kernel", "--m", "1", "--n", "1024", "--k", "1024", "--iterations", "3", "--warmup", "1")
    assert k["benchmark"] == "matmul_f16[1,1024,1024]" and k["throughput_unit"] == "TFLOP/s"
    assert {"mean_ms", "median_ms", "p95_ms", "gpu_mean_ms", "allocated_bytes"} <= set(k)
    at = run("attention", "--length", "256", "--iterations", "3", "--warmup", "1")
    assert set(at["attention_comparison"]) == {"reference", "tiled", "flash_prefill",
                                               "decode_split_kv", "flash_decode"}
    assert all(v["max_abs_error"] < 5e-2 for v in at["attention_comparison"].values())
    for mode in ("persistent", "pipelined", "synchronous"):
        m = run("model", "--random", "0.6b", "--prompt", "32", "--generate", "8", "--iterations", "2",
                "--warmup", "1", "--decode-mode", mode)
        assert m["benchmark"] == "qwen3_model" and m["decode_mode"] == mode
        assert m["prefill"]["tokens"] == 32 and m["decode"]["tokens_per_second"] > 0
    m = run("model", "--random", "0.6b", "--prompt", "16", "--generate", "4", "--iterations", "1",
            "--warmup", "0", "--profile-kernels")
    assert m["kernel_profile"]["diagnostic_only"] and m["kernel_profile"]["decode"]["kernels"]
    w = dict(schema_version=1, case_id="case", prompt_text="hi", prompt_token_ids=[1, 2, 3],
             forced_decode_ids=[5, 6, 7], output_tokens=4)
    path = tmp_path / "w.json"
    path.write_text(json.dumps(w))
    for mode in ("fixed", "autoregressive"):
        r = run("inference", "--random", "0.6b", "--workload", str(path), "--mode", mode,
                "--iterations", "2", "--warmup", "1")
        assert r["schema_version"] == 2 and r["kind"] == "inference" and r["mode"] == mode
        s = r["samples"][0]
        assert len(s["sampled_token_ids"]) == 4 and len(s["token_times_ms"]) == 4
        if mode == "fixed":
            assert s["fed_token_ids"] == [5, 6, 7]
        else:
            assert s["fed_token_ids"] == s["sampled_token_ids"][:3]


@pytest.mark.gpu
def test_attention_compare_against_oracle():
    """`attention --kind compare` reports each kind's error against the
    engine's reference kind; here every kind's output on the subcommand's own
    seeded inputs is pinned to the CPU oracle (the reference semantics of
    transformer.metal:1579-1612 for the prefill kinds, the oracle's flash
    decode for the decode kinds), and the CLI's error column to those outputs."""
    import metal_infer as mi
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    T, L, qh, kvh, hd = 1, 640, 16, 8, 128
    qf, kf, vf = B.attention_inputs(T, L, qh, kvh, hd)
    qb, kb, vb = O.f16_bits(qf), O.f16_bits(kf), O.f16_bits(vf)
    ctx = mi.MetalContext(0)
    q = ctx.tensor_f16_bits(qb, [T, qh, hd])
    k = ctx.tensor_f16_bits(kb, [L, kvh, hd])
    v = ctx.tensor_f16_bits(vb, [L, kvh, hd])
    cfg = mi.AttentionConfig(qh, kvh, hd, 1, L - T)
    want = O.f32(O.attention(qb, kb, vb, qh, kvh, hd, True, L - T)).ravel()
    outs = {}
    for name, kind in B.ATTENTION_KINDS.items():
        outs[name] = ctx.attention(q, k, v, cfg, kind).to_f32_vec()
        # per-op tolerance of the north star: max relative error 2e-3
        err = np.max(np.abs(outs[name] - want)) / np.max(np.abs(want))
        assert err <= 2e-3, (name, err)
    np.testing.assert_array_equal(
        outs["flash-decode"], O.f32(O.attention_decode(qb, kb, vb, qh, kvh, hd)).ravel())
    out = subprocess.run([sys.executable, "-m", "metal_infer.bench_cli", "--format", "json",
                          "attention", "--kind", "compare", "--tokens", "1", "--length", str(L),
                          "--iterations", "2", "--warmup", "1"],
                         capture_output=True, text=True, env=ENV, timeout=600)
    assert out.returncode == 0, out.stderr
    cmp_ = json.loads(out.stdout)["attention_comparison"]
    for name in B.ATTENTION_KINDS:
        got = cmp_[name.replace("-", "_")]["max_abs_error"]
        assert got == pytest.approx(float(np.max(np.abs(outs[name] - outs["reference"]))), abs=1e-6)


"""Generates the golden fixtures of tests/golden/ with the CPU oracle.

    python tests/golden/make_golden.py

The reference has no CPU path and no stored outputs, so the model-level
fixtures are the oracle's own outputs on the BASELINE.json configs (seeded
synthetic weights and inputs). They pin the oracle across changes; the GPU
tests compare the engine against them and against the oracle directly.
"""
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

INPUT_STREAM = 1 << 20


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def config2():
    """Full Qwen3-0.6B, seed 2: 128-token prompt, 256 greedy decode steps."""
    cfg = dict(O.QWEN3_0_6B)
    m = O.Qwen3(cfg, seed=2, capacity=2048)
    prompt = O.gen_tokens(2, INPUT_STREAM, 128, cfg["vocab_size"])
    ids = m.generate_greedy(prompt, 257)
    m.reset()
    logits = m.forward(prompt)
    return {"config": cfg, "seed": 2, "prompt_stream": INPUT_STREAM, "prompt_len": 128,
            "prompt_sha256": sha(prompt), "max_tokens": 257, "ids": ids.tolist(),
            "prefill_logits_sha256": sha(logits),
            "prefill_logits_head": logits[:16].tolist()}


def config0():
    """One Qwen3-0.6B block, seed 0: 64-token hidden prefill + 16 decode steps."""
    cfg = dict(O.QWEN3_0_6B)
    cfg["num_hidden_layers"] = 1
    m = O.Qwen3(cfg, seed=0, capacity=2048)
    h = cfg["hidden_size"]
    prefill = O.gen_normal_f16(0, INPUT_STREAM, 64 * h, 1.0).reshape(64, h)
    outs = [m.forward_hidden(prefill)]
    for step in range(16):
        x = O.gen_normal_f16(0, INPUT_STREAM + 1 + step, h, 1.0).reshape(1, h)
        outs.append(m.forward_hidden(x))
    allout = np.concatenate([o.reshape(-1, h) for o in outs])
    np.save(os.path.join(HERE, "block0_hidden.npy"), allout)
    return {"config": cfg, "seed": 0, "rows": int(allout.shape[0]), "sha256": sha(allout)}


def generator():
    normals = O.gen_normal_f16(0, 1, 64, 1.0)
    tokens = O.gen_tokens(2, INPUT_STREAM, 64, 151936)
    return {"normal_seed0_stream1_first64": normals.tolist(),
            "tokens_seed2_input_first64": tokens.tolist()}


if __name__ == "__main__":
    t = time.time()
    with open(os.path.join(HERE, "generator.json"), "w") as f:
        json.dump(generator(), f)
    with open(os.path.join(HERE, "block0.json"), "w") as f:
        json.dump(config0(), f)
    with open(os.path.join(HERE, "qwen3_0_6b_greedy.json"), "w") as f:
        json.dump(config2(), f)
    print(f"golden fixtures written in {time.time() - t:.1f} s")

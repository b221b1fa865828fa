"""The serving layer on the engine (crates/metal-infer-cli): a random Qwen3
checkpoint exported to safetensors with a synthetic tokenizer, served over
HTTP and run through the generate CLI; the tokens must be those of
generate_with on the same prompt and options, and those in turn the CPU
oracle's greedy and sampled ids for the same seeded model (cut at the first
end-of-sequence id, where the engine stops)."""
import json
import os
import subprocess
import sys
import threading
import urllib.request

import numpy as np
import pytest

import metal_infer as mi
from metal_infer import serving as S
from test_loader_gpu import export, small_cfg
from tokenizer_fixture import write_tokenizer
import oracle as O

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("qwen3_ckpt"))
    cfg = small_cfg()
    ctx = mi.MetalContext(0)
    export(mi.Qwen3Model.random(ctx, cfg, seed=31), cfg, d)
    write_tokenizer(d, cfg["vocab_size"])
    return d, cfg


def oracle_ids(cfg, prompt, max_tokens, stops, **sampling):
    """The oracle's ids for the seed-31 model of the checkpoint: greedy, or
    sampled with the engine's options, cut before the first stop id."""
    ref = O.Qwen3(cfg, seed=31, capacity=256)
    if sampling.get("temperature", 0.0) > 0.0:
        ids = ref.generate_sampled(prompt, max_tokens, sampling["temperature"],
                                   sampling.get("top_p", 1.0), sampling.get("top_k", 0),
                                   sampling.get("seed", 0))
    else:
        ids = ref.generate_greedy(prompt, max_tokens)
    ref.close()
    cut = [i for i, t in enumerate(ids.tolist()) if t in set(stops)]
    return ids[:cut[0]] if cut else ids


def _post(url, body):
    req = urllib.request.Request(url, data=json.dumps(body).encode(),
                                 headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=120) as r:
        return r.read()


def test_server_matches_generate_with(checkpoint):
    d, cfg = checkpoint
    engine = S.load_engine(d, context=256)
    assert engine.model_id == os.path.basename(d)
    srv = S.make_server(engine, "127.0.0.1:0")
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    base = f"http://127.0.0.1:{srv.server_address[1]}"
    try:
        messages = [{"role": "system", "content": "Be concise."}, {"role": "user", "content": "hello world"}]
        prompt = engine.tokenizer.encode_chat([S.ChatMessage(**m) for m in messages])
        for opts in (dict(), dict(temperature=0.8, top_p=0.9, top_k=40, seed=5)):
            want = engine.model.generate_with(prompt, dict(dict(max_tokens=12, temperature=0.0, top_p=1.0,
                                                               top_k=0, seed=0), **opts,
                                                          stop_token_ids=engine.tokenizer.eos_token_ids),
                                              engine.model.kv_cache(256))
            np.testing.assert_array_equal(
                np.asarray(want, np.uint32),
                oracle_ids(cfg, np.asarray(prompt, np.uint32), 12, engine.tokenizer.eos_token_ids,
                           **opts))
            r = json.loads(_post(base + "/v1/chat/completions",
                                 dict(messages=messages, max_tokens=12, **opts)))
            assert r["usage"]["prompt_tokens"] == len(prompt)
            assert r["usage"]["completion_tokens"] == len(want)
            text = engine.tokenizer.decode(want)
            assert r["choices"][0]["message"]["content"] == S.split_reasoning(text)[1]
            body = _post(base + "/v1/chat/completions", dict(messages=messages, max_tokens=12,
                                                               stream=True, **opts)).decode()
            events = [e[6:] for e in body.split("\n\n") if e.startswith("data: ")]
            assert events[-1] == "[DONE]"
            streamed = "".join(json.loads(e)["choices"][0]["delta"].get("content", "")
                               for e in events[:-1])
            assert streamed == S.stream_channels(text)[1]
    finally:
        srv.shutdown()
        srv.server_close()


def test_generate_cli(checkpoint):
    d, cfg = checkpoint
    env = dict(os.environ, PYTHONPATH=os.path.join(ROOT, "metal-infer-rs_b200"))
    out = subprocess.run([sys.executable, "-m", "metal_infer", "generate", "--model", d, "--prompt",
                          "hello world", "--max-tokens", "10"], capture_output=True, text=True,
                         env=env, timeout=300)
    assert out.returncode == 0, out.stderr
    ctx = mi.MetalContext(0)
    tk = S.ModelTokenizer.from_directory(d)
    model = mi.Qwen3Model.load(d, ctx)
    ids = model.generate_with(tk.encode("hello world"), dict(max_tokens=10, stop_token_ids=tk.eos_token_ids),
                              model.kv_cache(2048))
    assert out.stdout == tk.decode(ids)
    prompt = np.asarray(tk.encode("hello world"), np.uint32)
    np.testing.assert_array_equal(np.asarray(ids, np.uint32),
                                  oracle_ids(cfg, prompt, 10, tk.eos_token_ids))
    bad = subprocess.run([sys.executable, "-m", "metal_infer", "generate", "--model", d, "--prompt",
                          "hello", "--max-tokens", "5000", "--context", "64"], capture_output=True,
                         text=True, env=env, timeout=300)
    assert bad.returncode == 1 and "exceeds context" in bad.stderr

"""CPU tests of the serving layer (crates/metal-infer-cli/src/server.rs,
lib.rs, crates/metal-infer-models/src/tokenizer.rs): the reference's unit
tests restated, the tokenizer wrapper, model path resolution, and the HTTP
server end to end over a fake model."""
import json
import os
import threading
import urllib.error
import urllib.request

import pytest

from metal_infer import serving as S
from tokenizer_fixture import write_tokenizer


def test_renders_qwen_chat_boundaries():
    # tokenizer.rs:130-148
    prompt = S.render_qwen_chat([S.ChatMessage("system", "Be concise."),
                                 S.ChatMessage("user", "Hello")])
    assert prompt == ("<|im_start|>system\nBe concise.<|im_end|>\n<|im_start|>user\nHello"
                      "<|im_end|>\n<|im_start|>assistant\n")
    with pytest.raises(S.ServingError, match="at least one message"):
        S.render_qwen_chat([])
    with pytest.raises(S.ServingError, match="unsupported chat role `robot`"):
        S.render_qwen_chat([S.ChatMessage("robot", "x")])


def test_stop_sequences_are_not_returned():
    # server.rs:640-647
    assert S.truncate_stop("hello STOP later", ["STOP"]) == "hello "
    assert S.safe_stream_boundary("hello ST", ["STOP"]) == 6
    assert S.truncate_stop("a b", ["", "zz"]) == "a b"


def test_reasoning_is_split_from_answer():
    # server.rs:649-660
    assert S.split_reasoning("<think>work</think> answer") == ("work", "answer")
    assert S.split_reasoning("<think> partial") == ("partial", "")
    assert S.split_reasoning("plain") == (None, "plain")
    assert S.stream_channels("<thi") == ("", "")
    assert S.stream_channels("<think>work</thi") == ("work", "")
    assert S.stream_channels("<think>work</think>answer") == ("work", "answer")


def test_hugging_face_ids_and_model_id():
    # lib.rs:104-117, server.rs:662-670
    assert S.hugging_face_model_id("Qwen/Qwen3-8B") == "Qwen/Qwen3-8B"
    assert S.hugging_face_model_id("local-model") is None
    assert S.hugging_face_model_id("a/b/c") is None
    assert S.infer_model_id("/cache/models--Qwen--Qwen3-8B/snapshots/revision") == "Qwen/Qwen3-8B"
    assert S.infer_model_id("/models/my-qwen") == "my-qwen"


def test_resolve_model_path_through_the_cache(tmp_path, monkeypatch):
    monkeypatch.setenv("HUGGINGFACE_HUB_CACHE", str(tmp_path))
    local = tmp_path / "local"
    local.mkdir()
    assert S.resolve_model_path(str(local)) == local
    with pytest.raises(S.ServingError, match="does not exist"):
        S.resolve_model_path(str(tmp_path / "missing"))
    with pytest.raises(S.ServingError, match="not available in the local cache"):
        S.resolve_model_path("Qwen/Qwen3-0.6B")
    repo = tmp_path / "models--Qwen--Qwen3-0.6B"
    old = repo / "snapshots" / "aaa"
    new = repo / "snapshots" / "bbb"
    for d in (old, new):
        d.mkdir(parents=True)
        (d / "config.json").write_text("{}")
        (d / "tokenizer.json").write_text("{}")
    os.utime(old, (1, 1))
    assert S.resolve_model_path("Qwen/Qwen3-0.6B") == new  # newest snapshot
    (repo / "refs").mkdir()
    (repo / "refs" / "main").write_text("aaa\n")
    assert S.resolve_model_path("Qwen/Qwen3-0.6B") == old  # refs/main wins
    monkeypatch.delenv("HUGGINGFACE_HUB_CACHE")
    monkeypatch.setenv("HF_HOME", str(tmp_path / "hf"))
    assert S.hugging_face_cache_root() == tmp_path / "hf" / "hub"


def test_tokenizer_wrapper(tmp_path):
    vocab = write_tokenizer(str(tmp_path), 64)
    tk = S.ModelTokenizer.from_directory(tmp_path)
    assert tk.eos_token_ids == [vocab["<|im_end|>"]]
    ids = tk.encode_chat([S.ChatMessage("user", "hello world")])
    assert ids[0] == vocab["<|im_start|>"] and vocab["hello"] in ids and vocab["world"] in ids
    assert tk.decode([vocab["hello"], vocab["<|im_end|>"], vocab["world"]]) == "hello world"
    # eos_token as a list of strings / dicts (collect_special_tokens)
    with open(tmp_path / "tokenizer_config.json", "w") as f:
        json.dump({"eos_token": ["<|endoftext|>", {"content": "<|im_end|>"}, "not-a-token"]}, f)
    tk = S.ModelTokenizer.from_directory(tmp_path)
    assert tk.eos_token_ids == [vocab["<|endoftext|>"], vocab["<|im_end|>"]]
    with pytest.raises(S.ServingError, match="failed to load tokenizer"):
        S.ModelTokenizer.from_directory(tmp_path / "nowhere")


class FakeModel:
    """generate_with as the engine's: a fixed continuation, stops at
    stop_token_ids, on_token may end early."""

    def __init__(self, continuation):
        self.continuation = continuation
        self.calls = []

    def kv_cache(self, capacity):
        return object()

    def generate_with(self, prompt, options, cache, on_token=None):
        self.calls.append((list(prompt), dict(options)))
        out = []
        for tok in self.continuation[:options["max_tokens"]]:
            if tok in options["stop_token_ids"]:
                break
            out.append(tok)
            if on_token and not on_token(tok):
                break
        return out


@pytest.fixture()
def server(tmp_path):
    vocab = write_tokenizer(str(tmp_path), 64)
    tk = S.ModelTokenizer.from_directory(tmp_path)
    words = ["<think>", "work", "</think>", "hello", "world", "STOP", "answer", "<|im_end|>", "t1"]
    model = FakeModel([vocab[w] for w in words])
    engine = S.ChatEngine(model, tk, context=64, model_id="qwen3-test")
    srv = S.make_server(engine, "127.0.0.1:0")
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    yield f"http://127.0.0.1:{srv.server_address[1]}", model, vocab
    srv.shutdown()
    srv.server_close()


def _post(url, body, raw=False):
    data = body if raw else json.dumps(body).encode()
    req = urllib.request.Request(url, data=data, headers={"Content-Type": "application/json"})
    try:
        with urllib.request.urlopen(req, timeout=30) as r:
            return r.status, r.read()
    except urllib.error.HTTPError as e:
        return e.code, e.read()


def test_http_routes(server):
    base, model, vocab = server
    with urllib.request.urlopen(base + "/health", timeout=30) as r:
        assert json.loads(r.read()) == {"status": "ok"}
    with urllib.request.urlopen(base + "/v1/models?x=1", timeout=30) as r:
        assert json.loads(r.read())["data"][0]["id"] == "qwen3-test"
    code, body = _post(base + "/nope", {})
    assert code == 404 and json.loads(body)["error"]["message"] == "route not found"
    code, body = _post(base + "/v1/chat/completions", b"{bad", raw=True)
    assert code == 400 and "invalid JSON" in json.loads(body)["error"]["message"]


def test_chat_completion(server):
    base, model, vocab = server
    code, body = _post(base + "/v1/chat/completions", {
        "model": "qwen3-test", "messages": [{"role": "user", "content": "hello"}],
        "max_tokens": 8, "temperature": 0.7, "top_p": 0.9, "top_k": 5, "seed": 3})
    r = json.loads(body)
    assert code == 200 and r["object"] == "chat.completion"
    msg = r["choices"][0]["message"]
    assert msg["reasoning_content"] == "work" and msg["content"] == "hello world STOP answer"
    assert r["choices"][0]["finish_reason"] == "stop"  # <|im_end|> (EOS) ended it
    assert r["usage"]["completion_tokens"] == 7
    prompt, opts = model.calls[-1]
    assert opts == dict(max_tokens=8, temperature=0.7, top_p=pytest.approx(0.9), top_k=5, seed=3,
                        stop_token_ids=[vocab["<|im_end|>"]])
    # stop sequence + length finish
    code, body = _post(base + "/v1/chat/completions", {
        "messages": [{"role": "user", "content": [{"type": "text", "text": "hello"}]}],
        "max_tokens": 4, "stop": "world"})
    r = json.loads(body)
    assert r["choices"][0]["message"]["content"] == "hello" and r["choices"][0]["finish_reason"] == "length"
    # errors
    for req, text in (({"model": "other", "messages": [{"role": "user", "content": "x"}]}, "not loaded"),
                      ({"messages": [{"role": "user", "content": "x"}], "max_tokens": 100}, "exceeds context"),
                      ({"messages": [{"role": "user", "content": [{"type": "image_url"}]}]}, "not supported"),
                      ({"messages": []}, "at least one message")):
        code, body = _post(base + "/v1/chat/completions", req)
        assert code == 400 and text in json.loads(body)["error"]["message"], req


def test_streaming_chat_completion(server):
    base, model, vocab = server
    code, body = _post(base + "/v1/chat/completions", {
        "messages": [{"role": "user", "content": "hello"}], "max_tokens": 8, "stream": True,
        "stop": ["STOP"]})
    assert code == 200
    events = [line[len("data: "):] for line in body.decode().split("\n\n") if line.startswith("data: ")]
    assert events[-1] == "[DONE]"
    chunks = [json.loads(e) for e in events[:-1]]
    assert chunks[0]["choices"][0]["delta"] == {"role": "assistant"}
    reasoning = "".join(c["choices"][0]["delta"].get("reasoning_content", "") for c in chunks)
    content = "".join(c["choices"][0]["delta"].get("content", "") for c in chunks)
    # stream_channels does not trim (server.rs:598-615); the word-level test
    # tokenizer joins tokens with spaces
    assert reasoning == " work " and content == " hello world "
    assert chunks[-1]["choices"][0]["finish_reason"] == "stop"
    # generation ended at the stop sequence (on_token returned False)
    assert len(model.calls) >= 1

"""OpenAI-compatible chat server and the tokenizer it needs, over the engine's
C ABI (the `metal_infer` binding). Mirrors crates/metal-infer-cli/src/server.rs
(routes, request fields and defaults, stop sequences, `<think>` reasoning
split, SSE streaming), crates/metal-infer-cli/src/lib.rs (model path
resolution through the Hugging Face cache) and
crates/metal-infer-models/src/tokenizer.rs (tokenizer.json, EOS ids from
tokenizer_config.json, the Qwen chat template).

The HTTP server serves one request at a time, as the reference does: one
model, one KV cache.
"""
from __future__ import annotations

import json
import os
import time
from dataclasses import dataclass
from http.server import BaseHTTPRequestHandler, HTTPServer
from pathlib import Path
from typing import Callable, Iterable, List, Optional, Sequence, Tuple

MAX_REQUEST_BYTES = 4 * 1024 * 1024  # server.rs:13
DEFAULT_MAX_TOKENS = 256             # server.rs:387-389
DEFAULT_TOP_P = 1.0                  # server.rs:391-393
THINK_OPEN, THINK_CLOSE = "<think>", "</think>"


class ServingError(ValueError):
    """Invalid request or arguments (CliError::InvalidArguments / ModelError::Config)."""


# ---- tokenizer (tokenizer.rs) ----------------------------------------------------
@dataclass
class ChatMessage:
    role: str
    content: str


def render_qwen_chat(messages: Sequence[ChatMessage]) -> str:
    """render_qwen_chat (tokenizer.rs:79-102)."""
    if not messages:
        raise ServingError("chat completion requires at least one message")
    prompt = []
    for m in messages:
        if m.role not in ("system", "user", "assistant", "tool"):
            raise ServingError(f"unsupported chat role `{m.role}`")
        prompt.append(f"<|im_start|>{m.role}\n{m.content}<|im_end|>\n")
    prompt.append("<|im_start|>assistant\n")
    return "".join(prompt)


def _collect_special_tokens(value, visit: Callable[[str], None]) -> None:
    """collect_special_tokens (tokenizer.rs:104-123)."""
    if isinstance(value, str):
        visit(value)
    elif isinstance(value, list):
        for v in value:
            _collect_special_tokens(v, visit)
    elif isinstance(value, dict) and isinstance(value.get("content"), str):
        visit(value["content"])


class ModelTokenizer:
    """ModelTokenizer (tokenizer.rs:9-77) over the `tokenizers` package."""

    def __init__(self, inner, eos_token_ids: List[int]):
        self.inner = inner
        self.eos_token_ids = eos_token_ids

    @classmethod
    def from_directory(cls, directory) -> "ModelTokenizer":
        from tokenizers import Tokenizer  # the HF tokenizers package
        directory = Path(directory)
        path = directory / "tokenizer.json"
        try:
            inner = Tokenizer.from_file(str(path))
        except Exception as e:
            raise ServingError(f"failed to load tokenizer from {path}") from e
        eos: List[int] = []
        cfg = directory / "tokenizer_config.json"
        if cfg.exists():
            config = json.loads(cfg.read_bytes())
            if "eos_token" in config:
                def visit(token: str) -> None:
                    tid = inner.token_to_id(token)
                    if tid is not None and tid not in eos:
                        eos.append(tid)
                _collect_special_tokens(config["eos_token"], visit)
        return cls(inner, eos)

    def encode(self, text: str) -> List[int]:
        return list(self.inner.encode(text, add_special_tokens=True).ids)

    def decode(self, tokens: Iterable[int]) -> str:
        return self.inner.decode([int(t) for t in tokens], skip_special_tokens=True)

    def encode_chat(self, messages: Sequence[ChatMessage]) -> List[int]:
        return list(self.inner.encode(render_qwen_chat(messages), add_special_tokens=False).ids)


# ---- model path resolution (lib.rs) ---------------------------------------------------
def hugging_face_model_id(model) -> Optional[str]:
    """hugging_face_model_id / is_hugging_face_id (lib.rs:58-66): `owner/name`."""
    parts = str(model).split("/")
    if len(parts) == 2 and parts[0] and parts[1]:
        return str(model)
    return None


def hugging_face_cache_root() -> Optional[Path]:
    """lib.rs:68-76: HUGGINGFACE_HUB_CACHE, then HF_HOME/hub, then ~/.cache/huggingface/hub."""
    if os.environ.get("HUGGINGFACE_HUB_CACHE"):
        return Path(os.environ["HUGGINGFACE_HUB_CACHE"])
    if os.environ.get("HF_HOME"):
        return Path(os.environ["HF_HOME"]) / "hub"
    if os.environ.get("HOME"):
        return Path(os.environ["HOME"]) / ".cache" / "huggingface" / "hub"
    return None


def resolve_model_path(model) -> Path:
    """resolve_model_path (lib.rs:20-56): a directory as given, else a
    Hugging Face repository id looked up in the local cache (refs/main, else
    the newest snapshot) holding config.json and tokenizer.json."""
    path = Path(model)
    if path.is_dir():
        return path
    ident = hugging_face_model_id(model)
    if ident is None:
        raise ServingError(f"model directory `{model}` does not exist")
    cache = hugging_face_cache_root()
    if cache is None:
        raise ServingError("cannot locate the Hugging Face cache because HOME, HF_HOME, and "
                           "HUGGINGFACE_HUB_CACHE are unset")
    repo = cache / ("models--" + ident.replace("/", "--"))
    snapshots = repo / "snapshots"
    revision = None
    try:
        value = (repo / "refs" / "main").read_text().strip()
        if value and "/" not in value and ".." not in value:
            revision = value
    except OSError:
        pass
    missing = ServingError(f"Hugging Face model `{ident}` is not available in the local cache; "
                           f"download it with `hf download {ident}`")
    if revision is not None:
        snapshot = snapshots / revision
    else:
        try:
            dirs = [d for d in snapshots.iterdir() if d.is_dir()]
        except FileNotFoundError:
            dirs = []
        if not dirs:
            raise missing
        snapshot = max(dirs, key=lambda d: d.stat().st_mtime)
    if (snapshot / "config.json").is_file() and (snapshot / "tokenizer.json").is_file():
        return snapshot
    raise missing


def infer_model_id(path) -> str:
    """infer_model_id (server.rs:617-631)."""
    p = Path(path)
    for part in [p] + list(p.parents):
        name = part.name
        if name.startswith("models--"):
            return name[len("models--"):].replace("--", "/")
    return p.name or "qwen3"


# ---- text post-processing (server.rs:565-615) ------------------------------------------
def truncate_stop(value: str, stops: Sequence[str]) -> str:
    hits = [value.find(s) for s in stops if s and s in value]
    return value[:min(hits)] if hits else value


def safe_stream_boundary(value: str, stops: Sequence[str]) -> int:
    """Length of `value` that cannot be the start of a stop sequence."""
    withheld = 0
    for stop in stops:
        for i in range(1, len(stop)):
            if value.endswith(stop[:i]):
                withheld = max(withheld, i)
    return max(0, len(value) - withheld)


def split_reasoning(value: str) -> Tuple[Optional[str], str]:
    if not value.startswith(THINK_OPEN):
        return None, value
    rest = value[len(THINK_OPEN):]
    if THINK_CLOSE not in rest:
        return rest.strip(), ""
    reasoning, content = rest.split(THINK_CLOSE, 1)
    return reasoning.strip(), content.strip()


def stream_channels(value: str) -> Tuple[str, str]:
    if len(value) < len(THINK_OPEN) and THINK_OPEN.startswith(value):
        return "", ""
    if not value.startswith(THINK_OPEN):
        return "", value
    rest = value[len(THINK_OPEN):]
    if THINK_CLOSE in rest:
        reasoning, content = rest.split(THINK_CLOSE, 1)
        return reasoning, content
    return rest[:safe_stream_boundary(rest, [THINK_CLOSE])], ""


# ---- chat completions (server.rs:172-355) ----------------------------------------------
def _message(wire: dict) -> ChatMessage:
    """WireMessage::into_chat_message (server.rs:357-378)."""
    if not isinstance(wire, dict) or "role" not in wire or "content" not in wire:
        raise ServingError("invalid message: expected `role` and `content`")
    content = wire["content"]
    if isinstance(content, list):
        out = []
        for part in content:
            kind = part.get("type") if isinstance(part, dict) else None
            if kind != "text":
                raise ServingError(f"message content type `{kind}` is not supported yet")
            out.append(part.get("text") or "")
        content = "".join(out)
    elif not isinstance(content, str):
        raise ServingError("invalid message content")
    return ChatMessage(str(wire["role"]), content)


class ChatEngine:
    """ServerState (server.rs:22-28): model, tokenizer, one KV cache."""

    def __init__(self, model, tokenizer: ModelTokenizer, context: int, model_id: str):
        self.model = model
        self.tokenizer = tokenizer
        self.context = context
        self.model_id = model_id
        self.cache = model.kv_cache(context)

    def prepare(self, request: dict):
        model = request.get("model")
        if model is not None and model != self.model_id:
            raise ServingError(f"requested model `{model}` is not loaded")
        if not isinstance(request.get("messages"), list):
            raise ServingError("invalid request: `messages` must be a list")
        messages = [_message(m) for m in request["messages"]]
        prompt = self.tokenizer.encode_chat(messages)
        max_tokens = int(request.get("max_tokens", DEFAULT_MAX_TOKENS))
        required = len(prompt) + max_tokens
        if required > self.context:
            raise ServingError(f"prompt + generated tokens ({required}) exceeds context "
                               f"{self.context}")
        stop = request.get("stop")
        stops = [] if stop is None else ([stop] if isinstance(stop, str) else list(stop))
        options = dict(max_tokens=max_tokens, temperature=float(request.get("temperature", 0.0)),
                       top_p=float(request.get("top_p", DEFAULT_TOP_P)),
                       top_k=int(request.get("top_k", 0)), seed=int(request.get("seed", 0)),
                       stop_token_ids=list(self.tokenizer.eos_token_ids))
        return prompt, options, stops

    def complete(self, request: dict) -> dict:
        """complete_once (server.rs:214-257)."""
        prompt, options, stops = self.prepare(request)
        generated = self.model.generate_with(prompt, options, self.cache)
        decoded = truncate_stop(self.tokenizer.decode(generated), stops)
        reasoning, content = split_reasoning(decoded)
        message = {"role": "assistant", "content": content}
        if reasoning is not None:
            message["reasoning_content"] = reasoning
        return {
            "id": completion_id(), "object": "chat.completion", "created": int(time.time()),
            "model": self.model_id,
            "choices": [{"index": 0, "message": message,
                         "finish_reason": "length" if len(generated) == options["max_tokens"]
                         else "stop"}],
            "usage": {"prompt_tokens": len(prompt), "completion_tokens": len(generated),
                      "total_tokens": len(prompt) + len(generated)},
        }

    def stream(self, request: dict, emit: Callable[[dict], None]) -> None:
        """stream_completion (server.rs:259-355): role chunk, reasoning /
        content deltas as tokens arrive (text that may begin a stop sequence
        or `</think>` is withheld), the final chunk."""
        prompt, options, stops = self.prepare(request)
        cid, model_id = completion_id(), self.model_id

        def chunk(delta: dict, finish=None) -> dict:
            return {"id": cid, "object": "chat.completion.chunk", "created": int(time.time()),
                    "model": model_id, "choices": [{"index": 0, "delta": delta,
                                                    "finish_reason": finish}]}

        emit(chunk({"role": "assistant"}))
        tokens: List[int] = []
        sent = {"reasoning_content": 0, "content": 0}

        def flush(reasoning: str, content: str) -> None:
            for field, text in (("reasoning_content", reasoning), ("content", content)):
                delta = text[sent[field]:]
                if delta:
                    emit(chunk({field: delta}))
                    sent[field] = len(text)

        def on_token(token: int) -> bool:
            tokens.append(token)
            decoded = self.tokenizer.decode(tokens)
            stopped = any(s in decoded for s in stops if s)
            visible = truncate_stop(decoded, stops)
            safe = visible if stopped else visible[:safe_stream_boundary(visible, stops)]
            flush(*stream_channels(safe))
            return not stopped

        generated = self.model.generate_with(prompt, options, self.cache, on_token=on_token)
        flush(*stream_channels(truncate_stop(self.tokenizer.decode(generated), stops)))
        emit(chunk({}, "length" if len(generated) == options["max_tokens"] else "stop"))


def completion_id() -> str:
    return f"chatcmpl-metal-{int(time.time())}"


# ---- HTTP (server.rs:84-170, 425-546) ---------------------------------------------------
def make_handler(engine: ChatEngine):
    class Handler(BaseHTTPRequestHandler):
        protocol_version = "HTTP/1.1"

        def log_message(self, fmt, *args):  # quiet, as the reference
            pass

        def _headers(self, status: int, ctype: Optional[str], length: Optional[int]):
            self.send_response(status)
            if ctype:
                self.send_header("Content-Type", ctype)
            if length is not None:
                self.send_header("Content-Length", str(length))
            self.send_header("Connection", "close")
            self.send_header("Access-Control-Allow-Origin", "*")

        def _json(self, status: int, value: dict):
            body = json.dumps(value).encode()
            self._headers(status, "application/json", len(body))
            self.end_headers()
            self.wfile.write(body)
            self.close_connection = True

        def _error(self, status: int, message: str):
            self._json(status, {"error": {"message": message, "type": "invalid_request_error"}})

        def _path(self) -> str:
            return self.path.split("?", 1)[0]

        def do_OPTIONS(self):
            self._headers(204, None, 0)
            self.send_header("Access-Control-Allow-Headers", "Content-Type, Authorization")
            self.send_header("Access-Control-Allow-Methods", "GET, POST, OPTIONS")
            self.end_headers()
            self.close_connection = True

        def do_GET(self):
            if self._path() == "/health":
                self._json(200, {"status": "ok"})
            elif self._path() == "/v1/models":
                self._json(200, {"object": "list", "data": [
                    {"id": engine.model_id, "object": "model", "owned_by": "metal-infer"}]})
            else:
                self._error(404, "route not found")

        def do_POST(self):
            if self._path() != "/v1/chat/completions":
                self._error(404, "route not found")
                return
            try:
                length = int(self.headers.get("Content-Length", "0"))
            except ValueError:
                self._error(400, "invalid Content-Length")
                return
            if length > MAX_REQUEST_BYTES:
                self._error(400, "request is too large")
                return
            try:
                request = json.loads(self.rfile.read(length) or b"null")
                if not isinstance(request, dict):
                    raise ValueError("expected a JSON object")
            except ValueError as e:
                self._error(400, f"invalid JSON: {e}")
                return
            if request.get("stream"):
                try:
                    engine.prepare(request)  # reject before the event stream starts
                except Exception as e:
                    self._error(400, str(e))
                    return
                self._headers(200, "text/event-stream", None)
                self.send_header("Cache-Control", "no-cache")
                self.end_headers()

                def emit(value: dict):
                    self.wfile.write(b"data: " + json.dumps(value).encode() + b"\n\n")
                    self.wfile.flush()
                try:
                    engine.stream(request, emit)
                except Exception:  # headers are out: end the stream
                    pass
                self.wfile.write(b"data: [DONE]\n\n")
                self.wfile.flush()
                self.close_connection = True
                return
            try:
                self._json(200, engine.complete(request))
            except Exception as e:
                self._error(400, str(e))

    return Handler


def make_server(engine: ChatEngine, bind: str = "127.0.0.1:8080") -> HTTPServer:
    host, port = bind.rsplit(":", 1)
    return HTTPServer((host, int(port)), make_handler(engine))


def load_engine(model, context: int, model_id: Optional[str] = None, device: int = 0):
    """serve() setup (server.rs:84-112): resolve, load tokenizer and model,
    allocate the cache."""
    import metal_infer as mi
    requested = hugging_face_model_id(model)
    path = resolve_model_path(model)
    ctx = mi.MetalContext(device)
    tokenizer = ModelTokenizer.from_directory(path)
    qwen = mi.Qwen3Model.load(str(path), ctx)
    return ChatEngine(qwen, tokenizer, context, model_id or requested or infer_model_id(path))

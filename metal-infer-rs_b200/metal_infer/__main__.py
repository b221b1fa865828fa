"""metal-infer command line (crates/metal-infer-cli/src/main.rs):

    python -m metal_infer generate --model DIR_OR_HF_ID --prompt TEXT [--max-tokens 32]
        [--context 2048] [--temperature 0] [--top-p 1] [--top-k 0] [--seed 0]
        [--attention tiled|reference|flash-prefill]
    python -m metal_infer serve --model DIR_OR_HF_ID [--model-id ID]
        [--bind 127.0.0.1:8080] [--context 8192]
"""
from __future__ import annotations

import argparse
import sys


def _generate(a) -> int:
    import metal_infer as mi
    from metal_infer import serving
    path = serving.resolve_model_path(a.model)
    ctx = mi.MetalContext(0)
    print(f"CUDA device: {ctx.device_name()}", file=sys.stderr)
    print(f"Loading {path}", file=sys.stderr)
    tokenizer = serving.ModelTokenizer.from_directory(path)
    prompt = tokenizer.encode(a.prompt)
    model = mi.Qwen3Model.load(str(path), ctx)
    model.set_attention_kind({"reference": mi.AttentionKind.REFERENCE,
                              "tiled": mi.AttentionKind.TILED,
                              "flash-prefill": mi.AttentionKind.FLASH_PREFILL}[a.attention])
    required = len(prompt) + a.max_tokens
    if required > a.context:
        raise serving.ServingError(f"prompt + generated tokens ({required}) exceeds context "
                                   f"{a.context}")
    cache = model.kv_cache(a.context)
    generated = model.generate_with(prompt, dict(
        max_tokens=a.max_tokens, temperature=a.temperature, top_p=a.top_p, top_k=a.top_k,
        seed=a.seed, stop_token_ids=list(tokenizer.eos_token_ids)), cache)
    sys.stdout.write(tokenizer.decode(generated))
    sys.stdout.flush()
    return 0


def _serve(a) -> int:
    from metal_infer import serving
    engine = serving.load_engine(a.model, a.context, a.model_id)
    server = serving.make_server(engine, a.bind)
    print(f"OpenAI-compatible server listening on http://{a.bind}", file=sys.stderr)
    server.serve_forever()
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="metal-infer", description="Qwen3 inference on B200")
    sub = ap.add_subparsers(dest="command", required=True)
    g = sub.add_parser("generate")
    g.add_argument("--model", required=True)
    g.add_argument("--prompt", required=True)
    g.add_argument("--max-tokens", type=int, default=32)
    g.add_argument("--context", type=int, default=2048)
    g.add_argument("--temperature", type=float, default=0.0)
    g.add_argument("--top-p", type=float, default=1.0)
    g.add_argument("--top-k", type=int, default=0)
    g.add_argument("--seed", type=int, default=0)
    g.add_argument("--attention", choices=["reference", "tiled", "flash-prefill"], default="tiled")
    s = sub.add_parser("serve")
    s.add_argument("--model", required=True)
    s.add_argument("--model-id")
    s.add_argument("--bind", default="127.0.0.1:8080")
    s.add_argument("--context", type=int, default=8192)
    a = ap.parse_args(argv)
    try:
        return _generate(a) if a.command == "generate" else _serve(a)
    except Exception as e:  # main.rs: print the error, exit 1
        print(e, file=sys.stderr)
        return 1


if __name__ == "__main__":
    sys.exit(main())

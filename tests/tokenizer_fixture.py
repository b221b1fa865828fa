"""A synthetic Qwen-style tokenizer.json for the serving tests (no real
checkpoint exists here): a word-level vocabulary covering every id of a
small model (`t<id>` words, a few English words) plus the chat special
tokens, and a tokenizer_config.json naming the EOS tokens."""
import json
import os

SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "[UNK]"]
WORDS = ["hello", "world", "be", "concise.", "Be", "Hello", "say", "something", "STOP",
         "<think>", "</think>", "answer", "work"]


def write_tokenizer(directory: str, vocab_size: int, eos=("<|im_end|>", "<|endoftext|>")):
    from tokenizers import Tokenizer, models, pre_tokenizers, decoders  # noqa: F401
    from tokenizers import AddedToken
    vocab = {}
    for tok in SPECIALS + WORDS:
        vocab[tok] = len(vocab)
    i = 0
    while len(vocab) < vocab_size:
        vocab[f"t{i}"] = len(vocab)
        i += 1
    tk = Tokenizer(models.WordLevel(vocab, unk_token="[UNK]"))
    tk.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tk.add_special_tokens([AddedToken(t, special=True) for t in SPECIALS[:3]])
    os.makedirs(directory, exist_ok=True)
    tk.save(os.path.join(directory, "tokenizer.json"))
    with open(os.path.join(directory, "tokenizer_config.json"), "w") as f:
        json.dump({"eos_token": {"content": eos[0]}, "additional_special_tokens": list(eos)}, f)
    return vocab

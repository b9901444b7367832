"""Tokenizer loading, with a byte-level fallback for runs without tokenizer files.

Text environments (TextWorld, math) need a tokenizer. Real runs load the model directory's HF
tokenizer (``AutoTokenizer``, local files only). Random-init runs of a named shape have no tokenizer
files, so ``ByteTokenizer`` maps UTF-8 bytes to ids ``3..258`` (0 pad, 1 eos, 2 bos); any model with a
vocabulary of at least 259 can run on it. Its ``decode`` drops ids outside the byte range.
"""

from __future__ import annotations

import os
from typing import List, Optional


class ByteTokenizer:
    pad_token_id = 0
    eos_token_id = 1
    bos_token_id = 2
    offset = 3
    pad_token = "<pad>"
    eos_token = "<eos>"

    def __init__(self, vocab_size: int = 259):
        if vocab_size < 259:
            raise ValueError("ByteTokenizer needs a vocabulary of at least 259 ids")
        self.vocab_size = vocab_size

    def encode(self, text: str, add_special_tokens: bool = False) -> List[int]:
        return [b + self.offset for b in text.encode("utf-8")]

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        data = bytes(int(i) - self.offset for i in ids if self.offset <= int(i) < self.offset + 256)
        return data.decode("utf-8", errors="replace")

    def apply_chat_template(self, messages, tokenize: bool = False, add_generation_prompt: bool = True, **_):
        text = "".join(f"<|{m['role']}|>\n{m['content']}\n" for m in messages)
        if add_generation_prompt:
            text += "<|assistant|>\n"
        return self.encode(text) if tokenize else text


def load_tokenizer(model_path: str, trust_remote_code: bool = False, vocab_size: Optional[int] = None,
                   fallback: bool = False):
    """HF tokenizer of ``model_path`` when it has one; else ``ByteTokenizer`` if ``fallback`` (needs
    ``vocab_size``), else None."""
    if os.path.isdir(model_path):
        try:
            from transformers import AutoTokenizer

            tok = AutoTokenizer.from_pretrained(model_path, local_files_only=True, trust_remote_code=trust_remote_code)
            if tok.pad_token is None:
                tok.pad_token = tok.eos_token
            return tok
        except Exception:
            pass
    if fallback:
        return ByteTokenizer(vocab_size or 259)
    return None

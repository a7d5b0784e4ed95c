"""Tokenizers.  A local Hugging Face tokenizer directory is used when given; otherwise a
byte-level tokenizer (256 byte tokens + specials) serves random-weight models offline."""
from __future__ import annotations

import os
from typing import Optional


class ByteTokenizer:
    """Bytes 0..255 map to ids 3..258; 0 = <pad>, 1 = <bos>, 2 = <eos>.  Ids >= 259 (random
    models have larger vocabularies) decode to nothing."""
    pad_token_id = 0
    bos_token_id = 1
    eos_token_id = 2
    OFFSET = 3

    def __init__(self, vocab_size: int = 4096):
        self.vocab_size = vocab_size

    def encode(self, text: str, add_bos: bool = False) -> list[int]:
        ids = [b + self.OFFSET for b in text.encode("utf-8")]
        return ([self.bos_token_id] if add_bos else []) + ids

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        bs = bytes(i - self.OFFSET for i in ids if self.OFFSET <= i < 256 + self.OFFSET)
        return bs.decode("utf-8", errors="replace")

    def apply_chat_template(self, messages: list[dict], add_generation_prompt: bool = True,
                            **kw) -> str:
        """ChatML layout (the Qwen family's template)."""
        out = []
        enable_thinking = kw.get("enable_thinking", True)
        for m in messages:
            content = m.get("content") or ""
            if isinstance(content, list):
                content = "".join(p.get("text", "") for p in content if isinstance(p, dict))
            out.append(f"<|im_start|>{m['role']}\n{content}<|im_end|>\n")
        if add_generation_prompt:
            out.append("<|im_start|>assistant\n")
            if not enable_thinking:
                out.append("<think>\n\n</think>\n\n")
        return "".join(out)


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer
        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.eos_token_id = self.tok.eos_token_id
        self.vocab_size = len(self.tok)

    def encode(self, text: str, add_bos: bool = False) -> list[int]:
        return self.tok.encode(text, add_special_tokens=add_bos)

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        return self.tok.decode(ids, skip_special_tokens=skip_special_tokens)

    def apply_chat_template(self, messages, add_generation_prompt=True, **kw) -> str:
        return self.tok.apply_chat_template(messages, tokenize=False,
                                            add_generation_prompt=add_generation_prompt, **kw)


def get_tokenizer(path: Optional[str], vocab_size: int):
    if path and os.path.isdir(path) and any(
            os.path.exists(os.path.join(path, f)) for f in ("tokenizer.json", "tokenizer_config.json")):
        return HFTokenizer(path)
    return ByteTokenizer(vocab_size)


class IncrementalDetokenizer:
    """Streams text deltas; holds back an incomplete UTF-8 tail and stop-string prefixes."""

    def __init__(self, tokenizer, stop: Optional[list[str]] = None):
        self.tok = tokenizer
        self.stop = [s for s in (stop or []) if s]
        self.text = ""
        self.emitted = 0
        self.stopped = False

    def update(self, all_output_ids) -> str:
        if self.stopped:
            return ""
        self.text = self.tok.decode(all_output_ids)
        visible = self.text
        if visible.endswith("�"):
            visible = visible.rstrip("�")
        for s in self.stop:
            i = visible.find(s)
            if i >= 0:
                visible = visible[:i]
                self.text = visible
                self.stopped = True
                break
        if not self.stopped and self.stop:
            hold = max(len(s) - 1 for s in self.stop)
            for k in range(min(hold, len(visible)), 0, -1):
                if any(s.startswith(visible[-k:]) for s in self.stop):
                    visible = visible[:-k]
                    break
        delta = visible[self.emitted:]
        self.emitted = len(visible)
        return delta

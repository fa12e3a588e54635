"""Tokenizers and chat-template rendering for the API.

* :class:`ByteTokenizer` is the tokenizer of random-init models (no
  checkpoint, no network): UTF-8 bytes mapped to ids ``offset + byte``.
* :class:`HFTokenizer` wraps a local HuggingFace tokenizer directory (the
  ``tokenizer/`` folder of a shard tree) when one exists.
* :class:`ChatPromptRenderer` renders ``messages`` through the tokenizer's
  Jinja chat template (``enable_thinking`` and ``tools`` passed through, as the
  reference's minijinja renderer does, crates/cascadia-api/src/lib.rs:1280,
  :1659) and falls back to a plain role-prefixed transcript.
"""
from __future__ import annotations

import json
import os
from typing import List, Optional, Sequence


class ByteTokenizer:
    def __init__(self, vocab_size: int = 512, offset: int = 3, eos_id: int = 1):
        self.vocab_size = vocab_size
        self.offset = offset
        self.eos_id = eos_id
        self.chat_template: Optional[str] = None

    def encode(self, text: str) -> List[int]:
        return [self.offset + b for b in text.encode("utf-8")]

    def decode(self, ids: Sequence[int]) -> str:
        bs = bytes(i - self.offset for i in ids if self.offset <= i < self.offset + 256)
        return bs.decode("utf-8", errors="replace")

    def decode_incremental(self, ids: Sequence[int], emitted: int) -> (str, int):
        """Text of ids[emitted_tokens:] that forms complete characters."""
        full = bytes(i - self.offset for i in ids if self.offset <= i < self.offset + 256)
        text = full.decode("utf-8", errors="ignore")
        return text, len(ids)


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer  # local files only

        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.vocab_size = len(self.tok)
        self.eos_id = self.tok.eos_token_id
        self.chat_template = getattr(self.tok, "chat_template", None)

    def encode(self, text: str) -> List[int]:
        return self.tok.encode(text, add_special_tokens=False)

    def decode(self, ids: Sequence[int]) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=True)


def load_tokenizer(path: Optional[str], vocab_size: int, eos_id: int):
    if path and os.path.isdir(path):
        try:
            return HFTokenizer(path)
        except Exception:  # noqa: BLE001 - no usable tokenizer files
            pass
    return ByteTokenizer(vocab_size=vocab_size, eos_id=eos_id)


class IncrementalDecoder:
    """Emit only newly-completed text as tokens arrive (advance_emitted)."""

    def __init__(self, tokenizer):
        self.tok = tokenizer
        self.ids: List[int] = []
        self.text = ""

    def push(self, token_ids: Sequence[int]) -> str:
        self.ids.extend(int(t) for t in token_ids)
        full = self.tok.decode(self.ids)
        if full.endswith("�"):  # incomplete UTF-8 sequence: wait
            return ""
        delta = full[len(self.text):] if full.startswith(self.text) else full
        self.text = full
        return delta


class ChatPromptRenderer:
    def __init__(self, template: Optional[str] = None, bos: str = "", eos: str = ""):
        self.template = template
        self.bos, self.eos = bos, eos
        self._compiled = None
        if template:
            try:
                import jinja2

                env = jinja2.Environment(undefined=jinja2.ChainableUndefined,
                                         trim_blocks=True, lstrip_blocks=True)
                env.filters["tojson"] = lambda v, indent=None, **kw: json.dumps(
                    v, indent=indent, ensure_ascii=False)
                self._compiled = env.from_string(template)
            except Exception:  # noqa: BLE001 - fall back to the legacy format
                self._compiled = None

    def render(self, messages: List[dict], enable_thinking: bool = True,
               tools: Optional[list] = None, add_generation_prompt: bool = True) -> str:
        if self._compiled is not None:
            try:
                return self._compiled.render(messages=messages, tools=tools,
                                             add_generation_prompt=add_generation_prompt,
                                             enable_thinking=enable_thinking,
                                             bos_token=self.bos, eos_token=self.eos)
            except Exception:  # noqa: BLE001
                pass
        parts = []
        for m in messages:
            content = m.get("content")
            if isinstance(content, list):  # OpenAI content parts
                content = "".join(p.get("text", "") for p in content if isinstance(p, dict))
            parts.append(f"{m.get('role', 'user')}: {content or ''}")
        if add_generation_prompt:
            parts.append("assistant:")
        return "\n".join(parts)

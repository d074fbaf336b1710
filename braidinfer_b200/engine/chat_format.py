"""Chat-template fragments for chunks.

A chunk caches the tokens of its own chat-template *fragment* (for Qwen:
``<|im_start|>user\\n{content}<|im_end|>\\n``), so the concatenation of a
composition's chunk tokens plus the generation prompt is exactly the token
sequence the HF chat template produces for the whole conversation.  The
reference cached raw content tokens but then decoded against the templated
conversation, so cached and attended tokens disagreed (its
``braidinfer/engine/llm_engine.py:453-493`` vs ``braidinfer/chunked_llm.py:561-564``).

Fragments are derived from the tokenizer's own template by rendering with and
without the message and taking the textual difference.  Tokenizers without a
chat template fall back to raw content tokens and an empty generation prompt.
"""
from __future__ import annotations

from typing import List, Optional

from ..chunks import ChunkType

ROLE_OF = {ChunkType.SYSTEM_PROMPT: "system", ChunkType.CONTEXT: "user", ChunkType.QUERY: "user",
           ChunkType.OUTPUT: "assistant"}
_DUMMY_SYS = {"role": "system", "content": "x"}


class ChatFormat:
    def __init__(self, tokenizer, use_template: bool = True):
        self.tok = tokenizer
        self.enabled = bool(use_template and tokenizer is not None and getattr(tokenizer, "chat_template", None))
        self._gen_prompt: Optional[List[int]] = None

    def _render(self, msgs, gen: bool = False) -> str:
        return self.tok.apply_chat_template(msgs, tokenize=False, add_generation_prompt=gen)

    def encode(self, text: str) -> List[int]:
        return list(self.tok.encode(text, add_special_tokens=False)) if self.tok is not None else []

    def fragment(self, role: str, content: str) -> str:
        msg = {"role": role, "content": content}
        if role == "system":
            return self._render([msg])
        base = self._render([_DUMMY_SYS])
        full = self._render([_DUMMY_SYS, msg])
        if full.startswith(base):
            return full[len(base):]
        return full

    def chunk_tokens(self, chunk_type: ChunkType, content: str, role: Optional[str] = None) -> List[int]:
        if not self.enabled or chunk_type == ChunkType.OUTPUT:
            return self.encode(content)
        return self.encode(self.fragment(role or ROLE_OF[chunk_type], content))

    def generation_prompt(self) -> List[int]:
        """Tokens that open the assistant turn (rendered once, then cached)."""
        if self._gen_prompt is None:
            if not self.enabled:
                self._gen_prompt = []
            else:
                msgs = [_DUMMY_SYS, {"role": "user", "content": "x"}]
                a, b = self._render(msgs, False), self._render(msgs, True)
                self._gen_prompt = self.encode(b[len(a):]) if b.startswith(a) else []
        return list(self._gen_prompt)

"""Byte-level tokenizer for text I/O with random-initialised weights (no checkpoint vocabulary is available
offline): token id = byte value + 16 (ids 0..15 reserved: 0 = mask / pad, 1 = BOS, 2 = EOS); ids that do not map to
a byte decode to nothing."""

from __future__ import annotations

OFFSET = 16
BOS, EOS = 1, 2


class ByteTokenizer:
    def __init__(self, vocab: int):
        if vocab < OFFSET + 256:
            raise ValueError("vocabulary too small for the byte tokenizer")
        self.vocab = vocab
        self.eos_token_id = EOS
        self.bos_token_id = BOS

    def encode(self, text: str, bos: bool = True) -> list[int]:
        ids = [b + OFFSET for b in text.encode("utf-8")]
        return ([BOS] if bos else []) + ids

    def decode(self, ids) -> str:
        bs = bytes(i - OFFSET for i in ids if OFFSET <= i < OFFSET + 256)
        return bs.decode("utf-8", errors="replace")

    def apply_chat_template(self, messages: list[dict], add_generation_prompt: bool = True,
                            reasoning_effort: str | None = None, tools: list | None = None) -> str:
        """``reasoning_effort`` becomes a system line placed before the first user turn (so the cached prompt head
        -- system prompt and tool list -- stays identical across efforts: the reference's chat-template option,
        code/launcher-patches/chat_template-reasoning-effort-placement.patch:1-40); ``tools`` are listed in a
        system block as JSON."""
        parts = []
        if tools:
            import json
            parts.append("<|system|>\n# Tools\n" + "\n".join(json.dumps(t, sort_keys=True) for t in tools) + "\n")
        placed = reasoning_effort is None
        for m in messages:
            if not placed and m.get("role") == "user":
                parts.append(f"<|system|>\nReasoning effort: {reasoning_effort}\n")
                placed = True
            content = m.get("content", "")
            if isinstance(content, list):       # OpenAI content parts: keep the text ones
                content = "".join(p.get("text", "") for p in content if isinstance(p, dict))
            parts.append(f"<|{m.get('role', 'user')}|>\n{content}\n")
        if not placed:
            parts.append(f"<|system|>\nReasoning effort: {reasoning_effort}\n")
        if add_generation_prompt:
            parts.append("<|assistant|>\n")
        return "".join(parts)

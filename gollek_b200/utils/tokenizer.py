"""Tokenizers: Hugging Face ``tokenizer.json``, GGUF-embedded vocabularies, and a byte fallback.

The reference ships BPE / HF-BPE / SentencePiece / WordPiece tokenizers and a GGUF
metadata tokenizer (core/gollek-tokenizer-core/…/tokenizer/impl/*.java; runner/gguf/
gollek-gguf-tokenizer/…/GGUFTokenizer.java:1-335) plus a streaming decoder. Here the HF path
uses the ``tokenizers`` library, GGUF vocabularies get a greedy longest-match SentencePiece-style
encoder over the stored pieces (scores break ties), and random-init presets use a byte-level
tokenizer so text requests still work end to end.
"""
from __future__ import annotations

import json
import os
from typing import Dict, List, Optional


def _gpt2_byte_decoder() -> Dict[str, int]:
    """Inverse of the GPT-2 byte-level BPE alphabet: printable Latin-1 bytes stand for themselves,
    the remaining bytes are shifted to code points 256 + n in byte order."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + list(range(ord("®"), ord("ÿ") + 1))
    chars = list(keep)
    n = 0
    for b in range(256):
        if b not in keep:
            keep.append(b)
            chars.append(256 + n)
            n += 1
    return {chr(c): b for b, c in zip(keep, chars)}


def _piece_bytes(piece: str, byte_level: bool, dec: Dict[str, int]) -> bytes:
    """Bytes a vocabulary piece stands for (byte-level BPE or SentencePiece conventions)."""
    if byte_level:
        try:
            return bytes(dec[ch] for ch in piece)
        except KeyError:
            return piece.encode("utf-8")
    if len(piece) == 6 and piece.startswith("<0x") and piece.endswith(">"):
        try:
            return bytes([int(piece[3:5], 16)])
        except ValueError:
            pass
    return piece.replace("▁", " ").encode("utf-8")


class ByteTokenizer:
    """UTF-8 bytes mapped to ids 3..258 (0 = pad, 1 = bos, 2 = eos)."""
    offset = 3

    def __init__(self, vocab_size: int = 32000, eos_token_id: int = 2):
        self.vocab_size = vocab_size
        self.eos_token_id = eos_token_id

    def encode(self, text: str) -> List[int]:
        return [b + self.offset for b in text.encode("utf-8")]

    def decode(self, ids: List[int]) -> str:
        bs = bytes(i - self.offset for i in ids if self.offset <= i < self.offset + 256)
        return bs.decode("utf-8", errors="replace")

    def token_bytes(self) -> List[bytes]:
        out = [b""] * self.vocab_size
        for b in range(256):
            if b + self.offset < self.vocab_size:
                out[b + self.offset] = bytes([b])
        return out

    def apply_chat_template(self, messages: List[dict], tools: Optional[List[dict]] = None) -> str:
        return default_chat_template(messages, tools)


class HFTokenizer:
    def __init__(self, path: str):
        from tokenizers import Tokenizer
        self.tok = Tokenizer.from_file(path)
        self.vocab_size = self.tok.get_vocab_size()
        self.chat_template: Optional[str] = None
        cfg = os.path.join(os.path.dirname(path), "tokenizer_config.json")
        if os.path.exists(cfg):
            with open(cfg) as f:
                self.chat_template = json.load(f).get("chat_template")

    def encode(self, text: str) -> List[int]:
        return self.tok.encode(text, add_special_tokens=True).ids

    def decode(self, ids: List[int]) -> str:
        return self.tok.decode(ids, skip_special_tokens=True)

    def token_bytes(self) -> List[bytes]:
        vocab = self.tok.get_vocab(with_added_tokens=True)
        special = {t.content for t in self.tok.get_added_tokens_decoder().values() if t.special} \
            if hasattr(self.tok, "get_added_tokens_decoder") else set()
        byte_level = any(("Ġ" in p or "Ċ" in p) for p in list(vocab)[:5000])
        dec = _gpt2_byte_decoder()
        out = [b""] * max(self.vocab_size, max(vocab.values()) + 1)
        for piece, i in vocab.items():
            if piece not in special:
                out[i] = _piece_bytes(piece, byte_level, dec)
        return out

    def apply_chat_template(self, messages: List[dict], tools: Optional[List[dict]] = None) -> str:
        """The checkpoint's Jinja chat template; tool definitions go to the template's ``tools``
        variable when it has one, else into a system message."""
        if self.chat_template:
            try:
                import jinja2
                msgs = messages
                if tools and "tools" not in self.chat_template:
                    msgs, tools = _with_tools_system(messages, tools), None
                return jinja2.Template(self.chat_template).render(messages=msgs, tools=tools,
                                                                  add_generation_prompt=True, bos_token="",
                                                                  eos_token="")
            except Exception:
                pass
        return default_chat_template(messages, tools)


class GGUFTokenizer:
    """Vocabulary from ``tokenizer.ggml.tokens`` (+ scores); SentencePiece-style greedy encode."""

    def __init__(self, tokens: List[str], scores: Optional[List[float]] = None, bos: int = 1, eos: int = 2):
        self.tokens = tokens
        self.vocab_size = len(tokens)
        self.scores = scores or [0.0] * len(tokens)
        self.bos, self.eos_token_id = bos, eos
        self.index: Dict[str, int] = {}
        for i, t in enumerate(tokens):
            if t not in self.index or self.scores[i] > self.scores[self.index[t]]:
                self.index[t] = i
        self.max_len = max((len(t) for t in tokens), default=1)
        self.byte_ids = {}
        for i, t in enumerate(tokens):
            if len(t) == 6 and t.startswith("<0x") and t.endswith(">"):
                try:
                    self.byte_ids[int(t[3:5], 16)] = i
                except ValueError:
                    pass

    @staticmethod
    def from_metadata(meta: dict) -> "GGUFTokenizer":
        return GGUFTokenizer(meta.get("tokenizer.ggml.tokens", []), meta.get("tokenizer.ggml.scores"),
                             int(meta.get("tokenizer.ggml.bos_token_id", 1)), int(meta.get("tokenizer.ggml.eos_token_id", 2)))

    def encode(self, text: str) -> List[int]:
        s = "▁" + text.replace(" ", "▁")
        ids, i = [], 0
        while i < len(s):
            for L in range(min(self.max_len, len(s) - i), 0, -1):
                piece = s[i:i + L]
                if piece in self.index:
                    ids.append(self.index[piece])
                    i += L
                    break
            else:
                for b in s[i].encode("utf-8"):
                    ids.append(self.byte_ids.get(b, 0))
                i += 1
        return ids

    def token_bytes(self) -> List[bytes]:
        byte_level = any(("Ġ" in p or "Ċ" in p) for p in self.tokens[:5000])
        dec = _gpt2_byte_decoder()
        return [b"" if (p.startswith("<") and p.endswith(">") and len(p) != 6) else _piece_bytes(p, byte_level, dec)
                for p in self.tokens]

    def decode(self, ids: List[int]) -> str:
        out = bytearray()
        inv_bytes = {v: k for k, v in self.byte_ids.items()}
        for i in ids:
            if i in inv_bytes:
                out.append(inv_bytes[i])
            elif 0 <= i < len(self.tokens):
                out += self.tokens[i].replace("▁", " ").encode("utf-8")
        return out.decode("utf-8", errors="replace").lstrip(" ")

    def apply_chat_template(self, messages: List[dict], tools: Optional[List[dict]] = None) -> str:
        return default_chat_template(messages, tools)


def _with_tools_system(messages: List[dict], tools: List[dict]) -> List[dict]:
    from ..server.tools import tools_preamble
    pre = tools_preamble(tools)
    if messages and messages[0].get("role") == "system":
        first = dict(messages[0])
        first["content"] = f"{first.get('content') or ''}\n\n{pre}"
        return [first] + list(messages[1:])
    return [{"role": "system", "content": pre}] + list(messages)


def default_chat_template(messages: List[dict], tools: Optional[List[dict]] = None) -> str:
    if tools:
        messages = _with_tools_system(messages, tools)
    parts = []
    for m in messages:
        if m.get("tool_calls"):  # an assistant turn that called tools
            calls = "".join("<tool_call>" + json.dumps({"name": tc.get("function", {}).get("name"),
                                                        "arguments": tc.get("function", {}).get("arguments")})
                            + "</tool_call>" for tc in m["tool_calls"])
            parts.append(f"<|assistant|>\n{m.get('content') or ''}{calls}\n")
            continue
        content = m.get("content", "")
        if isinstance(content, list):
            content = "".join(c.get("text", "") for c in content if isinstance(c, dict))
        parts.append(f"<|{m.get('role', 'user')}|>\n{content}\n")
    parts.append("<|assistant|>\n")
    return "".join(parts)


def load_tokenizer(directory: str):
    p = os.path.join(directory, "tokenizer.json")
    if os.path.exists(p):
        return HFTokenizer(p)
    return None

"""Tokenizers: Hugging Face ``tokenizer.json``, GGUF-embedded vocabularies, and a byte fallback.

The reference ships BPE / HF-BPE / SentencePiece / WordPiece tokenizers and a GGUF
metadata tokenizer (core/gollek-tokenizer-core/…/tokenizer/impl/*.java; runner/gguf/
gollek-gguf-tokenizer/…/GGUFTokenizer.java:1-335) plus a streaming decoder. Here the HF path
uses the ``tokenizers`` library; GGUF vocabularies are tokenized by their own metadata
(SentencePiece BPE by piece scores, or byte-level BPE by ``tokenizer.ggml.merges``; checked
against sentencepiece and HF ``tokenizers`` on the same vocabularies); random-init presets use a
byte-level tokenizer so text requests still work end to end.
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

    def token_text(self, i: int) -> Optional[str]:
        """The vocabulary string of token ``i`` (special tokens included)."""
        return self.tok.id_to_token(i)

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


# Pre-tokenizer split patterns of byte-level BPE vocabularies, by ``tokenizer.ggml.pre``: GPT-2's
# (the default) and the one Llama-3 vocabularies were trained with (digits in groups of up to three).
_PRE_PATTERNS = {
    "default": r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+""",
    "llama-bpe": r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*"""
                 r"""|\s*[\r\n]+|\s+(?!\S)|\s+""",
}
_PRE_PATTERNS["llama3"] = _PRE_PATTERNS["llama-bpe"]
_PRE_PATTERNS["gpt2"] = _PRE_PATTERNS["default"]

# ggml token types (tokenizer.ggml.token_type)
_TT_NORMAL, _TT_UNKNOWN, _TT_CONTROL, _TT_USER_DEFINED, _TT_UNUSED, _TT_BYTE = 1, 2, 3, 4, 5, 6


class GGUFTokenizer:
    """Tokenizer built from a GGUF file's ``tokenizer.ggml.*`` metadata.

    * ``model == "llama"``: SentencePiece BPE. The text gets a leading space and spaces become
      ``▁``; starting from single characters, the adjacent pair whose concatenation is a vocabulary
      piece with the highest score is merged first (leftmost on ties) until no pair is in the
      vocabulary; characters left outside it fall back to their ``<0xXX>`` byte pieces.
    * ``model == "gpt2"``: byte-level BPE. The text is split by the vocabulary's pre-tokenizer
      pattern (``tokenizer.ggml.pre``), each chunk's UTF-8 bytes are mapped to the GPT-2 byte
      alphabet, and ``tokenizer.ggml.merges`` are applied lowest rank first.
    * ``model == "bert"``: WordPiece. The text is cleaned (control characters dropped, whitespace
      unified), lower-cased with accents stripped (``lowercase``), CJK ideographs and punctuation
      become words of their own, and each whitespace-separated word is split greedily into the
      longest vocabulary pieces from its start; a word with no such split (or longer than 100
      characters) becomes the unknown token. The vocabulary may be in the ``##`` continuation form
      (as HF writes it) or in GGUF's phantom-space form (word-initial pieces carry ``▁``, continuation
      pieces are bare). The ids are wrapped in the classifier / separator tokens.
    Control / user-defined tokens that appear literally in the text are matched as single ids.
    ``add_bos`` follows ``tokenizer.ggml.add_bos_token``; ``tokenizer.chat_template`` (Jinja) is used
    by ``apply_chat_template`` when present.

    Reference: runner/gguf/gollek-gguf-tokenizer/…/gguf/tokenizer/GGUFTokenizer.java:53-78 (merges and
    vocabulary loading from the same metadata keys).
    """

    def __init__(self, tokens: List[str], scores: Optional[List[float]] = None, bos: int = 1, eos: int = 2,
                 model: str = "llama", merges: Optional[List[str]] = None, token_types: Optional[List[int]] = None,
                 pre: str = "default", add_bos: Optional[bool] = None, chat_template: Optional[str] = None,
                 add_eos: Optional[bool] = None, unk: Optional[int] = None, lowercase: bool = True):
        self.tokens = tokens
        self.vocab_size = len(tokens)
        self.model = model
        self.scores = scores or [0.0] * len(tokens)
        self.bos, self.eos_token_id = bos, eos
        self.token_types = token_types or [_TT_NORMAL] * len(tokens)
        self.add_bos = (model in ("llama", "bert")) if add_bos is None else bool(add_bos)
        self.add_eos = (model == "bert") if add_eos is None else bool(add_eos)
        self.wordpiece = model == "bert"
        self.lowercase = lowercase
        self.chat_template = chat_template
        self.index: Dict[str, int] = {}
        for i, t in enumerate(tokens):
            if t not in self.index or self.scores[i] > self.scores[self.index[t]]:
                self.index[t] = i
        self.byte_ids = {}
        for i, t in enumerate(tokens):
            if len(t) == 6 and t.startswith("<0x") and t.endswith(">"):
                try:
                    self.byte_ids[int(t[3:5], 16)] = i
                except ValueError:
                    pass
        self.special = {t: i for i, t in enumerate(tokens)
                        if self.token_types[i] in (_TT_CONTROL, _TT_USER_DEFINED) and t}
        self._special_re = None
        if self.special:
            import regex
            self._special_re = regex.compile("|".join(regex.escape(t) for t in
                                                      sorted(self.special, key=len, reverse=True)))
        self.byte_level = model == "gpt2"
        self.ranks: Dict[tuple, int] = {}
        if self.byte_level:
            import regex
            for r, m in enumerate(merges or []):
                a, _, b = m.partition(" ")
                self.ranks[(a, b)] = r
            self._pre = regex.compile(_PRE_PATTERNS.get(pre, _PRE_PATTERNS["default"]))
            enc = {v: k for k, v in _gpt2_byte_decoder().items()}
            self._byte_enc = [enc[b] for b in range(256)]
        self._dec = _gpt2_byte_decoder()
        self._cache: Dict[str, List[int]] = {}
        if self.wordpiece:
            self.hash_form = any(t.startswith("##") and len(t) > 2 for t in tokens)
            self.unk = unk if unk is not None else self.index.get("[UNK]", 0)

    @staticmethod
    def from_metadata(meta: dict) -> "GGUFTokenizer":
        return GGUFTokenizer(meta.get("tokenizer.ggml.tokens", []), meta.get("tokenizer.ggml.scores"),
                             int(meta.get("tokenizer.ggml.bos_token_id", 1)),
                             int(meta.get("tokenizer.ggml.eos_token_id", 2)),
                             model=str(meta.get("tokenizer.ggml.model", "llama")),
                             merges=meta.get("tokenizer.ggml.merges"),
                             token_types=meta.get("tokenizer.ggml.token_type"),
                             pre=str(meta.get("tokenizer.ggml.pre", "default")),
                             add_bos=meta.get("tokenizer.ggml.add_bos_token"),
                             chat_template=meta.get("tokenizer.chat_template"),
                             add_eos=meta.get("tokenizer.ggml.add_eos_token"),
                             unk=meta.get("tokenizer.ggml.unknown_token_id"))

    # -- encoding
    def encode(self, text: str, add_special: bool = True) -> List[int]:
        ids: List[int] = [self.bos] if (add_special and self.add_bos) else []
        parts = [(text, False)]
        if self._special_re is not None:
            parts, pos = [], 0
            for m in self._special_re.finditer(text):
                if m.start() > pos:
                    parts.append((text[pos:m.start()], False))
                parts.append((m.group(0), True))
                pos = m.end()
            if pos < len(text):
                parts.append((text[pos:], False))
        first = True
        for chunk, is_special in parts:
            if is_special:
                ids.append(self.special[chunk])
            elif self.wordpiece:
                ids += self._encode_wpm(chunk)
            elif self.byte_level:
                ids += self._encode_bpe(chunk)
            else:
                ids += self._encode_spm(chunk, first)
            first = False
        if add_special and self.add_eos:
            ids.append(self.eos_token_id)
        return ids

    @staticmethod
    def _wpm_words(text: str, lowercase: bool) -> List[str]:
        import unicodedata
        out, cur = [], []

        def flush():
            if cur:
                out.append("".join(cur))
                cur.clear()
        if lowercase:
            text = "".join(c for c in unicodedata.normalize("NFD", text.lower()) if unicodedata.category(c) != "Mn")
        for c in text:
            o = ord(c)
            cat = unicodedata.category(c)
            if o == 0 or o == 0xFFFD or (cat.startswith("C") and c not in "\t\n\r"):
                continue
            if c.isspace():
                flush()
            elif (33 <= o <= 47 or 58 <= o <= 64 or 91 <= o <= 96 or 123 <= o <= 126 or cat.startswith("P")
                  or 0x4E00 <= o <= 0x9FFF or 0x3400 <= o <= 0x4DBF or 0x20000 <= o <= 0x2A6DF
                  or 0xF900 <= o <= 0xFAFF or 0x2F800 <= o <= 0x2FA1F):
                flush()
                out.append(c)
            else:
                cur.append(c)
        flush()
        return out

    def _encode_wpm(self, text: str) -> List[int]:
        ids: List[int] = []
        for w in self._wpm_words(text, self.lowercase):
            if len(w) > 100:
                ids.append(self.unk)
                continue
            pieces, start = [], 0
            while start < len(w):
                for end in range(len(w), start, -1):
                    sub = w[start:end]
                    key = (("##" + sub) if start else sub) if self.hash_form else (sub if start else "▁" + sub)
                    if key in self.index:
                        pieces.append(self.index[key])
                        break
                else:
                    pieces = [self.unk]
                    break
                start = end
            ids += pieces
        return ids

    def _encode_bpe(self, text: str) -> List[int]:
        out: List[int] = []
        for word in self._pre.findall(text):
            hit = self._cache.get(word)
            if hit is None:
                hit = self._bpe_word("".join(self._byte_enc[b] for b in word.encode("utf-8")))
                if len(self._cache) < 100000:
                    self._cache[word] = hit
            out += hit
        return out

    def _bpe_word(self, w: str) -> List[int]:
        syms = list(w)
        ranks = self.ranks
        while len(syms) > 1:
            best, bi = None, -1
            for i in range(len(syms) - 1):
                r = ranks.get((syms[i], syms[i + 1]))
                if r is not None and (best is None or r < best):
                    best, bi = r, i
            if best is None:
                break
            a, b = syms[bi], syms[bi + 1]
            merged, i = [], 0
            while i < len(syms):  # every occurrence of the pair, left to right
                if i < len(syms) - 1 and syms[i] == a and syms[i + 1] == b:
                    merged.append(a + b)
                    i += 2
                else:
                    merged.append(syms[i])
                    i += 1
            syms = merged
        out = []
        for sym in syms:
            i = self.index.get(sym)
            if i is not None:
                out.append(i)
            else:  # a piece outside the vocabulary: its single-byte pieces
                out += [self.index.get(ch, 0) for ch in sym]
        return out

    def _encode_spm(self, text: str, leading: bool) -> List[int]:
        import heapq
        s = ("▁" if leading else "") + text.replace(" ", "▁")
        if not s:
            return []
        syms = list(s)
        n = len(syms)
        prev = list(range(-1, n - 1))
        nxt = list(range(1, n + 1))
        alive = [True] * n
        heap = []

        def push(i):
            j = nxt[i]
            if j >= n:
                return
            piece = syms[i] + syms[j]
            t = self.index.get(piece)
            if t is not None:
                heapq.heappush(heap, (-self.scores[t], i, piece))

        for i in range(n - 1):
            push(i)
        while heap:
            _, i, piece = heapq.heappop(heap)
            j = nxt[i] if alive[i] else n
            if not alive[i] or j >= n or syms[i] + syms[j] != piece:
                continue  # stale entry
            syms[i] = piece
            alive[j] = False
            nxt[i] = nxt[j]
            if nxt[j] < n:
                prev[nxt[j]] = i
            if prev[i] >= 0:
                push(prev[i])
            push(i)
        ids: List[int] = []
        i = 0
        while i < n:
            t = self.index.get(syms[i])
            if t is not None:
                ids.append(t)
            else:
                ids += [self.byte_ids.get(b, 0) for b in syms[i].encode("utf-8")]
            i = nxt[i]
        return ids

    # -- decoding
    def token_text(self, i: int) -> Optional[str]:
        return self.tokens[i] if 0 <= i < len(self.tokens) else None

    def token_bytes(self) -> List[bytes]:
        out = []
        for i, p in enumerate(self.tokens):
            tt = self.token_types[i]
            if tt in (_TT_CONTROL, _TT_UNUSED) or (p.startswith("<") and p.endswith(">") and len(p) != 6
                                                  and tt != _TT_USER_DEFINED and not self.byte_level):
                out.append(b"")
            else:
                out.append(_piece_bytes(p, self.byte_level, self._dec))
        return out

    def decode(self, ids: List[int]) -> str:
        out = bytearray()
        if self.wordpiece:
            words: List[str] = []
            for i in ids:
                if not (0 <= i < len(self.tokens)) or self.token_types[i] == _TT_CONTROL:
                    continue
                t = self.tokens[i]
                if self.hash_form:
                    cont = t.startswith("##")
                    t = t[2:] if cont else t
                else:
                    cont = not t.startswith("▁")
                    t = t if cont else t[1:]
                if cont and words:
                    words[-1] += t
                else:
                    words.append(t)
            return " ".join(words)
        if self.byte_level:
            for i in ids:
                if 0 <= i < len(self.tokens) and self.token_types[i] != _TT_CONTROL:
                    out += _piece_bytes(self.tokens[i], True, self._dec)
            return out.decode("utf-8", errors="replace")
        inv_bytes = {v: k for k, v in self.byte_ids.items()}
        for i in ids:
            if i in inv_bytes:
                out.append(inv_bytes[i])
            elif 0 <= i < len(self.tokens) and self.token_types[i] != _TT_CONTROL:
                out += self.tokens[i].replace("▁", " ").encode("utf-8")
        text = out.decode("utf-8", errors="replace")
        return text[1:] if text.startswith(" ") else text

    def apply_chat_template(self, messages: List[dict], tools: Optional[List[dict]] = None) -> str:
        """The file's Jinja ``tokenizer.chat_template`` when present (``bos_token`` / ``eos_token`` set
        to the vocabulary's pieces), else the built-in role-tag template."""
        if self.chat_template:
            try:
                import jinja2
                msgs = messages
                if tools and "tools" not in self.chat_template:
                    msgs, tools = _with_tools_system(messages, tools), None
                env = jinja2.Environment()
                env.globals["raise_exception"] = lambda m: (_ for _ in ()).throw(ValueError(m))
                bos = self.tokens[self.bos] if 0 <= self.bos < len(self.tokens) else ""
                eos = self.tokens[self.eos_token_id] if 0 <= self.eos_token_id < len(self.tokens) else ""
                text = env.from_string(self.chat_template).render(messages=msgs, tools=tools,
                                                                  add_generation_prompt=True, bos_token=bos,
                                                                  eos_token=eos)
                # encode() adds BOS itself: drop a rendered leading BOS so it is not doubled
                if self.add_bos and bos and text.startswith(bos):
                    text = text[len(bos):]
                return text
            except Exception:
                pass
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

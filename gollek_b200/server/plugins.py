"""Request / response plugins of the server: PII redaction, content safety, reasoning-block split and
a semantic response cache.

Reference behaviour: plugins/gollek-plugin-pii-redaction/…/PIIRedactionService.java:60-107 (e-mail,
phone, card, US SSN, IPv4 address, API-key assignment and AWS access-key patterns replaced by typed
``[REDACTED_*]`` markers; custom patterns can be added), plugins/gollek-plugin-content-
safety/…/ContentSafetyPlugin.java:64-110 (blocked keywords, case-insensitive, and blocked regular
expressions reject the request), plugins/gollek-plugin-reasoning/…/OutputParser.java:111-112
(``<think>`` / ``<reasoning>`` blocks separated from the answer) and plugins/gollek-plugin-semantic-
cache/…/SemanticCacheService.java (responses reused for prompts whose embedding is within a cosine
threshold, 0.85 by default, bounded size and age). Embeddings come from the served model.
"""
from __future__ import annotations

import os
import re
import threading
import time
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

_OCTET = r"(?:25[0-5]|2[0-4]\d|1\d\d|[1-9]?\d)"
PII_PATTERNS: List[Tuple[str, "re.Pattern"]] = [
    # secrets first: their values may contain digit runs the later kinds would take
    ("AWS_KEY", re.compile(r"\b(?:AKIA|ABIA|ACCA|ASIA)[0-9A-Z]{16}\b")),
    ("API_KEY", re.compile(r"\b(?:api[_-]?key|apikey|secret[_-]?key|access[_-]?token)\s*[=:]\s*['\"]?[\w\-]{20,}['\"]?",
                           re.IGNORECASE)),
    ("EMAIL", re.compile(r"\b[\w.%+-]+@[\w-]+(?:\.[\w-]+)*\.[A-Za-z]{2,}\b")),
    # before PHONE: a dotted IPv4 address has enough digits to pass for a phone number
    ("IP", re.compile(rf"(?<![\d.]){_OCTET}(?:\.{_OCTET}){{3}}(?![\d.])")),
    ("SSN", re.compile(r"\b\d{3}-\d{2}-\d{4}\b")),
    ("CC", re.compile(r"\b(?:\d[ -]?){12,18}\d\b")),
    ("PHONE", re.compile(r"(?<![\w-])\+?\(?\d{1,4}\)?(?:[ .-]?\(?\d{2,4}\)?){2,4}(?![\w-])")),
]


def add_pii_pattern(kind: str, pattern: str, flags: int = 0, first: bool = False) -> None:
    """Register a custom PII kind: matches become ``[REDACTED_<KIND>]`` (appended to the list, or
    checked before the built-in kinds with ``first``)."""
    entry = (kind.upper(), re.compile(pattern, flags))
    if first:
        PII_PATTERNS.insert(0, entry)
    else:
        PII_PATTERNS.append(entry)


def redact_pii(text: str) -> Tuple[str, int]:
    """Replace AWS access keys, API-key assignments, e-mail addresses, IPv4 addresses, US social
    security numbers, card numbers and phone numbers (in that order, so a card number is not taken
    for a phone number) by ``[REDACTED_<KIND>]``; returns the text and the number of replacements."""
    n = 0
    for kind, rx in PII_PATTERNS:
        def sub(m, kind=kind):
            nonlocal n
            if kind == "PHONE" and sum(c.isdigit() for c in m.group(0)) < 10:
                return m.group(0)  # short digit runs (years, counts) are not phone numbers
            n += 1
            return f"[REDACTED_{kind}]"
        text = rx.sub(sub, text)
    return text, n


class UnsafeContent(ValueError):
    pass


@dataclass
class ContentSafety:
    blocked_keywords: List[str] = field(default_factory=list)
    blocked_patterns: List[str] = field(default_factory=list)

    def __post_init__(self):
        self._rx = [re.compile(p, re.IGNORECASE) for p in self.blocked_patterns]

    def check(self, text: str) -> None:
        low = text.lower()
        for k in self.blocked_keywords:
            if k and k.lower() in low:
                raise UnsafeContent(f"content contains blocked keyword: {k}")
        for rx in self._rx:
            if rx.search(text):
                raise UnsafeContent(f"content matches blocked pattern: {rx.pattern}")


_REASONING = re.compile(r"<(think|reasoning)>(.*?)(?:</\1>|$)", re.DOTALL)


def split_reasoning(text: str) -> Tuple[Optional[str], str]:
    """(reasoning, answer): the contents of ``<think>`` / ``<reasoning>`` blocks (an unterminated
    block runs to the end) and the text without them."""
    parts = [m.group(2).strip() for m in _REASONING.finditer(text)]
    if not parts:
        return None, text
    return "\n\n".join(p for p in parts if p), _REASONING.sub("", text).strip()


class SemanticCache:
    """Responses keyed by (request options, prompt embedding); a lookup returns the most similar
    entry with cosine >= ``threshold`` under the same options, entries expire after ``ttl_s`` and the
    least recently used one is dropped beyond ``max_size``."""

    def __init__(self, threshold: float = 0.85, max_size: int = 1024, ttl_s: float = 3600.0):
        self.threshold, self.max_size, self.ttl_s = threshold, max_size, ttl_s
        self._entries: "OrderedDict[int, Tuple[str, np.ndarray, dict, float]]" = OrderedDict()
        self._next = 0
        self._lock = threading.Lock()
        self.hits = self.misses = 0

    def lookup(self, key: str, vec: List[float]) -> Optional[dict]:
        q = np.asarray(vec, dtype=np.float32)
        q = q / max(float(np.linalg.norm(q)), 1e-12)
        now = time.time()
        with self._lock:
            best, best_sim = None, self.threshold
            for i, (k, v, resp, t) in list(self._entries.items()):
                if now - t > self.ttl_s:
                    del self._entries[i]
                    continue
                if k == key:
                    sim = float(v @ q)
                    if sim >= best_sim:
                        best, best_sim = i, sim
            if best is None:
                self.misses += 1
                return None
            self._entries.move_to_end(best)
            self.hits += 1
            return dict(self._entries[best][2], similarity=best_sim)

    def store(self, key: str, vec: List[float], response: dict) -> None:
        v = np.asarray(vec, dtype=np.float32)
        v = v / max(float(np.linalg.norm(v)), 1e-12)
        with self._lock:
            self._entries[self._next] = (key, v, response, time.time())
            self._next += 1
            while len(self._entries) > self.max_size:
                self._entries.popitem(last=False)


@dataclass
class ServerPlugins:
    pii_redaction: bool = False
    safety: Optional[ContentSafety] = None
    semantic_cache: Optional[SemanticCache] = None
    reasoning_split: bool = True

    @staticmethod
    def from_env() -> "ServerPlugins":
        e = os.environ
        kw = [k.strip() for k in e.get("GOLLEK_BLOCKED_KEYWORDS", "").split(",") if k.strip()]
        pats = [p for p in e.get("GOLLEK_BLOCKED_PATTERNS", "").split("\n") if p.strip()]
        sc = e.get("GOLLEK_SEMANTIC_CACHE")
        return ServerPlugins(pii_redaction=e.get("GOLLEK_PII_REDACTION", "0") not in ("0", "", "false"),
                             safety=ContentSafety(kw, pats) if (kw or pats) else None,
                             semantic_cache=SemanticCache(float(sc)) if sc else None)

    def configure(self, d: Dict) -> None:
        if "pii_redaction" in d:
            self.pii_redaction = bool(d["pii_redaction"])
        if "blocked_keywords" in d or "blocked_patterns" in d:
            kw, pats = d.get("blocked_keywords") or [], d.get("blocked_patterns") or []
            self.safety = ContentSafety(list(kw), list(pats)) if (kw or pats) else None
        if "semantic_cache" in d:
            c = d["semantic_cache"]
            self.semantic_cache = None if not c else SemanticCache(
                float(c.get("threshold", 0.85)), int(c.get("max_size", 1024)), float(c.get("ttl_s", 3600.0)))
        if "reasoning_split" in d:
            self.reasoning_split = bool(d["reasoning_split"])

    def describe(self) -> Dict:
        sc = self.semantic_cache
        return {"pii_redaction": self.pii_redaction, "reasoning_split": self.reasoning_split,
                "blocked_keywords": self.safety.blocked_keywords if self.safety else [],
                "blocked_patterns": self.safety.blocked_patterns if self.safety else [],
                "semantic_cache": None if sc is None else {"threshold": sc.threshold, "max_size": sc.max_size,
                                                           "ttl_s": sc.ttl_s, "hits": sc.hits, "misses": sc.misses}}

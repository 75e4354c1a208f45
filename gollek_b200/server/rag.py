"""Retrieval-augmented generation: documents are chunked, embedded with the served model and kept
in named collections; a question retrieves its most similar chunks, which go into the prompt as
cited context blocks.

Reference behaviour: the REST surface of runner/safetensor/gollek-safetensor-api/…/api/
RagResource.java:28-283 (``/v1/rag/ingest``, ``/v1/rag/query``, ``/v1/rag/collections[/{name}]``,
answer + ``context_used`` + ``sources`` of ``source_id`` / ``excerpt`` / ``similarity``) and the
pipeline of inference/gollek-runtime-inference/…/rag/RAGPipeline.java:140-330 (embed the query,
top-K search, optional rerank down to top-N, ``[Source: id]`` context blocks cut to a token budget,
template fill). The reference stores vectors in Qdrant; here a collection is a matrix of unit-norm
embeddings on the host (cosine similarity is one matrix-vector product), saved to and loaded from
an ``.npz`` file.
"""
from __future__ import annotations

import json
import threading
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

import numpy as np

DEFAULT_TEMPLATE = ("Answer the question using the context below. Cite sources by their id when you use "
                    "them. If the context does not contain the answer, say so.\n\nContext:\n{context}")


def chunk_text(text: str, chunk_chars: int = 800, overlap: int = 100) -> List[str]:
    """Split ``text`` into pieces of at most ``chunk_chars`` characters that overlap by about
    ``overlap`` characters, cutting at whitespace where one is near the limit."""
    text = " ".join(text.split())
    if chunk_chars <= 0:
        raise ValueError("chunk size must be positive")
    overlap = max(0, min(overlap, chunk_chars // 2))
    out, i, n = [], 0, len(text)
    while i < n:
        end = min(n, i + chunk_chars)
        if end < n:
            cut = text.rfind(" ", i + chunk_chars // 2, end)
            if cut > i:
                end = cut
        piece = text[i:end].strip()
        if piece:
            out.append(piece)
        if end >= n:
            break
        i = max(end - overlap, i + 1)
        while 0 < i < n and text[i - 1] != " " and text[i] != " " and i < end:
            i += 1  # start the next chunk at a word boundary inside the overlap
    return out


@dataclass
class Hit:
    source_id: str
    text: str
    similarity: float

    def source(self, excerpt_chars: int = 200) -> dict:
        return {"source_id": self.source_id, "excerpt": self.text[:excerpt_chars], "similarity": self.similarity}


@dataclass
class Collection:
    name: str
    dim: int = 0
    source_ids: List[str] = field(default_factory=list)
    texts: List[str] = field(default_factory=list)
    vecs: np.ndarray = field(default_factory=lambda: np.zeros((0, 0), np.float32))

    def __len__(self) -> int:
        return len(self.texts)

    def add(self, source_id: str, chunks: Sequence[str], vecs: np.ndarray) -> None:
        v = np.asarray(vecs, dtype=np.float32)
        if v.ndim != 2 or v.shape[0] != len(chunks):
            raise ValueError("one embedding per chunk expected")
        if self.dim and v.shape[1] != self.dim:
            raise ValueError(f"collection {self.name!r} holds {self.dim}-d embeddings, got {v.shape[1]}-d")
        v = v / np.maximum(np.linalg.norm(v, axis=1, keepdims=True), 1e-12)
        self.dim = v.shape[1]
        self.vecs = v if len(self.vecs) == 0 else np.concatenate([self.vecs, v], 0)
        self.source_ids.extend([source_id] * len(chunks))
        self.texts.extend(chunks)

    def search(self, query_vec: Sequence[float], top_k: int, min_similarity: float = -1.0) -> List[Hit]:
        if len(self) == 0 or top_k <= 0:
            return []
        q = np.asarray(query_vec, dtype=np.float32)
        q = q / max(float(np.linalg.norm(q)), 1e-12)
        sims = self.vecs @ q
        k = min(top_k, len(sims))
        idx = np.argpartition(-sims, k - 1)[:k]
        idx = idx[np.lexsort((idx, -sims[idx]))]  # by similarity, ties to the earlier chunk
        return [Hit(self.source_ids[i], self.texts[i], float(sims[i])) for i in idx if sims[i] >= min_similarity]


class RagStore:
    """Named collections (thread-safe for the server's worker threads)."""

    def __init__(self):
        self.collections: Dict[str, Collection] = {}
        self._lock = threading.Lock()

    def get(self, name: str, create: bool = False) -> Optional[Collection]:
        with self._lock:
            c = self.collections.get(name)
            if c is None and create:
                c = self.collections[name] = Collection(name)
            return c

    def drop(self, name: str) -> bool:
        with self._lock:
            return self.collections.pop(name, None) is not None

    def save(self, path: str) -> None:
        with self._lock:
            meta = {n: {"dim": c.dim, "source_ids": c.source_ids, "texts": c.texts} for n, c in self.collections.items()}
            arrays = {f"v{i}": c.vecs for i, c in enumerate(self.collections.values())}
        np.savez(path, meta=np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8), **arrays)

    @staticmethod
    def load(path: str) -> "RagStore":
        z = np.load(path)
        meta = json.loads(bytes(z["meta"]).decode())
        st = RagStore()
        for i, (n, m) in enumerate(meta.items()):
            st.collections[n] = Collection(n, m["dim"], list(m["source_ids"]), list(m["texts"]), z[f"v{i}"])
        return st


def build_context(hits: Sequence[Hit], max_context_tokens: int, count_tokens: Callable[[str], int]) -> str:
    """``[Source: id]`` blocks in similarity order, cut at whole blocks (or inside the first one)
    to ``max_context_tokens``."""
    blocks, used = [], 0
    for h in hits:
        b = f"[Source: {h.source_id}]\n{h.text}"
        n = count_tokens(b)
        if used + n > max_context_tokens:
            if not blocks:  # keep a cut first block rather than no context at all
                words = b.split(" ")
                while words and count_tokens(" ".join(words)) > max_context_tokens:
                    words = words[: max(1, len(words) * 3 // 4)] if len(words) > 1 else []
                if words:
                    blocks.append(" ".join(words))
            break
        blocks.append(b)
        used += n
    return "\n\n".join(blocks)


def augment_messages(messages: List[dict], context: str, template: str = DEFAULT_TEMPLATE) -> List[dict]:
    """The conversation with the retrieved context as a system message in front (merged into an
    existing leading system message)."""
    sys_text = template.format(context=context)
    msgs = [dict(m) for m in messages]
    if msgs and msgs[0].get("role") == "system":
        msgs[0]["content"] = f"{msgs[0].get('content') or ''}\n\n{sys_text}".strip()
    else:
        msgs.insert(0, {"role": "system", "content": sys_text})
    return msgs


def last_user_text(messages: List[dict]) -> str:
    for m in reversed(messages):
        if m.get("role") == "user":
            c = m.get("content")
            if isinstance(c, list):  # OpenAI content parts
                return " ".join(p.get("text", "") for p in c if isinstance(p, dict))
            return str(c or "")
    return ""

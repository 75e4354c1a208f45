"""Retrieval-augmented generation: chunking, cosine retrieval, context budget, persistence, and the
/v1/rag REST surface plus the chat-completions ``rag`` option over a served tiny model (whose
embeddings are mean-pooled hidden states: an exact-text query must retrieve its own chunk)."""
import numpy as np
import pytest

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.models.reference import init_random_weights
from gollek_b200.server.rag import (Collection, Hit, RagStore, augment_messages, build_context, chunk_text,
                                    last_user_text)
from gollek_b200.utils.tokenizer import ByteTokenizer


def test_chunk_text_covers_with_overlap():
    words = [f"w{i:03d}" for i in range(400)]
    text = " ".join(words)
    chunks = chunk_text(text, chunk_chars=200, overlap=40)
    assert all(len(c) <= 200 for c in chunks) and len(chunks) > 5
    seen = set(" ".join(chunks).split())
    assert seen == set(words)  # every word lands in some chunk, none is cut
    for a, b in zip(chunks, chunks[1:]):  # consecutive chunks share words
        assert set(a.split()) & set(b.split())
    assert chunk_text("short text", 100) == ["short text"]
    with pytest.raises(ValueError):
        chunk_text("x", 0)


def test_collection_search_order_and_persistence(tmp_path):
    c = Collection("c")
    c.add("a", ["alpha", "beta"], np.array([[1.0, 0.0, 0.0], [0.6, 0.8, 0.0]]))
    c.add("b", ["gamma"], np.array([[0.0, 0.0, 2.0]]))
    hits = c.search([1.0, 0.1, 0.0], top_k=2)
    assert [h.text for h in hits] == ["alpha", "beta"]
    assert hits[0].similarity == pytest.approx(1 / np.sqrt(1.01), rel=1e-5)
    assert [h.text for h in c.search([0, 0, 1], 5, min_similarity=0.5)] == ["gamma"]
    with pytest.raises(ValueError):
        c.add("x", ["bad"], np.ones((1, 4)))
    st = RagStore()
    st.collections["c"] = c
    st.save(str(tmp_path / "rag.npz"))
    back = RagStore.load(str(tmp_path / "rag.npz"))
    assert back.get("c").texts == c.texts and np.allclose(back.get("c").vecs, c.vecs)


def test_context_budget_and_messages():
    hits = [Hit("d1", "one two three four", 0.9), Hit("d2", "five six seven eight", 0.8)]
    count = lambda s: len(s.split())  # noqa: E731
    full = build_context(hits, 100, count)
    assert full.index("[Source: d1]") < full.index("[Source: d2]")
    only_first = build_context(hits, 7, count)
    assert "d1" in only_first and "d2" not in only_first
    assert count(build_context(hits, 3, count)) <= 3  # a cut first block
    msgs = augment_messages([{"role": "system", "content": "Be brief."}, {"role": "user", "content": "q?"}], "CTX")
    assert len(msgs) == 2 and msgs[0]["content"].startswith("Be brief.") and "CTX" in msgs[0]["content"]
    assert augment_messages([{"role": "user", "content": "q"}], "CTX")[0]["role"] == "system"
    assert last_user_text([{"role": "user", "content": [{"type": "text", "text": "hi"}]}]) == "hi"


def _engine():
    cfg = preset("tiny-llama")
    w = init_random_weights(cfg, seed=0)
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=256, max_model_len=1024,
                      use_cuda_graphs=False)
    return LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=192,
                     tokenizer=ByteTokenizer(cfg.vocab_size, cfg.eos_token_id))


def test_rag_api_ingest_query_chat_drop():
    from fastapi.testclient import TestClient

    from gollek_b200.server.app import create_app
    from gollek_b200.server.async_engine import AsyncEngine
    docs = [{"id": "paris", "content": "Paris is the capital of France and sits on the Seine."},
            {"id": "oslo", "content": "Oslo is the capital of Norway, at the head of the Oslofjord."},
            {"id": "lima", "content": "Lima is the capital of Peru, on the Pacific coast."}]
    ae = AsyncEngine(_engine()).start()
    try:
        with TestClient(create_app(ae)) as c:
            r = c.post("/v1/rag/ingest", json={"collection": "geo", "documents": docs})
            assert r.json() == {"collection": "geo", "chunks": 3, "status": "indexed"}
            assert c.get("/v1/rag/collections").json() == {"collections": [{"name": "geo", "chunks": 3}]}
            q = c.post("/v1/rag/query", json={"collection": "geo", "question": docs[1]["content"], "topK": 2,
                                              "maxTokens": 4, "temperature": 0.0}).json()
            assert q["context_used"] is True and len(q["sources"]) == 2
            assert q["sources"][0]["source_id"] == "oslo" and q["sources"][0]["similarity"] > 0.999
            assert isinstance(q["answer"], str)
            base = {"messages": [{"role": "user", "content": docs[2]["content"]}], "max_tokens": 2,
                    "temperature": 0.0}
            plain = c.post("/v1/chat/completions", json=base).json()
            aug = c.post("/v1/chat/completions", json={**base, "rag": {"collection": "geo", "top_k": 1}}).json()
            assert aug["rag_sources"][0]["source_id"] == "lima"
            assert aug["usage"]["prompt_tokens"] > plain["usage"]["prompt_tokens"] + len(docs[2]["content"])
            assert c.delete("/v1/rag/collections/geo").status_code == 204
            assert c.post("/v1/rag/query", json={"collection": "geo", "question": "x"}).status_code == 404
            assert c.get("/v1/rag/collections/geo").status_code == 404
    finally:
        ae.shutdown()

"""KV eviction (EVICPRESS-style): native block drop + batch metadata, the scoring / protection /
retention policy, decoding over evicted KV against a masked fp32 oracle, and the REST routes."""
import pytest
import torch

from gollek_b200 import ops
from gollek_b200.config import EngineConfig
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.evicpress import KVEvictor
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.models.reference import ReferenceDecoder
from gollek_b200.native import host_ext
from gollek_b200.utils.tokenizer import ByteTokenizer


def test_seqtables_drop_and_batch():
    h = host_ext()
    pool = h.BlockPool(32, 4)
    t = h.SeqTables(pool)
    t.add(7)
    assert t.ensure_capacity(7, 18)                 # 5 blocks of 4
    blocks = t.blocks(7)
    assert t.drop(7, [1, 2]) == 2 and t.dropped(7) == 8
    assert t.blocks(7) == [blocks[0], blocks[3], blocks[4]]
    assert pool.num_free() == 32 - 3
    with pytest.raises(Exception):
        t.drop(7, [2])                               # the last block stays
    # position 18 (the 19th token): KV index 10 -> third kept block, offset 2
    pos = torch.zeros(4, dtype=torch.int32)
    slots = torch.zeros(4, dtype=torch.int32)
    bt = torch.zeros(1, 8, dtype=torch.int32)
    lens = torch.zeros(1, dtype=torch.int32)
    qs = torch.zeros(2, dtype=torch.int32)
    n = t.build_batch(torch.tensor([7]), torch.tensor([18], dtype=torch.int32), torch.tensor([1], dtype=torch.int32),
                      pos, slots, bt, lens, qs)
    assert n == 1 and int(pos[0]) == 18 and int(lens[0]) == 11
    assert int(slots[0]) == blocks[4] * 4 + 2
    assert t.blocks_needed(7, 20) == 0 and t.blocks_needed(7, 21) == 1   # 20 - 8 tokens fit in 3 blocks
    t.remove(7)
    assert pool.num_free() == 32


def test_policy_protect_and_retention():
    ev = KVEvictor(retention_target=0.5, sink_blocks=1, recent=0.2)
    assert ev.protect_mask(10) == [True] + [False] * 7 + [True, True]
    norms = torch.tensor([1.0, 9.0, 1.0, 8.0, 2.0, 7.0, 3.0, 6.0, 5.0, 5.0])
    drop = ev.plan(norms)
    assert len(drop) == 5 and 0 not in drop and 8 not in drop and 9 not in drop
    # high key norm and old -> least important
    assert 1 in drop and 3 in drop
    assert KVEvictor(retention_target=1.0).plan(norms) == []
    with pytest.raises(ValueError):
        KVEvictor(retention_target=0.0)


def test_key_norms_cpu():
    cache = torch.randn(2, 6, 2, 3, 4, 8)
    ids = torch.tensor([5, 1, 2], dtype=torch.int32)
    got = ops.kv_key_norms(cache, ids)
    want = torch.stack([cache[:, b, 0].norm(dim=-1).mean() for b in (5, 1, 2)])
    torch.testing.assert_close(got, want)


def _engine(cfg, weights, **kw):
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=512, max_model_len=512,
                      use_cuda_graphs=False, async_scheduling=False, kv_eviction=True, kv_eviction_threshold=1.1,
                      kv_retention_target=0.6, kv_eviction_min_blocks=4, **kw)
    return LLMEngine(ec, model_cfg=cfg, weights=weights.__getitem__, num_blocks=128,
                     tokenizer=ByteTokenizer(cfg.vocab_size, cfg.eos_token_id))


def test_decode_over_evicted_kv_matches_masked_oracle(tiny_cfg, tiny_weights):
    eng = _engine(tiny_cfg, tiny_weights)
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(3, 250, (200,), generator=g).tolist()
    eng.add_request("r", prompt, SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True))
    eng.step()                                       # prefill + first token
    seq = eng.seqs["r"]
    before = eng.kv.tables.blocks(seq.seq_id)
    freed = eng.evictor.run(eng, force=True)
    after = eng.kv.tables.blocks(seq.seq_id)
    assert freed == len(before) - len(after) > 0 and eng.kv.dropped_tokens(seq) == 16 * freed
    dropped_idx = [i for i, b in enumerate(before) if b not in after]
    out = None
    while eng.has_unfinished():
        for o in eng.step():
            if o.finished:
                out = o
    toks = prompt + list(out.output_token_ids)
    S = len(toks)
    key_mask = torch.ones(S, S, dtype=torch.bool)
    gone = [p for i in dropped_idx for p in range(16 * i, 16 * i + 16)]
    key_mask[len(prompt):, gone] = False             # queries after the eviction do not see those keys
    logits = ReferenceDecoder(tiny_cfg, tiny_weights).forward(torch.tensor(toks), key_mask)
    want = logits[len(prompt) - 1: S - 1].argmax(-1).tolist()
    assert list(out.output_token_ids) == want
    assert eng.evictor.stats.blocks_dropped == freed


def test_eviction_guards_and_routes(tiny_cfg, tiny_weights):
    from fastapi.testclient import TestClient

    from gollek_b200.server.app import create_app
    from gollek_b200.server.async_engine import AsyncEngine
    with pytest.raises(ValueError):
        _engine(tiny_cfg, tiny_weights, tensor_parallel_size=2)
    ae = AsyncEngine(_engine(tiny_cfg, tiny_weights)).start()
    try:
        with TestClient(create_app(ae)) as c:
            s = c.get("/v1/kvcache/stats").json()
            assert s["eviction_enabled"] and s["retention_target"] == 0.6
            assert c.put("/v1/kvcache/retention", params={"target": 0.5}).json() == {"previous": 0.6, "current": 0.5}
            assert c.put("/v1/kvcache/retention", params={"target": 1.5}).status_code == 400
            assert c.post("/v1/kvcache/evict-now").json()["blocks_dropped"] == 0   # nothing running
    finally:
        ae.shutdown(drain=False)

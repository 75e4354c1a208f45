"""Checkpoint / resume: prefix-cache snapshots reload into a fresh engine (prefix hits, identical
outputs), mismatched snapshots are refused, and drained requests resume after a restart."""
import pytest
import torch

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.models.reference import ReferenceDecoder, init_random_weights


def _engine(cfg, w, device="cpu", **kw):
    ec = EngineConfig(model="tiny", device=device, dtype="float32" if device == "cpu" else "bfloat16",
                      block_size=16, max_num_seqs=8, max_num_batched_tokens=64, max_model_len=256,
                      use_cuda_graphs=False, **kw)
    return LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64)


def test_prefix_cache_snapshot_roundtrip(tiny_cfg, tiny_weights, tmp_path):
    g = torch.Generator().manual_seed(31)
    shared = torch.randint(0, tiny_cfg.vocab_size, (50,), generator=g).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True)
    a = _engine(tiny_cfg, tiny_weights)
    a.generate([shared + [1, 2]], sp)
    path = str(tmp_path / "prefix.safetensors")
    n = a.save_prefix_cache(path)
    assert n >= 3
    b = _engine(tiny_cfg, tiny_weights)
    assert b.load_prefix_cache(path) == n
    hits0 = b.kv.prefix_hits
    out = b.generate([shared + [9]], sp)[0]
    assert b.kv.prefix_hits - hits0 >= 3
    ref = ReferenceDecoder(tiny_cfg, tiny_weights)
    assert out.output_token_ids == ref.greedy(shared + [9], 5)[0]


def test_prefix_snapshot_signature_checked(tiny_cfg, tiny_weights, tmp_path):
    a = _engine(tiny_cfg, tiny_weights)
    a.generate([list(range(40))], SamplingParams(temperature=0.0, max_tokens=2, ignore_eos=True))
    path = str(tmp_path / "p.safetensors")
    a.save_prefix_cache(path)
    other = preset("tiny-llama", num_hidden_layers=2)
    b = _engine(other, init_random_weights(other, seed=1))
    with pytest.raises(ValueError, match="snapshot was written for"):
        b.load_prefix_cache(path)


def test_drain_and_restart_resumes_requests(tiny_cfg, tiny_weights):
    g = torch.Generator().manual_seed(32)
    prompts = [torch.randint(0, tiny_cfg.vocab_size, (n,), generator=g).tolist() for n in (12, 30)]
    ref = ReferenceDecoder(tiny_cfg, tiny_weights)
    expect = [ref.greedy(p, 10)[0] for p in prompts]
    a = _engine(tiny_cfg, tiny_weights)
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True)
    for i, p in enumerate(prompts):
        a.add_request(f"r{i}", p, SamplingParams(**vars(sp)))
    for _ in range(4):  # partway through
        a.step()
    snap = a.snapshot_requests()
    done = {r["request_id"]: r["output_token_ids"] for r in snap}
    assert snap and all(len(v) < 10 for v in done.values())
    b = _engine(tiny_cfg, tiny_weights)  # "restarted" process
    b.restore_requests(snap)
    final = {}
    while b.has_unfinished():
        for o in b.step():
            if o.finished:
                final[o.request_id] = done[o.request_id] + o.output_token_ids
    assert [final[f"r{i}"] for i in range(2)] == expect


@pytest.mark.gpu
def test_prefix_cache_snapshot_gpu(tiny_cfg, tiny_weights, tmp_path):
    g = torch.Generator().manual_seed(33)
    shared = torch.randint(0, tiny_cfg.vocab_size, (64,), generator=g).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True)
    a = _engine(tiny_cfg, tiny_weights, device="cuda")
    first = a.generate([shared + [3]], sp)[0]
    path = str(tmp_path / "g.safetensors")
    n = a.save_prefix_cache(path)
    b = _engine(tiny_cfg, tiny_weights, device="cuda")
    assert b.load_prefix_cache(path) == n
    hits0 = b.kv.prefix_hits
    again = b.generate([shared + [3]], sp)[0]
    assert b.kv.prefix_hits - hits0 >= 4
    assert again.output_token_ids == first.output_token_ids


def test_prefix_cache_snapshot_turboquant(tiny_cfg, tiny_weights, tmp_path):
    """A prefix snapshot compressed with TurboQuant (2.5 bits per KV value): much smaller than the
    plain one, reloads as prefix hits, and the restored blocks stay close to the computed ones."""
    import os
    g = torch.Generator().manual_seed(32)
    shared = torch.randint(0, tiny_cfg.vocab_size, (64,), generator=g).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True)
    a = _engine(tiny_cfg, tiny_weights)
    a.generate([shared + [1, 2]], sp)
    plain, small = str(tmp_path / "plain.safetensors"), str(tmp_path / "tq.safetensors")
    n = a.save_prefix_cache(plain)
    assert a.save_prefix_cache(small, compress="turboquant") == n >= 3
    assert os.path.getsize(small) < os.path.getsize(plain) / 5  # fp32 cache here: ~12x less
    b = _engine(tiny_cfg, tiny_weights)
    assert b.load_prefix_cache(small) == n
    from gollek_b200 import ops
    ha = dict(a.kv.pool.cached_items())
    hb = dict(b.kv.pool.cached_items())
    common = [h for h in ha if h in hb]
    assert len(common) == n
    ka = ops.kv_gather_blocks(a.kv_cache, torch.tensor([ha[h] for h in common], dtype=torch.int32))
    kb = ops.kv_gather_blocks(b.kv_cache, torch.tensor([hb[h] for h in common], dtype=torch.int32))
    # 2.5 bits per value; this toy model's head_dim of 32 leaves more error than 128 does (0.2)
    assert float((ka - kb).norm() / ka.norm()) < 0.3
    hits0 = b.kv.prefix_hits
    out = b.generate([shared + [9]], sp)[0]
    assert b.kv.prefix_hits - hits0 >= 3 and len(out.output_token_ids) == 3

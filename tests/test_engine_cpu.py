"""The serving engine on CPU (plain-PyTorch op path) against the dense oracle.

Tiny Llama (4 layers, d 256, 8/2 heads, hd 32, ffn 688, vocab 32000, seed 0), prompt of 32 ids,
32 greedy tokens through the paged KV cache with block size 16.
"""
import torch

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.models.reference import ReferenceDecoder, init_random_weights


def _engine(cfg, weights, **kw):
    ec = EngineConfig(device="cpu", dtype="float32", block_size=16, max_num_seqs=8,
                      max_num_batched_tokens=kw.pop("budget", 64), max_model_len=256, use_cuda_graphs=False, **kw)
    return LLMEngine(ec, model_cfg=cfg, weights=weights.__getitem__, num_blocks=64)


def test_greedy_matches_oracle(tiny_cfg, tiny_weights):
    prompt = torch.randint(0, tiny_cfg.vocab_size, (32,), generator=torch.Generator().manual_seed(0)).tolist()
    ref_tokens, ref_logits = ReferenceDecoder(tiny_cfg, tiny_weights).greedy(prompt, 32)
    eng = _engine(tiny_cfg, tiny_weights)
    out = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=32, ignore_eos=True))[0]
    assert out.output_token_ids == ref_tokens
    assert out.finish_reason == "length"


def test_chunked_prefill_and_batching(tiny_cfg, tiny_weights):
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, tiny_cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 40, 17, 70)]
    ref = ReferenceDecoder(tiny_cfg, tiny_weights)
    expect = [ref.greedy(p, 6)[0] for p in prompts]
    eng = _engine(tiny_cfg, tiny_weights, budget=24)  # forces multi-step chunked prefill
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
    assert [o.output_token_ids for o in outs] == expect


def test_prefix_cache_reuse(tiny_cfg, tiny_weights):
    g = torch.Generator().manual_seed(4)
    shared = torch.randint(0, tiny_cfg.vocab_size, (48,), generator=g).tolist()
    p1 = shared + [1, 2, 3]
    p2 = shared + [7, 8]
    ref = ReferenceDecoder(tiny_cfg, tiny_weights)
    eng = _engine(tiny_cfg, tiny_weights)
    sp = SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True)
    o1 = eng.generate([p1], sp)[0]
    hits0 = eng.kv.prefix_hits
    o2 = eng.generate([p2], sp)[0]
    assert eng.kv.prefix_hits - hits0 >= 3  # 48 shared tokens = 3 full blocks
    assert o1.output_token_ids == ref.greedy(p1, 4)[0]
    assert o2.output_token_ids == ref.greedy(p2, 4)[0]


def test_preemption_recompute(tiny_cfg, tiny_weights):
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, tiny_cfg.vocab_size, (30,), generator=g).tolist() for _ in range(4)]
    ref = ReferenceDecoder(tiny_cfg, tiny_weights)
    expect = [ref.greedy(p, 20)[0] for p in prompts]
    ec = EngineConfig(device="cpu", dtype="float32", block_size=16, max_num_seqs=4, max_num_batched_tokens=128,
                      max_model_len=128, use_cuda_graphs=False, enable_prefix_caching=False)
    eng = LLMEngine(ec, model_cfg=tiny_cfg, weights=tiny_weights.__getitem__, num_blocks=9)  # too few for all
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=20, ignore_eos=True))
    assert eng.scheduler.num_preemptions > 0
    assert [o.output_token_ids for o in outs] == expect


def test_sampling_seeded_reproducible(tiny_cfg, tiny_weights):
    prompt = list(range(10, 30))
    eng = _engine(tiny_cfg, tiny_weights)
    sp = SamplingParams(temperature=0.8, top_k=50, top_p=0.9, max_tokens=8, seed=123, ignore_eos=True)
    a = eng.generate([prompt], sp)[0].output_token_ids
    b = eng.generate([prompt], sp)[0].output_token_ids
    assert a == b and len(a) == 8


def test_mixtral_engine_matches_oracle():
    cfg = preset("tiny-mixtral")
    w = init_random_weights(cfg, seed=2)
    prompt = torch.randint(0, cfg.vocab_size, (20,), generator=torch.Generator().manual_seed(2)).tolist()
    ref_tokens, _ = ReferenceDecoder(cfg, w).greedy(prompt, 8)
    eng = _engine(cfg, w)
    out = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))[0]
    assert out.output_token_ids == ref_tokens

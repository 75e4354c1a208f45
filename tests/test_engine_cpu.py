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


def test_prefill_schedule_forms_cover_every_tile_once():
    """The prefill work list covers every (head, 128-row query tile) exactly once in both forms,
    heaviest items first; row-tile pairs are consecutive tiles; head pairs are the default when the
    GQA group size is even."""
    from gollek_b200 import ops
    qs, lens = [0, 300, 560, 561, 690, 1330], [300, 1260, 8, 329, 640]
    for H, Hk in ((32, 8), (28, 4), (12, 4)):
        for form in (None, "rows", "pairs"):
            if form == "pairs" and (H // Hk) % 2:
                continue
            w = ops.prefill_schedule(qs, lens, H, Hk, 128, form=form)
            seen = []
            costs = []
            for b, o0, o1, code in w.tolist():
                pair, h = code >> 16, code & 0xFFFF
                ctx0 = lens[b] - (qs[b + 1] - qs[b])
                c = lambda o: (min(lens[b], ctx0 + o + 128) + 127) // 128  # noqa: E731
                if pair:
                    assert o0 == o1 and h % 2 == 0
                    seen += [(b, o0, h), (b, o0, h + 1)]
                    costs.append(2 * c(o0))
                else:
                    seen.append((b, o0, h))
                    costs.append(max(c(o0), c(o1) if o1 >= 0 else 0))
                    if o1 >= 0:
                        assert o1 == o0 + 128
                        seen.append((b, o1, h))
            want = [(b, o, h) for b in range(5) for o in range(0, qs[b + 1] - qs[b], 128) for h in range(H)]
            assert sorted(seen) == sorted(want), (H, Hk, form)
            assert costs == sorted(costs, reverse=True)
    one = ops.prefill_schedule([0, 1088], [1088], 32, 8, 128, form="rows")
    assert (one[:, 3] >> 16 == 0).all() and one.shape[0] == 32 * 5
    assert sorted({(o0, o1) for _, o0, o1, _ in one.tolist()}) == [(0, 128), (256, 384), (512, 640), (768, 896),
                                                                 (1024, -1)]
    many = ops.prefill_schedule(list(range(0, 8 * 1024 + 1, 1024)), [1024] * 8, 32, 8, 128)
    assert (many[:, 3] >> 16 == 1).all() and many.shape[0] == 8 * 8 * 16

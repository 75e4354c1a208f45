"""Split batches: a step run as two halves (the tensor-parallel overlap path) gives the same
results as the unsplit forward — halves at sequence boundaries, inside a prefill sequence, inside
the decode rows — on the CPU engine (single process: the halves' collectives are local)."""
import torch

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams


def _engine(cfg, w, split: bool):
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=8, max_num_batched_tokens=96, max_model_len=256,
                      use_cuda_graphs=False, enable_prefix_caching=False)
    eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64)
    if split:
        eng.runner.split_min_tokens = 4
        eng.model.can_split_batch = lambda: True
    return eng


def test_split_forward_matches_unsplit(tiny_cfg, tiny_weights):
    g = torch.Generator().manual_seed(4)
    # prompts long enough that chunked prefill puts a sequence across the middle of a step, plus
    # several decodes next to the prefill chunks
    prompts = [torch.randint(0, tiny_cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 70, 33, 9, 120)]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True, logprobs=3)
    ref = _engine(tiny_cfg, tiny_weights, split=False).generate(prompts, sp)
    calls = []
    eng = _engine(tiny_cfg, tiny_weights, split=True)
    orig = eng.model._forward_split

    def spy(ids, meta, cache):
        calls.append((ids.shape[0], meta.halves[0], meta.halves[1].num_tokens, meta.halves[2].num_tokens))
        return orig(ids, meta, cache)

    eng.model._forward_split = spy
    got = eng.generate(prompts, sp)
    assert calls and all(a + b == T and t == a for T, t, a, b in calls)
    for r, o in zip(ref, got):
        assert r.output_token_ids == o.output_token_ids
        for lr, lo in zip(r.logprobs or [], o.logprobs or []):
            assert abs(lr["logprob"] - lo["logprob"]) < 1e-4


def test_half_metadata_cut_inside_a_prefill_sequence(tiny_cfg, tiny_weights):
    """A step of 3 decodes + one 40-token prefill chunk splits inside the chunk: the first half sees
    the sequence's KV up to the cut, the second half the rest with the full KV length."""
    eng = _engine(tiny_cfg, tiny_weights, split=True)
    g = torch.Generator().manual_seed(1)
    for i in range(3):
        eng.add_request(f"d{i}", torch.randint(0, 1000, (4,), generator=g).tolist(),
                        SamplingParams(temperature=0.0, max_tokens=20, ignore_eos=True))
    eng.step()  # the three short prompts prefilled; they decode from now on
    eng.add_request("p", torch.randint(0, 1000, (40,), generator=g).tolist(),
                    SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True))
    seen = []
    orig = eng.model._forward_split

    def spy(ids, meta, cache):
        seen.append(meta)
        return orig(ids, meta, cache)

    eng.model._forward_split = spy
    eng.step()
    meta = seen[-1]
    tA, mA, mB = meta.halves
    assert ids_total(meta) == 43 and tA == 21
    assert mA.num_decode == 3 and mA.num_prefill_tokens == 18 and mB.num_decode == 0 and mB.num_prefill_tokens == 22
    assert mA.prefill_seq_lens.tolist() == [18] and mB.prefill_seq_lens.tolist() == [40]
    assert mA.prefill_query_start.tolist() == [0, 18] and mB.prefill_query_start.tolist() == [0, 22]


def ids_total(meta):
    return meta.positions.shape[0]

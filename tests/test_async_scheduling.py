"""Async scheduling (host work of step N+1 overlapping step N) produces exactly the tokens of
synchronous scheduling: greedy and seeded sampling, EOS and stop tokens reached while the next
step is already in flight, max_tokens, aborts, preemption under KV pressure, prefix reuse."""
import pytest
import torch

from gollek_b200.config import EngineConfig
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams


def _engine(cfg, w, asyn, device="cpu", **kw):
    ec = EngineConfig(device=device, dtype="float32" if device == "cpu" else "bfloat16", block_size=16,
                      max_num_seqs=kw.pop("seqs", 8), max_num_batched_tokens=kw.pop("budget", 48), max_model_len=256,
                      use_cuda_graphs=device != "cpu", async_scheduling=asyn, **kw)
    return LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=kw.pop("nb", 96) if "nb" in kw else 96)


def _prompts(cfg, seed, lens=(5, 40, 17, 70, 9)):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]


def _run(eng, prompts, params):
    for i, (p, sp) in enumerate(zip(prompts, params)):
        eng.add_request(f"r{i}", p, sp)
    done = {}
    while eng.has_unfinished():
        for o in eng.step():
            if o.finished:
                done[o.request_id] = (list(o.output_token_ids), o.finish_reason)
    assert all(t >= 0 for v in done.values() for t in v[0])
    return [done[f"r{i}"] for i in range(len(prompts))]


@pytest.mark.parametrize("mode", ["greedy", "sampled"])
def test_async_equals_sync(tiny_cfg, tiny_weights, mode):
    prompts = _prompts(tiny_cfg, 1)
    if mode == "greedy":
        params = [SamplingParams(temperature=0.0, max_tokens=n, ignore_eos=True) for n in (1, 7, 12, 3, 9)]
    else:
        params = [SamplingParams(temperature=0.9, top_k=30, top_p=0.9, max_tokens=n, ignore_eos=True, seed=11 + i)
                  for i, n in enumerate((4, 8, 11, 2, 6))]
    a = _run(_engine(tiny_cfg, tiny_weights, True), prompts, params)
    b = _run(_engine(tiny_cfg, tiny_weights, False), prompts, [SamplingParams(**vars(p)) for p in params])
    assert a == b


def test_async_stop_tokens_in_flight(tiny_cfg, tiny_weights):
    """A stop token sampled at step N while step N+1 is already launched: the extra token is
    dropped and the sequence ends exactly where synchronous scheduling ends it."""
    prompts = _prompts(tiny_cfg, 2)
    ref = _run(_engine(tiny_cfg, tiny_weights, False), prompts,
               [SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True) for _ in prompts])
    stops = [toks[min(3, len(toks) - 1)] for toks, _ in ref]  # stop on the 4th token of each
    mk = lambda: [SamplingParams(temperature=0.0, max_tokens=12, stop_token_ids=[s]) for s in stops]  # noqa: E731
    a = _run(_engine(tiny_cfg, tiny_weights, True), prompts, mk())
    b = _run(_engine(tiny_cfg, tiny_weights, False), prompts, mk())
    assert a == b
    assert all(r == "stop" for _, r in a)


def test_async_abort_and_preemption(tiny_cfg, tiny_weights):
    prompts = _prompts(tiny_cfg, 3, lens=(60, 61, 62, 63))
    params = [SamplingParams(temperature=0.0, max_tokens=40, ignore_eos=True) for _ in prompts]
    outs = {}
    for asyn in (True, False):
        ec = EngineConfig(device="cpu", dtype="float32", block_size=16, max_num_seqs=4, max_num_batched_tokens=128,
                          max_model_len=256, use_cuda_graphs=False, async_scheduling=asyn)
        eng = LLMEngine(ec, model_cfg=tiny_cfg, weights=tiny_weights.__getitem__, num_blocks=20)  # forces preemption
        for i, (p, sp) in enumerate(zip(prompts, params)):
            eng.add_request(f"r{i}", p, SamplingParams(**vars(sp)))
        done, steps = {}, 0
        while eng.has_unfinished():
            for o in eng.step():
                if o.finished:
                    done[o.request_id] = list(o.output_token_ids)
            steps += 1
            if steps == 6:
                eng.abort_request("r1")
        outs[asyn] = done
        assert eng.scheduler.num_preemptions > 0
        assert eng.kv.num_free_blocks() == eng.num_blocks
    assert outs[True] == outs[False]


@pytest.mark.gpu
def test_async_equals_sync_gpu(tiny_cfg, tiny_weights):
    prompts = _prompts(tiny_cfg, 4)
    params = [SamplingParams(temperature=0.0, max_tokens=n, ignore_eos=True) for n in (2, 9, 16, 5, 12)]
    a = _run(_engine(tiny_cfg, tiny_weights, True, device="cuda"), prompts, params)
    b = _run(_engine(tiny_cfg, tiny_weights, False, device="cuda"), prompts,
             [SamplingParams(**vars(p)) for p in params])
    assert a == b

"""Hybrid gated-delta-rule / attention stacks (H1 / H2 schedules): the scan oracle's chunk and step
consistency, the serving engine (chunked prefill, decode, state slots) against the dense oracle, and
the schedules."""
import math

import pytest
import torch

from gollek_b200 import ops
from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.models.reference import ReferenceDecoder, init_random_weights
from gollek_b200.ops import reference as R
from gollek_b200.utils.tokenizer import ByteTokenizer


def _proj(T, Hg, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(T, (4 * Hg * 128 + 2 * Hg + 7) // 8 * 8, generator=g)   # rows padded to 16 bytes


def test_schedules():
    h1 = preset("tiny-llama", hybrid_schedule="H1", num_hidden_layers=12)
    h2 = preset("tiny-llama", hybrid_schedule="H2", num_hidden_layers=6)
    assert [h1.is_gdn_layer(i) for i in range(12)] == [True] * 4 + [False, True] * 1 + [True] * 4 + [False, True]
    assert [h2.is_gdn_layer(i) for i in range(6)] == [True, True, False, True, True, False]
    assert not preset("tiny-llama").is_gdn_layer(0)
    with pytest.raises(ValueError):
        preset("tiny-llama", hybrid_schedule="H9").is_gdn_layer(0)


def test_scan_chunks_equal_one_pass():
    Hg, T = 2, 40
    proj = _proj(T, Hg, 1)
    a_log, dt = torch.tensor([0.3, 1.2]), torch.tensor([0.1, -0.4])
    st1 = torch.zeros(1, Hg, 128, 128)
    o1 = R.gdn_scan(proj, st1, torch.tensor([0]), torch.tensor([1]), torch.tensor([0, T]), a_log, dt, Hg)
    st2 = torch.zeros(1, Hg, 128, 128)
    oa = R.gdn_scan(proj[:25], st2, torch.tensor([0]), torch.tensor([1]), torch.tensor([0, 25]), a_log, dt, Hg)
    ob = R.gdn_scan(proj[25:], st2, torch.tensor([0]), torch.tensor([0]), torch.tensor([0, T - 25]), a_log, dt, Hg)
    torch.testing.assert_close(torch.cat([oa, ob]), o1, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(st2, st1, rtol=1e-5, atol=1e-5)


def test_scan_matches_recurrence_definition():
    """One head, three tokens, written out from the delta-rule update."""
    Hg, T = 1, 3
    proj = _proj(T, Hg, 2)
    a_log, dt = torch.tensor([0.5]), torch.tensor([0.2])
    st = torch.zeros(1, 1, 128, 128)
    o = R.gdn_scan(proj, st, torch.tensor([0]), torch.tensor([1]), torch.tensor([0, T]), a_log, dt, Hg)
    silu = torch.nn.functional.silu
    S = torch.zeros(128, 128)
    for t in range(T):
        q = silu(proj[t, :128])
        q = q / q.norm() / math.sqrt(128)
        k = silu(proj[t, 128:256])
        k = k / k.norm()
        v = silu(proj[t, 256:384])
        alpha = math.exp(-math.exp(0.5) * math.log1p(math.exp(float(proj[t, 512]) + 0.2)))
        beta = 1 / (1 + math.exp(-float(proj[t, 513])))
        S = alpha * S
        S = S + torch.outer(k, beta * (v - S.t() @ k))
        torch.testing.assert_close(o[t, 0], S.t() @ q, rtol=1e-4, atol=1e-5)


def _engine(cfg, w, **kw):
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=512,
                      use_cuda_graphs=False, **kw)
    return LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=128,
                     tokenizer=ByteTokenizer(cfg.vocab_size, cfg.eos_token_id))


@pytest.mark.parametrize("schedule", ["H1", "H2"])
def test_engine_matches_oracle(schedule):
    cfg = preset("tiny-hybrid", hybrid_schedule=schedule)
    w = init_random_weights(cfg, seed=4)
    eng = _engine(cfg, w)
    assert eng.hybrid and not eng.cfg.enable_prefix_caching
    assert eng.model.num_gdn_layers == sum(cfg.is_gdn_layer(i) for i in range(cfg.num_hidden_layers))
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(3, 1000, (n,), generator=g).tolist() for n in (150, 9, 70)]   # chunked prefills
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
    ref = ReferenceDecoder(cfg, w)
    for p, o in zip(prompts, outs):
        want, _ = ref.greedy(p, 6)
        assert list(o.output_token_ids) == list(want)
    assert sorted(eng.kv.free_state_slots) == list(range(cfg_slots(eng)))


def cfg_slots(eng):
    return eng.cfg.max_num_seqs + 1


def test_hybrid_guards():
    cfg = preset("tiny-hybrid")
    w = init_random_weights(cfg, seed=0)
    with pytest.raises(ValueError):
        _engine(cfg, w, speculative_method="ngram")


@pytest.mark.gpu
def test_gdn_scan_kernel_matches_oracle():
    """K14 scan on the GPU: varlen sequences, state slots, reset vs carried state."""
    Hg, lens = 3, [1, 37, 70, 5]
    T = sum(lens)
    proj = _proj(T, Hg, 9).mul_(0.7)
    qs = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    slots = torch.tensor([2, 0, 3, 1], dtype=torch.int32)
    reset = torch.tensor([1, 0, 1, 0], dtype=torch.int32)
    g = torch.Generator().manual_seed(10)
    state = torch.randn(5, Hg, 128, 128, generator=g) * 0.1
    a_log, dt = torch.tensor([0.1, 0.9, 2.0]), torch.tensor([0.3, -0.2, 0.0])
    ref_state = state.clone()
    want = R.gdn_scan(proj.bfloat16().float(), ref_state, slots, reset, qs, a_log, dt, Hg)
    st = state.cuda()
    got = ops.gdn_scan(proj.bfloat16().cuda(), st, slots.cuda(), reset.cuda(), qs.cuda(), a_log.cuda(), dt.cuda(), Hg)
    torch.testing.assert_close(got.float().cpu(), want, rtol=2e-2, atol=2e-3)
    torch.testing.assert_close(st.cpu(), ref_state, rtol=1e-3, atol=1e-4)
    # gated head norm
    o = torch.randn(T, Hg, 128, generator=g).bfloat16()
    gt = torch.randn(T, Hg * 128, generator=g).bfloat16()
    wn = (1 + 0.1 * torch.randn(128, generator=g)).bfloat16()
    y = ops.gdn_gated_norm(o.cuda(), gt.cuda(), wn.cuda(), 1e-6)
    torch.testing.assert_close(y.float().cpu(), R.gdn_gated_norm(o.float(), gt.float(), wn.float(), 1e-6),
                               rtol=2e-2, atol=2e-2)


@pytest.mark.gpu
def test_hybrid_engine_gpu_near_oracle():
    cfg = preset("tiny-hybrid")
    w = init_random_weights(cfg, seed=5)
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(3, 1000, (n,), generator=g).tolist() for n in (3, 40, 70)]
    ec = EngineConfig(device="cuda", max_num_seqs=8, max_num_batched_tokens=48, max_model_len=512)
    eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64)
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    ref = ReferenceDecoder(cfg, w)
    for p, o in zip(prompts, outs):
        logits = ref.forward(torch.tensor(p + o.output_token_ids))
        for i, tok in enumerate(o.output_token_ids):
            row = logits[len(p) - 1 + i]
            assert row[tok] >= row.max() - 0.05 * max(1.0, float(row.abs().max()) / 10), (i, tok)

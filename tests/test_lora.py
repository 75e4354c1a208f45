"""Multi-LoRA serving against the merged-weight oracle (W + alpha/r * B A)."""
import pytest
import torch

from gollek_b200.config import EngineConfig
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.lora import merged_weights
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.models.reference import ReferenceDecoder


def _engine(cfg, w, device="cpu"):
    ec = EngineConfig(device=device, dtype="float32" if device == "cpu" else "bfloat16", block_size=16,
                      max_num_seqs=8, max_num_batched_tokens=128, max_model_len=256, use_cuda_graphs=device != "cpu",
                      enable_lora=True, max_loras=2, max_lora_rank=16, enable_prefix_caching=False)
    return LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64)


def test_multi_lora_batch_matches_merged_oracle_cpu(tiny_cfg, tiny_weights):
    eng = _engine(tiny_cfg, tiny_weights)
    a1 = eng.add_lora("a1", seed=1)
    a2 = eng.add_lora("a2", seed=2)
    a3 = eng.add_lora("a3", seed=3)  # 3 adapters, 2 slots: exercises LRU paging
    lm = eng.lora_manager
    for aid in (a1, a2, a3):  # make the adapters strong enough to change greedy tokens
        for L in lm.adapters[aid].layers:
            for m in L:
                A, B = L[m]
                L[m] = (A, B * 200)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, tiny_cfg.vocab_size, (n,), generator=g).tolist() for n in (12, 30, 7)]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    # batch 1: base + a1 + a2 together; batch 2: a3 evicts the LRU slot
    outs = eng.generate(prompts, sp, lora_ids=[0, a1, a2])
    outs3 = eng.generate([prompts[0]], sp, lora_ids=[a3])
    expect = []
    for p, aid in zip(prompts, [0, a1, a2]):
        w = tiny_weights if aid == 0 else merged_weights(tiny_weights, lm.adapters[aid])
        expect.append(ReferenceDecoder(tiny_cfg, w).greedy(p, 6)[0])
    assert [o.output_token_ids for o in outs] == expect
    w3 = merged_weights(tiny_weights, lm.adapters[a3])
    assert outs3[0].output_token_ids == ReferenceDecoder(tiny_cfg, w3).greedy(prompts[0], 6)[0]
    assert lm.loads >= 3
    # the adapter actually changes the output
    assert expect[1] != ReferenceDecoder(tiny_cfg, tiny_weights).greedy(prompts[1], 6)[0]


@pytest.mark.gpu
@pytest.mark.parametrize("T,mods", [(37, 3), (300, 3), (300, 1), (12, 3)])
def test_lora_kernels_match_reference(T, mods):
    """Shrink (tensor cores) and expand over 64-token tiles of adapter segments, one segment
    spanning several tiles, fused q/k/v (three rank blocks) or a single module."""
    from gollek_b200.native import cuda_ext
    torch.manual_seed(0)
    K, r = 4096, 16
    S = 5
    N = 6144 if mods == 3 else 4096
    N1, N2 = (4096, 5120) if mods == 3 else (N, N)
    x = torch.randn(T, K, device="cuda").bfloat16()
    A = (torch.randn(S, mods * r, K, device="cuda") * 0.02).bfloat16()
    B = (torch.randn(S, N, r, device="cuda") * 0.02).bfloat16()
    scales = torch.rand(S, device="cuda") + 0.5
    y = torch.randn(T, N, device="cuda").bfloat16()
    g = torch.Generator().manual_seed(1)
    slots = torch.multinomial(torch.tensor([0.1, 0.6, 0.1, 0.1, 0.1]), T, replacement=True, generator=g).tolist()
    groups = {}
    for t, s in enumerate(slots):
        if s:
            groups.setdefault(s, []).append(t)
    seg_slot = sorted(groups)
    seg_ptr, tok, tiles = [0], [], []
    for i, s in enumerate(seg_slot):
        tiles += [[i, p] for p in range(len(tok), len(tok) + len(groups[s]), 64)]
        tok += groups[s]
        seg_ptr.append(len(tok))
    d = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")  # noqa: E731
    V = torch.zeros(T, mods * r, device="cuda")
    y2 = y.clone()
    ext = cuda_ext()
    ext.lora_shrink(V, x, A, d(seg_ptr), d(tok), d(seg_slot), d(tiles), max(len(v) for v in groups.values()))
    ext.lora_expand(y2, V, B, N1, N2, scales, d(seg_ptr), d(tok), d(seg_slot), d(tiles))
    ref = y.float().clone()
    for t, s in enumerate(slots):
        if not s:
            continue
        v = x[t].float() @ A[s].float().t()
        torch.testing.assert_close(V[t], v, rtol=2e-2, atol=2e-3)
        bounds = ((0, N1, 0), (N1, N2, r), (N2, N, 2 * r)) if mods == 3 else ((0, N, 0),)
        for lo, hi, ro in bounds:
            ref[t, lo:hi] += scales[s] * (B[s][lo:hi].float() @ v[ro:ro + r])
    torch.testing.assert_close(y2.float(), ref, rtol=2e-2, atol=3e-2)


@pytest.mark.gpu
def test_multi_lora_engine_gpu(tiny_cfg, tiny_weights):
    eng = _engine(tiny_cfg, tiny_weights, device="cuda")
    a1 = eng.add_lora("a1", seed=1)
    lm = eng.lora_manager
    for L in lm.adapters[a1].layers:
        for m in L:
            A, B = L[m]
            L[m] = (A, B * 200)
    lm._upload(a1, lm.slot_of[a1]) if a1 in lm.slot_of else None
    prompt = torch.randint(0, tiny_cfg.vocab_size, (20,), generator=torch.Generator().manual_seed(5)).tolist()
    out = eng.generate([prompt, prompt], SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True),
                       lora_ids=[0, a1])
    ref_base = ReferenceDecoder(tiny_cfg, tiny_weights).greedy(prompt, 1)[0]
    ref_lora = ReferenceDecoder(tiny_cfg, merged_weights(tiny_weights, lm.adapters[a1])).greedy(prompt, 1)[0]
    assert out[0].output_token_ids[0] == ref_base[0]
    assert out[1].output_token_ids[0] == ref_lora[0]

"""fp8 (e4m3) paged KV cache: per-token scales written with each token, decode attention reading the
fp8 cache on tensor cores, prefill over dequantized blocks; against fp32 oracles."""
import math

import pytest
import torch

from gollek_b200 import ops
from gollek_b200.ops import reference as ref


def _case(seed, lens, Hk=2, G=4, D=128, dev="cpu"):
    g = torch.Generator().manual_seed(seed)
    bs = 16
    mb = max((l + bs - 1) // bs for l in lens)
    NB = len(lens) * mb + 3
    kv = torch.randn(NB * bs, 2, Hk, D, generator=g) * 2.0
    slots = torch.randperm(NB * bs, generator=g)[: NB * bs].int()
    cache = torch.zeros(NB, 2, Hk, bs, D, dtype=torch.uint8)
    scales = torch.zeros(NB, 2, Hk, bs)
    ops.kv_quant_fp8(kv, slots, cache, scales)
    bt = torch.zeros(len(lens), mb, dtype=torch.int32)
    perm = torch.randperm(NB, generator=g).int()
    k = 0
    for b, l in enumerate(lens):
        n = (l + bs - 1) // bs
        bt[b, :n] = perm[k:k + n]
        k += n
    q = torch.randn(len(lens), Hk * G, D, generator=g)
    return q, kv, slots, cache, scales, bt, torch.tensor(lens, dtype=torch.int32)


def test_quantization_roundtrip_and_scale_rule():
    q, kv, slots, cache, scales, bt, sl = _case(0, [40])
    deq = ops.kv_dequant_fp8(cache, scales)
    bs = cache.shape[3]
    for t in range(0, kv.shape[0], 37):
        s = int(slots[t])
        x, y = kv[t], deq[s // bs, :, :, s % bs]
        amax = x.abs().amax(-1)
        assert torch.allclose(scales[s // bs, :, :, s % bs], amax / 448.0)
        # e4m3: 3 mantissa bits -> relative rounding error <= 2^-4 of each value's magnitude
        assert bool(((x - y).abs() <= x.abs() * 2 ** -4 + amax[..., None] * 2 ** -9 / 448 * 8).all())


def test_cpu_decode_over_fp8_matches_dequantized_oracle():
    q, kv, slots, cache, scales, bt, sl = _case(1, [5, 100, 33])
    scale = 1 / math.sqrt(128)
    got = ops.paged_decode_attention(q, cache, bt, sl, scale, kv_scales=scales)
    want = ref.paged_attention(q, ops.kv_dequant_fp8(cache, scales), bt, sl, torch.arange(4, dtype=torch.int32),
                               scale)
    torch.testing.assert_close(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("G,splits", [(4, 1), (4, 3), (8, 2), (1, 1), (16, 2)])
def test_gpu_decode_fp8_kernel_vs_fp32_oracle(G, splits):
    lens = [7, 300, 1029, 16, 64]
    q, kv, slots, cache, scales, bt, sl = _case(2 + G, lens, G=G)
    dev = "cuda"
    scale = 1 / math.sqrt(128)
    qd = q.bfloat16().to(dev)
    # quantize on the GPU as well: bit-identical cache and scales to the CPU restatement
    cache_d = torch.zeros_like(cache, device=dev)
    scales_d = torch.zeros_like(scales, device=dev)
    ops.kv_quant_fp8(kv.bfloat16().to(dev), slots.to(dev), cache_d, scales_d)
    cache_c = torch.zeros_like(cache)
    scales_c = torch.zeros_like(scales)
    ops.kv_quant_fp8(kv.bfloat16().float(), slots, cache_c, scales_c)
    assert torch.equal(cache_d.cpu(), cache_c) and torch.equal(scales_d.cpu(), scales_c)
    out = ops.paged_decode_attention(qd, cache_d, bt.to(dev), sl.to(dev), scale, num_splits=splits,
                                     kv_scales=scales_d)
    want = ref.paged_attention(qd.float().cpu(), ops.kv_dequant_fp8(cache_c, scales_c), bt, sl,
                               torch.arange(len(lens) + 1, dtype=torch.int32), scale)
    torch.testing.assert_close(out.float().cpu(), want, rtol=2e-2, atol=2e-2)


@pytest.mark.gpu
def test_gpu_prefill_over_fp8_and_engine():
    from gollek_b200.config import EngineConfig, preset
    from gollek_b200.engine.engine import LLMEngine
    from gollek_b200.engine.sequence import SamplingParams
    from gollek_b200.models.reference import ReferenceDecoder, init_random_weights
    cfg = preset("llama-3-8b", num_hidden_layers=2, vocab_size=4096)
    w = init_random_weights(cfg, seed=5)
    prompts = [torch.randint(0, 4096, (n,), generator=torch.Generator().manual_seed(n)).tolist() for n in (90, 17)]
    ec = EngineConfig(device="cuda", max_num_seqs=4, max_num_batched_tokens=256, max_model_len=512,
                      kv_cache_dtype="fp8", cuda_graph_batch_sizes=(1, 2, 4))
    eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64)
    assert eng.kv_cache.dtype == torch.uint8 and eng.model.kv_scales is not None
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
    refm = ReferenceDecoder(cfg, w)
    for p, o in zip(prompts, outs):
        ts = o.output_token_ids
        logits = refm.forward(torch.tensor(p + ts))[len(p) - 1: len(p) - 1 + len(ts)]
        gap = (logits.max(-1).values - logits[torch.arange(len(ts)), torch.tensor(ts)]) / logits.std(-1)
        assert float(gap.max()) < 0.25, gap  # fp8 K/V: a little more rounding than bf16

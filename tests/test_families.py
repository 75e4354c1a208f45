"""Serving the non-Llama families (Qwen2/3, Mistral, Gemma 1/2/3, Phi-3, Cohere-2) through the engine:
greedy tokens equal the fp32 oracle (itself checked against transformers) on CPU, with chunked
prefill, prompts longer than the sliding windows and prefix reuse; on the GPU the sm_100a kernels
(windows, softcaps, QK-norm, biases, GeGLU, head_dim 256) produce near-argmax tokens."""
import pytest
import torch

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.models.reference import ReferenceDecoder, init_random_weights

FAMILIES = ["tiny-qwen2", "tiny-qwen3", "tiny-mistral", "tiny-gemma", "tiny-gemma2", "tiny-gemma3", "tiny-phi3",
            "tiny-cohere2"]


def _prompts(cfg, seed, lens):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]


@pytest.mark.parametrize("name", FAMILIES)
def test_family_engine_cpu_matches_oracle(name):
    cfg = preset(name)
    w = init_random_weights(cfg, seed=5)
    prompts = _prompts(cfg, 6, (7, 45, 60))
    ref = ReferenceDecoder(cfg, w)
    expect = [ref.greedy(p, 5)[0] for p in prompts]
    ec = EngineConfig(device="cpu", dtype="float32", block_size=16, max_num_seqs=8, max_num_batched_tokens=32,
                      max_model_len=256, use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64)
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True))
    assert [o.output_token_ids for o in outs] == expect


@pytest.mark.gpu
@pytest.mark.parametrize("name", FAMILIES)
def test_family_engine_gpu_near_oracle(name):
    cfg = preset(name)
    w = init_random_weights(cfg, seed=5)
    prompts = _prompts(cfg, 7, (3, 40, 70))
    ref = ReferenceDecoder(cfg, w)
    ec = EngineConfig(device="cuda", max_num_seqs=8, max_num_batched_tokens=48, max_model_len=512,
                      use_cuda_graphs=True, cuda_graph_batch_sizes=[1, 2, 4, 8])
    eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64)
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    for p, o in zip(prompts, outs):
        full = p + o.output_token_ids
        logits = ref.forward(torch.tensor(full))
        assert o.output_token_ids[0] == int(logits[len(p) - 1].argmax())
        for i, tok in enumerate(o.output_token_ids):
            row = logits[len(p) - 1 + i]
            assert row[tok] >= row.max() - 0.05 * max(1.0, float(row.abs().max()) / 10), (name, i, tok)

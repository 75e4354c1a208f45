"""Weight-only int8 serving (``quantization="int8"``): dense linear weights become Q8_0 blocks (32 int8
values, one fp16 scale) at load; greedy tokens equal the oracle run on the same rounded weights (CPU)
and are near its argmax on the GPU (Q8_0 GEMV for decode, dequant + tcgen05 GEMM for prefill)."""
import pytest
import torch

from gollek_b200.config import EngineConfig
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.models.reference import ReferenceDecoder
from gollek_b200.native import host_ext


def _q8_roundtrip(v):
    """What the engine stores for one linear weight (K zero-padded to a multiple of 64, as the FFN
    width is), dequantized back."""
    h = host_ext()
    K = v.shape[1]
    Kp = (K + 63) // 64 * 64
    vp = torch.nn.functional.pad(v.float(), (0, Kp - K)).contiguous()
    return h.dequantize_q8_0(h.quantize_q8_0(vp.reshape(-1)), vp.numel()).view(v.shape[0], Kp)[:, :K]


def _oracle(cfg, w):
    lin = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
    return ReferenceDecoder(cfg, {k: (_q8_roundtrip(v) if any(s in k for s in lin) else v) for k, v in w.items()})


def _prompts(cfg, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (7, 33)]


def test_int8_engine_cpu_matches_rounded_oracle(tiny_cfg, tiny_weights):
    ref = _oracle(tiny_cfg, tiny_weights)
    prompts = _prompts(tiny_cfg, 8)
    expect = [ref.greedy(p, 6)[0] for p in prompts]
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=128,
                      use_cuda_graphs=False, quantization="int8")
    eng = LLMEngine(ec, model_cfg=tiny_cfg, weights=tiny_weights.__getitem__, num_blocks=32)
    assert type(eng.model.layers[0]["w_qkv"]).__name__ == "QWeight"
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
    assert [o.output_token_ids for o in outs] == expect


@pytest.mark.gpu
def test_int8_engine_gpu(tiny_cfg, tiny_weights):
    ref = _oracle(tiny_cfg, tiny_weights)
    prompts = _prompts(tiny_cfg, 9)
    ec = EngineConfig(device="cuda", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=128,
                      quantization="int8")
    eng = LLMEngine(ec, model_cfg=tiny_cfg, weights=tiny_weights.__getitem__, num_blocks=32)
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
    for p, o in zip(prompts, outs):
        logits = ref.forward(torch.tensor(p + o.output_token_ids))
        for i, tok in enumerate(o.output_token_ids):
            row = logits[len(p) - 1 + i]
            assert row[tok] >= row.max() - 0.05, (i, tok)

"""Serving GGUF-quantized checkpoints with the blocks kept quantized (Q4_K linears, Q8_0 embed/output)."""
import pytest
import torch

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.loaders import gguf as G
from gollek_b200.models.reference import ReferenceDecoder, init_random_weights


def _q_model(tmp_path):
    cfg = preset("tiny-llama", intermediate_size=768)  # Q4_K needs K % 256 == 0 (down_proj K = ffn)
    w = init_random_weights(cfg, seed=11)
    p = str(tmp_path / "q.gguf")
    G.write_llama_gguf(p, cfg, w, G.GGML_Q4_K, embed_type=G.GGML_Q8_0)
    cfg_q, wq, _ = G.load_llama_gguf(p, keep_quantized=True)
    deq = {k: (v.dequantize() if isinstance(v, G.QuantizedWeight) else v) for k, v in wq.items()}
    return cfg_q, wq, deq


def test_quantized_cpu_engine_matches_dequantized_oracle(tmp_path):
    cfg, wq, deq = _q_model(tmp_path)
    assert isinstance(wq["model.layers.0.mlp.down_proj.weight"], G.QuantizedWeight)
    assert isinstance(wq["model.embed_tokens.weight"], G.QuantizedWeight)
    prompt = torch.randint(0, cfg.vocab_size, (20,), generator=torch.Generator().manual_seed(1)).tolist()
    ref = ReferenceDecoder(cfg, deq).greedy(prompt, 6)[0]
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=128,
                      use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=cfg, weights=wq.__getitem__, num_blocks=32)
    from gollek_b200.quant.gguf_weights import QWeight
    assert isinstance(eng.model.layers[0]["w_qkv"], QWeight)
    out = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))[0]
    assert out.output_token_ids == ref


@pytest.mark.gpu
def test_gguf_gemv_and_dequant_kernels(host):
    from gollek_b200 import ops
    from gollek_b200.quant.gguf_weights import QWeight, interleave_rows
    g = torch.Generator().manual_seed(2)
    N, K = 1024, 4096
    w = torch.randn(N, K, generator=g) * 0.02
    for qtype, quant in ((12, host.quantize_q4_k), (8, host.quantize_q8_0)):
        raw = quant(w.flatten())
        qw = QWeight(raw.cuda(), N, K, qtype)
        wd = qw.dequantize().float()
        host_deq = (host.dequantize_q4_k if qtype == 12 else host.dequantize_q8_0)(raw, N * K).view(N, K)
        torch.testing.assert_close(wd.cpu(), host_deq, rtol=1e-2, atol=1e-3)
        for M in (1, 3, 16, 40):
            x = torch.randn(M, K, device="cuda").bfloat16()
            y = ops.linear(x, qw)
            ref = x.float() @ wd.t()
            torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=3e-2)
    # SwiGLU epilogue on interleaved gate/up rows (Q4_K)
    gq = QWeight(host.quantize_q4_k(w[:512].flatten()).cuda(), 512, K, 12)
    uq = QWeight(host.quantize_q4_k(w[512:].flatten()).cuda(), 512, K, 12)
    gu = interleave_rows(gq, uq)
    x = torch.randn(5, K, device="cuda").bfloat16()
    y = ops.linear_swiglu(x, gu)
    ref = torch.nn.functional.silu(x.float() @ gq.dequantize().float().t()) * (x.float() @ uq.dequantize().float().t())
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=3e-2)
    # Q8_0 embedding gather
    tab = QWeight(host.quantize_q8_0(w.flatten()).cuda(), N, K, 8)
    ids = torch.randint(0, N, (9,), device="cuda").int()
    torch.testing.assert_close(ops.embedding(ids, tab).float(), tab.dequantize().float()[ids.long()], rtol=0, atol=0)


@pytest.mark.gpu
def test_quantized_gpu_engine(tmp_path):
    cfg, wq, deq = _q_model(tmp_path)
    prompt = torch.randint(0, cfg.vocab_size, (20,), generator=torch.Generator().manual_seed(1)).tolist()
    ref = ReferenceDecoder(cfg, deq)
    ec = EngineConfig(device="cuda", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=128,
                      cuda_graph_batch_sizes=(1, 2, 4))
    eng = LLMEngine(ec, model_cfg=cfg, weights=wq.__getitem__, num_blocks=32)
    out = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))[0].output_token_ids
    logits = ref.forward(torch.tensor(prompt + out))[len(prompt) - 1: len(prompt) - 1 + len(out)]
    chosen = logits[torch.arange(len(out)), torch.tensor(out)]
    assert bool(((logits.max(-1).values - chosen) <= 0.05).all())

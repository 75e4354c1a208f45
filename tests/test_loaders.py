"""safetensors + GGUF readers/writers and the GGUF block quantizers (oracle: gguf-py)."""
import json
import os

import numpy as np
import pytest
import torch

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.loaders import gguf as G
from gollek_b200.loaders.safetensors import SafetensorsCheckpoint, save_file, save_sharded
from gollek_b200.models.reference import ReferenceDecoder, init_random_weights


def test_q8_0_matches_gguf_py(host):
    import gguf
    x = torch.randn(64 * 32, generator=torch.Generator().manual_seed(0)) * 0.1
    raw = host.quantize_q8_0(x)
    assert raw.numel() == 64 * 34
    ours = host.dequantize_q8_0(raw, x.numel())
    theirs = gguf.quants.dequantize(raw.numpy(), gguf.GGMLQuantizationType.Q8_0).reshape(-1)
    np.testing.assert_allclose(ours.numpy(), theirs, rtol=0, atol=1e-6)
    assert (ours - x).abs().max() < x.abs().max() / 127 + 1e-6
    # gguf-py's own quantizer agrees byte-for-byte on a random block set
    q2 = gguf.quants.quantize(x.numpy().reshape(-1, 32), gguf.GGMLQuantizationType.Q8_0).reshape(-1)
    deq2 = gguf.quants.dequantize(q2, gguf.GGMLQuantizationType.Q8_0).reshape(-1)
    np.testing.assert_allclose(ours.numpy(), deq2, atol=2e-3)


def test_q4_k_matches_gguf_py(host):
    import gguf
    g = torch.Generator().manual_seed(1)
    x = torch.randn(16 * 256, generator=g) * 0.05 + torch.randn(16 * 256, generator=g) * 0.01
    raw = host.quantize_q4_k(x)
    assert raw.numel() == 16 * 144
    ours = host.dequantize_q4_k(raw, x.numel())
    theirs = gguf.quants.dequantize(raw.numpy(), gguf.GGMLQuantizationType.Q4_K).reshape(-1)
    np.testing.assert_allclose(ours.numpy(), theirs, rtol=1e-6, atol=1e-7)
    rel = ((ours - x).norm() / x.norm()).item()
    assert rel < 0.12, rel


def test_safetensors_roundtrip(tmp_path):
    t = {"a": torch.randn(3, 4), "b": torch.arange(10, dtype=torch.int32), "c": torch.randn(5).bfloat16()}
    p = str(tmp_path / "x.safetensors")
    save_file(t, p, {"k": "v"})
    ck = SafetensorsCheckpoint(p)
    for k, v in t.items():
        assert torch.equal(ck.get(k), v)
    # interoperates with the safetensors package
    from safetensors.torch import load_file
    other = load_file(p)
    assert torch.equal(other["a"], t["a"])
    d = str(tmp_path / "sharded")
    save_sharded(t, d, max_shard_bytes=40)
    ck2 = SafetensorsCheckpoint(d)
    assert sorted(ck2.keys()) == sorted(t)
    assert torch.equal(ck2.get("c"), t["c"])


def test_gguf_writer_readable_by_gguf_py(tmp_path, tiny_cfg, tiny_weights):
    import gguf
    p = str(tmp_path / "m.gguf")
    G.write_llama_gguf(p, tiny_cfg, tiny_weights, G.GGML_F32)
    r = gguf.GGUFReader(p)
    names = {t.name for t in r.tensors}
    assert "blk.0.attn_q.weight" in names and "token_embd.weight" in names
    f = G.GGUFFile(p)
    assert f.metadata["llama.block_count"] == tiny_cfg.num_hidden_layers
    for t in r.tensors[:5]:
        ours = f.get(t.name).numpy().reshape(-1)
        np.testing.assert_array_equal(ours, np.asarray(t.data).reshape(-1))


def _engine(cfg, weights, tok=None):
    ec = EngineConfig(device="cpu", dtype="float32", block_size=16, max_num_seqs=4, max_num_batched_tokens=64,
                      max_model_len=128, use_cuda_graphs=False)
    return LLMEngine(ec, model_cfg=cfg, weights=weights, num_blocks=32)


def test_tiny_llama_safetensors_and_gguf_f32_same_tokens(tmp_path, tiny_cfg, tiny_weights):
    """the same random model saved as safetensors and as GGUF F32 decodes the
    same 32 greedy tokens as the oracle (prompt of 32 ids, paged KV block 16)."""
    prompt = torch.randint(0, tiny_cfg.vocab_size, (32,), generator=torch.Generator().manual_seed(0)).tolist()
    ref_tokens, _ = ReferenceDecoder(tiny_cfg, tiny_weights).greedy(prompt, 32)
    d = tmp_path / "st"
    d.mkdir()
    save_file(tiny_weights, str(d / "model.safetensors"))
    with open(d / "config.json", "w") as f:
        json.dump(tiny_cfg.to_hf(), f)
    sp = SamplingParams(temperature=0.0, max_tokens=32, ignore_eos=True)
    from gollek_b200.engine.engine import load_model_source
    cfg_st, w_st, _ = load_model_source(str(d))
    out_st = _engine(cfg_st, w_st).generate([prompt], sp)[0].output_token_ids
    gp = str(tmp_path / "m.gguf")
    G.write_llama_gguf(gp, tiny_cfg, tiny_weights, G.GGML_F32)
    cfg_g, w_g, f = G.load_llama_gguf(gp)
    assert cfg_g.rope_theta == tiny_cfg.rope_theta and cfg_g.num_key_value_heads == 2
    for k in tiny_weights:  # Q/K un-permuted back to HF order
        torch.testing.assert_close(w_g[k], tiny_weights[k])
    out_g = _engine(cfg_g, w_g.__getitem__).generate([prompt], sp)[0].output_token_ids
    assert out_st == ref_tokens
    assert out_g == ref_tokens


def test_gguf_quantized_keeps_blocks(tmp_path, tiny_cfg, tiny_weights, host):
    gp = str(tmp_path / "q.gguf")
    G.write_llama_gguf(gp, tiny_cfg, tiny_weights, G.GGML_Q4_K, embed_type=G.GGML_Q8_0)
    cfg, w, f = G.load_llama_gguf(gp, keep_quantized=True)
    qw = w["model.layers.0.mlp.gate_proj.weight"]
    assert isinstance(qw, G.QuantizedWeight) and qw.ggml_type == G.GGML_Q4_K
    deq = qw.dequantize()
    ref = tiny_weights["model.layers.0.mlp.gate_proj.weight"]
    assert ((deq - ref).norm() / ref.norm()) < 0.12
    # Q rows come back in HF order even though the blocks stayed quantized
    qq = w["model.layers.0.self_attn.q_proj.weight"].dequantize()
    rq = tiny_weights["model.layers.0.self_attn.q_proj.weight"]
    assert ((qq - rq).norm() / rq.norm()) < 0.12

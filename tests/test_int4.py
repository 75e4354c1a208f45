"""4-bit weights: AWQ/GPTQ checkpoint conversion, RTN/NF4/GPTQ quantizers, engine serving, and the
GPU GEMV / dequant + tcgen05 GEMM kernels against dequantized fp32 references."""
import pytest
import torch

from gollek_b200 import ops
from gollek_b200.config import EngineConfig
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.models.reference import ReferenceDecoder
from gollek_b200.quant import int4 as I4


def _rand_codes(shape, seed):
    return torch.randint(0, 16, shape, generator=torch.Generator().manual_seed(seed))


def test_awq_and_gptq_conversion_roundtrip():
    K, N, g = 256, 64, 128
    codes = _rand_codes((K, N), 1)
    # zero points 1..15: GPTQ stores zero - 1 in a nibble, so 0 is not representable in that format
    zeros = torch.randint(1, 16, (K // g, N), generator=torch.Generator().manual_seed(2))
    scales = (torch.rand(K // g, N, generator=torch.Generator().manual_seed(3)) * 0.02 + 0.001).half()
    ref = ((codes.float() - zeros.float().repeat_interleave(g, 0)) * scales.float().repeat_interleave(g, 0)).t()
    # AWQ: qweight [K, N/8] and qzeros [K/g, N/8], 8 columns per word in AWQ order
    w = I4.from_awq(I4._pack_words(codes, I4.AWQ_ORDER), I4._pack_words(zeros, I4.AWQ_ORDER), scales, g)
    torch.testing.assert_close(w.dequantize(), ref, rtol=1e-2, atol=1e-4)
    # GPTQ: qweight [K/8, N] (8 consecutive k per word), qzeros store zero - 1
    qw = I4._pack_words(codes.t().contiguous()).t().contiguous()
    qz = I4._pack_words(zeros - 1)
    w = I4.from_gptq(qw, qz, scales, g, torch.arange(K) // g)
    torch.testing.assert_close(w.dequantize(), ref, rtol=1e-2, atol=1e-4)
    # act-order g_idx: dequantized to bf16 with the per-column group map
    gi = torch.randperm(K, generator=torch.Generator().manual_seed(4)) % (K // g)
    dense = I4.from_gptq(qw, qz, scales, g, gi)
    ref2 = ((codes.float() - zeros.float()[gi]) * scales.float()[gi]).t()
    torch.testing.assert_close(dense.float(), ref2, rtol=1e-2, atol=1e-3)


def test_quantizers_and_slicing():
    g = torch.Generator().manual_seed(5)
    w = torch.randn(96, 512, generator=g) * 0.05
    rt = I4.quantize_rtn(w, 128)
    assert (rt.dequantize() - w).abs().max() < 0.05 * 0.25
    nf = I4.quantize_nf4(w, 64)
    assert (nf.dequantize() - w).abs().mean() < 0.01
    # TP slicing: rows and group-aligned K slices are views of the same codes
    torch.testing.assert_close(rt[10:20].dequantize(), rt.dequantize()[10:20])
    torch.testing.assert_close(rt[:, 128:384].dequantize(), rt.dequantize()[:, 128:384])
    # GPTQ beats round-to-nearest on correlated calibration inputs
    X = torch.randn(512, 2048, generator=g)
    X[:256] += 3 * X[256:]  # correlated channels
    H = 2 * X @ X.t()
    gq = I4.quantize_gptq(w, H, 128)
    err_gptq = ((gq.dequantize() - w) @ X).pow(2).mean()
    err_rtn = ((rt.dequantize() - w) @ X).pow(2).mean()
    assert err_gptq < err_rtn, (float(err_gptq), float(err_rtn))


def _rtn_like_engine(v):
    """What the engine does to one linear weight: zero-pad K to a multiple of 64, quantize with the
    largest group of 128/64 dividing it, drop the padding."""
    K = v.shape[1]
    Kp = (K + 63) // 64 * 64
    vp = torch.nn.functional.pad(v, (0, Kp - K))
    g = 128 if Kp % 128 == 0 else 64
    return I4.quantize_rtn(vp, g).dequantize()[:, :K]


def _oracle_weights(cfg, w):
    lin = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
    return {k: (_rtn_like_engine(v) if any(s in k for s in lin) else v) for k, v in w.items()}


def test_int4_engine_cpu_matches_dequantized_oracle(tiny_cfg, tiny_weights):
    ref = ReferenceDecoder(tiny_cfg, _oracle_weights(tiny_cfg, tiny_weights))
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, tiny_cfg.vocab_size, (n,), generator=g).tolist() for n in (7, 33)]
    expect = [ref.greedy(p, 6)[0] for p in prompts]
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=128,
                      use_cuda_graphs=False, quantization="int4")
    eng = LLMEngine(ec, model_cfg=tiny_cfg, weights=tiny_weights.__getitem__, num_blocks=32)
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
    assert [o.output_token_ids for o in outs] == expect


@pytest.mark.gpu
@pytest.mark.parametrize("nf4", [False, True])
@pytest.mark.parametrize("M", [1, 3, 8, 300])
@pytest.mark.parametrize("swiglu", [False, True])
def test_int4_kernels_gpu(nf4, M, swiglu):
    g = torch.Generator().manual_seed(M)
    N, K = 1024, 2048
    w = torch.randn(N, K, generator=g) * 0.03
    q = (I4.quantize_nf4(w, 64) if nf4 else I4.quantize_rtn(w, 128))
    wd = q.dequantize()  # CPU reference dequantization
    qg = q.to("cuda")
    torch.testing.assert_close(qg.dequantize().cpu(), wd, rtol=1e-2, atol=1e-3)  # dequant kernel
    x = torch.randn(M, K, generator=g).bfloat16()
    y = ops.linear_swiglu(x.cuda(), qg) if swiglu else ops.linear(x.cuda(), qg)
    ref = ops.reference.gemm_swiglu(x.float(), wd, 64) if swiglu else x.float() @ wd.t()
    torch.testing.assert_close(y.float().cpu(), ref.float(), rtol=3e-2, atol=3e-2)


@pytest.mark.gpu
def test_int4_engine_gpu(tiny_cfg, tiny_weights):
    ref = ReferenceDecoder(tiny_cfg, _oracle_weights(tiny_cfg, tiny_weights))
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, tiny_cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 40)]
    ec = EngineConfig(device="cuda", max_num_seqs=4, max_num_batched_tokens=64, max_model_len=128,
                      quantization="int4")
    eng = LLMEngine(ec, model_cfg=tiny_cfg, weights=tiny_weights.__getitem__, num_blocks=32)
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
    for p, o in zip(prompts, outs):
        logits = ref.forward(torch.tensor(p + o.output_token_ids))
        for i, tok in enumerate(o.output_token_ids):
            row = logits[len(p) - 1 + i]
            assert row[tok] >= row.max() - 0.05, (i, tok)


def test_cli_dequantize_awq_checkpoint(tmp_path):
    """``gollek dequantize``: an AWQ checkpoint directory becomes dense bf16 safetensors whose
    weights equal the 4-bit values, with unquantized tensors copied and the quant block removed."""
    import json

    from gollek_b200.cli import main
    from gollek_b200.loaders.safetensors import SafetensorsCheckpoint, save_file
    K, N, g = 256, 64, 128
    codes = _rand_codes((K, N), 11)
    zeros = torch.randint(1, 16, (K // g, N), generator=torch.Generator().manual_seed(12))
    scales = (torch.rand(K // g, N, generator=torch.Generator().manual_seed(13)) * 0.02 + 0.001).half()
    ref = ((codes.float() - zeros.float().repeat_interleave(g, 0)) * scales.float().repeat_interleave(g, 0)).t()
    src, dst = tmp_path / "awq", tmp_path / "dense"
    src.mkdir()
    norm = torch.rand(K)
    save_file({"model.layers.0.mlp.up_proj.qweight": I4._pack_words(codes, I4.AWQ_ORDER),
               "model.layers.0.mlp.up_proj.qzeros": I4._pack_words(zeros, I4.AWQ_ORDER),
               "model.layers.0.mlp.up_proj.scales": scales,
               "model.layers.0.input_layernorm.weight": norm}, str(src / "model.safetensors"))
    (src / "config.json").write_text(json.dumps({"model_type": "llama", "quantization_config": {
        "quant_method": "awq", "bits": 4, "group_size": g, "version": "gemm"}}))
    main(["dequantize", str(src), str(dst)])
    ck = SafetensorsCheckpoint(str(dst))
    assert sorted(ck.keys()) == ["model.layers.0.input_layernorm.weight", "model.layers.0.mlp.up_proj.weight"]
    w = ck.get("model.layers.0.mlp.up_proj.weight")
    assert w.dtype == torch.bfloat16 and w.shape == (N, K)
    torch.testing.assert_close(w.float(), ref, rtol=1e-2, atol=1e-4)
    torch.testing.assert_close(ck.get("model.layers.0.input_layernorm.weight").float(), norm, rtol=1e-2, atol=1e-3)
    assert "quantization_config" not in json.loads((dst / "config.json").read_text())

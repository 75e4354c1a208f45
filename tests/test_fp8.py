"""Block-scaled FP8 (128x128 weight blocks, 1x128 activation groups): kernels vs the fp32 oracle."""
import pytest
import torch

from gollek_b200.quant import fp8 as F8


def test_fp8_reference_quantisation_cpu():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(300, 512, generator=g) * 0.02
    fw = F8.quantize_weight(w)
    assert fw.scale.shape == (3, 4)
    err = (fw.dequantize().float() - w).norm() / w.norm()
    assert err < 0.05
    x = torch.randn(7, 512, generator=g)
    xq, sa = F8.quantize_act(x)
    y = F8.reference_gemm(xq, sa, fw)
    assert ((y - x @ w.t()).norm() / (x @ w.t()).norm()) < 0.08


def test_fp8_engine_cpu_runs(tiny_cfg):
    from gollek_b200.config import EngineConfig, preset
    from gollek_b200.engine.engine import LLMEngine
    from gollek_b200.engine.sequence import SamplingParams
    from gollek_b200.models.reference import ReferenceDecoder, init_random_weights
    cfg = preset("tiny-llama", intermediate_size=768)
    w = init_random_weights(cfg, seed=4)
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=2, max_num_batched_tokens=64, max_model_len=128,
                      use_cuda_graphs=False, quantization="fp8")
    eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=32)
    assert type(eng.model.layers[0]["w_qkv"]).__name__ == "FP8Weight"
    prompt = list(range(100, 116))
    out = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True))[0].output_token_ids
    ref = ReferenceDecoder(cfg, w)
    logits = ref.forward(torch.tensor(prompt + out))[len(prompt) - 1:len(prompt) - 1 + len(out)]
    chosen = logits[torch.arange(len(out)), torch.tensor(out)]
    assert bool(((logits.max(-1).values - chosen) <= 0.1).all())


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(1, 1280, 8192), (64, 8192, 1024), (300, 1024, 4096), (2048, 2048, 2048)])
def test_fp8_gemm_matches_oracle(M, N, K):
    from gollek_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(M + N)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    fw = F8.quantize_weight(w)
    fw_cpu = F8.quantize_weight(w.float().cpu())
    torch.testing.assert_close(fw.scale.cpu(), fw_cpu.scale, rtol=1e-2, atol=1e-6)
    xq, sa = F8.quantize_act(x)
    xq_c, sa_c = F8.quantize_act(x.float().cpu())
    torch.testing.assert_close(sa.cpu(), sa_c, rtol=1e-2, atol=1e-6)
    ref = F8.reference_gemm(xq.cpu(), sa.cpu(), F8.FP8Weight(fw.q.cpu(), fw.scale.cpu(), N, K))
    tiles = ((M + 127) // 128) * (N // 128)
    cnt = torch.zeros(tiles, dtype=torch.int32, device="cuda")
    for splits, fixup in ((1, False), (3, False), (3, True), (5, True), (3, True)):
        # fixup: the tile's last split unit sums the partials (counters must come back to zero)
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        ws = torch.empty(splits * M * N, device="cuda") if splits > 1 else None
        ops.cuda_ext().gemm_fp8(out, xq, sa, fw.q, fw.scale, 0, splits, ws, cnt if fixup else None)
        torch.testing.assert_close(out.float().cpu(), ref, rtol=2e-2, atol=2e-2 * max(1.0, float(ref.abs().max()) / 4))
        assert int(cnt.abs().sum()) == 0
    y = ops.linear(x, fw)  # automatic split choice
    torch.testing.assert_close(y.float().cpu(), ref, rtol=2e-2, atol=2e-2 * max(1.0, float(ref.abs().max()) / 4))


@pytest.mark.gpu
@pytest.mark.parametrize("M,F,K", [(33, 1024, 2048), (64, 3584, 8192)])
def test_fp8_swiglu(M, F, K):
    from gollek_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(9)
    wg = (torch.randn(F, K, device="cuda", generator=g) * 0.03).bfloat16()
    wu = (torch.randn(F, K, device="cuda", generator=g) * 0.03).bfloat16()
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    fw = F8.quantize_weight(ops.interleave_gate_up(wg, wu).contiguous())
    y = ops.linear_swiglu(x, fw)
    xq, sa = F8.quantize_act(x)
    full = F8.reference_gemm(xq.cpu(), sa.cpu(), F8.FP8Weight(fw.q.cpu(), fw.scale.cpu(), fw.N, K)).view(M, -1, 2, 64)
    ref = (torch.nn.functional.silu(full[:, :, 0]) * full[:, :, 1]).reshape(M, -1)
    # bf16 output rounding grows with the magnitude (K = 8192 gives values of several units)
    torch.testing.assert_close(y.float().cpu(), ref, rtol=2e-2, atol=3e-2 * max(1.0, float(ref.abs().max()) / 4))

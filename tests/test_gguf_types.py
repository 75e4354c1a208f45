"""Every GGUF tensor type of stock llama.cpp files (oracle: gguf-py), the Q4_K_M-style mixture, and
serving a mixed Q4_K / Q6_K file unchanged."""
import numpy as np
import pytest
import torch

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.loaders import gguf as G
from gollek_b200.models.reference import ReferenceDecoder, init_random_weights

# ggml type -> byte offsets of its fp16 scale fields inside one block
_SCALE_FIELDS = {G.GGML_Q4_0: [0], G.GGML_Q4_1: [0, 2], G.GGML_Q5_0: [0], G.GGML_Q5_1: [0, 2],
                 G.GGML_Q2_K: [80, 82], G.GGML_Q3_K: [108], G.GGML_Q5_K: [0, 2], G.GGML_Q6_K: [208]}


def _random_blocks(gt: int, nb: int, seed: int) -> np.ndarray:
    """Random bytes for ``nb`` blocks with finite, modest fp16 scales."""
    rng = np.random.default_rng(seed)
    _, _, bb = G.GGML_TYPES[gt]
    raw = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    for off in _SCALE_FIELDS[gt]:
        raw[:, off:off + 2] = (rng.standard_normal(nb) * 0.05).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return raw.reshape(-1)


@pytest.mark.parametrize("gt", sorted(_SCALE_FIELDS))
def test_dequant_bit_exact_vs_gguf_py(gt):
    import gguf
    name, bs, _ = G.GGML_TYPES[gt]
    raw = _random_blocks(gt, 96, seed=gt)
    theirs = gguf.quants.dequantize(raw, gguf.GGMLQuantizationType[name]).reshape(-1).astype(np.float32)
    ours = G.dequantize_blocks(torch.from_numpy(raw.copy()), gt, 96 * bs).numpy()
    assert np.array_equal(theirs.view(np.uint32), ours.view(np.uint32)), name


# relative L2 error bound of the round-to-nearest quantizers on Gaussian weights
_RT_BOUND = {G.GGML_Q4_0: 0.12, G.GGML_Q4_1: 0.11, G.GGML_Q5_0: 0.06, G.GGML_Q5_1: 0.055, G.GGML_Q2_K: 0.40,
             G.GGML_Q3_K: 0.20, G.GGML_Q5_K: 0.06, G.GGML_Q6_K: 0.03}


@pytest.mark.parametrize("gt", sorted(_RT_BOUND))
def test_quantize_roundtrip_and_gguf_py_decodes_our_blocks(gt):
    import gguf
    name, bs, bb = G.GGML_TYPES[gt]
    x = torch.randn(64 * bs, generator=torch.Generator().manual_seed(gt)) * 0.02
    q = G.quantize_blocks(x, gt)
    assert q.numel() == 64 * bb
    y = G.dequantize_blocks(q, gt, x.numel())
    assert float((y - x).norm() / x.norm()) < _RT_BOUND[gt], name
    theirs = gguf.quants.dequantize(q.numpy(), gguf.GGMLQuantizationType[name]).reshape(-1)
    assert np.array_equal(theirs.astype(np.float32), y.numpy())


def test_q4_k_m_mixture_types():
    n = 32
    t = G.mixture_type
    assert t("Q4_K_M", "lm_head.weight", n) == G.GGML_Q6_K
    assert t("Q4_K_M", "model.embed_tokens.weight", n) == G.GGML_Q4_K
    assert t("Q4_K_M", "model.layers.0.self_attn.v_proj.weight", n) == G.GGML_Q6_K   # first eighth
    assert t("Q4_K_M", "model.layers.5.self_attn.v_proj.weight", n) == G.GGML_Q4_K
    assert t("Q4_K_M", "model.layers.6.mlp.down_proj.weight", n) == G.GGML_Q6_K      # (6 - 4) % 3 == 2
    assert t("Q4_K_M", "model.layers.31.mlp.down_proj.weight", n) == G.GGML_Q6_K     # last eighth
    assert t("Q4_K_M", "model.layers.10.self_attn.q_proj.weight", n) == G.GGML_Q4_K
    assert t("Q5_K_M", "model.layers.10.mlp.up_proj.weight", n) == G.GGML_Q5_K


def _mixed_file(tmp_path):
    cfg = preset("tiny-llama", intermediate_size=768, num_hidden_layers=8)  # K-quants need K % 256 == 0
    w = init_random_weights(cfg, seed=21)
    p = str(tmp_path / "m.gguf")
    G.write_llama_gguf(p, cfg, w, "Q4_K_M")
    return cfg, w, p


def test_mixed_file_readable_by_gguf_py_and_loads(tmp_path):
    import gguf
    cfg, w, p = _mixed_file(tmp_path)
    r = gguf.GGUFReader(p)
    types = {t.name: t.tensor_type.name for t in r.tensors}
    assert types["output.weight"] == "Q6_K" and types["blk.0.attn_v.weight"] == "Q6_K"
    assert types["blk.3.attn_q.weight"] == "Q4_K" and types["blk.7.ffn_down.weight"] == "Q6_K"
    f = G.GGUFFile(p)
    for t in r.tensors:  # our dequant of every tensor equals gguf-py's
        ours = f.get(t.name).numpy().reshape(-1)
        theirs = gguf.quants.dequantize(t.data, t.tensor_type).reshape(-1)
        assert np.array_equal(ours, theirs.astype(np.float32)), t.name
    f.close()


def test_gguf_py_written_q6_k_file_loads(tmp_path):
    """A file written by gguf-py's own writer (Q5_0 and Q6_K tensors) loads through our reader."""
    import gguf
    p = str(tmp_path / "w.gguf")
    wr = gguf.GGUFWriter(p, "llama")
    rng = np.random.default_rng(0)
    vals = {}
    for name, gt, typ in (("a.weight", G.GGML_Q6_K, gguf.GGMLQuantizationType.Q6_K),
                          ("b.weight", G.GGML_Q5_0, gguf.GGMLQuantizationType.Q5_0)):
        x = torch.from_numpy((rng.standard_normal((8, 512)) * 0.02).astype(np.float32))
        q = G.quantize_blocks(x, gt).numpy().reshape(8, -1)
        wr.add_tensor(name, q, raw_shape=q.shape, raw_dtype=typ)
        vals[name] = G.dequantize_blocks(torch.from_numpy(q.reshape(-1).copy()), gt, x.numel()).view(8, 512)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    f = G.GGUFFile(p)
    for name, v in vals.items():
        assert tuple(f.tensors[name].shape) == (8, 512)
        assert torch.equal(f.get(name), v)
    f.close()


def test_serve_mixed_q4_k_m_file_on_cpu(tmp_path):
    """Q4_K and Q6_K tensors stay in their blocks (dequant-fused kernels; a fused q/k/v whose parts
    differ in type is dequantized for that layer); the greedy tokens match the fp32 oracle over the
    file's dequantized weights."""
    cfg, _, p = _mixed_file(tmp_path)
    cfg_q, wq, _ = G.load_llama_gguf(p, keep_quantized=True)
    assert isinstance(wq["model.layers.3.self_attn.q_proj.weight"], G.QuantizedWeight)
    assert isinstance(wq["model.layers.0.self_attn.v_proj.weight"], G.QuantizedWeight)  # Q6_K
    assert wq["model.layers.0.self_attn.v_proj.weight"].ggml_type == G.GGML_Q6_K
    deq = {k: (v.dequantize() if isinstance(v, G.QuantizedWeight) else v) for k, v in wq.items()}
    prompt = torch.randint(0, cfg.vocab_size, (16,), generator=torch.Generator().manual_seed(2)).tolist()
    ref = ReferenceDecoder(cfg_q, deq).greedy(prompt, 5)[0]
    ec = EngineConfig(device="cpu", dtype="float32", max_num_seqs=2, max_num_batched_tokens=64, max_model_len=128,
                      use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=cfg_q, weights=wq.__getitem__, num_blocks=16)
    out = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True))[0]
    assert out.output_token_ids == ref


@pytest.mark.gpu
def test_q6_k_gpu_dequant_and_gemv():
    """Q6_K weights kept in their blocks on the GPU: dequantization equals the host decoder (bf16 of
    the same fp32 values) and the decode GEMV matches x @ W^T for 1..16 tokens."""
    from gollek_b200 import ops
    from gollek_b200.quant.gguf_weights import QWeight
    N, K = 768, 1024
    w = torch.randn(N, K, generator=torch.Generator().manual_seed(6)) * 0.02
    raw = G.quantize_blocks(w, G.GGML_Q6_K)
    qw = QWeight(raw.cuda(), N, K, G.GGML_Q6_K)
    host = G.dequantize_blocks(raw, G.GGML_Q6_K, N * K).view(N, K)
    wd = qw.dequantize()
    assert torch.equal(wd.cpu(), host.bfloat16())
    for M in (1, 3, 16, 40):  # GEMV up to 16 rows, dequant + tcgen05 GEMM above
        x = torch.randn(M, K, device="cuda").bfloat16()
        y = ops.linear(x, qw)
        ref = x.float() @ host.cuda().t()
        torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(5, 256, 512), (64, 1024, 4096), (130, 6144, 4096), (300, 512, 2048)])
def test_q4_k_fused_tcgen05_gemm(M, N, K):
    """Q4_K super-blocks decoded inside the tcgen05 GEMM (more than 4 tokens): equal to x @ W^T over
    the host dequantization of the same blocks; with split-K (small M) and whole tiles, and the
    SwiGLU epilogue over gate/up rows interleaved in groups of 64."""
    from gollek_b200 import ops
    from gollek_b200.quant.gguf_weights import QWeight
    g = torch.Generator().manual_seed(M + N)
    w = torch.randn(N, K, generator=g) * 0.02
    raw = G.quantize_blocks(w, G.GGML_Q4_K)
    host = G.dequantize_blocks(raw, G.GGML_Q4_K, N * K).view(N, K)
    qw = QWeight(raw.cuda(), N, K, G.GGML_Q4_K)
    x = torch.randn(M, K, generator=g).bfloat16()
    ref = x.float() @ host.bfloat16().float().t()
    y = ops.linear(x.cuda(), qw)
    torch.testing.assert_close(y.float().cpu(), ref, rtol=2e-2, atol=2e-2 * max(1.0, float(ref.abs().max()) / 4))
    assert ops.cuda_ext().gemm_q4k_splits(M, N, K) >= 1
    # SwiGLU: gate/up rows interleaved in groups of 64 (the layout the loader gives fused gate/up)
    F = N // 2
    wg, wu = torch.randn(F, K, generator=g) * 0.02, torch.randn(F, K, generator=g) * 0.02
    wgu = ops.interleave_gate_up(wg, wu).contiguous()
    raw2 = G.quantize_blocks(wgu, G.GGML_Q4_K)
    host2 = G.dequantize_blocks(raw2, G.GGML_Q4_K, N * K).view(N, K).bfloat16().float()
    qw2 = QWeight(raw2.cuda(), N, K, G.GGML_Q4_K)
    y2 = ops.linear_swiglu(x.cuda(), qw2)
    ref2 = ops.reference.gemm_swiglu(x.float(), host2)
    torch.testing.assert_close(y2.float().cpu(), ref2, rtol=2e-2, atol=3e-2 * max(1.0, float(ref2.abs().max()) / 4))


@pytest.mark.gpu
@pytest.mark.parametrize("N,K", [(4096, 14336), (4097, 4096), (768, 1024), (6144, 2304)])
@pytest.mark.parametrize("swiglu", [False, True])
def test_q4_k_gemv_k_split(N, K, swiglu, monkeypatch):
    """The Q4_K decode GEMV with several warps per row pair (each over part of the super-blocks,
    partial sums added in shared memory) and with one warp per pair: both against x @ W^T over the
    host dequantization, for 1..16 tokens, an odd row count and the SwiGLU epilogue."""
    from gollek_b200 import ops
    from gollek_b200.quant.gguf_weights import QWeight
    if swiglu:
        N = (N // 128) * 128
    g = torch.Generator().manual_seed(N + K)
    w = torch.randn(N, K, generator=g) * 0.02
    raw = G.quantize_blocks(w, G.GGML_Q4_K)
    host = G.dequantize_blocks(raw, G.GGML_Q4_K, N * K).view(N, K).bfloat16().float()
    qw = QWeight(raw.cuda(), N, K, G.GGML_Q4_K)
    for M in (1, 3, 4, 7, 16):
        if M > ops.GGUF_GEMV_MAX_TOKENS and N % 8:
            continue  # the tcgen05 path above the GEMV sizes needs 16-byte output rows
        x = torch.randn(M, K, generator=g).bfloat16().cuda()
        ref = ops.reference.gemm_swiglu(x.float().cpu(), host) if swiglu else x.float().cpu() @ host.t()
        for split in ("1", "0"):
            monkeypatch.setenv("GOLLEK_GEMV_KSPLIT", split)
            y = ops.linear_swiglu(x, qw) if swiglu else ops.linear(x, qw)
            torch.testing.assert_close(y.float().cpu(), ref, rtol=2e-2, atol=2e-2 * max(1.0, float(ref.abs().max()) / 4),
                                       msg=lambda m: f"{M} ksplit={split}: {m}")

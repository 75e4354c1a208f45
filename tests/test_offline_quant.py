"""Offline quantizers: QuIP#-style lattice codes, AutoRound, AWQ scale search, and the checkpoint
pipeline that writes what the engine serves (CPU)."""
import json

import pytest
import torch

from gollek_b200.config import preset
from gollek_b200.loaders.safetensors import save_file
from gollek_b200.models.reference import ReferenceDecoder, init_random_weights
from gollek_b200.quant import quip as Q
from gollek_b200.quant.autoround import from_autoround, quantize_autoround, to_autoround
from gollek_b200.quant.awq import awq_search, to_awq
from gollek_b200.quant.int4 import Int4Weight, from_awq, quantize_rtn


def _rel(a, b):
    return float((a - b).norm() / b.norm())


def test_e8_codebook_and_nearest_point():
    cb = Q.codebook()
    assert cb.shape == (56881, 8)  # 1 + 240 + 2160 + 6720 + 17520 + 30240 points of squared norm <= 10
    n2 = (cb ** 2).sum(1)
    assert sorted(set(n2.tolist())) == [0.0, 2.0, 4.0, 6.0, 8.0, 10.0]
    x = torch.randn(3000, 8, generator=torch.Generator().manual_seed(1))
    p = Q.nearest_e8(x)
    bf = cb[((x[:, None, :] - cb[None]) ** 2).sum(-1).argmin(1)]
    inside = (p * p).sum(1) <= 10
    assert inside.sum() > 2000 and torch.equal(p[inside], bf[inside])
    assert torch.equal(cb[Q._index(bf)], bf)


@pytest.mark.parametrize("N,K", [(256, 1792), (96, 512)])
def test_quip_roundtrip_and_error(N, K):
    g = torch.Generator().manual_seed(N)
    w = torch.randn(N, K, generator=g) * 0.02
    w[3, 5] = 0.5  # an outlier: spread by the incoherence transform
    assert _rel(Q.coherent(Q.incoherent(w, 4), 4), w) < 1e-5
    q1, q2 = Q.quantize_quip(w, stages=1, seed=4), Q.quantize_quip(w, stages=2, seed=4)
    assert q1.bits_per_weight() == pytest.approx(2.25) and q2.bits_per_weight() == pytest.approx(4.25)
    e1, e2 = _rel(q1.dequantize(), w), _rel(q2.dequantize(), w)
    assert e1 < 0.34 and e2 < 0.12 and e2 < e1 / 2.5


def test_autoround_lowers_output_error_and_native_format():
    g = torch.Generator().manual_seed(0)
    N, K = 128, 512
    W = torch.randn(N, K, generator=g) * 0.02
    X = torch.randn(768, K, generator=g)
    X[:, :8] *= 10  # a few large activation channels
    ref = X @ W.t()
    oerr = lambda q: _rel(X @ q.dequantize().t(), ref)  # noqa: E731
    q = quantize_autoround(W, X, 128, iters=150)
    assert oerr(q) < 0.95 * oerr(quantize_rtn(W, 128))
    t = to_autoround(q)
    assert t["weight"].dtype == torch.int32 and t["weight"].shape == (N // 8, K) and t["zp"].dtype == torch.int32
    assert torch.equal(from_autoround(t["weight"], t["scale"], t["zp"], 128).dequantize(), q.dequantize())
    sym = from_autoround(t["weight"], t["scale"], None, 128)  # symmetric checkpoints: zero point 8
    assert torch.equal(sym.zero.float(), torch.full_like(sym.zero.float(), 8.0))


def test_awq_search_lowers_output_error_and_awq_format():
    g = torch.Generator().manual_seed(2)
    K = 512
    Ws = [torch.randn(n, K, generator=g) * 0.02 for n in (256, 128)]
    X = torch.randn(1024, K, generator=g)
    X[:, 100:104] *= 30
    s, qs = awq_search(Ws, X, 128)
    err = sum(float(((X @ (q.dequantize() / s[None]).t() - X @ w.t()) ** 2).sum()) for q, w in zip(qs, Ws))
    err_rtn = sum(float(((X @ quantize_rtn(w, 128).dequantize().t() - X @ w.t()) ** 2).sum()) for w in Ws)
    assert err < 0.9 * err_rtn
    t = to_awq(qs[0])
    back = from_awq(t["qweight"], t["qzeros"], t["scales"].float(), 128)
    torch.testing.assert_close(back.dequantize(), qs[0].dequantize(), rtol=1e-2, atol=1e-4)  # fp16 scales


@pytest.mark.parametrize("method", ["awq", "autoround", "quip"])
def test_quantize_checkpoint_serves(tmp_path, method):
    """A small Llama-family checkpoint quantized by each method: the engine loads it (int4 weights for
    AWQ / AutoRound, bf16 for QuIP), the dense model rebuilt from what it loads stays close to the fp32
    model, and the engine decodes from it."""
    from gollek_b200.config import EngineConfig
    from gollek_b200.engine.engine import LLMEngine, load_model_source
    from gollek_b200.engine.sequence import SamplingParams
    from gollek_b200.quant.offline import quantize_checkpoint
    cfg = preset("tiny-llama", intermediate_size=512, num_hidden_layers=2)
    w = init_random_weights(cfg, seed=0)
    src, dst = tmp_path / "src", tmp_path / "dst"
    src.mkdir()
    save_file(w, str(src / "model.safetensors"))
    (src / "config.json").write_text(json.dumps(cfg.to_hf()))
    summary = quantize_checkpoint(str(src), str(dst), method, group=64, calib_seqs=2, calib_len=64, iters=60,
                                  stages=2 if method == "quip" else 1)
    assert summary["linears"] == 7 * cfg.num_hidden_layers
    qcfg, get, _ = load_model_source(str(dst))
    dense = {}
    for k in w:
        v = get(k)
        if isinstance(v, Int4Weight):
            assert method in ("awq", "autoround")
            v = v.dequantize(torch.float32)
        dense[k] = v.float()
    ids = torch.randint(0, cfg.vocab_size, (48,), generator=torch.Generator().manual_seed(7))
    lf = ReferenceDecoder(cfg, w).forward(ids)
    lq = ReferenceDecoder(cfg, dense).forward(ids)
    assert _rel(lq, lf) < 0.2, _rel(lq, lf)
    ec = EngineConfig(device="cpu", dtype="float32", block_size=16, max_num_seqs=2, max_num_batched_tokens=128,
                      max_model_len=128, use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=qcfg, weights=get, num_blocks=16)
    out = eng.generate([ids[:20].tolist()], SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True))[0]
    assert len(out.output_token_ids) == 4


@pytest.mark.parametrize("method", ["autoround", "quip"])
def test_cli_quantize_then_dequantize(tmp_path, method):
    """``gollek quantize --method`` then ``gollek dequantize``: a dense bf16 checkpoint with every
    original tensor name, close to the original weights."""
    import argparse
    from gollek_b200 import cli
    from gollek_b200.loaders.safetensors import SafetensorsCheckpoint
    cfg = preset("tiny-llama", intermediate_size=512, num_hidden_layers=1)
    w = init_random_weights(cfg, seed=1)
    src = tmp_path / "src"
    src.mkdir()
    save_file(w, str(src / "model.safetensors"))
    (src / "config.json").write_text(json.dumps(cfg.to_hf()))
    cli.cmd_quantize(argparse.Namespace(src=str(src), dst=str(tmp_path / "q"), method=method, group=64, iters=20,
                                        stages=2, calib_file=None, type="Q4_K"))
    cli.cmd_dequantize(argparse.Namespace(src=str(tmp_path / "q"), dst=str(tmp_path / "dq")))
    ck = SafetensorsCheckpoint(str(tmp_path / "dq"))
    assert set(ck.keys()) == set(w.keys())
    k = "model.layers.0.mlp.down_proj.weight"
    assert ck.get(k).dtype == torch.bfloat16 and _rel(ck.get(k).float(), w[k].float()) < 0.2
    assert "quantization_config" not in json.loads((tmp_path / "dq" / "config.json").read_text())


def test_turboquant_distortion_unbiased_inner_products_and_kv_split():
    """TurboQuant: MSE distortion of unit vectors at 1-4 bits near the values the method's analysis
    gives (0.36 / 0.117 / 0.03 / 0.009), unbiased inner products of the residual-sketch form, and the
    2.5-bit KV split beating uniform 2 bits on data with outlier channels."""
    import math
    from gollek_b200.quant import turboquant as T
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3000, 128, generator=g)
    x = x / x.norm(dim=1, keepdim=True)
    for b, want in ((1, 0.36), (2, 0.117), (3, 0.03), (4, 0.009)):
        q = T.TurboQuantMSE(128, b, seed=3)
        mse = float(((q.dequantize(q.quantize(x)) - x) ** 2).sum(1).mean())
        assert abs(mse - want) < 0.2 * want, (b, mse)
    P = T.TurboQuantProd(128, 3, seed=5)
    xs, y = torch.randn(3000, 128, generator=g), torch.randn(1, 128, generator=g)
    err = P.inner(y, P.quantize(xs))[0] - (y @ xs.t())[0]
    assert abs(float(err.mean())) < 3 * float(err.std()) / math.sqrt(err.numel())
    kv = torch.randn(512, 128, generator=g)
    kv[:, 40:72] *= 6
    qk = T.quantize_kv(kv, 2, 32)
    assert sorted(qk.outlier_idx.tolist()) == list(range(40, 72))
    assert 8 * qk.nbytes() / kv.numel() == pytest.approx(2.5, abs=0.02)
    u = T.TurboQuantMSE(128, 2)
    assert _rel(T.dequantize_kv(qk), kv) < 0.7 * _rel(u.dequantize(u.quantize(kv)), kv)


@pytest.mark.parametrize("double_quant", [False, True])
def test_bitsandbytes_checkpoint_loading(tmp_path, double_quant):
    """bitsandbytes-serialized NF4 (plain and double-quantized statistics), FP4-style code maps and
    LLM.int8 rows: NF4 loads as an NF4 Int4Weight (served by the int4 kernels), the others as bf16,
    all close to the original matrix; the engine decodes from such a checkpoint."""
    from gollek_b200.config import EngineConfig
    from gollek_b200.engine.engine import LLMEngine, load_model_source
    from gollek_b200.engine.sequence import SamplingParams
    from gollek_b200.quant.bnb import to_bnb4
    cfg = preset("tiny-llama", intermediate_size=512, num_hidden_layers=1)
    w = init_random_weights(cfg, seed=3)
    out = {}
    fp4_map = torch.tensor([0.0, 0.0052, 0.6667, 1.0, 0.3333, 0.5, 0.1667, 0.25,
                            -0.0, -0.0052, -0.6667, -1.0, -0.3333, -0.5, -0.1667, -0.25])
    for k, v in w.items():
        if k.endswith("proj.weight"):
            if "o_proj" in k:  # LLM.int8 rows
                scb = v.float().abs().amax(1)
                out[k] = torch.round(v.float() / scb[:, None] * 127).to(torch.int8)
                out[k[:-7] + ".SCB"] = scb
            else:
                qm = fp4_map if "down_proj" in k else None
                for suf, t in to_bnb4(v, 64, qm, double_quant, "fp4" if qm is not None else "nf4").items():
                    out[k + suf] = t
        else:
            out[k] = v
    d = tmp_path / "bnb"
    d.mkdir()
    save_file(out, str(d / "model.safetensors"))
    hf = cfg.to_hf()
    hf["quantization_config"] = {"quant_method": "bitsandbytes", "load_in_4bit": True, "bnb_4bit_quant_type": "nf4",
                                 "bnb_4bit_use_double_quant": double_quant}
    (d / "config.json").write_text(json.dumps(hf))
    qcfg, get, _ = load_model_source(str(d))
    g = get("model.layers.0.mlp.gate_proj.weight")
    assert isinstance(g, Int4Weight) and g.nf4 and g.group == 64
    for n, tol in (("mlp.gate_proj", 0.12), ("mlp.down_proj", 0.35), ("self_attn.o_proj", 0.02)):
        k = f"model.layers.0.{n}.weight"
        v = get(k)
        v = v.dequantize() if isinstance(v, Int4Weight) else v.float()
        assert _rel(v, w[k].float()) < tol, (n, _rel(v, w[k].float()))
    ec = EngineConfig(device="cpu", dtype="float32", block_size=16, max_num_seqs=2, max_num_batched_tokens=64,
                      max_model_len=64, use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=qcfg, weights=get, num_blocks=8)
    outp = eng.generate([[5, 6, 7, 8]], SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True))[0]
    assert len(outp.output_token_ids) == 3


def test_squeezellm_dense_and_sparse(tmp_path):
    """SqueezeLLM: on a heavy-tailed matrix the per-channel k-means codebooks plus exact outliers beat
    uniform int4; the checkpoint tensors round-trip, and the engine serves such a checkpoint."""
    from gollek_b200.quant.squeezellm import from_tensors, quantize_squeezellm, to_tensors
    g = torch.Generator().manual_seed(5)
    W = torch.distributions.StudentT(3.0).sample((256, 512)) * 0.01
    q = quantize_squeezellm(W, 4, 0.005)
    assert q.val.numel() == round(0.005 * W.numel())
    e = _rel(q.dequantize(), W)
    assert e < 0.8 * _rel(quantize_rtn(W, 128).dequantize(), W), e
    t = to_tensors(q)
    back = from_tensors(t["qweight"], t["lookup_table"], t["dense_ptr"], t["dense_idx"], t["weight_nnz"])
    assert torch.equal(back.dequantize(), q.dequantize())
    # a checkpoint served by the engine
    from gollek_b200.config import EngineConfig
    from gollek_b200.engine.engine import LLMEngine, load_model_source
    from gollek_b200.engine.sequence import SamplingParams
    cfg = preset("tiny-llama", intermediate_size=512, num_hidden_layers=1)
    w = init_random_weights(cfg, seed=4)
    out = {}
    for k, v in w.items():
        if k.endswith("proj.weight"):
            for suf, tt in to_tensors(quantize_squeezellm(v, 4, 0.005)).items():
                out[k[:-7] + "." + suf] = tt
        else:
            out[k] = v
    d = tmp_path / "sq"
    d.mkdir()
    save_file(out, str(d / "model.safetensors"))
    hf = cfg.to_hf()
    hf["quantization_config"] = {"quant_method": "squeezellm", "wbits": 4}
    (d / "config.json").write_text(json.dumps(hf))
    qcfg, get, _ = load_model_source(str(d))
    k = "model.layers.0.mlp.down_proj.weight"
    assert get(k).dtype == torch.bfloat16 and _rel(get(k).float(), w[k].float()) < 0.12
    ec = EngineConfig(device="cpu", dtype="float32", block_size=16, max_num_seqs=2, max_num_batched_tokens=64,
                      max_model_len=64, use_cuda_graphs=False)
    o = LLMEngine(ec, model_cfg=qcfg, weights=get, num_blocks=8).generate(
        [[5, 6, 7]], SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True))[0]
    assert len(o.output_token_ids) == 3


def test_e2m1_rounding_and_fp4_formats():
    """e2m1: nearest code, ties to the even code, saturation at 6; NVFP4 (e4m3 scale per 16 and a
    tensor scale) and MXFP4 (power-of-two scale per 32) round-trip through their checkpoint tensors,
    and the W4A4 oracle matches the dequantized product."""
    from gollek_b200.quant import fp4 as F
    x = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, -0.3, -5.0, 0.74, 0.76])
    assert F.decode_e2m1(F.encode_e2m1(x)).tolist() == [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, -0.5, -4.0, 0.5, 1.0]
    c = torch.arange(16, dtype=torch.uint8)
    assert torch.equal(F.encode_e2m1(F.decode_e2m1(c))[c != 8], c[c != 8])  # -0 encodes as +0
    assert torch.equal(F.unpack_nibbles(F.pack_nibbles(c.view(2, 8))), c.view(2, 8))
    g = torch.Generator().manual_seed(3)
    w = torch.randn(96, 256, generator=g) * 0.02
    w[:, :16] *= 50.0  # one block of large magnitude per row: the per-block scales absorb it
    for fmt in ("nvfp4", "mxfp4"):
        q = F.quantize_nvfp4(w) if fmt == "nvfp4" else F.quantize_mxfp4(w)
        assert _rel(q.dequantize(), w) < 0.12, (fmt, _rel(q.dequantize(), w))
        t = F.to_tensors(q)
        back = (F.from_nvfp4(t[""], t["_scale"], t["_scale_2"]) if fmt == "nvfp4"
                else F.from_mxfp4(t["_blocks"], t["_scales"]))
        assert torch.equal(back.dequantize(), q.dequantize())
        xa = torch.randn(5, 256, generator=g)
        ref = F.fp4_matmul_reference(xa, q, quantize_activations=False)
        assert torch.allclose(ref, xa @ q.dequantize().t(), atol=1e-5)
        assert _rel(F.fp4_matmul_reference(xa, q), xa @ w.t()) < 0.2
    # every NVFP4 element with a non-zero block is within half an e2m1 step of its scaled value
    q = F.quantize_nvfp4(w)
    s = (q.scale * q.global_scale).repeat_interleave(16, 1)
    assert ((q.dequantize() - w).abs() <= s * 1.0 + 1e-12).all()


@pytest.mark.parametrize("method", ["nvfp4", "mxfp4"])
def test_fp4_checkpoint_serves_and_dequantizes(tmp_path, method):
    """``gollek quantize --method nvfp4|mxfp4`` writes ModelOpt / MXFP4 tensors that the engine loads
    and serves, and ``gollek dequantize`` turns back into bf16 close to the original."""
    import subprocess
    import sys
    from gollek_b200.config import EngineConfig
    from gollek_b200.engine.engine import LLMEngine, load_model_source
    from gollek_b200.engine.sequence import SamplingParams
    from gollek_b200.loaders.safetensors import SafetensorsCheckpoint
    cfg = preset("tiny-llama", intermediate_size=512, num_hidden_layers=1)
    w = init_random_weights(cfg, seed=6)
    src, dst, deq = tmp_path / "src", tmp_path / method, tmp_path / "deq"
    src.mkdir()
    save_file({k: v.to(torch.bfloat16) for k, v in w.items()}, str(src / "model.safetensors"))
    (src / "config.json").write_text(json.dumps(cfg.to_hf()))
    run = lambda *a: subprocess.run([sys.executable, "-m", "gollek_b200", *a], check=True, capture_output=True, text=True)
    run("quantize", str(src), str(dst), "--method", method)
    ck = SafetensorsCheckpoint(str(dst))
    k = "model.layers.0.mlp.down_proj.weight"
    if method == "nvfp4":
        assert ck.get(k).dtype == torch.uint8 and ck.get(k + "_scale").dtype == torch.float8_e4m3fn
    else:
        assert ck.get(k + "_blocks").shape[-1] == 16 and ck.get(k + "_scales").dtype == torch.uint8
    qcfg, get, _ = load_model_source(str(dst))
    assert get(k).dtype == torch.bfloat16 and _rel(get(k).float(), w[k].float()) < 0.12
    ec = EngineConfig(device="cpu", dtype="float32", block_size=16, max_num_seqs=2, max_num_batched_tokens=64,
                      max_model_len=64, use_cuda_graphs=False)
    o = LLMEngine(ec, model_cfg=qcfg, weights=get, num_blocks=8).generate(
        [[5, 6, 7]], SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True))[0]
    assert len(o.output_token_ids) == 3
    r = run("dequantize", str(dst), str(deq))
    assert "7 " in r.stdout, r.stdout  # q, k, v, o, gate, up, down
    back = SafetensorsCheckpoint(str(deq)).get(k)
    assert back.dtype == torch.bfloat16 and torch.equal(back, get(k))


def test_modelopt_hf_quant_config_and_fp8(tmp_path):
    """A ModelOpt checkpoint described only by hf_quant_config.json; its FP8 linears (e4m3 weight,
    per-tensor scale) load as bf16."""
    from gollek_b200.loaders.safetensors import SafetensorsCheckpoint
    from gollek_b200.quant.int4 import checkpoint_quant_config, quantized_checkpoint_getter
    w = torch.randn(64, 128) * 0.05
    s = w.abs().max() / 448.0
    d = tmp_path / "mo"
    d.mkdir()
    save_file({"l.weight": (w / s).to(torch.float8_e4m3fn), "l.weight_scale": s.reshape(()).float(),
               "n.weight": torch.ones(8)}, str(d / "model.safetensors"))
    (d / "config.json").write_text(json.dumps({"model_type": "llama"}))
    (d / "hf_quant_config.json").write_text(json.dumps({"quantization": {"quant_algo": "FP8"}}))
    qc = checkpoint_quant_config(str(d))
    assert qc["quant_method"] == "modelopt" and qc["quant_algo"] == "FP8"
    get = quantized_checkpoint_getter(SafetensorsCheckpoint(str(d)), qc)
    assert get("l.weight").dtype == torch.bfloat16 and _rel(get("l.weight").float(), w) < 0.05
    assert torch.equal(get("n.weight"), torch.ones(8))

"""DeepSeek-V3 family (also DeepSeek-R1 / Kimi-K2 checkpoints): multi-head latent attention, YaRN
RoPE, sigmoid group-limited routing with a correction bias, shared experts and dense first layers.

The fp32 oracle is checked against transformers' DeepseekV3ForCausalLM; the serving model (MLA
decompressed into the paged cache, the K12 router in sigmoid mode) against the oracle on CPU, over
two gloo ranks (tensor- and expert-parallel), and on the GPU."""
import multiprocessing as mp

import pytest
import torch

from gollek_b200 import ops
from gollek_b200.config import EngineConfig, ModelConfig, RopeScaling, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.models.reference import ReferenceDecoder, init_random_weights
from gollek_b200.ops import reference as R

YARN = RopeScaling(kind="yarn", factor=8.0, original_max_position_embeddings=256, mscale=0.7, mscale_all_dim=1.0)


def _hf_deepseek(cfg, w):
    """transformers' model with our checkpoint-named weights (its experts are stacked per layer)."""
    import transformers
    d = cfg.to_hf()
    mt, arch = d.pop("model_type"), d.pop("architectures")[0]
    d.pop("torch_dtype", None)
    hc = transformers.AutoConfig.for_model(mt, **d)
    hc._attn_implementation = "eager"
    model = getattr(transformers, arch)(hc).eval()
    sd = model.state_dict()
    new = {k: w[k] for k in sd if k in w}
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}.mlp."
        for k in sd:
            if not k.startswith(p):
                continue
            E = cfg.num_local_experts
            if k.endswith("experts.gate_up_proj"):
                new[k] = torch.stack([torch.cat([w[p + f"experts.{e}.gate_proj.weight"],
                                                 w[p + f"experts.{e}.up_proj.weight"]], 0) for e in range(E)])
            elif k.endswith("experts.down_proj"):
                new[k] = torch.stack([w[p + f"experts.{e}.down_proj.weight"] for e in range(E)])
            if k in new and new[k].shape != sd[k].shape:
                new[k] = new[k].transpose(1, 2)
    assert not [k for k in sd if k not in new and "rotary" not in k]
    model.load_state_dict(new, strict=False)
    return model


@pytest.mark.parametrize("variant", ["q_lora", "no_q_lora_yarn", "yarn"])
def test_reference_deepseek_v3_matches_hf(variant):
    over = {"no_q_lora_yarn": dict(q_lora_rank=0, rope_scaling=YARN), "yarn": dict(rope_scaling=YARN)}.get(variant, {})
    cfg = preset("tiny-deepseek-v3", **over)
    w = init_random_weights(cfg, seed=3)
    ids = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(3))
    ours = ReferenceDecoder(cfg, w).forward(ids)
    with torch.no_grad():
        theirs = _hf_deepseek(cfg, w)(ids[None]).logits[0]
    torch.testing.assert_close(ours, theirs, rtol=1e-4, atol=1e-5)


def test_deepseek_config_round_trip():
    for cfg in (preset("tiny-deepseek-v3"), preset("deepseek-v3")):
        back = ModelConfig.from_hf(cfg.to_hf())
        for f in ("architecture", "head_dim", "q_lora_rank", "kv_lora_rank", "qk_nope_head_dim", "qk_rope_head_dim",
                  "v_head_dim", "num_local_experts", "num_experts_per_tok", "moe_intermediate_size",
                  "n_shared_experts", "moe_scoring", "n_group", "topk_group", "routed_scaling_factor",
                  "norm_topk_prob", "first_k_dense_replace", "rope_interleaved", "num_key_value_heads"):
            assert getattr(back, f) == getattr(cfg, f), f
        assert back.rope_scaling == cfg.rope_scaling
        assert abs(back.attn_scale - cfg.attn_scale) < 1e-9
    full = preset("deepseek-v3")
    assert 670e9 < full.num_params() < 672e9 and 36e9 < full.flops_per_token() / 2 < 38e9


def test_sigmoid_group_limited_routing():
    """Groups are ranked by their two best choice scores (bias included); experts outside the kept
    groups are not chosen even when their own score is higher; weights are the unbiased sigmoid
    scores, renormalised, times the routed scale."""
    logit = torch.tensor([[4.0, -4.0, -4.0, -4.0, 1.0, 1.0, 0.5, 0.5]])  # 4 groups of 2
    bias = torch.tensor([0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.2, 0.2])
    ids, w = R.moe_route(logit, 2, scoring="sigmoid", bias=bias, n_group=4, topk_group=2, scale=2.5)
    # group scores: g0 = s(4)+s(-4) = 1.0, g1 = 0.018+0.018, g2 = 2*0.731 = 1.462, g3 = 2*(0.622+0.2) = 1.645
    assert sorted(ids[0].tolist()) == [6, 7]  # best two experts inside groups {2, 3}: the biased 6 and 7
    s = torch.sigmoid(logit[0, 6])
    torch.testing.assert_close(w[0], torch.stack([s, s]) / (2 * s) * 2.5)
    ids1, _ = R.moe_route(logit, 2, scoring="sigmoid", bias=bias, n_group=4, topk_group=3)
    assert ids1[0].tolist() == [0, 6]  # group 0 now kept: expert 0 (0.982) first, then 6 (0.822) over 4 (0.731)


def _prompts(cfg, seed, lens):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]


def test_deepseek_engine_cpu_matches_oracle():
    """Chunked prefill (32-token budget), decode and the paged cache: greedy tokens equal the oracle's
    and the top-5 log-probabilities of every step match its log-softmax."""
    cfg = preset("tiny-deepseek-v3")
    w = init_random_weights(cfg, seed=5)
    prompts = _prompts(cfg, 6, (7, 45, 60))
    ref = ReferenceDecoder(cfg, w)
    ec = EngineConfig(device="cpu", dtype="float32", block_size=16, max_num_seqs=8, max_num_batched_tokens=32,
                      max_model_len=256, use_cuda_graphs=False)
    eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64)
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True, logprobs=5))
    for p, o in zip(prompts, outs):
        logits = ref.forward(torch.tensor(p + o.output_token_ids))
        lp = torch.log_softmax(logits, -1)
        assert o.output_token_ids == [int(x) for x in logits[len(p) - 1:-1].argmax(-1)]
        for i, entry in enumerate(o.logprobs):
            for tok, v in entry["top"].items():
                assert abs(v - float(lp[len(p) - 1 + i, tok])) < 1e-3, (i, tok)


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("expert_parallel", [False, True])
def test_deepseek_tp2_gloo_matches_oracle(expert_parallel):
    """Two ranks: MLA heads, dense MLP and shared experts split by width; experts split by width
    (tensor parallel) or by expert (expert parallel)."""
    from tests.tp_worker import run_tp
    cfg = preset("tiny-deepseek-v3")
    w = init_random_weights(cfg, seed=0)
    prompts = _prompts(cfg, 11, (5, 21))
    ref = ReferenceDecoder(cfg, w)
    expect = [ref.greedy(p, 5)[0] for p in prompts]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=run_tp, args=(r, 2, port, "gloo", "nccl", prompts, 5, q, None, "tiny-deepseek-v3",
                                              expert_parallel)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, toks, err in res:
        assert err is None, err
        assert toks == expect, (rank, toks, expect)


# ---------------------------------------------------------------------------- GPU
def _route_margin(logits, bias, k, n_group, topk_group):
    """Smallest gap at the group and expert cut-offs (rows under 1e-4 may flip between fp32 sums)."""
    s = torch.sigmoid(logits.double())
    c = s + bias.double()
    T, E = c.shape
    gs = c.view(T, n_group, E // n_group).topk(2, -1).values.sum(-1).sort(-1, descending=True).values
    gm = (gs[:, topk_group - 1] - gs[:, topk_group]) if topk_group < n_group else torch.full((T,), 1.0)
    ids, _ = R.moe_route(logits, k, scoring="sigmoid", bias=bias, n_group=n_group, topk_group=topk_group)
    keep = torch.zeros(T, E, dtype=torch.bool)
    groups = torch.zeros(T, n_group, dtype=torch.bool)
    groups.scatter_(1, ids // (E // n_group), True)
    keep = groups.repeat_interleave(E // n_group, 1)
    cm = c.masked_fill(~keep, 0.0).sort(-1, descending=True).values
    em = cm[:, k - 1] - cm[:, k]
    return torch.minimum(gm, em)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 9, 300])
@pytest.mark.parametrize("E,k,n_group,topk_group", [(256, 8, 8, 4), (16, 4, 4, 2), (64, 6, 1, 1)])
def test_sigmoid_router_kernel_gpu(T, E, k, n_group, topk_group):
    """The K12 router in sigmoid mode picks the oracle's experts with its weights, and the MoE
    output (grouped tcgen05 GEMMs + combine) matches on those rows."""
    H, F = 256, 128
    g = torch.Generator().manual_seed(T + E)
    bf = torch.bfloat16
    x = torch.randn(T, H, generator=g).to(bf)
    router = (torch.randn(E, H, generator=g) * 0.1).to(bf)
    bias = torch.randn(E, generator=g) * 0.05
    gu = (torch.randn(E * 2 * F, H, generator=g) * 0.05).to(bf)
    dn = (torch.randn(E * H, F, generator=g) * 0.05).to(bf)
    opt = dict(scoring="sigmoid", n_group=n_group, topk_group=topk_group, scale=2.5)
    rr, rg = {}, {}
    ref = ops.fused_moe(x.float(), router.float(), gu.float(), dn.float(), k, bias=bias, routing=rr, **opt)
    out = ops.fused_moe(x.cuda(), router.cuda(), gu.cuda(), dn.cuda(), k, bias=bias.cuda(), routing=rg, **opt)
    torch.cuda.synchronize()
    ok = _route_margin(x.float() @ router.float().t(), bias, k, n_group, topk_group) > 1e-4
    assert ok.float().mean() > 0.9
    ids_g, ids_r = rg["ids"].cpu().long(), rr["ids"]
    assert torch.equal(ids_g.sort(-1).values[ok], ids_r.sort(-1).values[ok])
    wg = torch.gather(rg["wts"].cpu(), 1, ids_g.sort(-1).indices)
    wr = torch.gather(rr["wts"], 1, ids_r.sort(-1).indices)
    torch.testing.assert_close(wg[ok], wr[ok].float(), rtol=1e-3, atol=1e-4)
    atol = 1e-2 * float(ref.abs().max())
    torch.testing.assert_close(out.float().cpu()[ok], ref.float()[ok], rtol=3e-2, atol=atol)


@pytest.mark.gpu
def test_deepseek_engine_gpu_near_oracle():
    """MLA (D padded 96 -> 128: the tcgen05 prefill and decode kernels), the sigmoid router and the
    shared-expert GEMM served with CUDA graphs: each greedy token is (near) the oracle's argmax."""
    cfg = preset("tiny-deepseek-v3")
    w = init_random_weights(cfg, seed=5)
    prompts = _prompts(cfg, 7, (3, 40, 70))
    ref = ReferenceDecoder(cfg, w)
    ec = EngineConfig(device="cuda", max_num_seqs=8, max_num_batched_tokens=48, max_model_len=512,
                      use_cuda_graphs=True, cuda_graph_batch_sizes=[1, 2, 4, 8])
    eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64)
    outs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    for p, o in zip(prompts, outs):
        logits = ref.forward(torch.tensor(p + o.output_token_ids))
        for i, tok in enumerate(o.output_token_ids):
            row = logits[len(p) - 1 + i]
            assert row[tok] >= row.max() - 0.05 * max(1.0, float(row.abs().max()) / 10), (i, tok)

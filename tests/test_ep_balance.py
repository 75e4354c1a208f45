"""Expert-parallel rebalancing: the placement planner (balanced groups, fewest moves) and live
re-placement of Mixtral / DeepSeek-V3 experts over two gloo ranks (router rows permuted, expert
weights exchanged point to point) with unchanged greedy output."""
import multiprocessing as mp

import numpy as np
import pytest

from gollek_b200.config import preset
from gollek_b200.models.reference import ReferenceDecoder, init_random_weights
from gollek_b200.parallel.ep_balance import balanced_groups, imbalance, moves, plan_placement


def test_plan_balances_and_keeps_experts_in_place():
    loads = np.array([10.0, 9, 8, 7, 1, 1, 1, 1])
    ident = np.arange(8)
    assert imbalance(loads, ident, 2) == pytest.approx(34 / 19)
    groups = balanced_groups(loads, 2)
    assert sorted(len(g) for g in groups) == [4, 4]
    new = plan_placement(loads, ident, 2)
    assert sorted(new.tolist()) == list(range(8))
    assert imbalance(loads, new, 2) == pytest.approx(1.0)
    mv = moves(ident, new, 2)
    assert len(mv) == 4  # two hot experts leave rank 0, two cold ones come in
    for e, src, p_old, p_new in mv:
        assert ident[p_old] == e and new[p_new] == e and src == p_old // 4 != p_new // 4
    # an already balanced placement stays where it is
    assert np.array_equal(plan_placement(np.ones(8), ident, 4), ident)
    # four ranks, skewed loads: max/mean drops below 1.1
    rng = np.random.default_rng(0)
    ld = rng.zipf(1.5, 64).astype(float)
    assert imbalance(ld, plan_placement(ld, np.arange(64), 4), 4) < min(1.1, imbalance(ld, np.arange(64), 4))


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("model", ["tiny-mixtral", "tiny-deepseek-v3"])
def test_ep2_rebalance_keeps_output(model):
    from tests.tp_worker import run_ep_rebalance
    import torch
    cfg = preset(model)
    w = init_random_weights(cfg, seed=0)
    g = torch.Generator().manual_seed(21)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (6, 19)]
    ref = ReferenceDecoder(cfg, w)
    expect = [ref.greedy(p, 4)[0] for p in prompts]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=run_ep_rebalance, args=(r, 2, port, prompts, 4, q, model)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, out, err in res:
        assert err is None, err
        first, second, third, moved, n_rebalances = out
        assert moved > 0
        assert first == expect and second == expect and third == expect, (rank, first, second, third, expect)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [5, 300])
def test_expert_map_kernel_gpu(T):
    """The K12 router with a logical -> physical expert map: weights stored in a permuted order plus
    the map give the unpermuted layer's output (sigmoid group-limited routing), also as EP partials."""
    import torch
    from gollek_b200 import ops
    E, k, H, F = 16, 4, 256, 128
    g = torch.Generator().manual_seed(T)
    bf = torch.bfloat16
    x = torch.randn(T, H, generator=g).to(bf).cuda()
    router = (torch.randn(E, H, generator=g) * 0.1).to(bf).cuda()
    bias = (torch.randn(E, generator=g) * 0.05).cuda()
    gu = (torch.randn(E * 2 * F, H, generator=g) * 0.05).to(bf).cuda()
    dn = (torch.randn(E * H, F, generator=g) * 0.05).to(bf).cuda()
    opt = dict(scoring="sigmoid", bias=bias, n_group=4, topk_group=2, scale=2.5)
    ref = ops.fused_moe(x, router, gu, dn, k, **opt)
    perm = torch.randperm(E, generator=g)  # physical slot p holds logical expert perm[p]
    gu_p = gu.view(E, 2 * F, H)[perm.cuda()].reshape(E * 2 * F, H).contiguous()
    dn_p = dn.view(E, H, F)[perm.cuda()].reshape(E * H, F).contiguous()
    emap = torch.argsort(perm).to(torch.int32).cuda()
    out = ops.fused_moe(x, router, gu_p, dn_p, k, expert_map=emap, **opt)
    torch.cuda.synchronize()
    torch.testing.assert_close(out, ref, rtol=1e-2, atol=1e-3)
    half = E // 2
    parts = [ops.fused_moe(x, router, gu_p[r * half * 2 * F:(r + 1) * half * 2 * F],
                           dn_p[r * half * H:(r + 1) * half * H], k, e0=r * half, e_loc=half, expert_map=emap, **opt)
             for r in range(2)]
    # each partial is rounded to bf16 before the sum: allow a bf16 step of the output's scale
    atol = 1e-2 * float(ref.float().abs().max())
    torch.testing.assert_close((parts[0].float() + parts[1].float()), ref.float(), rtol=2e-2, atol=atol)

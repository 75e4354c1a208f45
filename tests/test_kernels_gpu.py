"""sm_100a kernels against the plain-PyTorch fp32 restatements (gollek_b200.ops.reference)."""
import math

import pytest
import torch

from gollek_b200 import ops
from gollek_b200.ops import reference as R

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _g(seed=0):
    return torch.Generator(device=DEV).manual_seed(seed)


def bf(x):
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("T,d", [(1, 256), (7, 4096), (33, 8192), (5, 1024),
                                 # warp-per-row kernel (T >= 512), 4 / 8 / 16 vectors per lane, ragged d
                                 (1344, 4096), (515, 2048), (600, 1000), (700, 8192)])
def test_rms_norm(T, d):
    x = bf(torch.randn(T, d, device=DEV, generator=_g(1)))
    w = bf(torch.randn(d, device=DEV, generator=_g(2)))
    torch.testing.assert_close(ops.rms_norm(x, w, 1e-5).float(), R.rms_norm(x.float(), w.float(), 1e-5),
                               rtol=2e-2, atol=2e-2)
    res = bf(torch.randn(T, d, device=DEV, generator=_g(3)))
    res_ref = res.clone()
    y = ops.fused_add_rms_norm(x, res, w, 1e-5)
    yr = R.fused_add_rms_norm(x, res_ref, w, 1e-5)
    torch.testing.assert_close(res, res_ref, rtol=0, atol=0)
    torch.testing.assert_close(y.float(), yr.float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("T,d", [(3, 256), (64, 4096), (5, 8192), (1100, 4096)])
def test_layer_norm(T, d):
    """K1 with center: bias-free LayerNorm (Cohere), plain and fused with the residual add."""
    x = bf(torch.randn(T, d, device=DEV, generator=_g(4)) + 0.5)
    w = bf(torch.randn(d, device=DEV, generator=_g(5)))
    torch.testing.assert_close(ops.rms_norm(x, w, 1e-5, center=True).float(),
                               R.rms_norm(x.float(), w.float(), 1e-5, center=True), rtol=2e-2, atol=2e-2)
    res = bf(torch.randn(T, d, device=DEV, generator=_g(6)))
    res_ref = res.clone()
    y = ops.fused_add_rms_norm(x, res, w, 1e-5, center=True)
    yr = R.fused_add_rms_norm(x, res_ref, w, 1e-5, center=True)
    torch.testing.assert_close(res, res_ref, rtol=0, atol=0)
    torch.testing.assert_close(y.float(), yr.float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("H,Hk,D", [(32, 8, 128), (8, 2, 32), (4, 1, 128)])
def test_rope_kv_write(H, Hk, D):
    from gollek_b200.config import preset
    from gollek_b200.models.reference import rope_cos_sin
    cfg = preset("tiny-llama", head_dim=D, rope_theta=500000.0)
    T, NB, bs = 37, 8, 16
    qkv = bf(torch.randn(T, (H + 2 * Hk) * D, device=DEV, generator=_g(4)))
    pos = torch.randint(0, 4000, (T,), device=DEV, generator=_g(5)).int()
    slots = torch.randperm(NB * bs, device=DEV, generator=_g(6))[:T].int()
    slots[3] = -1
    cs = rope_cos_sin(cfg, 4096, device=DEV)
    c1 = torch.zeros(NB, 2, Hk, bs, D, dtype=torch.bfloat16, device=DEV)
    c2 = c1.clone()
    q1 = ops.rope_kv_write(qkv, pos, cs, c1, slots, H, Hk, D)
    q2 = R.rope_kv_write(qkv.float(), pos, cs, c2, slots, H, Hk, D)
    torch.testing.assert_close(q1.float(), q2.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(c1.float(), c2.float(), rtol=2e-2, atol=2e-2)


def _paged_setup(B, Hk, D, lens, NB=None, bs=16, seed=0):
    g = _g(seed)
    max_blocks = max((l + bs - 1) // bs for l in lens)
    NB = NB or B * max_blocks + 3
    cache = bf(torch.randn(NB, 2, Hk, bs, D, device=DEV, generator=g))
    perm = torch.randperm(NB, device=DEV, generator=g)
    bt = torch.zeros(B, max_blocks, dtype=torch.int32, device=DEV)
    k = 0
    for b, l in enumerate(lens):
        n = (l + bs - 1) // bs
        bt[b, :n] = perm[k:k + n].int()
        k += n
    return cache, bt, torch.tensor(lens, dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("H,Hk,D", [(32, 8, 128), (4, 1, 128), (8, 2, 32), (64, 8, 128)])
@pytest.mark.parametrize("splits", [1, 3])
def test_paged_decode_attention(H, Hk, D, splits):
    lens = [1, 17, 100, 513, 40]
    B = len(lens)
    cache, bt, sl = _paged_setup(B, Hk, D, lens, seed=7)
    q = bf(torch.randn(B, H, D, device=DEV, generator=_g(8)))
    scale = 1 / math.sqrt(D)
    out = ops.paged_decode_attention(q, cache, bt, sl, scale, num_splits=splits)
    qsl = torch.arange(B + 1, dtype=torch.int32)
    ref = R.paged_attention(q.float().cpu(), cache.float().cpu(), bt.cpu(), sl.cpu(), qsl, scale)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("H,Hk,D", [(32, 8, 128), (8, 2, 32), (8, 8, 64)])
def test_paged_prefill_attention(H, Hk, D):
    # (prefix already cached, new tokens) per sequence
    specs = [(0, 70), (33, 20), (128, 1), (5, 130)]
    lens = [p + n for p, n in specs]
    B = len(specs)
    cache, bt, sl = _paged_setup(B, Hk, D, lens, seed=9)
    qs = [0]
    for _, n in specs:
        qs.append(qs[-1] + n)
    T = qs[-1]
    q = bf(torch.randn(T, H, D, device=DEV, generator=_g(10)))
    qsl = torch.tensor(qs, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(D)
    out = ops.paged_prefill_attention(q, cache, bt, sl, qsl, scale)
    ref = R.paged_attention(q.float().cpu(), cache.float().cpu(), bt.cpu(), sl.cpu(), qsl.cpu(), scale)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("H,Hk", [(32, 8), (28, 4), (8, 8), (12, 4)])
@pytest.mark.parametrize("emu", [0, 1, 2])
@pytest.mark.parametrize("qscale", [1.0, 6.0])
@pytest.mark.parametrize("D", [128, 64])
def test_prefill_two_tile_kernel(H, Hk, emu, qscale, D):
    """The two-tile tcgen05 prefill kernel at head_dim 128 and 64: head pairs (even GQA groups) and
    row-tile pairs (odd groups), FMA-pipe exponentials, and sharp score distributions (qscale 6) that
    move the running max across tiles (O rescaled in TMEM) against the fp32 oracle."""
    specs = [(0, 300), (1000, 260), (7, 1), (200, 129), (0, 640)]
    lens = [p + n for p, n in specs]
    cache, bt, sl = _paged_setup(len(specs), Hk, D, lens, seed=23)
    qs = [0]
    for _, n in specs:
        qs.append(qs[-1] + n)
    q = bf(torch.randn(qs[-1], H, D, device=DEV, generator=_g(24)) * qscale)
    qsl = torch.tensor(qs, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(D)
    ref = R.paged_attention(q.float().cpu(), cache.float().cpu(), bt.cpu(), sl.cpu(), qsl.cpu(), scale)
    forms = [None, "rows"] + (["pairs"] if (H // Hk) % 2 == 0 else [])
    for form in forms:  # the schedule's own choice, then each work-item form
        work = ops.prefill_schedule(qs, lens, H, Hk, D, form=form).to(DEV)
        assert work.shape[1] == 4
        out = ops.paged_prefill_attention(q, cache, bt, sl, qsl, scale, tiles=work, emu=emu)
        torch.testing.assert_close(out.float().cpu(), ref, rtol=2e-2, atol=2e-2, msg=lambda m: f"{form}: {m}")


@pytest.mark.parametrize("H,Hk", [(32, 8), (4, 1), (64, 8), (8, 8)])
@pytest.mark.parametrize("tensor_cores", [True, False])
def test_paged_prefill_attention_d128(H, Hk, tensor_cores):
    """head_dim 128: the tcgen05 kernel (128-row query tiles, several 128-key KV tiles, cached
    prefixes not on tile boundaries) and the mma.sync kernel against the fp32 oracle."""
    specs = [(0, 70), (33, 20), (128, 1), (5, 130), (300, 400), (1000, 260), (0, 129)]
    lens = [p + n for p, n in specs]
    B = len(specs)
    D = 128
    cache, bt, sl = _paged_setup(B, Hk, D, lens, seed=19)
    qs = [0]
    for _, n in specs:
        qs.append(qs[-1] + n)
    T = qs[-1]
    q = bf(torch.randn(T, H, D, device=DEV, generator=_g(20)))
    qsl = torch.tensor(qs, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(D)
    out = ops.paged_prefill_attention(q, cache, bt, sl, qsl, scale, tensor_cores=tensor_cores)
    ref = R.paged_attention(q.float().cpu(), cache.float().cpu(), bt.cpu(), sl.cpu(), qsl.cpu(), scale)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=2e-2, atol=2e-2)
    # a second call into a view of a larger buffer (the engine's decode-then-prefill layout)
    big = torch.full((T + 3, H, D), float("nan"), device=DEV, dtype=torch.bfloat16)
    qb = torch.zeros(T + 3, H, D, device=DEV, dtype=torch.bfloat16)
    qb[3:] = q
    ops.paged_prefill_attention(qb[3:], cache, bt, sl, qsl, scale, out=big[3:], tensor_cores=tensor_cores)
    torch.testing.assert_close(big[3:].float().cpu(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (77, 384, 256), (128, 4096, 4096), (300, 6144, 4096),
                                   (2048, 1024, 512), (16, 32000, 256)])
@pytest.mark.parametrize("bn", [0, 64, 128, 256])
def test_gemm(M, N, K, bn):
    a = bf(torch.randn(M, K, device=DEV, generator=_g(11)) * 0.5)
    b = bf(torch.randn(N, K, device=DEV, generator=_g(12)) * 0.05)
    y = ops.linear(a, b, bn=bn)
    ref = a.float() @ b.float().t()
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2 * max(1.0, ref.abs().max().item() / 4))


def test_gemm_residual():
    M, N, K = 200, 512, 384
    a = bf(torch.randn(M, K, device=DEV, generator=_g(13)))
    b = bf(torch.randn(N, K, device=DEV, generator=_g(14)) * 0.05)
    r = bf(torch.randn(M, N, device=DEV, generator=_g(15)))
    y = ops.linear(a, b, residual=r)
    torch.testing.assert_close(y.float(), a.float() @ b.float().t() + r.float(), rtol=2e-2, atol=5e-2)


@pytest.mark.parametrize("M,F,K", [(5, 704, 256), (300, 1792, 4096), (64, 14336, 4096)])
def test_gemm_swiglu(M, F, K):
    a = bf(torch.randn(M, K, device=DEV, generator=_g(16)))
    wg = bf(torch.randn(F, K, device=DEV, generator=_g(17)) * 0.03)
    wu = bf(torch.randn(F, K, device=DEV, generator=_g(18)) * 0.03)
    w = ops.interleave_gate_up(wg, wu).contiguous()
    y = ops.linear_swiglu(a, w)
    ref = torch.nn.functional.silu(a.float() @ wg.float().t()) * (a.float() @ wu.float().t())
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=3e-2)


def test_embedding_and_silu():
    table = bf(torch.randn(1000, 256, device=DEV, generator=_g(19)))
    ids = torch.randint(0, 1000, (50,), device=DEV, generator=_g(20)).int()
    torch.testing.assert_close(ops.embedding(ids, table), table[ids.long()])
    x = bf(torch.randn(9, 512, device=DEV, generator=_g(21)))
    torch.testing.assert_close(ops.silu_mul(x).float(), R.silu_mul(x.float()), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("V", [1000, 32000, 128256])
def test_argmax(V):
    logits = bf(torch.randn(33, V, device=DEV, generator=_g(22)))
    out = ops.argmax(logits)
    lf = logits.float()
    ref = torch.stack([torch.nonzero(r == r.max())[0, 0] for r in lf])
    assert torch.equal(out.cpu(), ref.cpu())


def test_sampler_matches_reference():
    B, V = 24, 32000
    logits = torch.randn(B, V, device=DEV, generator=_g(23)) * 3
    g = torch.Generator().manual_seed(0)
    temps = torch.rand(B, generator=g) * 1.5
    temps[0] = 0.0
    top_k = torch.randint(0, 100, (B,), generator=g).int()
    top_p = torch.rand(B, generator=g) * 0.5 + 0.5
    top_p[1] = 1.0
    min_p = torch.rand(B, generator=g) * 0.1
    min_p[2] = 0.0
    seeds = torch.randint(0, 2 ** 31, (B,), generator=g)
    offs = torch.randint(0, 1000, (B,), generator=g)
    out = ops.sample(logits, temps.to(DEV), top_k.to(DEV), top_p.to(DEV), min_p.to(DEV), seeds.to(DEV), offs.to(DEV))
    ref = R.sample(logits.cpu(), temps, top_k, top_p, min_p, seeds, offs)
    agree = (out.cpu() == ref).float().mean().item()
    assert agree >= 0.95, agree


def test_penalties():
    B, V = 4, 500
    logits = torch.randn(B, V, device=DEV, generator=_g(24))
    l2 = logits.clone().cpu()
    trip = torch.tensor([[0, 5, 2], [0, 7, 0], [2, 9, 1], [3, 499, 3]], dtype=torch.int32)
    rep = torch.tensor([1.3, 1.0, 1.1, 0.9])
    fr = torch.tensor([0.5, 0.0, 0.2, 0.1])
    pr = torch.tensor([0.3, 0.0, 0.1, 0.0])
    ops.apply_penalties(logits, trip.to(DEV), rep.to(DEV), fr.to(DEV), pr.to(DEV))
    R.apply_penalties_triples(l2, trip, rep, fr, pr)
    torch.testing.assert_close(logits.cpu(), l2)


@pytest.mark.parametrize("epi", [0, 1, 2])
@pytest.mark.parametrize("splits", [2, 3, 8])
def test_gemm_split_k(epi, splits):
    M, N, K = 200, 1024, 4096
    a = bf(torch.randn(M, K, device=DEV, generator=_g(30)) * 0.5)
    w = bf(torch.randn(N, K, device=DEV, generator=_g(31)) * 0.02)
    r = bf(torch.randn(M, N, device=DEV, generator=_g(32)))
    out = torch.empty(M, N // 2 if epi == 2 else N, dtype=torch.bfloat16, device=DEV)
    ws = torch.empty(splits * M * N, dtype=torch.float32, device=DEV)
    ops.cuda_ext().gemm_bf16(out, a, w, r if epi == 1 else None, epi, 256, None, 0, splits, ws)
    y = a.float() @ w.float().t()
    if epi == 1:
        y = y + r.float()
    elif epi == 2:
        y = R.gemm_swiglu(a.float(), w.float())
    torch.testing.assert_close(out.float(), y, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("M,N,K", [(256, 4096, 14336), (64, 6144, 4096), (256, 28672, 4096), (64, 4096, 14336),
                                   (128, 4096, 4096), (1, 4096, 4096), (200, 4096, 4096)])
@pytest.mark.parametrize("residual", [False, True])
def test_gemm_auto_plan_decode_shapes(M, N, K, residual):
    """The planned tile width / split-K factor at decode sizes (narrow outputs split K over the SMs,
    partials summed with the residual epilogue) against the fp32 oracle."""
    a = bf(torch.randn(M, K, device=DEV, generator=_g(33)) * 0.5)
    w = bf(torch.randn(N, K, device=DEV, generator=_g(34)) * 0.02)
    r = bf(torch.randn(M, N, device=DEV, generator=_g(35))) if residual else None
    bn, splits = ops.gemm_plan(M, N, K, ops.EPI_RESIDUAL if residual else ops.EPI_NONE)
    if N == 4096 and M <= 256 and K >= 4096:
        assert splits >= 2 and bn == 128, (bn, splits)
    y = ops.linear(a, w, residual=r)
    ref = a.float() @ w.float().t() + (r.float() if residual else 0)
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("G", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("splits", [1, 4])
@pytest.mark.parametrize("tc", [True, False])
def test_paged_decode_attention_hd128(G, splits, tc):
    if not tc and G == 16:
        pytest.skip("the CUDA-core decode kernel is instantiated for groups up to 8")
    Hk, D = 2, 128
    H = Hk * G
    lens = [1, 16, 17, 300, 1029, 64]
    B = len(lens)
    cache, bt, sl = _paged_setup(B, Hk, D, lens, seed=40 + G)
    q = bf(torch.randn(B, H, D, device=DEV, generator=_g(41)))
    scale = 1 / math.sqrt(D)
    out = ops.paged_decode_attention(q, cache, bt, sl, scale, num_splits=splits, tensor_cores=tc)
    qsl = torch.arange(B + 1, dtype=torch.int32)
    ref = R.paged_attention(q.float().cpu(), cache.float().cpu(), bt.cpu(), sl.cpu(), qsl, scale)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=2e-2, atol=2e-2)


# ---------------------------------------------------------------------------- family features
@pytest.mark.parametrize("H,Hk,D,tc", [(32, 8, 128, True), (32, 8, 128, False), (8, 2, 64, False),
                                       (4, 2, 256, False), (8, 1, 256, False)])
@pytest.mark.parametrize("window,softcap", [(0, 50.0), (40, 0.0), (100, 30.0)])
def test_attention_window_softcap(H, Hk, D, tc, window, softcap):
    """Sliding window (block skipping + mask) and tanh softcap in the decode and prefill kernels."""
    lens = [1, 17, 100, 513, 40]
    B = len(lens)
    cache, bt, sl = _paged_setup(B, Hk, D, lens, seed=31)
    q = bf(torch.randn(B, H, D, device=DEV, generator=_g(32)))
    scale = 1 / math.sqrt(D)
    qsl = torch.arange(B + 1, dtype=torch.int32)
    if not (tc and D == 128):
        if H // Hk not in (1, 2, 4, 8):
            pytest.skip("group size not instantiated")
    out = ops.paged_decode_attention(q, cache, bt, sl, scale, num_splits=3, tensor_cores=tc, window=window,
                                     softcap=softcap)
    ref = R.paged_attention(q.float().cpu(), cache.float().cpu(), bt.cpu(), sl.cpu(), qsl, scale, window, softcap)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=2e-2, atol=2e-2)
    # prefill with cached prefixes
    specs = [(0, 70), (33, 20), (300, 200), (5, 130)]
    plens = [p + n for p, n in specs]
    cache, bt, sl = _paged_setup(len(specs), Hk, D, plens, seed=33)
    qs = [0]
    for _, n in specs:
        qs.append(qs[-1] + n)
    qp = bf(torch.randn(qs[-1], H, D, device=DEV, generator=_g(34)))
    qslp = torch.tensor(qs, dtype=torch.int32, device=DEV)
    outp = ops.paged_prefill_attention(qp, cache, bt, sl, qslp, scale, tensor_cores=tc, window=window,
                                       softcap=softcap)
    refp = R.paged_attention(qp.float().cpu(), cache.float().cpu(), bt.cpu(), sl.cpu(), qslp.cpu(), scale, window,
                             softcap)
    torch.testing.assert_close(outp.float().cpu(), refp, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("D,rot,bias,qkn", [(128, 128, True, False), (128, 128, False, True), (64, 64, True, True),
                                            (128, 96, False, False), (256, 256, False, True), (32, 32, True, False),
                                            (256, 64, False, False), (128, 32, False, False)])
def test_rope_bias_qknorm_partial(D, rot, bias, qkn):
    from gollek_b200.config import preset
    from gollek_b200.models.reference import rope_cos_sin
    H, Hk, T = 4, 2, 37
    cfg = preset("tiny-llama", head_dim=rot)
    cs = rope_cos_sin(cfg, 512, device=DEV)
    qkv = bf(torch.randn(T, (H + 2 * Hk) * D, device=DEV, generator=_g(40)))
    b = bf(torch.randn((H + 2 * Hk) * D, device=DEV, generator=_g(41))) if bias else None
    qn = bf(1 + 0.1 * torch.randn(D, device=DEV, generator=_g(42))) if qkn else None
    kn = bf(1 + 0.1 * torch.randn(D, device=DEV, generator=_g(43))) if qkn else None
    pos = torch.randint(0, 500, (T,), device=DEV, generator=_g(44)).int()
    cache = torch.zeros(8, 2, Hk, 16, D, device=DEV, dtype=torch.bfloat16)
    slots = torch.randperm(8 * 16, device=DEV, generator=_g(45))[:T].int()
    q = ops.rope_kv_write(qkv, pos, cs, cache, slots, H, Hk, D, bias=b, q_norm=qn, k_norm=kn, norm_eps=1e-6)
    cache_ref = torch.zeros_like(cache).float().cpu()
    qr = R.rope_kv_write(qkv.float().cpu(), pos.cpu(), cs.cpu(), cache_ref, slots.cpu(), H, Hk, D,
                         None if b is None else b.float().cpu(), None if qn is None else qn.float().cpu(),
                         None if kn is None else kn.float().cpu(), 1e-6)
    torch.testing.assert_close(q.float().cpu(), qr.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(cache.float().cpu(), cache_ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("M,N,K", [(7, 512, 256), (300, 2048, 1024), (1024, 6144, 4096)])
@pytest.mark.parametrize("splits", [1, 2])
def test_gemm_geglu(M, N, K, splits):
    a = bf(torch.randn(M, K, device=DEV, generator=_g(50)))
    w = bf(torch.randn(N, K, device=DEV, generator=_g(51)) * 0.05)
    out = torch.empty(M, N // 2, device=DEV, dtype=torch.bfloat16)
    ws = torch.empty(splits * M * N, device=DEV)
    ops.cuda_ext().gemm_bf16(out, a, w, None, ops.EPI_GEGLU, 0, None, 0, splits, ws)
    ref = R.gemm_swiglu(a.float().cpu(), w.float().cpu(), 64, "gelu_tanh")
    torch.testing.assert_close(out.float().cpu(), ref, rtol=2e-2, atol=2e-2)


def test_embedding_scale():
    table = bf(torch.randn(100, 256, device=DEV, generator=_g(60)))
    ids = torch.tensor([3, 99, 0, 42], dtype=torch.int32, device=DEV)
    out = ops.embedding(ids, table, scale=16.0)
    torch.testing.assert_close(out.float(), table[ids.long()].float() * 16.0, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("D", [64, 128, 256])
def test_kv_key_norms(D):
    """K15 block scoring kernel (mean key L2 norm per block) against torch."""
    cache = bf(torch.randn(3, 40, 2, 4, 16, D, device=DEV, generator=_g(50)))
    ids = torch.tensor([39, 0, 17, 5], dtype=torch.int32, device=DEV)
    got = ops.kv_key_norms(cache, ids)
    want = torch.stack([cache[:, b, 0].float().norm(dim=-1).mean() for b in ids.tolist()])
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("M,N,K,epi", [(1344, 4096, 4096, 0), (1344, 4096, 14336, 1), (1344, 28672, 4096, 2),
                                       (1344, 28672, 4096, 3), (1200, 4096, 2048, 0), (2500, 6144, 4096, 1)])
def test_gemm_tail_retile(M, N, K, epi):
    """The tiles past the grid's whole waves run as narrower tiles (a short last wave): equal to
    the fp32 oracle for every epilogue."""
    a = bf(torch.randn(M, K, device=DEV, generator=_g(40)) * 0.5)
    w = bf(torch.randn(N, K, device=DEV, generator=_g(41)) * 0.02)
    r = bf(torch.randn(M, N, device=DEV, generator=_g(42)))
    bn, full, bnt = ops.cuda_ext().gemm_retile(M, N, K, epi)
    if (M, N) in ((1344, 4096), (1200, 4096)):
        assert full > 0 and bnt in (64, 128)  # the shapes this targets are re-tiled
    if epi in (2, 3):
        y = ops.linear_swiglu(a, w, act="silu" if epi == 2 else "gelu_tanh")
        ref = R.gemm_swiglu(a.float(), w.float(), act="silu" if epi == 2 else "gelu_tanh")
    else:
        y = ops.linear(a, w, residual=r if epi == 1 else None)
        ref = a.float() @ w.float().t() + (r.float() if epi == 1 else 0)
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("temp,top_k,top_p,min_p", [(1.0, 0, 1.0, 0.0), (0.7, 20, 1.0, 0.0), (1.3, 0, 0.8, 0.0),
                                                    (1.0, 40, 0.9, 0.05)])
def test_sampler_distribution_matches_filtered_softmax(temp, top_k, top_p, min_p):
    """Empirical token frequencies of many draws (one logits row, 16384 seeds) against the fp32
    softmax over the top-k / min-p / top-p survivors: no draw outside the kept set, and a chi-square
    test that accepts (p > 1e-4; fixed seeds, so the outcome is deterministic)."""
    from scipy.stats import chisquare
    V, N = 64, 16384
    row = torch.randn(V, generator=torch.Generator().manual_seed(50)) * 1.5
    logits = row[None].expand(N, V).contiguous()
    t = torch.full((N,), temp)
    k = torch.full((N,), top_k, dtype=torch.int32)
    p = torch.full((N,), top_p)
    mp = torch.full((N,), min_p)
    seeds = torch.arange(N, dtype=torch.int64) * 7919 + 13
    offs = torch.zeros(N, dtype=torch.int64)
    draws = ops.sample(logits.to(DEV), t.to(DEV), k.to(DEV), p.to(DEV), mp.to(DEV), seeds.to(DEV), offs.to(DEV)).cpu()
    probs = R.filtered_probs(row[None], t[:1], k[:1], p[:1], mp[:1])[0].double()
    assert bool((probs[draws] > 0).all())  # never a filtered-out token
    support = probs > 0
    counts = torch.bincount(draws, minlength=V).double()[support]
    expected = probs[support] * N
    # merge rare tokens into one cell so every expected count is >= 5
    order = expected.argsort(descending=True)
    exp_s, cnt_s = expected[order], counts[order]
    big = exp_s >= 5
    e = torch.cat([exp_s[big], exp_s[~big].sum()[None]]) if (~big).any() else exp_s
    c = torch.cat([cnt_s[big], cnt_s[~big].sum()[None]]) if (~big).any() else cnt_s
    pval = chisquare(c.numpy(), e.numpy() * c.sum().item() / e.sum().item()).pvalue
    assert pval > 1e-4, (pval, c.tolist(), e.tolist())


@pytest.mark.parametrize("T", [1, 37, 300, 1344])
def test_qkv_gemm_with_rope_kv_epilogue(T):
    """The QKV GEMM's RoPE + paged KV-write epilogue equals the unfused projection GEMM followed by
    rope_kv_write: q, and every cache row written (rows with slot -1 are not written)."""
    H, Hk, D, K, NB, BS = 32, 8, 128, 4096, 128, 16
    g = _g(60)
    x = bf(torch.randn(T, K, device=DEV, generator=g) * 0.5)
    w = bf(torch.randn((H + 2 * Hk) * D, K, device=DEV, generator=g) * 0.02)
    pos = torch.randint(0, 900, (T,), device=DEV, generator=g).int()
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, device=DEV).float() / D))
    ang = torch.arange(1024, device=DEV).float()[:, None] * inv[None]
    cos_sin = torch.cat([ang.cos(), ang.sin()], 1).contiguous()
    slots = torch.randperm(NB * BS, device=DEV, generator=g)[:T].int()
    if T > 2:
        slots[1] = -1
    c1 = torch.zeros(NB, 2, Hk, BS, D, dtype=torch.bfloat16, device=DEV)
    c2 = torch.zeros_like(c1)
    q1 = ops.linear_rope_kv(x, w, pos, cos_sin, c1, slots, H, Hk, D)
    qkv = ops.linear(x, w)
    q2 = ops.rope_kv_write(qkv, pos, cos_sin, c2, slots, H, Hk, D)
    torch.testing.assert_close(q1.float(), q2.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(c1.float(), c2.float(), rtol=1e-2, atol=1e-2)
    written = (c1.abs().sum(dim=(1, 2, 4)) > 0).sum().item()
    assert written == int((slots >= 0).sum())

"""Device bounds checks: with a status buffer bound, a block id at or beyond the declared KV pool
(and a slot or token id out of range) is reported in the status word with the first bad index, the
read uses a valid block instead, the KV write is skipped, and the context stays usable. The declared
pool is a 32-block view of a 64-block allocation, so even a missed check reads and writes memory
that exists: the test cannot fault the GPU."""
import math

import pytest
import torch

from gollek_b200 import ops

pytestmark = pytest.mark.gpu
NB_REAL, NB_DECL, BAD = 64, 32, 40


def _cache(dtype=torch.bfloat16):
    full = torch.randn(NB_REAL, 2, 8, 16, 128, device="cuda").to(dtype)
    return full, full[:NB_DECL]


def _table(bad: bool):
    bt = torch.arange(8, dtype=torch.int32, device="cuda").view(2, 4) + 1
    if bad:
        bt[1, 2] = BAD
    return bt


@pytest.mark.parametrize("kind", ["decode_tc", "decode_cuda_core", "decode_fp8", "prefill"])
def test_block_id_beyond_pool_is_reported(kind):
    full, cache = _cache()
    sl = torch.tensor([60, 60], dtype=torch.int32, device="cuda")
    scale = 1 / math.sqrt(128)

    def run(bt):
        if kind == "prefill":
            q = torch.randn(120, 32, 128, device="cuda").bfloat16()
            qs = torch.tensor([0, 60, 120], dtype=torch.int32, device="cuda")
            return ops.paged_prefill_attention(q, cache, bt, sl, qs, scale)
        q = torch.randn(2, 32, 128, device="cuda").bfloat16()
        if kind == "decode_fp8":
            c8 = torch.randint(0, 120, (NB_REAL, 2, 8, 16, 128), dtype=torch.uint8, device="cuda")
            sc = torch.rand(NB_REAL, 2, 8, 16, device="cuda") * 0.01
            return ops.paged_decode_attention(q, c8[:NB_DECL], bt, sl, scale, kv_scales=sc[:NB_DECL])
        return ops.paged_decode_attention(q, cache, bt, sl, scale, tensor_cores=(kind != "decode_cuda_core"))

    with ops.BoundsCheck() as bc:
        run(_table(False))
        torch.cuda.synchronize()
        assert bc.status() == (0, None)
        out = run(_table(True))
        torch.cuda.synchronize()
        flags, idx = bc.status()
    assert flags & ops.BoundsCheck.BOUNDS and idx == BAD
    assert torch.isfinite(out.float()).all()
    run(_table(False))  # the context is still usable
    torch.cuda.synchronize()


def test_kv_write_beyond_pool_is_skipped_and_reported():
    full, cache = _cache()
    T, H, Hk, D = 3, 32, 8, 128
    qkv = torch.randn(T, (H + 2 * Hk) * D, device="cuda").bfloat16()
    pos = torch.arange(T, dtype=torch.int32, device="cuda")
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, device="cuda").float() / D))
    ang = torch.arange(64, device="cuda").float()[:, None] * inv[None]
    cos_sin = torch.cat([ang.cos(), ang.sin()], 1).contiguous()
    slots = torch.tensor([5, BAD * 16 + 3, 7], dtype=torch.int32, device="cuda")
    before = full[BAD].clone()
    with ops.BoundsCheck() as bc:
        ops.rope_kv_write(qkv, pos, cos_sin, cache, slots, H, Hk, D)
        torch.cuda.synchronize()
        flags, idx = bc.status()
    assert flags & ops.BoundsCheck.BOUNDS and idx == BAD
    assert torch.equal(full[BAD], before)  # the out-of-pool write was skipped
    c8 = torch.zeros(NB_REAL, 2, Hk, 16, D, dtype=torch.uint8, device="cuda")
    sc = torch.zeros(NB_REAL, 2, Hk, 16, device="cuda")
    with ops.BoundsCheck() as bc:
        ops.kv_quant_fp8(torch.randn(T, 2, Hk, D, device="cuda").bfloat16(), slots, c8[:NB_DECL], sc[:NB_DECL])
        torch.cuda.synchronize()
        flags, idx = bc.status()
    assert flags & ops.BoundsCheck.BOUNDS and idx == BAD
    assert int(c8[BAD].count_nonzero()) == 0 and int(c8[0].count_nonzero()) > 0


def test_token_id_beyond_vocab_is_reported():
    table = torch.randn(100, 64, device="cuda").bfloat16()
    ids = torch.tensor([3, 250, 7], dtype=torch.int32, device="cuda")
    with ops.BoundsCheck() as bc:
        out = ops.embedding(ids, table)
        torch.cuda.synchronize()
        flags, idx = bc.status()
    assert flags & ops.BoundsCheck.BOUNDS and idx == 250
    assert torch.equal(out[1], table[99])  # clamped to the last row, as without the check

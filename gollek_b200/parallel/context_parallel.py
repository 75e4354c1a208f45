"""Context parallelism: causal attention of one long sequence split over the ranks (ring attention).

The sequence of length S is cut into 2W chunks and rank r holds chunks r and 2W - 1 - r ("zigzag"),
so every rank owns the same amount of causal work. Each rank keeps its queries; the K/V blocks
travel around the ring: at step s, rank r attends to the block that originated at rank (r - s) mod W
and meanwhile sends the block it holds to rank r + 1 and receives the next one from rank r - 1
(non-blocking send / recv, so the transfer overlaps the step's attention). Partial results are
merged exactly with the online-softmax rule (running row max m, denominator l, unnormalised output
o). Causality uses global token positions, so the result equals full causal attention.

Prefills of at most 8K tokens fit one GPU, so the serving path here does not need it; this is the
building block for prompts beyond one GPU's memory or time budget. The reference has none.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def zigzag_indices(S: int, world: int, rank: int) -> torch.Tensor:
    """Global positions of rank ``rank``'s tokens (S a multiple of 2 * world)."""
    if S % (2 * world):
        raise ValueError(f"sequence length {S} must be a multiple of {2 * world}")
    c = S // (2 * world)
    a, b = rank, 2 * world - 1 - rank
    return torch.cat([torch.arange(a * c, (a + 1) * c), torch.arange(b * c, (b + 1) * c)])


def _partial(q, k, v, qpos, kpos, scale):
    """Unnormalised attention of q [Tq, H, D] over k / v [Tk, H, D] with the causal mask by global
    position: (o [Tq, H, D], m [H, Tq], l [H, Tq]); rows with no visible key get m = -inf."""
    s = torch.einsum("qhd,khd->hqk", q.float(), k.float()) * scale
    s = s.masked_fill(kpos[None, None, :] > qpos[None, :, None], float("-inf"))
    m = s.amax(-1)
    p = torch.exp(s - torch.where(torch.isinf(m), torch.zeros_like(m), m)[..., None])
    p = torch.where(torch.isinf(s), torch.zeros_like(p), p)
    return torch.einsum("hqk,khd->qhd", p, v.float()), m, p.sum(-1)


def _merge(acc, part):
    o, m, l = acc
    o2, m2, l2 = part
    mn = torch.maximum(m, m2)
    safe = torch.where(torch.isinf(mn), torch.zeros_like(mn), mn)
    a = torch.where(torch.isinf(m), torch.zeros_like(m), torch.exp(m - safe))
    b = torch.where(torch.isinf(m2), torch.zeros_like(m2), torch.exp(m2 - safe))
    o = o * a.t()[..., None] + o2 * b.t()[..., None]
    return o, mn, l * a + l2 * b


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor,
                   scale: float, group=None) -> torch.Tensor:
    """This rank's causal attention output [T, H, D] for its queries q [T, H, D] against the whole
    sequence, whose keys / values k, v [T, Hk, D] are spread over the ranks of ``group`` (this
    rank's rows at global ``positions`` [T]; every rank holds the same number of rows)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    H, Hk = q.shape[1], k.shape[1]
    rep = H // Hk
    T, D = q.shape[0], q.shape[2]
    acc = (torch.zeros(T, H, D, dtype=torch.float32, device=q.device),
           torch.full((H, T), float("-inf"), device=q.device), torch.zeros(H, T, device=q.device))
    blk = torch.cat([k.reshape(T, -1), v.reshape(T, -1)], 1).contiguous()
    pos = positions.to(torch.int64).contiguous()
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(world))
    for step in range(world):
        recv: Optional[torch.Tensor] = None
        reqs = []
        if step < world - 1:  # pass the block (and its positions) on while attending to it
            recv, recv_pos = torch.empty_like(blk), torch.empty_like(pos)
            reqs = [dist.isend(blk, ranks[nxt], group=group), dist.irecv(recv, ranks[prv], group=group),
                    dist.isend(pos, ranks[nxt], group=group), dist.irecv(recv_pos, ranks[prv], group=group)]
        kk = blk[:, :Hk * D].view(T, Hk, D).repeat_interleave(rep, 1)
        vv = blk[:, Hk * D:].view(T, Hk, D).repeat_interleave(rep, 1)
        acc = _merge(acc, _partial(q, kk, vv, positions, pos, scale))
        for r in reqs:
            r.wait()
        if recv is not None:
            blk, pos = recv, recv_pos
    o, m, l = acc
    return (o / l.t().clamp_min(1e-30)[..., None]).to(q.dtype)


def full_causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """Reference: causal attention over a whole sequence (q [S, H, D], k / v [S, Hk, D])."""
    rep = q.shape[1] // k.shape[1]
    pos = torch.arange(q.shape[0])
    o, m, l = _partial(q, k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1), pos, pos, scale)
    return (o / l.t()[..., None]).to(q.dtype)


def split_sequence(x: torch.Tensor, world: int, rank: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(rank's rows of x [S, ...], their global positions) in the zigzag layout."""
    idx = zigzag_indices(x.shape[0], world, rank)
    return x[idx], idx

"""Token-sharded expert parallelism: the MoE all-to-all dispatch → grouped expert GEMMs → combine
over NVLink (csrc/comm/ep_a2a.cu), and the same protocol restated with ``torch.distributed``
all-to-all for CPU ranks and as the NCCL baseline.

Layout: the rows of a step's tokens are split in contiguous chunks over the ranks (rank r owns
rows [r·c, (r+1)·c), c = ceil(T / world): the sequence-parallel residual of the NVLS collectives);
rank r holds the experts [r·E_loc, (r+1)·E_loc) (physical ids). A MoE layer sends each owned
token's row to the owners of its top-k experts, runs the experts there on the received rows
(grouped per local expert), returns every expert output row to its source, and the source sums
its token's k rows with the routing weights, adds the residual and applies the next RMSNorm.

Reference: the intended dispatch/combine boundary of core/optimization/gollek-plugin-elastic-ep/…/
elasticep/binding/ElasticEpBinding.java:19-45 (ep_dispatch / ep_combine over a token batch) and the
runner's per-layer flow, …/elasticep/ElasticExpertParallelismRunner.java:253-299.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist

HEADER_BYTES = 4096


def owned_rows(T: int, rank: int, world: int) -> Tuple[int, int]:
    """(first row, row count) of the tokens ``rank`` owns."""
    c = (T + world - 1) // world
    r0 = min(T, rank * c)
    return r0, min(T, r0 + c) - r0


def _rnd(n: int, a: int = 4096) -> int:
    return (n + a - 1) // a * a


class EPAllToAll:
    """Expert-parallel MoE layers over NVLink peer memory, on its own multicast-bound symmetric
    region. ``moe(x_own, residual, L, w_next, eps)`` runs one layer and returns the next layer's
    input rows gathered on every rank (a view of the shared region, valid until the next call)."""

    def __init__(self, rank: int, world: int, max_tokens: int, hidden: int, ffn: int, num_experts: int,
                 top_k: int, cpu_group=None, pg=None, timeout_s: float = 5.0):
        from ..native import cuda_ext
        from .symm import SymmHeap
        if num_experts % world:
            raise ValueError(f"{num_experts} experts do not split over {world} ranks")
        self.rank, self.world, self.H, self.F, self.k = rank, world, hidden, ffn, top_k
        self.E, self.e_loc = num_experts, num_experts // world
        self.max_tokens = max_tokens
        self.cap_tok = (max_tokens + world - 1) // world
        self.cap_src = self.cap_tok * top_k
        self.timeout_s = timeout_s
        off = HEADER_BYTES
        lay = {}
        lay["flags"] = off
        off += 4096
        lay["counts"] = off
        off += _rnd(world * self.e_loc * 4)
        lay["recv"] = off
        off += _rnd(world * self.cap_src * hidden * 2)
        lay["meta"] = off
        off += _rnd(world * self.cap_src * 16)
        lay["comb"] = off
        off += _rnd(self.cap_tok * top_k * hidden * 2)
        lay["x"] = off
        off += _rnd(max_tokens * hidden * 2)
        self.heap = SymmHeap(off, rank, world, group=cpu_group, multicast=True, pg=pg)
        if self.heap.mc == 0:
            raise RuntimeError("the expert-parallel all-to-all needs an NVLink multicast object: "
                               + (self.heap.multicast_error or "not available"))
        self.off_x = lay["x"]
        self.layout = [lay["flags"], lay["counts"], lay["recv"], lay["meta"], lay["comb"], lay["x"],
                       self.cap_src, self.cap_tok]
        dev = torch.device("cuda", torch.cuda.current_device())
        C = cuda_ext()
        self.cap_dst = _rnd(world * self.cap_src + 127 * self.e_loc, 128)
        self.ids = torch.empty(self.cap_tok * top_k, dtype=torch.int32, device=dev)
        self.wts = torch.empty(self.cap_tok * top_k, dtype=torch.float32, device=dev)
        self.ws = torch.zeros(C.ep_ws_ints(world, self.e_loc), dtype=torch.int32, device=dev)
        self.scratch = torch.zeros(1024, dtype=torch.int32, device=dev)
        self.xg = torch.empty(self.cap_dst, hidden, dtype=torch.bfloat16, device=dev)
        self.hbuf = torch.empty(self.cap_dst, ffn, dtype=torch.bfloat16, device=dev)
        self.comb_ptr = torch.zeros(self.cap_dst, dtype=torch.int64, device=dev)
        self.tile_group = torch.zeros(self.cap_dst // 128, dtype=torch.int32, device=dev)
        self.num_m = torch.zeros(1, dtype=torch.int32, device=dev)
        self.logits = None
        if world > 1:
            dist.barrier(group=cpu_group)

    def x_view(self, T: int) -> torch.Tensor:
        return self.heap.view(self.off_x, (T, self.H))

    def moe(self, x_own: torch.Tensor, residual: torch.Tensor, router: torch.Tensor, w_gu: torch.Tensor,
            w_down: torch.Tensor, w_next: torch.Tensor, eps: float, T: int, renorm: bool = True,
            scoring: str = "softmax", bias: Optional[torch.Tensor] = None, n_group: int = 1, topk_group: int = 1,
            scale: float = 1.0, expert_map: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One MoE layer on this rank's owned rows ``x_own`` ([Tn, H], normalised). The owned rows of
        ``residual`` ([T, H]) get the layer's output added; returns rms_norm(residual) * w_next for
        all T rows, gathered on every rank."""
        from ..native import cuda_ext
        C = cuda_ext()
        r0, Tn = owned_rows(T, self.rank, self.world)
        if x_own.shape[0] != Tn:
            raise ValueError(f"x_own has {x_own.shape[0]} rows, this rank owns {Tn}")
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the all-to-all buffers ({self.max_tokens})")
        lay = self.layout
        b, mc, r, el, k = self.heap.bases, self.heap.mc, self.rank, self.e_loc, self.k
        if Tn:
            C.moe_route(x_own, router, k, renorm, 0 if scoring == "softmax" else 1, bias, n_group, topk_group,
                        float(scale), expert_map, self.logits, self.ids, self.wts, self.scratch)
        C.ep_dispatch(b, mc, lay, r, el, k, x_own, self.ids, self.ws, self.timeout_s)
        C.ep_compact(b, mc, lay, r, el, k, self.xg, self.comb_ptr, self.tile_group, self.num_m, self.timeout_s)
        C.gemm_grouped(self.hbuf, self.xg, w_gu, 2 * self.F, el, 2, self.tile_group, self.num_m)
        C.gemm_grouped(self.comb_ptr, self.hbuf, w_down, self.H, el, 5, self.tile_group, self.num_m)
        C.ep_signal(b, mc, lay, r, el, k, self.H, self.timeout_s)
        C.ep_combine_norm(b, mc, lay, r, el, k, r0, Tn, self.wts, residual, w_next, float(eps), self.timeout_s)
        from ..ops import LAUNCHES
        LAUNCHES.add(7 if Tn else 6)
        return self.x_view(T)

    def check(self) -> None:
        st = self.heap.status()
        if st:
            raise RuntimeError(f"expert-parallel all-to-all failed on rank {self.rank}: status 0x{st:x}")


# --------------------------------------------------------------------------- torch.distributed restatement
def _all_to_all(out: list, inp: list, group=None) -> None:
    """out[p] <- what rank p sent this rank (``dist.all_to_all`` on NCCL; paired point-to-point
    messages where the backend has no all-to-all, e.g. gloo)."""
    if dist.get_backend(group) == "nccl":
        dist.all_to_all(out, inp, group=group)
        return
    me, world = dist.get_rank(group), dist.get_world_size(group)
    ops = []
    for p in range(world):
        if p == me:
            out[p].copy_(inp[p])
            continue
        if inp[p].numel():
            ops.append(dist.P2POp(dist.isend, inp[p].contiguous(), p, group=group))
        if out[p].numel():
            ops.append(dist.P2POp(dist.irecv, out[p], p, group=group))
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()


def moe_all_to_all_reference(x_own: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor, w_gu_local: torch.Tensor,
                             w_down_local: torch.Tensor, e_loc: int, group=None,
                             expert_fn=None) -> torch.Tensor:
    """The same dispatch → per-owner expert compute → combine protocol with ``dist.all_to_all``
    as the transport (gloo on CPU ranks, or NCCL: the baseline the NVLink kernels are measured
    against). ``ids`` [Tn, k] physical expert ids, ``wts`` [Tn, k]; ``w_gu_local`` /
    ``w_down_local`` the rank's experts in the fused layouts (gate/up interleaved in groups of 64).
    Returns the weighted sum of the k expert outputs per owned token, [Tn, H] fp32."""
    from ..ops import reference as ref
    world = dist.get_world_size(group)
    Tn, k = ids.shape
    H = x_own.shape[1]
    F_ = w_down_local.shape[1]
    flat_ids = ids.reshape(-1).long()
    dest = flat_ids // e_loc
    order = torch.argsort(dest * (Tn * k) + torch.arange(Tn * k, device=ids.device), stable=True)
    send_counts = torch.bincount(dest, minlength=world)
    rows = x_own.index_select(0, (order // k)).contiguous()
    le = (flat_ids % e_loc).index_select(0, order).to(torch.int64)
    # exchange counts, rows and local expert ids
    recv_counts = [torch.zeros(1, dtype=torch.int64, device=x_own.device) for _ in range(world)]
    _all_to_all(recv_counts, [c.reshape(1).to(torch.int64) for c in send_counts], group=group)
    rc = [int(c) for c in recv_counts]
    sc = [int(c) for c in send_counts]
    recv_rows = [torch.empty(n, H, dtype=x_own.dtype, device=x_own.device) for n in rc]
    _all_to_all(recv_rows, list(rows.split(sc)), group=group)
    recv_le = [torch.empty(n, dtype=torch.int64, device=x_own.device) for n in rc]
    _all_to_all(recv_le, list(le.split(sc)), group=group)
    xr = torch.cat(recv_rows) if recv_rows else x_own.new_zeros(0, H)
    lr = torch.cat(recv_le) if recv_le else le.new_zeros(0)
    y = torch.zeros(xr.shape[0], H, dtype=torch.float32, device=x_own.device)
    for e in range(e_loc):
        sel = (lr == e).nonzero().flatten()
        if sel.numel() == 0:
            continue
        xe = xr.index_select(0, sel)
        if expert_fn is not None:
            ye = expert_fn(xe, e)
        else:
            he = ref.gemm_swiglu(xe, w_gu_local[e * 2 * F_:(e + 1) * 2 * F_])
            ye = ref.gemm(he, w_down_local[e * H:(e + 1) * H])
        y.index_copy_(0, sel, ye.float())
    y = y.to(x_own.dtype)
    # return every row to its source, in the order it was sent
    back = [torch.empty(n, H, dtype=x_own.dtype, device=x_own.device) for n in sc]
    _all_to_all(back, list(y.split(rc)), group=group)
    yb = torch.cat(back) if back else y.new_zeros(0, H)
    out_rows = torch.empty_like(yb)
    out_rows.index_copy_(0, order, yb)
    wf = wts.reshape(-1, 1).float()
    return (out_rows.float() * wf).view(Tn, k, H).sum(1)

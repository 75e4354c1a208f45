"""Process-group bootstrap and the NCCL baseline collectives for tensor parallelism.

One process per GPU (``torchrun``/``torch.distributed.run``): RANK / LOCAL_RANK / WORLD_SIZE /
MASTER_ADDR / MASTER_PORT from the environment. NCCL carries tensors (and is the baseline and
correctness oracle for the fused P2P kernels in ``gollek_b200.parallel.symm``); a gloo group
carries host-side control messages (heartbeats, failure notices).

Replaces the reference's cluster plumbing (inference/gollek-cluster/…/GollekClusterManager.java:
26-37 node roles; gRPC hand-off src/main/proto/gollek_internal.proto:9-44), which moves no tensors.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops
from ..models.llama import TPComm


@dataclass
class DistInfo:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    backend: str = "none"

    @property
    def is_main(self) -> bool:
        return self.rank == 0


_INFO = DistInfo()
_CPU_GROUP = None


def init_distributed(backend: Optional[str] = None, timeout_s: float = 120.0) -> DistInfo:
    """Initialise the default process group from the environment (no-op for a single process)."""
    global _INFO, _CPU_GROUP
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws <= 1:
        _INFO = DistInfo()
        return _INFO
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(local)
    if not dist.is_initialized():
        kw = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(**kw)
    _CPU_GROUP = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=timeout_s)) \
        if backend == "nccl" else dist.group.WORLD
    _INFO = DistInfo(rank, ws, local, backend)
    return _INFO


def info() -> DistInfo:
    return _INFO


def cpu_group():
    return _CPU_GROUP


def barrier() -> None:
    if _INFO.world_size > 1:
        dist.barrier()


def shutdown() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()


class NcclComm(TPComm):
    """Tensor-parallel collectives through NCCL (the baseline path): NCCL all-reduce followed by
    the fused residual-add + RMSNorm kernel."""

    def __init__(self, rank: int, size: int, group=None):
        super().__init__(rank, size)
        self.group = group

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def argmax_last(self, t: torch.Tensor, vocab_offset: int) -> torch.Tensor:
        """Greedy ids from vocab shards: all-gather each rank's (max, id) per row, take the best."""
        if self.size == 1:
            return ops.argmax(t)
        v, i = t.float().max(-1)
        pair = torch.stack([v, (i + vocab_offset).float()], -1).contiguous()  # ids < 2^24: exact in fp32
        parts = [torch.empty_like(pair) for _ in range(self.size)]
        dist.all_gather(parts, pair, group=self.group)
        allp = torch.stack(parts, 0)  # [W, B, 2]; ranks hold ascending id ranges, so the first max wins ties
        best = allp[..., 0].argmax(0)
        return allp[..., 1].gather(0, best[None])[0].long()

    def all_gather_last(self, t: torch.Tensor) -> torch.Tensor:
        """[B, V/tp] shards → [B, V] (vocab-parallel lm_head)."""
        if self.size == 1:
            return t
        B, v = t.shape
        if t.is_cuda:
            buf = torch.empty(self.size, B, v, dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(buf, t.contiguous(), group=self.group)
            return buf.permute(1, 0, 2).reshape(B, self.size * v)
        parts = [torch.empty_like(t) for _ in range(self.size)]
        dist.all_gather(parts, t.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)

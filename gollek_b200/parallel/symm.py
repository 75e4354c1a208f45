"""Symmetric-memory heap and the fused tensor-parallel collectives (P2P over NVLink/NVSwitch).

Every rank allocates one region of the same size (``symm_alloc``: cudaMalloc + zero fill), the
CUDA IPC handles are all-gathered over the gloo control group, and each rank maps every peer's
region (``cudaIpcOpenMemHandle``). Region layout:

    [0, 4 KiB)          header: barrier flags (written by peers), arrive counter, epoch, status
    partial[0], [1]     [max_tokens, hidden] bf16 each: the row-parallel GEMM writes its partial
                        sum straight here (alternating per call, so a slow peer still reading
                        call k never sees call k+1's data)
    gather              [max_tokens, hidden] bf16: reduced row chunks (two-shot mode)

``FusedTPComm.allreduce_add_rmsnorm`` replaces "NCCL all-reduce → residual add → RMSNorm" with
one kernel (csrc/comm/symm.cu). Decode-sized batches use the one-shot variant (one barrier,
every rank sums all partials); larger ones the two-shot variant (reduce-scatter by rows, then
all-gather fused with RMSNorm: 2(N-1)/N of the data crosses NVLink per rank instead of N-1).
NCCL (``NcclComm``) remains the baseline and the correctness oracle.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from ..models.llama import TPComm
from ..native import cuda_ext

HEADER_BYTES = 4096
STATUS_PEER_TIMEOUT = 2


class SymmHeap:
    def __init__(self, nbytes: int, rank: int, world: int, group=None, device: Optional[int] = None):
        ext = cuda_ext()
        self.rank, self.world = rank, world
        dev = torch.cuda.current_device() if device is None else device
        self.region = ext.symm_alloc(nbytes, dev)  # uint8 tensor over the local region
        self.nbytes = nbytes
        handle = ext.symm_ipc_handle(self.region)
        handles: List[bytes] = [b""] * world
        if world > 1:
            dist.all_gather_object(handles, handle, group=group)
        else:
            handles = [handle]
        self.peer_ptrs = {}
        bases = []
        for i in range(world):
            if i == rank:
                bases.append(self.region.data_ptr())
            else:
                p = ext.symm_open_peer(handles[i])
                self.peer_ptrs[i] = p
                bases.append(p)
        self.bases = bases

    def view(self, offset: int, shape, dtype=torch.bfloat16) -> torch.Tensor:
        n = 1
        for s in shape:
            n *= s
        nbytes = n * torch.finfo(dtype).bits // 8 if dtype.is_floating_point else n * torch.iinfo(dtype).bits // 8
        return self.region.narrow(0, offset, nbytes).view(dtype).view(*shape)

    def status(self) -> int:
        return int(cuda_ext().symm_status(self.region))

    def close(self) -> None:
        ext = cuda_ext()
        for p in self.peer_ptrs.values():
            ext.symm_close_peer(p)
        self.peer_ptrs = {}


class FusedTPComm(TPComm):
    """Tensor-parallel collectives on the symmetric heap (own kernels), NCCL only for the logits gather."""

    fused_ar = True

    def __init__(self, rank: int, size: int, max_tokens: int, hidden: int, cpu_group=None,
                 timeout_s: float = 5.0, one_shot_max_tokens: int = 128, grid: int = 0):
        super().__init__(rank, size)
        self.max_tokens, self.hidden = max_tokens, hidden
        buf = max_tokens * hidden * 2
        buf = (buf + 4095) // 4096 * 4096
        self.off_p = [HEADER_BYTES, HEADER_BYTES + buf]
        self.off_g = HEADER_BYTES + 2 * buf
        self.heap = SymmHeap(HEADER_BYTES + 3 * buf, rank, size, group=cpu_group)
        self.timeout_s = timeout_s
        self.one_shot_max_tokens = one_shot_max_tokens
        self.calls = 0
        self.grid = grid or torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        if size > 1:
            dist.barrier(group=cpu_group)

    # the GEMM that precedes the next collective writes into this buffer
    def partial_buffer(self, T: int) -> torch.Tensor:
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the symmetric buffer ({self.max_tokens})")
        return self.heap.view(self.off_p[self.calls % 2], (T, self.hidden))

    def _ensure_in_partial(self, h: torch.Tensor) -> None:
        buf = self.partial_buffer(h.shape[0])
        if h.data_ptr() != buf.data_ptr():
            buf.copy_(h)

    def allreduce_add_rmsnorm(self, h: torch.Tensor, residual: torch.Tensor, w: torch.Tensor,
                              eps: float) -> torch.Tensor:
        """residual += all_reduce(h); returns rms_norm(residual) * w (residual updated in place)."""
        T = h.shape[0]
        self._ensure_in_partial(h)
        x = torch.empty_like(residual)
        one_shot = T <= self.one_shot_max_tokens
        cuda_ext().tp_allreduce_add_rmsnorm(self.heap.bases, self.rank, self.off_p[0], self.off_p[1], self.off_g,
                                            self.calls % 2, one_shot, residual, w, x, float(eps), self.timeout_s,
                                            min(self.grid, max(1, T)))
        self.calls += 1
        return x

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return t
        flat = t.reshape(-1)
        n = flat.numel()
        if n % self.hidden == 0 and n // self.hidden <= self.max_tokens and t.dtype == torch.bfloat16:
            self._ensure_in_partial(t.reshape(-1, self.hidden))
            cuda_ext().tp_allreduce(self.heap.bases, self.rank, self.off_p[0], self.off_p[1], self.calls % 2,
                                    t, self.timeout_s, self.grid)
            self.calls += 1
            return t
        dist.all_reduce(t)
        return t

    def all_gather_last(self, t: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return t
        B, v = t.shape
        buf = torch.empty(self.size, B, v, dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(buf, t.contiguous())
        return buf.permute(1, 0, 2).reshape(B, self.size * v)

    def check(self) -> None:
        """Raise if a device-side wait timed out (a peer missed a barrier)."""
        st = self.heap.status()
        if st:
            raise RuntimeError(f"tensor-parallel collective failed on rank {self.rank}: status 0x{st:x} "
                               f"(a peer did not reach the barrier within {self.timeout_s} s)")

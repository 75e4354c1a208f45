"""Symmetric-memory heap and the fused tensor-parallel collectives (P2P over NVLink/NVSwitch).

Every rank allocates one region of the same size (``symm_alloc``: cudaMalloc + zero fill), the
CUDA IPC handles are all-gathered over the gloo control group, and each rank maps every peer's
region (``cudaIpcOpenMemHandle``). Region layout:

    [0, 4 KiB)          header: barrier flags (written by peers), arrive counter, epoch, status
    partial[0], [1]     [max_tokens, hidden] bf16 each: the row-parallel GEMM writes its partial
                        sum straight here (alternating per call, so a slow peer still reading
                        call k never sees call k+1's data)
    gather              [max_tokens, hidden] bf16: reduced row chunks (two-shot mode)
    inbox[0], [1]       [world, push_max_tokens, hidden] bf16 each: the push path's per-source slots
    flags               uint32 [world, push_max_tokens / 32, hidden / 64]: per-tile ready epochs

``FusedTPComm.allreduce_add_rmsnorm`` replaces "NCCL all-reduce → residual add → RMSNorm" with
one kernel (csrc/comm/symm.cu). Decode-sized batches use the one-shot variant (one barrier,
every rank sums all partials); larger ones the two-shot variant (reduce-scatter by rows, then
all-gather fused with RMSNorm: 2(N-1)/N of the data crosses NVLink per rank instead of N-1).
NCCL (``NcclComm``) remains the baseline and the correctness oracle.

Push path (GEMM → all-reduce fused, decode-sized T ≤ ``push_max_tokens``): ``push_linear`` runs
the row-parallel GEMM whose epilogue stores every finished tile into this rank's slot of *every*
rank's inbox over NVLink and raises a ready flag per (source, 32-row group, n-tile); the
following ``allreduce_add_rmsnorm`` waits for the flags of each row group and reduces the
partials from local memory. The NVLink transfer overlaps the GEMM tile by tile and there is no
barrier: the flags are the synchronisation.
"""
from __future__ import annotations

import os
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
                 timeout_s: float = 5.0, one_shot_max_tokens: int = 128, grid: int = 0,
                 push_max_tokens: Optional[int] = None):
        super().__init__(rank, size)
        self.max_tokens, self.hidden = max_tokens, hidden
        rnd = lambda n: (n + 4095) // 4096 * 4096  # noqa: E731
        buf = rnd(max_tokens * hidden * 2)
        self.off_p = [HEADER_BYTES, HEADER_BYTES + buf]
        self.off_g = HEADER_BYTES + 2 * buf
        end = HEADER_BYTES + 3 * buf
        if push_max_tokens is None and os.environ.get("GOLLEK_TP_PUSH_MAX"):
            push_max_tokens = int(os.environ["GOLLEK_TP_PUSH_MAX"])
        if push_max_tokens is None:
            # Off by default: measured at Llama-3-8B TP2 shapes (benchmarks/tp_collectives_bench.py) the
            # push GEMM + local reduce (62.8 us at T=256, 186 us at T=1344) loses to GEMM + the pull
            # kernel (46.2 / 89.8 us; NCCL 52.3 / 96.6): one-row-per-lane 16-byte remote stores and a
            # system-scope fence per tile cost more than the pull kernel's single barrier at these sizes.
            push_max_tokens = 0
        self.push_max = min(push_max_tokens, max_tokens) if (size > 1 and hidden % 8 == 0) else 0
        self.slot = self.push_max * hidden
        inbox = rnd(size * self.slot * 2)
        self.off_inbox = [end, end + inbox]
        self.g_max = max(1, (self.push_max + 31) // 32)
        self.nt_max = (hidden + 63) // 64
        self.off_flags = end + 2 * inbox
        end = self.off_flags + rnd(size * self.g_max * self.nt_max * 4)
        # C5 argmax candidates: [2 parities][world][max_tokens] packed (logit key, id) words
        self.off_cand = end
        end = self.off_cand + rnd(2 * size * max_tokens * 8)
        self.heap = SymmHeap(end, rank, size, group=cpu_group)
        self._pushed = None  # (T, n-tiles) of a push GEMM awaiting its consumer
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

    def push_linear(self, a: torch.Tensor, w: torch.Tensor) -> Optional[torch.Tensor]:
        """Row-parallel ``a @ w.T`` with the push epilogue when it applies (bf16 weight producing
        the hidden width, T within the push buffers); None = use partial_buffer + linear."""
        T = a.shape[0]
        if (not self.push_max or T == 0 or T > self.push_max or not isinstance(w, torch.Tensor) or not a.is_cuda
                or w.dtype != torch.bfloat16 or a.dtype != torch.bfloat16 or w.shape[0] != self.hidden):
            return None
        ext = cuda_ext()
        bn = ext.gemm_pick_bn(T, self.hidden, 0)
        parity = self.calls % 2
        out = self.heap.view(self.off_inbox[parity] + self.rank * self.slot * 2, (T, self.hidden))
        ext.gemm_push(out, a, w, bn, self.heap.bases, self.rank, self.off_inbox[parity], self.slot, self.off_flags,
                      self.g_max, self.nt_max)
        self._pushed = (T, (self.hidden + bn - 1) // bn)
        return out

    def _ensure_in_partial(self, h: torch.Tensor) -> None:
        buf = self.partial_buffer(h.shape[0])
        if h.data_ptr() != buf.data_ptr():
            buf.copy_(h)

    def allreduce_add_rmsnorm(self, h: torch.Tensor, residual: torch.Tensor, w: torch.Tensor,
                              eps: float) -> torch.Tensor:
        """residual += all_reduce(h); returns rms_norm(residual) * w (residual updated in place)."""
        T = h.shape[0]
        if self._pushed is not None:
            Tp, nt = self._pushed
            self._pushed = None
            if Tp != T:
                raise RuntimeError("push GEMM and its all-reduce disagree on the token count")
            x = torch.empty_like(residual)
            cuda_ext().tp_push_allreduce_add_rmsnorm(self.heap.bases, self.rank, self.off_inbox[self.calls % 2],
                                                     self.slot, self.off_flags, self.g_max, self.nt_max, nt,
                                                     residual, w, x, float(eps), self.timeout_s,
                                                     min(self.grid, max(1, T)))
            self.calls += 1
            return x
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

    def argmax_last(self, t: torch.Tensor, vocab_offset: int) -> torch.Tensor:
        """C5: greedy ids from the vocab shards; per row one (logit, id) candidate per rank crosses
        NVLink (P2P kernel) instead of the all-gathered logits."""
        if self.size == 1 or t.dtype != torch.bfloat16 or t.shape[0] > self.max_tokens:
            return super().argmax_last(t, vocab_offset) if self.size == 1 else \
                self.all_gather_last(t).float().argmax(-1)
        out = torch.empty(t.shape[0], dtype=torch.int64, device=t.device)
        cuda_ext().tp_argmax(self.heap.bases, self.rank, t.contiguous(), int(vocab_offset), self.off_cand,
                             self.max_tokens, self.calls % 2, out, self.timeout_s)
        self.calls += 1
        return out

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

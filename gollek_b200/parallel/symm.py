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
    """One region of ``nbytes`` per rank, mapped by every peer.

    Two backends: ``multicast=True`` allocates through torch's symmetric memory (cuMem VMM
    allocations exchanged between the processes and bound to one NVLink multicast object), which
    gives the peer addresses *and* a multicast address ``mc`` for the NVLS kernels; otherwise (or
    when the driver/fabric offers no multicast) a cudaMalloc'd region shared by CUDA IPC handles.
    ``bases[i]`` is rank i's region as mapped in this process; ``mc`` is 0 without multicast.
    """

    def __init__(self, nbytes: int, rank: int, world: int, group=None, device: Optional[int] = None,
                 multicast: bool = False, pg=None):
        self.rank, self.world = rank, world
        dev = torch.cuda.current_device() if device is None else device
        self.nbytes = nbytes
        self.peer_ptrs = {}
        self.mc = 0
        self.backend = "ipc"
        self.multicast_error = ""
        if multicast and world > 1:
            try:
                self._init_multicast(nbytes, rank, dev, pg, group)
                return
            except Exception as e:  # no multicast on this system: P2P kernels over IPC instead
                self.multicast_error = f"{type(e).__name__}: {e}"
        ext = cuda_ext()
        self.region = ext.symm_alloc(nbytes, dev)  # uint8 tensor over the local region
        handle = ext.symm_ipc_handle(self.region)
        handles: List[bytes] = [b""] * world
        if world > 1:
            dist.all_gather_object(handles, handle, group=group)
        else:
            handles = [handle]
        bases = []
        for i in range(world):
            if i == rank:
                bases.append(self.region.data_ptr())
            else:
                p = ext.symm_open_peer(handles[i])
                self.peer_ptrs[i] = p
                bases.append(p)
        self.bases = bases

    def _init_multicast(self, nbytes: int, rank: int, dev: int, pg, group) -> None:
        import torch.distributed._symmetric_memory as symm_mem
        ok, why, t, hdl = False, "", None, None
        try:
            t = symm_mem.empty(nbytes, dtype=torch.uint8, device=torch.device("cuda", dev))
            hdl = symm_mem.rendezvous(t, pg if pg is not None else dist.group.WORLD)
            ptrs = [int(p) for p in hdl.buffer_ptrs]
            # the multicast mapping covers the whole block: use it only when this tensor is the block
            # (offset 0, large enough), so every offset the kernels touch lies inside the mapping
            if int(hdl.multicast_ptr) == 0:  # no multicast object: no NVLS on this system
                why = "no multicast support"
            elif t.data_ptr() != ptrs[rank] or int(hdl.buffer_size) < nbytes or int(getattr(hdl, "offset", 0)):
                why = f"symmetric tensor not at its block start ({t.data_ptr():#x} vs {ptrs[rank]:#x})"
            else:
                ok = True
        except Exception as e:  # noqa: BLE001 - reported through the agreement below
            why = f"{type(e).__name__}: {e}"
        # every rank reaches this agreement, or the ranks would pick different kernels
        flags = [None] * self.world
        dist.all_gather_object(flags, (ok, why), group=group)
        if not all(f[0] for f in flags):
            raise RuntimeError("; ".join(f"rank {i}: {f[1]}" for i, f in enumerate(flags) if not f[0]))
        t.zero_()
        torch.cuda.synchronize(dev)
        self.region = t
        self._symm_handle = hdl  # keeps the mappings alive
        self.bases = [int(p) for p in hdl.buffer_ptrs]
        self.mc = int(hdl.multicast_ptr)
        self.backend = "torch-symm+nvls"

    def view(self, offset: int, shape, dtype=torch.bfloat16) -> torch.Tensor:
        n = 1
        for s in shape:
            n *= s
        nbytes = n * torch.finfo(dtype).bits // 8 if dtype.is_floating_point else n * torch.iinfo(dtype).bits // 8
        return self.region.narrow(0, offset, nbytes).view(dtype).view(*shape)

    def status(self) -> int:
        return int(cuda_ext().symm_status(self.region))

    def close(self) -> None:
        if self.peer_ptrs:
            ext = cuda_ext()
            for p in self.peer_ptrs.values():
                ext.symm_close_peer(p)
        self.peer_ptrs = {}


class FusedTPComm(TPComm):
    """Tensor-parallel collectives on the symmetric heap (own kernels, no NCCL on the step's path)."""

    fused_ar = True

    def __init__(self, rank: int, size: int, max_tokens: int, hidden: int, cpu_group=None,
                 timeout_s: float = 5.0, one_shot_max_tokens: int = 128, grid: int = 0,
                 push_max_tokens: Optional[int] = None, nvls: Optional[bool] = None, pg=None):
        super().__init__(rank, size)
        if nvls is None:
            nvls = os.environ.get("GOLLEK_TP_NVLS", "1") != "0"
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
        self.cpu_group, self.pg = cpu_group, pg
        self.heap = SymmHeap(end, rank, size, group=cpu_group, multicast=nvls, pg=pg)
        # NVLS (multimem through the switch) when the region is bound to a multicast object; the
        # P2P pull kernels otherwise. Two-shot NVLS keeps the residual stream sharded by rows (each
        # rank updates only the rows it reduces) and gathers the normalised rows into `off_g`.
        self.nvls = self.heap.mc != 0
        self.nvls_one_shot_max = int(os.environ.get("GOLLEK_NVLS_ONE_SHOT_MAX", one_shot_max_tokens))
        self._pushed = None  # (T, n-tiles) of a push GEMM awaiting its consumer
        self.timeout_s = timeout_s
        self.one_shot_max_tokens = one_shot_max_tokens
        self.calls = 0
        self.lg_heap: Optional[SymmHeap] = None  # vocab-parallel logits gather (reserve_logits)
        self.lg_cap, self.lg_off, self.lg_calls = 0, [0, 0], 0
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
        if self.nvls:
            return self._nvls_add_rmsnorm(T, residual, w, eps)
        x = torch.empty_like(residual)
        one_shot = T <= self.one_shot_max_tokens
        cuda_ext().tp_allreduce_add_rmsnorm(self.heap.bases, self.rank, self.off_p[0], self.off_p[1], self.off_g,
                                            self.calls % 2, one_shot, residual, w, x, float(eps), self.timeout_s,
                                            min(self.grid, max(1, T)))
        self.calls += 1
        return x

    @property
    def supports_split(self) -> bool:
        return self.nvls

    @property
    def shares_x(self) -> bool:
        """True when ``allreduce_add_rmsnorm`` may return a view of the shared heap (valid until
        the next collective call): callers that keep it longer must copy it."""
        return self.nvls

    def residual_rows(self, T: int) -> slice:
        if self.nvls and T > self.nvls_one_shot_max:  # two-shot NVLS: sequence-parallel residual
            c = (T + self.size - 1) // self.size
            return slice(min(T, self.rank * c), min(T, (self.rank + 1) * c))
        return slice(0, T)

    def _nvls_grid(self, rows: int) -> int:
        # one warp per row, 8 warps per CTA, at most one CTA per SM (the kernel keeps one CTA
        # resident per SM): larger row counts loop, with the next row's reductions prefetched
        return max(1, min(self.grid, (rows + 7) // 8))

    def _nvls_add_rmsnorm(self, T: int, residual: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
        one_shot = T <= self.nvls_one_shot_max
        parity = self.calls % 2
        if one_shot:
            x = torch.empty_like(residual)
            rows = T
        else:
            x = self.heap.view(self.off_g, (T, self.hidden))
            rows = (T + self.size - 1) // self.size
        cuda_ext().tp_nvls_allreduce_add_rmsnorm(self.heap.bases[self.rank], self.heap.mc, self.rank, self.size,
                                                 self.off_p[0], self.off_p[1], self.off_g, parity, 0 if one_shot else 1,
                                                 residual, w, x if one_shot else None, float(eps), self.timeout_s,
                                                 self._nvls_grid(rows))
        self.calls += 1
        return x

    # ---- split batches: the rows of a step in two halves whose collectives overlap the other half's compute
    def half_partial_buffer(self, half: int, T: int) -> torch.Tensor:
        """Where the row-parallel GEMM of half ``half`` (0 or 1) of a split batch writes its partial."""
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the symmetric buffer ({self.max_tokens})")
        return self.heap.view(self.off_p[half], (T, self.hidden))

    def gathered_rows(self, T: int) -> torch.Tensor:
        """The [T, d] buffer the halves' normalised rows are gathered into."""
        return self.heap.view(self.off_g, (T, self.hidden))

    def allreduce_add_rmsnorm_half(self, half: int, row0: int, h: torch.Tensor, residual: torch.Tensor,
                                   w: torch.Tensor, eps: float) -> torch.Tensor:
        """Two-shot NVLS all-reduce + residual + RMSNorm of one half of a split batch: rows
        [row0, row0 + Th) of the step, partial in half buffer ``half``, ``residual`` the half's rows
        (row-sharded inside the half), normalised rows gathered into rows [row0, row0 + Th) of
        ``gathered_rows``. Every call waits for all ranks' stores (barrier C), so each half's
        buffers can be rewritten by its next GEMM as soon as the call completed on this rank."""
        Th = h.shape[0]
        buf = self.half_partial_buffer(half, Th)
        if h.data_ptr() != buf.data_ptr():
            buf.copy_(h)
        x_off = self.off_g + row0 * self.hidden * 2
        cuda_ext().tp_nvls_allreduce_add_rmsnorm(self.heap.bases[self.rank], self.heap.mc, self.rank, self.size,
                                                 self.off_p[half], self.off_p[half], x_off, 0, 1, residual, w, None,
                                                 float(eps), self.timeout_s,
                                                 self._nvls_grid((Th + self.size - 1) // self.size))
        self.calls += 1
        return self.heap.view(x_off, (Th, self.hidden))

    def reduce_scatter_add_rmsnorm(self, h: torch.Tensor, residual: torch.Tensor, w: torch.Tensor,
                                   eps: float) -> torch.Tensor:
        """Sequence-parallel step before an expert-parallel all-to-all: residual rows this rank owns
        (``residual_rows``) += the sum over ranks of h; returns a [T, d] tensor whose owned rows hold
        rms_norm(residual) * w (other rows unset). Needs NVLS."""
        if not self.nvls:
            raise RuntimeError("reduce_scatter_add_rmsnorm needs NVLS (an NVLink multicast object)")
        T = h.shape[0]
        self._ensure_in_partial(h)
        x = torch.empty_like(residual)
        rows = (T + self.size - 1) // self.size
        cuda_ext().tp_nvls_allreduce_add_rmsnorm(self.heap.bases[self.rank], self.heap.mc, self.rank, self.size,
                                                 self.off_p[0], self.off_p[1], self.off_g, self.calls % 2, 2,
                                                 residual, w, x, float(eps), self.timeout_s, self._nvls_grid(rows))
        self.calls += 1
        return x

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return t
        flat = t.reshape(-1)
        n = flat.numel()
        if (self.nvls and n % self.hidden == 0 and n // self.hidden <= self.max_tokens
                and t.dtype == torch.bfloat16):
            rows = n // self.hidden
            self._ensure_in_partial(t.reshape(rows, self.hidden))
            parity = self.calls % 2
            one_shot = rows <= self.nvls_one_shot_max
            grid = max(1, min(self.grid * 4, (n // 8 // (1 if one_shot else self.size) + 1023) // 1024))
            cuda_ext().tp_nvls_allreduce(self.heap.bases[self.rank], self.heap.mc, self.rank, self.size,
                                         self.off_p[0], self.off_p[1], parity, one_shot, n,
                                         t.reshape(-1) if one_shot else None, self.timeout_s, grid)
            self.calls += 1
            if one_shot:
                return t
            return self.heap.view(self.off_p[parity], tuple(t.shape))
        if n % self.hidden == 0 and n // self.hidden <= self.max_tokens and t.dtype == torch.bfloat16:
            self._ensure_in_partial(t.reshape(-1, self.hidden))
            cuda_ext().tp_allreduce(self.heap.bases, self.rank, self.off_p[0], self.off_p[1], self.calls % 2,
                                    t, self.timeout_s, self.grid)
            self.calls += 1
            return t
        if t.dtype == torch.bfloat16 and n % 8 == 0 and t.is_cuda:
            # any other bf16 size: chunks of the partial buffer's capacity, one-shot kernels in place
            work = flat if t.is_contiguous() else flat.clone()
            cap = self.max_tokens * self.hidden // 8 * 8
            for c0 in range(0, n, cap):
                self._all_reduce_flat(work[c0:c0 + cap])
            if work.data_ptr() != t.data_ptr():
                t.copy_(work.view(t.shape))
            return t
        # other dtypes (fp32 statistics such as expert loads) never occur on the step path
        dist.all_reduce(t)
        return t

    def _all_reduce_flat(self, c: torch.Tensor) -> None:
        """In-place sum over ranks of a contiguous bf16 vector of at most the partial buffer's size."""
        m = c.numel()
        parity = self.calls % 2
        self.heap.view(self.off_p[parity], (m,)).copy_(c)
        if self.nvls:
            grid = max(1, min(self.grid * 4, (m // 8 + 1023) // 1024))
            cuda_ext().tp_nvls_allreduce(self.heap.bases[self.rank], self.heap.mc, self.rank, self.size,
                                         self.off_p[0], self.off_p[1], parity, True, m, c, self.timeout_s, grid)
        else:
            cuda_ext().tp_allreduce(self.heap.bases, self.rank, self.off_p[0], self.off_p[1], parity, c,
                                    self.timeout_s, self.grid)
        self.calls += 1

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

    def reserve_logits(self, v_local: int, rows: int = 0) -> None:
        """Symmetric buffers for the vocab-parallel logits gather: two [rows, world * v_local] bf16
        buffers in a second heap (own barrier counters). Collective: every rank calls it at the same
        point of its collective sequence; the first sampled (non-greedy) step does, so greedy-only
        serving never allocates them."""
        if self.size == 1 or self.lg_heap is not None:
            return
        rows = rows or int(os.environ.get("GOLLEK_TP_LOGITS_ROWS", min(self.max_tokens, 256)))
        self.lg_cap = (rows * self.size * v_local * 2 + 4095) // 4096 * 4096
        self.lg_off = [HEADER_BYTES, HEADER_BYTES + self.lg_cap]
        self.lg_heap = SymmHeap(HEADER_BYTES + 2 * self.lg_cap, self.rank, self.size, group=self.cpu_group,
                                multicast=self.nvls, pg=self.pg)

    def all_gather_last(self, t: torch.Tensor) -> torch.Tensor:
        """[B, v] vocab shards → [B, world * v] with the column-gather kernel (NVLS multicast stores,
        or P2P stores). Rows that fit one buffer come back as a view of the symmetric buffer, valid
        until the second-next gather (the caller consumes them within the step); more rows are
        gathered in chunks into a fresh tensor. Any dtype is moved as its bf16-sized units."""
        if self.size == 1:
            return t
        if self.lg_heap is None:
            self.reserve_logits(t.shape[1] * t.element_size() // 2)
        B, v = t.shape
        src = t.contiguous()
        units = src if src.dtype == torch.bfloat16 else src.view(torch.bfloat16)
        vu = units.shape[1]
        ld = vu * self.size
        per = self.lg_cap // (ld * 2)
        if per < 1:
            raise ValueError(f"logits row of {ld} units exceeds the gather buffer")
        ext = cuda_ext()
        nvls = self.lg_heap.mc != 0 and vu % 8 == 0
        out = None if B <= per else torch.empty(B, ld, dtype=torch.bfloat16, device=t.device)
        res = None
        for r0 in range(0, B, per):
            n = min(per, B - r0)
            parity = self.lg_calls % 2
            vec = n * vu // 8
            grid = (max(1, min(2 * self.grid, (vec + 1023) // 1024)) if nvls
                    else max(1, min(self.grid, (vec + 2047) // 2048)))
            ext.tp_gather_cols(self.lg_heap.bases, self.lg_heap.mc if nvls else 0, self.rank, units[r0:r0 + n],
                               self.lg_off[parity], ld, self.timeout_s, grid)
            self.lg_calls += 1
            view = self.lg_heap.view(self.lg_off[parity], (n, ld))
            if out is None:
                res = view
            else:
                out[r0:r0 + n].copy_(view)
        res = res if out is None else out
        return res if t.dtype == torch.bfloat16 else res.view(t.dtype)

    def check(self) -> None:
        """Raise if a device-side wait timed out (a peer missed a barrier)."""
        st = self.heap.status() | (self.lg_heap.status() if self.lg_heap is not None else 0)
        if st:
            raise RuntimeError(f"tensor-parallel collective failed on rank {self.rank}: status 0x{st:x} "
                               f"(a peer did not reach the barrier within {self.timeout_s} s)")

"""KV-cache eviction under memory pressure (EVICPRESS-style keep / drop policy).

Reference behaviour: core/optimization/gollek-plugin-evicpress/…/evicpress/KvCacheEvicpressService.java
(applyEvictionPolicy :118-208: when pool utilisation passes a threshold, score a request's blocks,
protect blocks on the attention route, and act on the lowest-scored ones; REST stats / retention /
evict-now :212-243) and the kernels bound in …/binding/EvicpressBinding.java:17-50 (block scoring,
in-place compression, route protection; CPU fallback EvicpressCpuFallback.java:22-67: 0.5 recency
+ 0.5 attention, last 20 % of blocks protected).

Design here:
  score    K15 kernel ``ops.kv_key_norms``: mean key L2 norm of each block over all layers and KV
           heads (one pass over the block's keys in HBM). Low-norm keys draw the most attention
           (Devoto et al. 2024), so a block's importance is 0.5 * recency + 0.5 * (1 - its norm's
           rank among the sequence's blocks).
  protect  the first ``sink`` blocks (attention sinks) and the most recent ``recent`` fraction
           (which always contains the block being written) are never dropped.
  act      the lowest-importance unprotected blocks are dropped until the sequence keeps
           ``retention_target`` of its blocks. Dropping is a block-table edit in the native
           allocator (``SeqTables.drop``): later tokens keep their positions (RoPE), their KV slots
           shift down, and attention runs over the kept blocks. Compression to a narrower dtype is
           not offered: the attention kernels read bf16 blocks only.
Eviction is approximate attention and off by default. Sequences that lost blocks stop adding blocks
to the prefix cache (their block hashes no longer describe a contiguous prefix).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List

import torch

from .. import ops


@dataclass
class EvictionStats:
    cycles: int = 0
    sequences: int = 0
    blocks_scored: int = 0
    blocks_kept: int = 0
    blocks_dropped: int = 0
    blocks_protected: int = 0

    def as_dict(self) -> Dict[str, int]:
        return dict(vars(self))


@dataclass
class KVEvictor:
    threshold: float = 0.85
    retention_target: float = 0.6
    sink_blocks: int = 1
    recent: float = 0.2
    min_blocks: int = 8
    stats: EvictionStats = field(default_factory=EvictionStats)

    def __post_init__(self):
        if not 0.0 < self.retention_target <= 1.0:
            raise ValueError("retention_target must be in (0, 1]")

    # ------------------------------------------------------------------ policy pieces
    def protect_mask(self, nb: int) -> List[bool]:
        """Blocks that must stay: attention sinks and the recent window (incl. the last block)."""
        keep_recent = max(1, math.ceil(self.recent * nb))
        return [i < self.sink_blocks or i >= nb - keep_recent for i in range(nb)]

    @staticmethod
    def importance(norms: torch.Tensor) -> torch.Tensor:
        """0.5 * recency + 0.5 * (1 - rank of the key norm), per block of one sequence."""
        nb = norms.numel()
        recency = torch.arange(nb, dtype=torch.float32) / max(1, nb - 1)
        rank = torch.empty(nb, dtype=torch.float32)
        rank[norms.float().cpu().argsort()] = torch.arange(nb, dtype=torch.float32) / max(1, nb - 1)
        return 0.5 * recency + 0.5 * (1.0 - rank)

    def plan(self, norms: torch.Tensor) -> List[int]:
        """Block indices to drop for one sequence given its blocks' key norms."""
        nb = norms.numel()
        keep_n = max(1, math.ceil(self.retention_target * nb))
        protect = self.protect_mask(nb)
        imp = self.importance(norms)
        order = sorted((i for i in range(nb) if not protect[i]), key=lambda i: float(imp[i]))
        n_drop = max(0, nb - keep_n)
        self.stats.blocks_protected += sum(protect)
        return sorted(order[:n_drop])

    # ------------------------------------------------------------------ engine hook
    def over_threshold(self, kv) -> bool:
        return kv.usage() >= self.threshold

    def run(self, engine, force: bool = False) -> int:
        """Drop blocks of the longest running sequences until the pool is under the threshold
        (or, with ``force``, one pass over every eligible sequence). Returns blocks freed."""
        kv = engine.kv
        if engine.handoff_hook is not None:  # a P/D hand-off ships whole block tables
            return 0
        if not force and not self.over_threshold(kv):
            return 0
        self.stats.cycles += 1
        freed = 0
        cache = engine.kv_cache
        running = [q for q in engine.scheduler.running if kv.has(q)]
        for seq in sorted(running, key=lambda q: -kv.tables.num_blocks(q.seq_id)):
            if not force and not self.over_threshold(kv):
                break
            blocks = kv.tables.blocks(seq.seq_id)
            nb = len(blocks)
            if nb < self.min_blocks:
                continue
            norms = ops.kv_key_norms(cache, torch.tensor(blocks, dtype=torch.int32))
            drop = self.plan(norms)
            self.stats.blocks_scored += nb
            if not drop:
                continue
            freed += kv.drop_blocks(seq, drop)
            self.stats.sequences += 1
            self.stats.blocks_dropped += len(drop)
            self.stats.blocks_kept += nb - len(drop)
        return freed

"""Paged KV-cache manager: device pool + native block allocator + prefix cache.

The device pool is one tensor ``[layers, num_blocks, 2, kv_heads, block_size, head_dim]``
sized from free HBM (or an explicit block count). Block bookkeeping is the native
``BlockPool`` / ``SeqTables`` (csrc/host/block_allocator.cpp); this class adds the prefix
cache policy: a chain hash over each full block of tokens (seeded by the LoRA id) so two
requests with the same prompt prefix and adapter share KV blocks.

Reference behaviour covered: core/optimization/gollek-plugin-kv-cache/…/kvcache/
PagedKVCacheManager.java:79-222 (allocateForPrefill / appendToken / freeRequest / stats,
exhaustion errors :127-131) and the prompt cache's block-aligned rolling prefix hash
(core/optimization/gollek-plugin-prompt-cache/…/cache/PromptPrefixHasher.java,
PagedKVCacheManagerExtension.java).
"""
from __future__ import annotations

from typing import List, Optional

import torch

from ..native import host_ext
from .sequence import Sequence

_MASK63 = (1 << 63) - 1


def _salt(seq) -> object:
    """Hash salt of a sequence's blocks: its LoRA adapter, and for multimodal prompts the image
    content (placeholder token ids are equal for every image)."""
    return seq.lora_id if not getattr(seq, "cache_salt", 0) else (seq.lora_id, seq.cache_salt)


def block_hash(parent: int, tokens: List[int], salt: object = 0) -> int:
    """Chain hash of one full block (stable within a process; 63-bit, non-negative)."""
    return hash((parent, salt, tuple(tokens))) & _MASK63


class KVCacheManager:
    def __init__(self, num_blocks: int, block_size: int = 16, enable_prefix_caching: bool = True,
                 state_slots: int = 0):
        h = host_ext()
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.pool = h.BlockPool(num_blocks, block_size)
        self.tables = h.SeqTables(self.pool)
        self.enable_prefix_caching = enable_prefix_caching
        self.prefix_hits = 0
        self.prefix_queries = 0
        # recurrent-state slots of hybrid GDN models: taken with the sequence's block table
        self.free_state_slots = list(range(state_slots - 1, -1, -1)) if state_slots else None

    # ------------------------------------------------------------------ stats
    def num_free_blocks(self) -> int:
        return self.pool.num_free()

    def usage(self) -> float:
        return 1.0 - self.pool.num_free() / max(1, self.num_blocks)

    def blocks_for(self, n_tokens: int) -> int:
        return (n_tokens + self.block_size - 1) // self.block_size

    # ------------------------------------------------------------------ sequences
    def add(self, seq: Sequence) -> None:
        self.tables.add(seq.seq_id)
        seq.block_hashes = []
        if self.free_state_slots is not None:
            if not self.free_state_slots:
                raise RuntimeError("no recurrent-state slot free (more running sequences than max_num_seqs)")
            seq.state_slot = self.free_state_slots.pop()

    def free(self, seq: Sequence) -> None:
        self.tables.remove(seq.seq_id)
        seq.block_hashes = []
        if self.free_state_slots is not None and seq.state_slot >= 0:
            self.free_state_slots.append(seq.state_slot)
            seq.state_slot = -1

    def has(self, seq: Sequence) -> bool:
        return self.tables.has(seq.seq_id)

    def match_prefix(self, seq: Sequence) -> int:
        """Reuse cached blocks for the longest cached full-block prefix; returns tokens reused.

        At least one prompt token is always left to compute (its logits seed decoding).
        """
        if not self.enable_prefix_caching or seq.num_computed_tokens != 0:
            return 0
        bs = self.block_size
        max_blocks = (seq.num_tokens - 1) // bs
        parent = 0
        reused = 0
        for i in range(max_blocks):
            self.prefix_queries += 1
            hsh = block_hash(parent, seq.tokens(i * bs, (i + 1) * bs), _salt(seq))
            b = self.pool.lookup(hsh)
            if b < 0:
                break
            self.prefix_hits += 1
            self.tables.append_block(seq.seq_id, b)
            seq.block_hashes.append(hsh)
            parent = hsh
            reused += bs
        return reused

    def ensure(self, seq: Sequence, total_tokens: int) -> bool:
        return self.tables.ensure_capacity(seq.seq_id, total_tokens)

    def blocks_needed(self, seq: Sequence, total_tokens: int) -> int:
        return self.tables.blocks_needed(seq.seq_id, total_tokens)

    def drop_blocks(self, seq: Sequence, idx: List[int]) -> int:
        """KV eviction: release the blocks at table indices ``idx`` (never the last block); later
        tokens keep their positions and attend over the kept blocks. Returns blocks freed."""
        if not idx:
            return 0
        n = self.tables.drop(seq.seq_id, list(idx))
        del seq.block_hashes[min(idx):]
        return n

    def dropped_tokens(self, seq: Sequence) -> int:
        return self.tables.dropped(seq.seq_id) if self.tables.has(seq.seq_id) else 0

    def commit_full_blocks(self, seq: Sequence) -> None:
        """Register newly completed full blocks of ``seq`` in the prefix cache."""
        if not self.enable_prefix_caching:
            return
        bs = self.block_size
        full = seq.num_computed_tokens // bs
        if full <= len(seq.block_hashes) or self.tables.dropped(seq.seq_id):
            return
        blocks = self.tables.blocks(seq.seq_id)
        parent = seq.block_hashes[-1] if seq.block_hashes else 0
        for i in range(len(seq.block_hashes), full):
            hsh = block_hash(parent, seq.tokens(i * bs, (i + 1) * bs), _salt(seq))
            self.pool.insert(blocks[i], hsh)
            seq.block_hashes.append(hsh)
            parent = hsh


def allocate_kv_cache(shape: tuple, dtype: torch.dtype, device) -> torch.Tensor:
    """Zero-initialised so never-written slots hold finite values."""
    return torch.zeros(shape, dtype=dtype, device=device)


def num_blocks_from_memory(bytes_per_block: int, weight_bytes: int, device, utilization: float,
                           reserve_bytes: int = 4 << 30) -> int:
    """How many KV blocks fit in ``utilization`` of HBM after weights and activations."""
    free, total = torch.cuda.mem_get_info(device)
    budget = int(total * utilization) - (total - free) - reserve_bytes
    return max(16, budget // bytes_per_block)

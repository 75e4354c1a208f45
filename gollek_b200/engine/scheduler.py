"""Continuous-batching scheduler with chunked prefill, prefix reuse and preemption.

Each ``schedule()`` call builds one engine step under a token budget
(``max_num_batched_tokens``) and a sequence cap (``max_num_seqs``):

1. every running decode sequence gets one token (KV slot allocated first; when the pool is
   exhausted the most recently admitted running sequence is preempted — its blocks are freed
   and it re-enters the front of the waiting queue to be recomputed);
2. running sequences still in (chunked) prefill get the next prompt chunk;
3. waiting sequences are admitted in FCFS order while budget, sequence slots and KV blocks
   last. With ``scheduling_policy="wait"`` admission also requires the sequence's predicted
   total footprint (prompt + predicted output, from the native ``LengthPredictor``) to fit in
   ``wait_admission_fraction`` of the pool (the reference's WAIT rule).

Decode sequences come first in the step so the model runner can hand them to the decode
attention kernel and the rest to the prefill kernel.

Reference behaviour: inference/gollek-runtime-inference/…/batch/ContinuousBatchScheduler.java:
77-175,196-212,383-468 (iteration loop, KV-pressure rejection, retire finished);
core/optimization/gollek-plugin-wait-scheduler/…/ContinuousBatchingScheduler.java:288-320
(admission by free-block math) and …/waitscheduler/FluidInferenceScheduler.java:1-60 (WAIT:
admit iff used + E[blocks] <= total * fraction, E from ForeLen).
"""
from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional, Tuple

from ..config import EngineConfig
from .kv_cache import KVCacheManager
from .sequence import Sequence, SeqStatus


@dataclass
class ScheduledChunk:
    seq: Sequence
    start: int          # first absolute position processed this step
    num_tokens: int     # tokens processed this step
    sample: bool        # produce a token at the end of this chunk
    # speculative decoding: input tokens that are not (yet) the sequence's own (drafts), and the
    # number of trailing draft tokens whose verification needs logits at every position
    tokens: Optional[List[int]] = None
    verify: int = 0


@dataclass
class SchedulerOutput:
    decode: List[ScheduledChunk] = field(default_factory=list)
    prefill: List[ScheduledChunk] = field(default_factory=list)
    preempted: List[Sequence] = field(default_factory=list)

    @property
    def chunks(self) -> List[ScheduledChunk]:
        return self.decode + self.prefill

    @property
    def num_tokens(self) -> int:
        return len(self.decode) + sum(c.num_tokens for c in self.prefill)

    @property
    def empty(self) -> bool:
        return not self.decode and not self.prefill


class Scheduler:
    def __init__(self, cfg: EngineConfig, kv: KVCacheManager, predictor=None):
        self.cfg = cfg
        self.kv = kv
        self.waiting: Deque[Sequence] = deque()
        self.running: List[Sequence] = []
        self.predictor = predictor
        self.num_preemptions = 0

    # ------------------------------------------------------------------ queue management
    def add(self, seq: Sequence) -> None:
        max_len = self.cfg.max_model_len
        if seq.num_prompt_tokens + 1 > max_len:
            raise ValueError(f"prompt of {seq.num_prompt_tokens} tokens exceeds max_model_len {max_len}")
        if self.kv.blocks_for(seq.num_prompt_tokens + 1) > self.kv.num_blocks:
            raise ValueError("prompt does not fit in the KV cache")
        if self.predictor is not None:
            seq.predicted_len = float(self.predictor.predict(float(seq.num_prompt_tokens)))
        self.waiting.append(seq)

    def abort(self, request_id: str) -> Optional[Sequence]:
        for q in (self.running, self.waiting):
            for s in list(q):
                if s.request_id == request_id:
                    q.remove(s)
                    if self.kv.has(s):
                        self.kv.free(s)
                    s.status = SeqStatus.FINISHED_ABORTED
                    return s
        return None

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    # ------------------------------------------------------------------ scheduling
    def _preempt(self, seq: Sequence, out: SchedulerOutput) -> None:
        self.running.remove(seq)
        self.kv.free(seq)
        seq.num_computed_tokens = 0
        seq.status = SeqStatus.WAITING
        seq.num_preemptions += 1
        self.num_preemptions += 1
        self.waiting.appendleft(seq)
        out.preempted.append(seq)

    def _wait_admits(self, seq: Sequence) -> bool:
        if self.cfg.scheduling_policy != "wait" or seq.predicted_len is None:
            return True
        used = self.kv.num_blocks - self.kv.num_free_blocks()
        expect = self.kv.blocks_for(seq.num_prompt_tokens + int(seq.predicted_len))
        return used + expect <= self.cfg.wait_admission_fraction * self.kv.num_blocks

    def schedule(self) -> SchedulerOutput:
        out = SchedulerOutput()
        budget = self.cfg.max_num_batched_tokens
        # 1) decodes (oldest first; preempt from the back on KV exhaustion)
        for seq in list(self.running):
            if seq.status is not SeqStatus.RUNNING or not seq.is_decode:
                continue
            if len(seq.output_token_ids) >= seq.params.max_tokens or seq.num_tokens >= self.cfg.max_model_len:
                continue  # async scheduling: at its limit with a token in flight; finishes on read-back
            while not self.kv.ensure(seq, seq.num_tokens):
                victim = self.running[-1]
                self._preempt(victim, out)
                if victim is seq:
                    break
            if seq.status is not SeqStatus.RUNNING:
                continue
            out.decode.append(ScheduledChunk(seq, seq.num_computed_tokens, 1, True))
            budget -= 1
        # 2) running sequences mid-prefill
        for seq in list(self.running):
            if budget <= 0:
                break
            if seq.is_decode or seq.status is not SeqStatus.RUNNING:
                continue
            remaining = seq.num_tokens - seq.num_computed_tokens
            n = min(remaining, budget)
            if not self.kv.ensure(seq, seq.num_computed_tokens + n):
                continue
            out.prefill.append(ScheduledChunk(seq, seq.num_computed_tokens, n, n == remaining))
            budget -= n
        # 3) admit waiting sequences
        quotas = self.cfg.tenant_quotas
        usage = self._tenant_usage() if quotas else None
        skipped = []  # waiting requests of tenants at their quota keep their place in the queue
        while self.waiting and budget > 0 and len(self.running) < self.cfg.max_num_seqs:
            seq = self.waiting[0]
            if seq.pending:  # preempted with a token still in flight: admit after read-back
                break
            if usage is not None and not self._tenant_admits(seq, usage):
                skipped.append(self.waiting.popleft())
                continue
            if not self._wait_admits(seq):
                break
            self.kv.add(seq)
            reused = self.kv.match_prefix(seq)
            seq.num_computed_tokens = reused
            remaining = seq.num_tokens - reused
            n = min(remaining, budget)
            if not self.kv.ensure(seq, reused + n):
                self.kv.free(seq)
                seq.num_computed_tokens = 0
                break
            self.waiting.popleft()
            seq.status = SeqStatus.RUNNING
            if seq.scheduled_time is None:
                seq.scheduled_time = time.perf_counter()
            self.running.append(seq)
            out.prefill.append(ScheduledChunk(seq, reused, n, n == remaining))
            budget -= n
            if usage is not None and seq.tenant:
                u = usage.setdefault(seq.tenant, [0, 0])
                u[0] += 1
                u[1] += self.kv.tables.num_blocks(seq.seq_id)
        for seq in reversed(skipped):
            self.waiting.appendleft(seq)
        return out

    def _tenant_usage(self) -> Dict[str, List[int]]:
        use: Dict[str, List[int]] = {}
        for s in self.running:
            if s.tenant:
                u = use.setdefault(s.tenant, [0, 0])
                u[0] += 1
                u[1] += self.kv.tables.num_blocks(s.seq_id) if self.kv.has(s) else 0
        return use

    def _tenant_admits(self, seq, usage) -> bool:
        q = self.cfg.tenant_quotas.get(seq.tenant) if seq.tenant else None
        if not q:
            return True
        run, blocks = usage.get(seq.tenant, [0, 0])
        if run >= q.get("max_running", 1 << 30):
            return False
        need = (seq.num_tokens + self.kv.block_size - 1) // self.kv.block_size
        return blocks + need <= q.get("max_kv_blocks", 1 << 60)

    # ------------------------------------------------------------------ post-step update
    def finish(self, seq: Sequence, status: SeqStatus) -> None:
        seq.status = status
        if seq in self.running:
            self.running.remove(seq)
        if self.kv.has(seq):
            self.kv.free(seq)
        if self.predictor is not None and status != SeqStatus.FINISHED_ABORTED:
            self.predictor.observe(float(seq.num_prompt_tokens), float(len(seq.output_token_ids)))

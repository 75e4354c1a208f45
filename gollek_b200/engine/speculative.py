"""Speculative decoding inside continuous batching.

Each step, every running decode sequence may receive up to ``k`` draft tokens from a proposer:

* ``ngram`` — prompt lookup: the longest suffix of the sequence that occurred earlier proposes
  the tokens that followed it (native, ``csrc/host/spec_ngram.cpp``); no second model.
* ``draft`` — a small draft model (same tokenizer) decodes ``k`` greedy tokens. Its paged KV
  cache has the target's block layout and shares the target's block tables, so it needs no
  allocator of its own.

The target then verifies ``[last token] + drafts`` of every such sequence in one forward: each is
a varlen chunk of ``1 + k`` query tokens over its cached prefix (the prefill attention path), with
logits at every position. Acceptance is exact for greedy and sampled requests: with deterministic
proposals, draft ``x`` at position i is kept with probability p_i(x) (greedy: iff it is the
argmax), the first rejected position is resampled from p_i with ``x`` removed, and if every draft
survives one bonus token is drawn from p_k — so outputs follow the target distribution exactly. KV
written for rejected drafts lies beyond the sequence's computed length and is overwritten later.

Mirrors the draft → verify → accept → resample loop of the reference
(inference/gollek-runtime-inference/…/runtime/inference/speculative/SpeculativeDecoder.java:1-60,124),
batched over the running sequences instead of one request at a time.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from .. import ops
from ..ops import reference as ref
from .sequence import Sequence


@dataclass
class SpecStats:
    steps: int = 0
    proposed: int = 0
    accepted: int = 0

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / self.proposed if self.proposed else 0.0


class NgramProposer:
    def __init__(self, k: int, min_n: int = 1, max_n: int = 4):
        from ..native import host_ext
        self.k, self.min_n, self.max_n = k, min_n, max_n
        self.host = host_ext()

    def propose(self, seqs: List[Sequence], ks: List[int]) -> List[List[int]]:
        if not seqs:
            return []
        toks = [s.prompt_token_ids + s.output_token_ids for s in seqs]
        offs = [0]
        for t in toks:
            offs.append(offs[-1] + len(t))
        flat = torch.tensor([x for t in toks for x in t], dtype=torch.int32)
        d, c = self.host.ngram_propose(flat, torch.tensor(offs, dtype=torch.int64), self.min_n, self.max_n, self.k)
        d, c = d.tolist(), c.tolist()
        return [d[i][:min(c[i], ks[i])] for i in range(len(seqs))]


class DraftModelProposer:
    """Greedy proposals from a draft model sharing the target engine's block tables."""

    def __init__(self, engine, model_cfg, weights=None, k: int = 4):
        from ..models.llama import LlamaModel
        from .model_runner import ModelRunner
        self.k = k
        self.engine = engine
        tgt = engine.model
        if model_cfg.vocab_size != engine.model_cfg.vocab_size:
            raise ValueError("draft and target models must share the vocabulary")
        self.model = LlamaModel(model_cfg, device=str(tgt.device), dtype=tgt.dtype)
        if weights is not None:
            self.model.load_weights(weights)
        else:
            self.model.init_random(seed=engine.cfg.seed + 1)
        nb = engine.kv.num_blocks
        self.cache = torch.zeros(self.model.kv_cache_shape(nb, engine.cfg.block_size), dtype=tgt.dtype,
                                 device=tgt.device) if tgt.device.type == "cuda" else \
            torch.zeros(self.model.kv_cache_shape(nb, engine.cfg.block_size), dtype=tgt.dtype)
        self.runner = ModelRunner(self.model, engine.cfg, self.cache, engine.kv)
        self.runner.greedy_only = True
        self.budget = engine.cfg.max_num_batched_tokens
        self.done = {}  # seq_id -> positions whose draft KV is valid

    def propose(self, seqs: List[Sequence], ks: List[int]) -> List[List[int]]:
        from .scheduler import ScheduledChunk, SchedulerOutput
        if not seqs:
            return []
        drafts: List[List[int]] = [[] for _ in seqs]
        live = [i for i, k in enumerate(ks) if k > 0]
        if not live:
            return drafts
        # catch-up: run the draft over every token it has not seen, ending at the last token; the
        # prediction after the last token is the first draft. Chunked to the batch token budget.
        pos = {i: min(self.done.get(seqs[i].seq_id, 0), seqs[i].num_computed_tokens) for i in live}
        pending = list(live)
        while pending:
            chunks, owners, used = [], [], 0
            nxt = []
            for i in pending:
                s = seqs[i]
                left = s.num_tokens - pos[i]
                take = min(left, max(1, self.budget - used)) if chunks else min(left, self.budget)
                if used + take > self.budget and chunks:
                    nxt.append(i)
                    continue
                last = take == left
                chunks.append(ScheduledChunk(s, pos[i], take, last))
                owners.append((i, last))
                used += take
                pos[i] += take
                if not last:
                    nxt.append(i)
            toks = self.runner.execute(SchedulerOutput(prefill=chunks))
            j = 0
            for i, last in owners:
                if last:
                    drafts[i].append(int(toks[j][0]))
                    j += 1
            pending = nxt
        for i in live:
            self.done[seqs[i].seq_id] = seqs[i].num_tokens
        # k - 1 more greedy single-token steps over the sequences that still want drafts
        for step in range(1, max(ks[i] for i in live)):
            act = [i for i in live if ks[i] > step]
            if not act:
                break
            dec = [ScheduledChunk(seqs[i], seqs[i].num_tokens + step - 1, 1, True, tokens=[drafts[i][-1]])
                   for i in act]
            toks = self.runner.execute(SchedulerOutput(decode=dec))
            for j, i in enumerate(act):
                drafts[i].append(int(toks[j][0]))
        for i in live:
            self.done[seqs[i].seq_id] = seqs[i].num_tokens + len(drafts[i]) - 1
        return drafts

    def accepted(self, seq: Sequence) -> None:
        """After verification: draft KV stays valid up to the accepted prefix."""
        self.done[seq.seq_id] = min(self.done.get(seq.seq_id, 0), seq.num_computed_tokens)

    def forget(self, seq: Sequence) -> None:
        self.done.pop(seq.seq_id, None)


def accept_drafts(logits: torch.Tensor, chunks: list, seqs: List[Sequence], seed: int,
                  step: int) -> List[List[int]]:
    """Exact acceptance for the verify chunks. ``logits`` rows: for chunk j with k_j drafts, k_j + 1
    consecutive rows (predictions after the last token and after each draft). Returns the tokens to
    append per chunk: the accepted drafts plus one corrected or bonus token."""
    R = logits.shape[0]
    dev = logits.device
    greedy = all(s.params.greedy for s in seqs)
    rows_draft = []
    for c in chunks:
        rows_draft.extend(c.tokens[1:] + [-1])
    if greedy:
        am = ops.argmax(logits).tolist()
        out, r = [], 0
        for c in chunks:
            k = c.verify
            acc = []
            for i in range(k + 1):
                t = am[r + i]
                acc.append(t)
                if i == k or t != c.tokens[1 + i]:
                    break
            out.append(acc)
            r += k + 1
        return out
    # per-row sampling parameters (a greedy request in a mixed batch: temperature -> tiny)
    row_seq = []
    for c, s in zip(chunks, seqs):
        row_seq.extend([s] * (c.verify + 1))
    temps = torch.tensor([max(s.params.temperature, 1e-4) for s in row_seq], device=dev)
    topk = torch.tensor([s.params.top_k if s.params.temperature > 0 else 1 for s in row_seq], device=dev)
    topp = torch.tensor([s.params.top_p for s in row_seq], device=dev)
    minp = torch.tensor([s.params.min_p for s in row_seq], device=dev)
    p = ref.filtered_probs(logits, temps, topk, topp, minp)
    d = torch.tensor(rows_draft, device=dev)
    has = d >= 0
    pd = torch.where(has, p.gather(1, d.clamp_min(0)[:, None])[:, 0], torch.zeros(R, device=dev))
    g = torch.Generator(device=dev)
    g.manual_seed((seed * 1_000_003 + step) & 0x7FFFFFFFFFFF)
    u = torch.rand(R, generator=g, device=dev)
    accept = (u < pd) & has
    resid = p.clone()
    resid.scatter_(1, d.clamp_min(0)[:, None], 0.0)
    resid = torch.where(has[:, None], resid, p)
    resid = resid / resid.sum(-1, keepdim=True).clamp_min(1e-30)
    resid = torch.where(resid.sum(-1, keepdim=True) > 0, resid, p)
    draw = torch.multinomial(resid, 1, generator=g)[:, 0]
    acc_l, draw_l = accept.tolist(), draw.tolist()
    out, r = [], 0
    for c in chunks:
        k = c.verify
        toks = []
        for i in range(k + 1):
            if i < k and acc_l[r + i]:
                toks.append(c.tokens[1 + i])
                continue
            toks.append(draw_l[r + i])
            break
        out.append(toks)
        r += k + 1
    return out

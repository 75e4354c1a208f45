"""Per-row sampling modes beyond the fused sampling kernel: locally typical sampling, mirostat v2,
and log-probabilities of the chosen and top tokens.

* Typical (Meister et al., "Locally Typical Sampling", 2022): keep the tokens whose surprise
  -log p is closest to the distribution's entropy, in that order, until their mass reaches
  ``typical_p``; renormalise and sample.
* Mirostat v2 (Basu et al., "Mirostat", 2021): drop tokens whose surprise -log2 p exceeds the
  running target mu (keeping at least the most likely), sample from the renormalised rest, then
  mu -= eta * (observed surprise - tau); mu starts at 2 tau.
* Logprobs: log-softmax of the raw logits (before temperature and penalties), the chosen token
  and the ``logprobs`` most likely ones.

The reference exposes typical and mirostat through llama.cpp's sampler chain
(runner/llamacpp/gollek-runner-llamacpp/…/LlamaHandles.java:174-203).
"""
from __future__ import annotations

import math

import torch

from .sequence import Sequence


def _generator(seq: Sequence, base_seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    seed = seq.params.seed if seq.params.seed is not None else seq.seq_id * 7919 + base_seed
    g.manual_seed((int(seed) * 1_000_003 + len(seq.output_token_ids)) & 0x7FFFFFFFFFFF)
    return g


def sample_row(row: torch.Tensor, raw: torch.Tensor, seq: Sequence, base_seed: int) -> int:
    """row: penalised fp32 logits of one sequence; raw: its unpenalised logits (for logprobs).
    A constrained request (``seq.guide``) samples among the tokens its grammar allows."""
    p = seq.params
    if seq.guide is not None:
        allowed = seq.guide.mask().to(row.device)
        row = torch.where(allowed, row, torch.full_like(row, float("-inf")))
    if p.greedy:
        tok = int(row.argmax())
    else:
        x = row / max(p.temperature, 1e-6)
        V = x.shape[0]
        if 0 < p.top_k < V:
            kth = x.topk(p.top_k).values[-1]
            x = torch.where(x >= kth, x, torch.full_like(x, float("-inf")))
        probs = torch.softmax(x, -1)
        if p.min_p > 0:
            probs = torch.where(probs >= p.min_p * probs.max(), probs, torch.zeros_like(probs))
            probs = probs / probs.sum()
        if p.top_p < 1.0:
            sp, si = probs.sort(descending=True)
            keep = (sp.cumsum(0) - sp) < p.top_p
            probs = torch.zeros_like(probs).scatter(0, si[keep], sp[keep])
            probs = probs / probs.sum()
        if p.typical_p < 1.0:
            logp = torch.log(probs.clamp_min(1e-30))
            ent = -(probs * logp).sum()
            dev = (-logp - ent).abs()
            dev = torch.where(probs > 0, dev, torch.full_like(dev, float("inf")))
            order = dev.argsort()
            cum = probs[order].cumsum(0)
            n = int((cum < p.typical_p).sum()) + 1
            keep = order[:n]
            probs = torch.zeros_like(probs).scatter(0, keep, probs[keep])
            probs = probs / probs.sum()
        if p.mirostat == 2:
            mu = seq.mirostat_mu if seq.mirostat_mu is not None else 2.0 * p.mirostat_tau
            surprise = -torch.log2(probs.clamp_min(1e-30))
            top = int(probs.argmax())
            mask = surprise <= mu
            mask[top] = True
            probs = torch.where(mask, probs, torch.zeros_like(probs))
            probs = probs / probs.sum()
        g = _generator(seq, base_seed, probs.device)
        tok = int(torch.multinomial(probs, 1, generator=g))
        if p.mirostat == 2:
            observed = -math.log2(max(float(probs[tok]), 1e-30))
            seq.mirostat_mu = mu - p.mirostat_eta * (observed - p.mirostat_tau)
    if seq.guide is not None:
        seq.guide.advance(tok)
    if p.logprobs is not None:
        lp = torch.log_softmax(raw.float(), -1)
        entry = {"token": tok, "logprob": float(lp[tok])}
        if p.logprobs > 0:
            v, i = lp.topk(p.logprobs)
            entry["top"] = {int(a): float(b) for a, b in zip(i.tolist(), v.tolist())}
        seq.logprobs.append(entry)
    return tok

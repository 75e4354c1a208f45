"""Beam search over the serving engine.

Behaviour of the reference's decoder (runner/safetensor/gollek-safetensor-tooling/…/engine/tooling/
BeamSearchDecoder.java:97-163): K beams, each expanded by its top next tokens, the best K kept,
finished beams collected, the best length-normalised hypothesis returned (score = sum of token
log-probabilities / generated length ** length_penalty).

Design: the search is a host-side state machine (``BeamSearch``) that asks for one-token expansions
of up to K prefixes per step and never touches the KV cache itself. Each expansion is an ordinary
engine request (one greedy token, top-2K log-probabilities), so beams share every full KV block of
their common prefix through the prefix cache and only the last partial block is recomputed; beams
run batched with whatever else the engine serves. ``beam_search`` drives it on an ``LLMEngine``;
``abeam_search`` on the asynchronous server engine.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Awaitable, Callable, Dict, List, Optional, Sequence

from .sequence import SamplingParams


@dataclass
class BeamParams:
    beam_width: int = 4
    max_tokens: int = 64
    length_penalty: float = 1.0
    early_stopping: bool = False      # True: stop once beam_width hypotheses finished
    num_return: int = 1               # hypotheses returned, best first (<= beam_width)
    stop_token_ids: Sequence[int] = ()
    ignore_eos: bool = False

    def __post_init__(self):
        if self.beam_width < 1 or self.max_tokens < 1:
            raise ValueError("beam_width and max_tokens must be >= 1")
        if not 1 <= self.num_return <= self.beam_width:
            raise ValueError("num_return must be in [1, beam_width]")


@dataclass
class Hypothesis:
    tokens: List[int]
    logprob: float
    finished: bool = False
    finish_reason: str = "length"

    def score(self, alpha: float) -> float:
        return self.logprob / (max(1, len(self.tokens)) ** alpha)


@dataclass
class BeamSearch:
    """State machine: ``prefixes()`` -> expand each with its top tokens -> ``update(tops)``."""
    prompt: List[int]
    params: BeamParams
    eos_token_id: Optional[int]
    live: List[Hypothesis] = field(default_factory=lambda: [Hypothesis([], 0.0)])
    finished: List[Hypothesis] = field(default_factory=list)
    steps: int = 0

    @property
    def expansion_k(self) -> int:
        return 2 * self.params.beam_width  # enough candidates even if half of them end beams

    def prefixes(self) -> List[List[int]]:
        return [self.prompt + h.tokens for h in self.live]

    def _is_stop(self, tok: int) -> bool:
        if tok in self.params.stop_token_ids:
            return True
        return (not self.params.ignore_eos) and self.eos_token_id is not None and tok == self.eos_token_id

    def update(self, tops: List[Dict[int, float]]) -> None:
        K, alpha = self.params.beam_width, self.params.length_penalty
        cands = []
        for h, top in zip(self.live, tops):
            for tok, lp in top.items():
                cands.append((h.logprob + lp, h, int(tok)))
        cands.sort(key=lambda c: -c[0])
        nxt: List[Hypothesis] = []
        for rank, (lp, h, tok) in enumerate(cands):
            if self._is_stop(tok):
                if rank < K:  # an ending counts only if it ranks among the K best candidates
                    self.finished.append(Hypothesis(list(h.tokens), lp, True, "stop"))
            else:
                nxt.append(Hypothesis(h.tokens + [tok], lp))
            if len(nxt) == K:
                break
        self.live = nxt
        self.steps += 1
        self.finished.sort(key=lambda x: -x.score(alpha))
        del self.finished[K:]

    @property
    def done(self) -> bool:
        K, alpha = self.params.beam_width, self.params.length_penalty
        if not self.live or self.steps >= self.params.max_tokens:
            return True
        if len(self.finished) >= K:
            if self.params.early_stopping:
                return True
            # no live beam can still beat the worst kept hypothesis: a beam's log-probability only
            # falls, so with alpha > 0 its best reachable score is that sum over the longest length
            best_lp = max(h.logprob for h in self.live)
            n = self.params.max_tokens if alpha > 0 else max(1, max(len(h.tokens) for h in self.live))
            return best_lp / (n ** alpha) < self.finished[-1].score(alpha)
        return False

    def results(self) -> List[Hypothesis]:
        alpha = self.params.length_penalty
        pool = self.finished + [Hypothesis(h.tokens, h.logprob, False, "length") for h in self.live]
        pool.sort(key=lambda x: -x.score(alpha))
        return pool[: self.params.num_return]


def _expand_params(bs: BeamSearch) -> SamplingParams:
    return SamplingParams(temperature=0.0, max_tokens=1, logprobs=bs.expansion_k, ignore_eos=True)


def _top(out) -> Dict[int, float]:
    return dict(out.logprobs[0].get("top", {})) if out.logprobs else {}


def beam_search(engine, prompt: List[int], params: BeamParams, lora_id: int = 0) -> List[Hypothesis]:
    """Beam search on an ``LLMEngine`` (drives ``engine.generate``; the engine should not be serving
    other requests from another thread at the same time)."""
    bs = BeamSearch(list(prompt), params, engine.eos_token_id)
    sp = _expand_params(bs)
    while not bs.done:
        prefixes = bs.prefixes()
        outs = engine.generate(prefixes, sp, lora_ids=[lora_id] * len(prefixes))
        bs.update([_top(o) for o in outs])
    return bs.results()


async def abeam_search(expand: Callable[[List[int], SamplingParams], Awaitable], prompt: List[int],
                       params: BeamParams, eos_token_id: Optional[int]) -> List[Hypothesis]:
    """Beam search over an asynchronous engine: ``expand(prefix, params)`` returns the finished
    RequestOutput of one request; the K expansions of a step run concurrently."""
    import asyncio
    bs = BeamSearch(list(prompt), params, eos_token_id)
    sp = _expand_params(bs)
    while not bs.done:
        outs = await asyncio.gather(*(expand(p, sp) for p in bs.prefixes()))
        bs.update([_top(o) for o in outs])
    return bs.results()

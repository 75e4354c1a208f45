"""Requests, sequences and sampling parameters.

``SamplingParams`` covers the per-request knobs of the reference's request surface
(core/spi/gollek-spi-inference/…/InferenceRequest.java:32-73 ``parameters`` map; OpenAI
defaults in runner/safetensor/gollek-safetensor-api/…/OpenAiCompatibleResource.java:323-342;
SDK ``GenerationRequest`` sdk/gollek-sdk/…/sdk/model/GenerationRequest.java:36-112), with
validation equivalent to plugins/gollek-plugin-sampling/…/SamplingPolicyPlugin.java:111-152.
"""
from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass, field
from typing import List, Optional


@dataclass
class SamplingParams:
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0
    min_p: float = 0.0
    repetition_penalty: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    max_tokens: int = 16
    min_tokens: int = 0
    stop: List[str] = field(default_factory=list)
    stop_token_ids: List[int] = field(default_factory=list)
    ignore_eos: bool = False
    seed: Optional[int] = None
    logprobs: Optional[int] = None      # return the chosen token's and the top-k log-probabilities
    typical_p: float = 1.0              # locally typical sampling mass (1 = off)
    mirostat: int = 0                   # 2 = mirostat v2 (target surprise tau, learning rate eta)
    mirostat_tau: float = 5.0
    mirostat_eta: float = 0.1
    guided_json: bool = False           # constrain the output to a JSON object
    guided_regex: Optional[str] = None  # constrain the output to a full match of this regex

    def validate(self) -> "SamplingParams":
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if not 0.0 < self.top_p <= 1.0:
            raise ValueError("top_p must be in (0, 1]")
        if self.top_k < 0:
            raise ValueError("top_k must be >= 0 (0 disables)")
        if not 0.0 <= self.min_p <= 1.0:
            raise ValueError("min_p must be in [0, 1]")
        if self.repetition_penalty <= 0:
            raise ValueError("repetition_penalty must be > 0")
        if not -2.0 <= self.frequency_penalty <= 2.0 or not -2.0 <= self.presence_penalty <= 2.0:
            raise ValueError("frequency/presence penalties must be in [-2, 2]")
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if not 0.0 < self.typical_p <= 1.0:
            raise ValueError("typical_p must be in (0, 1]")
        if self.mirostat not in (0, 2):
            raise ValueError("mirostat must be 0 (off) or 2 (mirostat v2)")
        if self.logprobs is not None and not 0 <= self.logprobs <= 20:
            raise ValueError("logprobs must be in [0, 20]")
        if isinstance(self.stop, str):
            self.stop = [self.stop]
        return self

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0

    @property
    def needs_penalties(self) -> bool:
        return self.repetition_penalty != 1.0 or self.frequency_penalty != 0.0 or self.presence_penalty != 0.0

    @property
    def needs_host_sampling(self) -> bool:
        """Sampling modes served by the per-row host path (typical, mirostat, logprobs)."""
        return (self.typical_p < 1.0 or self.mirostat != 0 or self.logprobs is not None or self.guided_json
                or self.guided_regex is not None)

    @property
    def guided(self) -> bool:
        return self.guided_json or self.guided_regex is not None


class SeqStatus(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED_STOPPED = "stop"
    FINISHED_LENGTH = "length"
    FINISHED_ABORTED = "abort"
    FINISHED_HANDOFF = "handoff"  # prefill node: KV and first token handed to a decode node

    @property
    def finished(self) -> bool:
        return self in (SeqStatus.FINISHED_STOPPED, SeqStatus.FINISHED_LENGTH, SeqStatus.FINISHED_ABORTED,
                        SeqStatus.FINISHED_HANDOFF)


_seq_counter = itertools.count()


class Sequence:
    """One generation stream (one request, n = 1)."""

    __slots__ = ("seq_id", "request_id", "prompt_token_ids", "output_token_ids", "params", "lora_id",
                 "arrival_time", "num_computed_tokens", "status", "first_token_time", "finish_time",
                 "token_times", "block_hashes", "num_preemptions", "predicted_len", "stop_reason",
                 "output_text", "priority", "scheduled_time", "pending", "tenant", "mirostat_mu", "logprobs",
                 "guide", "state_slot", "mm_embeds", "mm_positions", "cache_salt")

    def __init__(self, request_id: str, prompt_token_ids: List[int], params: SamplingParams,
                 lora_id: int = 0, arrival_time: Optional[float] = None, priority: int = 0):
        self.seq_id = next(_seq_counter)
        self.request_id = request_id
        self.prompt_token_ids = list(prompt_token_ids)
        self.output_token_ids: List[int] = []
        self.params = params
        self.lora_id = lora_id
        self.arrival_time = time.perf_counter() if arrival_time is None else arrival_time
        self.num_computed_tokens = 0
        self.status = SeqStatus.WAITING
        self.first_token_time: Optional[float] = None
        self.finish_time: Optional[float] = None
        self.token_times: List[float] = []
        self.block_hashes: List[int] = []
        self.num_preemptions = 0
        self.predicted_len: Optional[float] = None
        self.stop_reason = None
        self.output_text = ""
        self.priority = priority
        self.scheduled_time: Optional[float] = None
        self.pending = 0  # async scheduling: sampled tokens not yet read back (placeholders -1)
        self.tenant = ""  # quota accounting (EngineConfig.tenant_quotas)
        self.mirostat_mu: Optional[float] = None
        self.logprobs: List[dict] = []  # per output token when params.logprobs is set
        # multimodal prompts: projected image rows [n, hidden] and the prompt positions they fill;
        # cache_salt (the image content) keeps their KV blocks apart in the prefix cache
        self.mm_embeds = None
        self.mm_positions: Optional[List[int]] = None
        self.cache_salt = 0
        self.guide = None  # constrained decoding: native GrammarMatcher of the output so far
        self.state_slot = -1  # hybrid GDN models: recurrent-state slot while the sequence holds KV

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    @property
    def num_prompt_tokens(self) -> int:
        return len(self.prompt_token_ids)

    def token_at(self, i: int) -> int:
        n = len(self.prompt_token_ids)
        return self.prompt_token_ids[i] if i < n else self.output_token_ids[i - n]

    def tokens(self, start: int, end: int) -> List[int]:
        n = len(self.prompt_token_ids)
        if end <= n:
            return self.prompt_token_ids[start:end]
        if start >= n:
            return self.output_token_ids[start - n:end - n]
        return self.prompt_token_ids[start:] + self.output_token_ids[: end - n]

    @property
    def is_decode(self) -> bool:
        """Every token but the last sampled one is in the KV cache."""
        return self.num_computed_tokens == self.num_tokens - 1 and len(self.output_token_ids) > 0

    def __repr__(self) -> str:
        return f"Sequence({self.request_id}, prompt={self.num_prompt_tokens}, out={len(self.output_token_ids)}, " \
               f"computed={self.num_computed_tokens}, {self.status.value})"


@dataclass
class RequestOutput:
    request_id: str
    prompt_token_ids: List[int]
    output_token_ids: List[int]
    new_token_ids: List[int]
    finished: bool
    finish_reason: Optional[str] = None
    text: str = ""
    metrics: dict = field(default_factory=dict)
    logprobs: Optional[List[dict]] = None  # per output token (SamplingParams.logprobs)

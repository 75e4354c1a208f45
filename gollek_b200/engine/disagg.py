"""Prefill/decode disaggregation: a prefill engine computes a prompt's KV and first token, then
hands the sequence to a decode engine that continues it.

* ``export_sequence`` gathers the sequence's paged KV blocks of every layer into one packed tensor
  ``[L, n_blocks, 2, Hk, block_size, head_dim]`` (``ops.kv_gather_blocks``, one CUDA kernel).
* The packed tensor moves to the decode side: a device-to-device copy when both engines share a
  node (copy engines over NVLink), or bytes over the cluster hand-off RPC between nodes
  (``gollek_b200.cluster``).
* ``import_sequence`` allocates blocks in the decode engine's pool, scatters the KV into them
  (``ops.kv_scatter_blocks``) and registers the sequence as running in its decode phase.

``DisaggregatedEngine`` pairs a prefill engine and a decode engine (e.g. on two GPUs of one node)
behind the ``LLMEngine`` request API. The reference partitions one block pool into prefill and
decode halves and copies blocks in process
(core/optimization/gollek-plugin-prefill-decode/…/prefilldecode/PrefillDecodeDisaggService.java:1-80,
DisaggregatedLLMProvider.java); here the two sides are separate engines with their own pools, so
each can run on its own GPU with its own batch composition.
"""
from __future__ import annotations

import dataclasses
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from .. import ops
from .sequence import RequestOutput, SamplingParams, SeqStatus, Sequence


@dataclass
class KVHandoff:
    request_id: str
    model_id: str
    prompt_token_ids: List[int]
    output_token_ids: List[int]          # the first token(s) sampled by the prefill side
    params: dict                         # SamplingParams fields
    block_size: int
    kv: torch.Tensor                     # packed [L, n, 2, Hk, bs, D] covering the prompt's KV
    lora_id: int = 0
    arrival_time: Optional[float] = None
    first_token_time: Optional[float] = None

    @property
    def num_kv_tokens(self) -> int:
        return len(self.prompt_token_ids) + len(self.output_token_ids) - 1

    def nbytes(self) -> int:
        return self.kv.numel() * self.kv.element_size()


def export_sequence(engine, seq: Sequence, model_id: str = "") -> KVHandoff:
    """Gather ``seq``'s KV (every computed position) from ``engine``'s paged cache."""
    n_tok = seq.num_computed_tokens
    nb = (n_tok + engine.cfg.block_size - 1) // engine.cfg.block_size
    blocks = engine.kv.tables.blocks(seq.seq_id)[:nb]
    ids = torch.tensor(blocks, dtype=torch.int32)
    if getattr(engine.model, "kv_scales", None) is not None:
        raise ValueError("moving KV blocks of an fp8 cache (values + per-token scales) is not supported")
    kv = ops.kv_gather_blocks(engine.kv_cache, ids.to(engine.kv_cache.device))
    return KVHandoff(seq.request_id, model_id or str(engine.cfg.model), list(seq.prompt_token_ids),
                     list(seq.output_token_ids), dataclasses.asdict(seq.params), engine.cfg.block_size, kv,
                     seq.lora_id, seq.arrival_time, seq.first_token_time)


def import_sequence(engine, h: KVHandoff) -> Sequence:
    """Register a handed-off sequence in ``engine`` (decode side) with its KV scattered into
    freshly allocated blocks; it joins the running batch at its next decode step."""
    if h.block_size != engine.cfg.block_size:
        raise ValueError("prefill and decode engines must use the same KV block size")
    exp = engine.model.kv_cache_shape(h.kv.shape[1], h.block_size)
    if tuple(h.kv.shape) != (exp[0], h.kv.shape[1]) + tuple(exp[2:]):
        raise ValueError(f"KV layout mismatch: got {tuple(h.kv.shape)}, this model stores {exp}")
    if h.request_id in engine.seqs:
        raise ValueError(f"duplicate request id {h.request_id}")
    params = SamplingParams(**h.params)
    seq = Sequence(h.request_id, list(h.prompt_token_ids), params, lora_id=h.lora_id, arrival_time=h.arrival_time)
    seq.output_token_ids = list(h.output_token_ids)
    seq.first_token_time = h.first_token_time
    engine.kv.add(seq)
    if not engine.kv.ensure(seq, seq.num_tokens):
        engine.kv.free(seq)
        raise RuntimeError("decode engine KV cache full: retry the hand-off later")
    nb = h.kv.shape[1]
    blocks = torch.tensor(engine.kv.tables.blocks(seq.seq_id)[:nb], dtype=torch.int32)
    ops.kv_scatter_blocks(engine.kv_cache, blocks.to(engine.kv_cache.device), h.kv)
    seq.num_computed_tokens = h.num_kv_tokens
    engine.kv.commit_full_blocks(seq)
    seq.status = SeqStatus.RUNNING
    seq.scheduled_time = time.perf_counter()
    engine.scheduler.running.append(seq)
    engine.seqs[seq.request_id] = seq
    engine.metrics.on_arrival()
    return seq


class DisaggregatedEngine:
    """A prefill engine and a decode engine behind one request API.

    Requests enter the prefill engine with ``max_tokens`` forced to 1; when a prompt has produced
    its first token its KV is exported, copied to the decode engine's device and imported there,
    and the decode engine generates the rest. ``step`` advances both engines once."""

    def __init__(self, prefill, decode):
        self.prefill = prefill
        self.decode = decode
        self.pending: Dict[str, SamplingParams] = {}
        self.handoff_bytes = 0
        self.handoffs = 0
        prefill.handoff_hook = self._on_prefill_done

    def add_request(self, request_id: Optional[str], prompt, params: Optional[SamplingParams] = None,
                    **kw) -> str:
        params = (params or SamplingParams()).validate()
        first = SamplingParams(**vars(params))
        first.max_tokens = 1
        rid = self.prefill.add_request(request_id, prompt, first, **kw)
        self.pending[rid] = params
        return rid

    def _on_prefill_done(self, seq: Sequence) -> bool:
        """Called by the prefill engine after a sequence's first token; True = handed off."""
        full = self.pending.pop(seq.request_id, None)
        if full is None:
            return False
        if len(seq.output_token_ids) >= full.max_tokens or seq.num_tokens >= self.decode.cfg.max_model_len:
            return False  # nothing left to decode
        h = export_sequence(self.prefill, seq)
        h.params = dataclasses.asdict(full)
        h.kv = h.kv.to(self.decode.kv_cache.device, non_blocking=True)
        self.handoff_bytes += h.nbytes()
        self.handoffs += 1
        import_sequence(self.decode, h)
        return True

    def step(self) -> List[RequestOutput]:
        out = [o for o in self.prefill.step() if o.finish_reason != SeqStatus.FINISHED_HANDOFF.value]
        out += self.decode.step()
        return out

    def has_unfinished(self) -> bool:
        return self.prefill.has_unfinished() or self.decode.has_unfinished()

    def generate(self, prompts, params: Optional[SamplingParams] = None) -> List[RequestOutput]:
        import uuid
        ids = [self.add_request(f"pd-{uuid.uuid4().hex[:8]}-{i}", p, SamplingParams(**vars(params or SamplingParams())))
               for i, p in enumerate(prompts)]
        final: Dict[str, RequestOutput] = {}
        while self.has_unfinished():
            for o in self.step():
                if o.finished:
                    final[o.request_id] = o
        return [final[i] for i in ids]

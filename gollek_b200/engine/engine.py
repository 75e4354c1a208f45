"""The serving engine: request intake → continuous-batching steps → outputs.

``LLMEngine`` is the synchronous core (``add_request`` / ``step`` / ``generate``); it owns the
model shard, the paged KV pool, the scheduler and the model runner. ``LLM`` is the
user-facing convenience wrapper (``LLM("llama-3-8b").generate(prompts, params)``).

Plays the role of the reference's engine stack (inference/gollek-engine/…/engine/inference/
PlatformInferenceService.java:74-103 → DefaultInferenceEngine.java:94-143 →
DefaultInferenceOrchestrator.java:122-200) together with its runtime continuous batcher
(inference/gollek-runtime-inference/…/batch/ContinuousBatchScheduler.java:383-468) and the
llama.cpp runner's decode loop (runner/llamacpp/gollek-runner-llamacpp/…/InferenceLogicExecutor.java:105-149).
"""
from __future__ import annotations

import os
import time
import uuid
from typing import Callable, Dict, Iterable, List, Optional, Sequence as Seq, Union

import torch

from ..config import EngineConfig, ModelConfig, PRESETS, preset
from ..models.llama import LlamaModel, TPComm
from ..native import host_ext
from .kv_cache import KVCacheManager, allocate_kv_cache, num_blocks_from_memory
from ..utils import tracing
from .model_runner import ModelRunner
from .scheduler import Scheduler
from .sequence import RequestOutput, SamplingParams, Sequence, SeqStatus
from ..utils.metrics import EngineMetrics


def _dtype(name: str) -> torch.dtype:
    return {"bfloat16": torch.bfloat16, "bf16": torch.bfloat16, "float32": torch.float32,
            "fp32": torch.float32, "float16": torch.float16}[name]


def _tune_gc() -> None:
    """Process-wide: rare full collections, and the start-up objects (weights' metadata, modules)
    moved out of the collector's scans. Long-lived sequences' token lists would otherwise be walked
    by every full collection."""
    import gc
    t0, t1, t2 = gc.get_threshold()
    gc.set_threshold(max(t0, 50000), max(t1, 50), max(t2, 100))
    gc.collect()
    gc.freeze()


class LLMEngine:
    def __init__(self, cfg: EngineConfig, model_cfg: Optional[ModelConfig] = None,
                 weights: Optional[Callable[[str], torch.Tensor]] = None, comm: Optional[TPComm] = None,
                 tokenizer=None, num_blocks: Optional[int] = None, vision=None):
        self.cfg = cfg
        self.comm = comm or TPComm()
        dev = cfg.device
        if dev == "cuda":
            dev = f"cuda:{torch.cuda.current_device()}" if torch.cuda.is_available() else "cpu"
        self.device = torch.device(dev)
        self.dtype = _dtype(cfg.dtype) if self.device.type == "cuda" else torch.float32
        self.tokenizer = tokenizer
        # image encoder + projector of a vision-language checkpoint (models/vlm.py), or None
        self.vision = vision
        # ---- model
        if model_cfg is None:
            if _is_llava(cfg.model):
                from ..models.vlm import load_llava
                from ..utils.tokenizer import load_tokenizer
                model_cfg, weights, self.vision = load_llava(cfg.model, str(self.device), self.dtype)
                tok = load_tokenizer(cfg.model)
            else:
                model_cfg, weights, tok = load_model_source(cfg.model, keep_quantized=cfg.quantization == "gguf")
            self.tokenizer = self.tokenizer or tok
        self.model_cfg = model_cfg
        self.model = LlamaModel(model_cfg, device=str(self.device), dtype=self.dtype, comm=self.comm,
                                expert_parallel=cfg.enable_expert_parallel)
        if weights is None:
            self.model.init_random(cfg.seed, fp8=cfg.quantization == "fp8")
        else:
            self.model.load_weights(weights)
            if cfg.quantization == "fp8":
                self.model.quantize_fp8()
            elif cfg.quantization in ("int4", "nf4"):
                self.model.quantize_int4(cfg.quantization)
            elif cfg.quantization == "int8":
                self.model.quantize_int8()
        if cfg.offload_layers > 0 and self.device.type == "cuda":
            self.model.enable_offload(cfg.offload_layers, cfg.offload_prefetch)
            cfg.use_cuda_graphs = False
        # ---- hybrid GDN stacks: one recurrent-state slot per running sequence (+1 scratch slot for
        # embeddings); the state is not block-addressable, so no prefix reuse, no speculative rollback
        self.hybrid = self.model.num_gdn_layers > 0
        if self.hybrid:
            if cfg.speculative_method != "none" or cfg.enable_lora or cfg.kv_eviction:
                raise ValueError("hybrid GDN models: speculative decoding, LoRA and KV eviction are not supported")
            cfg.enable_prefix_caching = False
            cfg.use_cuda_graphs = False
            self.model.alloc_gdn_state(cfg.max_num_seqs + 1)
        # ---- KV cache (bf16, or fp8 e4m3 with a scale per token and head)
        kv_fp8 = cfg.kv_cache_dtype in ("fp8", "fp8_e4m3")
        if kv_fp8:
            if self.model.D != 128 or model_cfg.is_mla:
                raise ValueError("kv_cache_dtype fp8: attention kernels are built for head_dim 128 (no MLA)")
            if cfg.kv_eviction:
                raise ValueError("kv_cache_dtype fp8: KV eviction moves blocks without their scales; not supported")
            self.model.kv_fp8 = True
        bpb = self.model.kv_bytes_per_block(cfg.block_size)
        nb = num_blocks or cfg.num_gpu_blocks
        if nb is None:
            if self.device.type == "cuda":
                nb = num_blocks_from_memory(bpb, self.model.weight_bytes(), self.device, cfg.gpu_memory_utilization)
            else:
                nb = 1024
        if self.comm.size > 1 and self.device.type == "cuda":
            t = torch.tensor([nb], device=self.device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
            nb = int(t)
        self.num_blocks = nb
        shape = self.model.kv_cache_shape(nb, cfg.block_size)
        self.kv_cache = allocate_kv_cache(shape, torch.uint8 if kv_fp8 else self.dtype, self.device)
        if kv_fp8:
            self.model.kv_scales = allocate_kv_cache(shape[:-1], torch.float32, self.device)
        if cfg.speculative_method == "draft" and cfg.enable_prefix_caching:
            # a reused prefix block may carry target KV whose draft-model KV was never computed
            cfg.enable_prefix_caching = False
        self.kv = KVCacheManager(nb, cfg.block_size, cfg.enable_prefix_caching,
                                 state_slots=cfg.max_num_seqs + 1 if self.hybrid else 0)
        predictor = None
        if cfg.scheduling_policy == "wait":
            predictor = host_ext().LengthPredictor(64, 1.0, float(cfg.max_model_len), 0.05, 8)
        self.scheduler = Scheduler(cfg, self.kv, predictor)
        self._steps = 0
        self.ep_reports: List[dict] = []  # rebalances done: {"step", "layers": {layer: before/after/moved}}
        if cfg.ep_rebalance_interval > 0 and getattr(self.model, "expert_parallel", False):
            self.model.enable_expert_load_tracking()
        if self.model.cfg.is_mla and cfg.enable_lora:
            raise ValueError("LoRA adapters on multi-head latent attention models are not supported")
        self.lora_manager = None
        if cfg.enable_lora:
            from .lora import LoRAManager
            self.lora_manager = LoRAManager(self.model, cfg.max_loras, cfg.max_lora_rank)
        if cfg.enable_expert_parallel and cfg.ep_all_to_all and self.device.type == "cuda" and self.comm.size > 1:
            # token-sharded MoE over the NVLink all-to-all when the comm supports it (collective)
            self.model.enable_ep_all_to_all(cfg.max_num_batched_tokens + cfg.max_num_seqs)
        self.model.split_sms = cfg.tp_overlap_sms
        self.runner = ModelRunner(self.model, cfg, self.kv_cache, self.kv)
        if getattr(cfg, "gc_tuning", False):
            _tune_gc()
        if cfg.kv_cache_dtype not in ("auto", cfg.dtype, "fp8", "fp8_e4m3"):
            raise ValueError(f"kv_cache_dtype {cfg.kv_cache_dtype!r}: auto (the model dtype) or fp8 (e4m3)")
        self.evictor = None
        if cfg.kv_eviction:
            from .evicpress import KVEvictor
            if cfg.tensor_parallel_size > 1:
                raise ValueError("kv_eviction: not supported with tensor parallelism (per-rank scores differ)")
            if model_cfg.sliding_window or model_cfg.layer_types:
                raise ValueError("kv_eviction: not supported with sliding-window layers")
            self.evictor = KVEvictor(cfg.kv_eviction_threshold, cfg.kv_retention_target, cfg.kv_protect_sink_blocks,
                                     cfg.kv_protect_recent, cfg.kv_eviction_min_blocks)
        self.seqs: Dict[str, Sequence] = {}
        self.metrics = EngineMetrics()
        self.eos_token_id = model_cfg.eos_token_id
        # prefill/decode disaggregation: called after a sequence's first token on a prefill engine;
        # returning True means its KV was handed to a decode engine (engine.disagg)
        self.handoff_hook = None
        self._inflight = None  # async scheduling: the launched step whose tokens are not read back yet
        self._n_host_sampling = 0  # live requests needing host-side sampling (forces synchronous steps)
        # ---- speculative decoding
        from .speculative import DraftModelProposer, NgramProposer, SpecStats
        self.spec = None
        self.spec_stats = SpecStats()
        if cfg.speculative_method == "ngram":
            self.spec = NgramProposer(cfg.num_speculative_tokens, cfg.ngram_min, cfg.ngram_max)
        elif cfg.speculative_method == "draft":
            if not cfg.draft_model:
                raise ValueError("speculative_method 'draft' needs draft_model")
            dcfg, dw, _ = load_model_source(cfg.draft_model)
            self.spec = DraftModelProposer(self, dcfg, dw, cfg.num_speculative_tokens)
        elif cfg.speculative_method != "none":
            raise ValueError(f"unknown speculative_method {cfg.speculative_method!r}")
        # ---- resume from a previous run's snapshots
        import os as _os
        if cfg.prefix_cache_snapshot and _os.path.exists(cfg.prefix_cache_snapshot):
            self.load_prefix_cache(cfg.prefix_cache_snapshot)
        if cfg.request_snapshot and _os.path.exists(cfg.request_snapshot):
            import json as _json
            with open(cfg.request_snapshot) as f:
                self.restore_requests(_json.load(f))
            _os.remove(cfg.request_snapshot)

    # ------------------------------------------------------------------ requests
    def add_request(self, request_id: Optional[str], prompt: Union[str, List[int]],
                    params: Optional[SamplingParams] = None, lora_id: int = 0,
                    arrival_time: Optional[float] = None, priority: int = 0, tenant: str = "",
                    images: Optional[list] = None) -> str:
        """``images``: PIL images, HxWx3 uint8 arrays or pixel tensors [3, S, S] of a vision-language
        model, one per image placeholder token in the prompt (in order)."""
        request_id = request_id or uuid.uuid4().hex
        if request_id in self.seqs:
            raise ValueError(f"duplicate request id {request_id}")
        params = (params or SamplingParams()).validate()
        if isinstance(prompt, str):
            if self.tokenizer is None:
                raise ValueError("text prompt given but the model has no tokenizer")
            ids = self.tokenizer.encode(prompt)
        else:
            ids = list(prompt)
        if not ids:
            raise ValueError("empty prompt")
        mm = None
        if images:
            ids, mm = self._image_rows(ids, images)
        if max(ids) >= self.model_cfg.vocab_size or min(ids) < 0:
            raise ValueError("prompt token id out of range")
        room = self.cfg.max_model_len - len(ids)
        if room < 1:
            raise ValueError("prompt too long for max_model_len")
        params.max_tokens = min(params.max_tokens, room)
        if lora_id and (self.lora_manager is None or lora_id not in self.lora_manager.adapters):
            raise ValueError(f"unknown LoRA adapter id {lora_id}")
        seq = Sequence(request_id, ids, params, lora_id=lora_id, arrival_time=arrival_time, priority=priority)
        seq.tenant = tenant or ""
        if mm is not None:
            seq.mm_embeds, seq.mm_positions, seq.cache_salt = mm
        if params.guided:
            seq.guide = self._make_guide(params)
        self.scheduler.add(seq)
        if params.needs_penalties or params.needs_host_sampling:
            self._n_host_sampling += 1
        self.seqs[request_id] = seq
        self.metrics.on_arrival()
        return request_id

    @property
    def image_placeholder(self) -> Optional[str]:
        """Prompt text that the tokenizer encodes to the image placeholder token (None: no vision)."""
        if self.vision is None:
            return None
        idx = self.vision.image_token_index
        fn = getattr(self.tokenizer, "token_text", None)
        t = fn(idx) if fn is not None else None
        return t if t else "<image>"

    def _image_rows(self, ids: List[int], images: list):
        """Expand the image placeholders of ``ids`` and encode the images: (ids, (projected rows,
        their prompt positions, a salt from the pixel content))."""
        if self.vision is None:
            raise ValueError("this model takes no images")
        from ..models.vlm import expand_image_tokens, preprocess_image
        v = self.vision
        n_ph = sum(1 for t in ids if t == v.image_token_index)
        if n_ph != len(images):
            raise ValueError(f"{len(images)} images for {n_ph} image placeholder tokens")
        size = v.vcfg.image_size
        pv = torch.stack([im.float() if isinstance(im, torch.Tensor) else preprocess_image(im, size)
                          for im in images])
        feats = v.encode(pv)  # [n, per_image, hidden]
        ids, pos = expand_image_tokens(ids, v.image_token_index, v.tokens_per_image)
        salt = hash(pv.numpy().tobytes()) & ((1 << 62) - 1) or 1
        rows = feats.reshape(-1, feats.shape[-1]).to(self.device, self.dtype)
        return ids, (rows, pos, salt)

    def _make_guide(self, params: SamplingParams):
        """A constrained-decoding matcher for one request (vocabulary trie built on first use)."""
        if self.tokenizer is None or not hasattr(self.tokenizer, "token_bytes"):
            raise ValueError("constrained decoding needs a tokenizer with a byte vocabulary")
        if getattr(self, "_grammar", None) is None:
            toks = self.tokenizer.token_bytes()
            toks = (toks + [b""] * self.model_cfg.vocab_size)[: self.model_cfg.vocab_size]
            self._grammar = host_ext().GrammarCompiler(toks, int(self.eos_token_id))
        try:
            if params.guided_regex is not None:
                return self._grammar.regex(params.guided_regex)
            return self._grammar.json(True)
        except Exception as e:
            raise ValueError(f"invalid constraint: {e}") from e

    def add_lora(self, name: str, path: Optional[str] = None, seed: Optional[int] = None, rank: int = 16) -> int:
        """Register a PEFT adapter directory (or a random adapter when ``path`` is None); returns its id."""
        if self.lora_manager is None:
            raise RuntimeError("engine was created without enable_lora")
        if path is not None:
            return self.lora_manager.load_peft(path, name)
        return self.lora_manager.random_adapter(name, seed if seed is not None else len(self.lora_manager.adapters),
                                                rank=rank)

    def abort_request(self, request_id: str) -> bool:
        seq = self.scheduler.abort(request_id)
        self.seqs.pop(request_id, None)
        if seq is not None and (seq.params.needs_penalties or seq.params.needs_host_sampling):
            self._n_host_sampling -= 1
        if seq is not None and self.spec is not None and hasattr(self.spec, "forget"):
            self.spec.forget(seq)
        return seq is not None

    def has_unfinished(self) -> bool:
        return self.scheduler.has_work() or self._inflight is not None

    # ------------------------------------------------------------------ stepping
    def _check_stop(self, seq: Sequence, tok: int, n_out: Optional[int] = None) -> Optional[SeqStatus]:
        """Stop test for ``tok``, the ``n_out``-th output token (default: the last one appended)."""
        p = seq.params
        n_out = len(seq.output_token_ids) if n_out is None else n_out
        if seq.guide is not None and tok == self.eos_token_id:
            seq.stop_reason = tok
            return SeqStatus.FINISHED_STOPPED  # a constrained output ends when the grammar lets it
        if n_out >= p.min_tokens:
            if not p.ignore_eos and tok == self.eos_token_id:
                seq.stop_reason = tok
                return SeqStatus.FINISHED_STOPPED
            if tok in p.stop_token_ids:
                seq.stop_reason = tok
                return SeqStatus.FINISHED_STOPPED
            if p.stop and self.tokenizer is not None:
                seq.output_text = self.tokenizer.decode(seq.output_token_ids[:n_out])
                for s in p.stop:
                    idx = seq.output_text.find(s)
                    if idx >= 0:
                        seq.output_text = seq.output_text[:idx]
                        seq.stop_reason = s
                        return SeqStatus.FINISHED_STOPPED
        if n_out >= p.max_tokens or seq.num_prompt_tokens + n_out >= self.cfg.max_model_len:
            return SeqStatus.FINISHED_LENGTH
        return None

    def _speculate(self, sched) -> None:
        """Turn decode chunks into verify chunks ``[last] + drafts`` where the proposer has drafts."""
        from .scheduler import ScheduledChunk
        K = self.cfg.num_speculative_tokens
        seqs, ks = [], []
        for c in sched.decode:
            s = c.seq
            room = min(s.params.max_tokens - len(s.output_token_ids), self.cfg.max_model_len - s.num_tokens) - 1
            k = 0 if (s.params.needs_penalties or s.params.needs_host_sampling) else max(0, min(K, room))
            if k and not self.kv.ensure(s, s.num_tokens + k):
                k = 0
            seqs.append(s)
            ks.append(k)
        drafts = self.spec.propose(seqs, ks)
        keep, verify = [], []
        for c, d in zip(sched.decode, drafts):
            if d:
                last = c.seq.tokens(c.start, c.start + 1)
                verify.append(ScheduledChunk(c.seq, c.start, 1 + len(d), True, tokens=list(last) + list(d),
                                             verify=len(d)))
                self.spec_stats.proposed += len(d)
            else:
                keep.append(c)
        if verify:
            self.spec_stats.steps += 1
            sched.decode = keep
            sched.prefill = verify + sched.prefill

    def _needs_sync(self) -> bool:
        if not self.cfg.async_scheduling or self.spec is not None or self.handoff_hook is not None:
            return True
        # live requests whose sampling needs host-visible history (penalties, typical, mirostat, logprobs)
        return self._n_host_sampling > 0

    def step(self) -> List[RequestOutput]:
        """One scheduler iteration. With async scheduling: schedule and launch this step, then read
        back the previous one (its outputs are returned), so the host work of a step overlaps the
        device work of the one before. Otherwise: schedule, (draft,) run, append, retire."""
        self._maybe_rebalance()
        if self._needs_sync():
            outs = self._resolve_inflight()
            return outs + self._step_sync()
        tracing.nvtx_push("schedule")
        if self.evictor is not None:
            self.evictor.run(self)
        sched = self.scheduler.schedule()
        tracing.nvtx_pop()
        if sched.empty:
            return self._resolve_inflight()
        t0 = time.perf_counter()
        tracing.nvtx_push("launch")
        h = self.runner.launch(sched, self._inflight)
        tracing.nvtx_pop()
        for c in sched.chunks:
            seq = c.seq
            seq.num_computed_tokens = c.start + c.num_tokens
            if c.sample:
                seq.output_token_ids.append(-1)
                seq.pending += 1
                h.records.append((seq, len(seq.output_token_ids) - 1))
        tracing.nvtx_push("read-back")
        outs = self._resolve_inflight()
        tracing.nvtx_pop()
        self._inflight = h
        self.metrics.on_step(time.perf_counter() - t0, sched.num_tokens, len(outs), len(self.scheduler.running),
                             len(self.scheduler.waiting), self.kv.usage(), len(sched.preempted))
        return outs

    def _maybe_rebalance(self) -> None:
        """Every ``ep_rebalance_interval`` steps (all ranks step in lockstep): re-place the experts by
        their routed load. In-place weight moves are ordered after the in-flight step on the stream."""
        self._steps += 1
        n = self.cfg.ep_rebalance_interval
        if n > 0 and self._steps % n == 0 and getattr(self.model, "expert_parallel", False):
            rep = self.model.rebalance_experts()
            if rep:
                self.ep_reports.append({"step": self._steps, "layers": rep})

    def _resolve_inflight(self) -> List[RequestOutput]:
        """Read back the in-flight step: fill placeholders, stop checks, retire finished sequences."""
        h = self._inflight
        if h is None:
            return []
        self._inflight = None
        toks = h.tokens()
        now = time.perf_counter()
        bs = self.kv.block_size
        outputs: List[RequestOutput] = []
        for (seq, idx), tok in zip(h.records, toks):
            seq.pending -= 1
            if seq.status.finished or idx >= len(seq.output_token_ids):
                continue  # stopped at an earlier token (this one was computed past the stop) or aborted
            tok = int(tok)
            seq.output_token_ids[idx] = tok
            seq.token_times.append(now)
            if seq.first_token_time is None:
                seq.first_token_time = now
            status = self._check_stop(seq, tok, idx + 1)
            finished = status is not None
            if finished:
                del seq.output_token_ids[idx + 1:]  # drop a token launched after the stop
                seq.finish_time = now
                self.scheduler.finish(seq, status)
                if seq.params.needs_penalties or seq.params.needs_host_sampling:
                    self._n_host_sampling -= 1
                self.seqs.pop(seq.request_id, None)
                self.metrics.on_finish(seq)
            elif (seq.num_computed_tokens // bs > len(seq.block_hashes) and seq.status is SeqStatus.RUNNING
                  and self.kv.has(seq)):
                # positions < num_computed_tokens are inputs of launched steps, all resolved by now
                # (the in-flight step's own placeholder sits at num_computed_tokens)
                self.kv.commit_full_blocks(seq)
            text = ""
            if self.tokenizer is not None and finished:
                text = seq.output_text or self.tokenizer.decode(seq.output_token_ids)
            outputs.append(RequestOutput(seq.request_id, seq.prompt_token_ids, seq.output_token_ids, [tok],
                                         finished, status.value if status else None, text,
                                         logprobs=seq.logprobs if seq.params.logprobs is not None else None))
        return outputs

    def _step_sync(self) -> List[RequestOutput]:
        if self.evictor is not None:
            self.evictor.run(self)
        sched = self.scheduler.schedule()
        if sched.empty:
            return []
        t0 = time.perf_counter()
        if self.spec is not None and sched.decode:
            self._speculate(sched)
        sampled = self.runner.execute(sched)
        now = time.perf_counter()
        outputs: List[RequestOutput] = []
        k = 0
        n_new = 0
        for c in sched.chunks:
            seq = c.seq
            new = sampled[k] if c.sample else []
            if c.verify:  # KV is valid for the last token and the accepted drafts
                seq.num_computed_tokens = c.start + len(new)
                self.spec_stats.accepted += len(new) - 1
                if hasattr(self.spec, "accepted"):
                    self.spec.accepted(seq)
            else:
                seq.num_computed_tokens = c.start + c.num_tokens
            self.kv.commit_full_blocks(seq)
            if not c.sample:
                continue
            k += 1
            status = None
            appended = []
            for tok in new:
                tok = int(tok)
                seq.output_token_ids.append(tok)
                seq.token_times.append(now)
                appended.append(tok)
                n_new += 1
                if seq.first_token_time is None:
                    seq.first_token_time = now
                status = self._check_stop(seq, tok)
                if status is not None:
                    break
            if (self.handoff_hook is not None and len(seq.output_token_ids) == 1
                    and status in (None, SeqStatus.FINISHED_LENGTH) and self.handoff_hook(seq)):
                status = SeqStatus.FINISHED_HANDOFF
            finished = status is not None
            if finished:
                seq.finish_time = now
                self.scheduler.finish(seq, status)
                if seq.params.needs_penalties or seq.params.needs_host_sampling:
                    self._n_host_sampling -= 1
                self.seqs.pop(seq.request_id, None)
                self.metrics.on_finish(seq)
                if self.spec is not None and hasattr(self.spec, "forget"):
                    self.spec.forget(seq)
            text = ""
            if self.tokenizer is not None and finished:
                text = seq.output_text or self.tokenizer.decode(seq.output_token_ids)
            outputs.append(RequestOutput(seq.request_id, seq.prompt_token_ids, seq.output_token_ids, appended,
                                         finished, status.value if status else None, text,
                                         logprobs=seq.logprobs if seq.params.logprobs is not None else None))
        self.metrics.on_step(now - t0, sched.num_tokens, n_new, len(self.scheduler.running),
                             len(self.scheduler.waiting), self.kv.usage(), len(sched.preempted))
        return outputs

    # ------------------------------------------------------------------ checkpoint / resume
    def save_prefix_cache(self, path: str, max_blocks: int = 0, compress: str = "") -> int:
        from .persistence import save_prefix_cache
        return save_prefix_cache(self, path, max_blocks, compress)

    def load_prefix_cache(self, path: str) -> int:
        from .persistence import load_prefix_cache
        return load_prefix_cache(self, path)

    def snapshot_requests(self) -> List[dict]:
        from .persistence import snapshot_requests
        return snapshot_requests(self)

    def restore_requests(self, reqs: List[dict]) -> List[str]:
        from .persistence import restore_requests
        return restore_requests(self, reqs)

    def embed(self, token_lists: List[List[int]]) -> List[List[float]]:
        """Mean-pooled, L2-normalised final hidden states (one prefill pass per input, KV blocks
        borrowed from the pool and returned). Must run between steps (the async front calls it on
        the engine thread)."""
        from .scheduler import ScheduledChunk, SchedulerOutput
        vecs: List[List[float]] = []
        for ids in token_lists:
            if not ids:
                raise ValueError("empty embedding input")
            ids = list(ids)[: self.cfg.max_model_len - 1]
            seq = Sequence(f"embed-{uuid.uuid4().hex[:8]}", ids, SamplingParams(max_tokens=1))
            self.kv.add(seq)
            try:
                if not self.kv.ensure(seq, len(ids)):
                    raise RuntimeError("KV cache full: retry the embedding request later")
                out = SchedulerOutput(prefill=[ScheduledChunk(seq, 0, len(ids), False)])
                hid = self.runner.run_hidden(out).float().mean(0)
                hid = hid / hid.norm().clamp_min(1e-12)
                vecs.append(hid.cpu().tolist())
            finally:
                self.kv.free(seq)
        return vecs

    def beam_search(self, prompt: Union[str, List[int]], params=None, lora_id: int = 0):
        """Beam search (engine.beam); returns the best hypotheses (tokens, logprob, finish_reason)."""
        from .beam import BeamParams, beam_search
        ids = self.tokenizer.encode(prompt) if isinstance(prompt, str) else list(prompt)
        return beam_search(self, ids, params or BeamParams(), lora_id)

    def generate(self, prompts: Seq[Union[str, List[int]]], params: Union[SamplingParams, List[SamplingParams], None] = None,
                 lora_ids: Optional[List[int]] = None, images: Optional[List[Optional[list]]] = None
                 ) -> List[RequestOutput]:
        ids = []
        for i, p in enumerate(prompts):
            sp = params[i] if isinstance(params, list) else (params or SamplingParams())
            sp = SamplingParams(**vars(sp))
            ids.append(self.add_request(f"gen-{uuid.uuid4().hex[:8]}-{i}", p, sp,
                                        lora_id=lora_ids[i] if lora_ids else 0,
                                        images=images[i] if images else None))
        final: Dict[str, RequestOutput] = {}
        while self.has_unfinished():
            for o in self.step():
                if o.finished:
                    final[o.request_id] = o
        return [final[i] for i in ids]


def _is_llava(source: str) -> bool:
    """A checkpoint directory of a LLaVA-layout vision-language model."""
    import json
    p = os.path.join(source, "config.json") if os.path.isdir(source) else None
    if p is None or not os.path.exists(p):
        return False
    with open(p) as fh:
        c = json.load(fh)
    archs = c.get("architectures") or []
    return c.get("model_type") == "llava" or any("Llava" in a for a in archs)


def load_model_source(source: str, keep_quantized: bool = False):
    """Resolve a preset name, a safetensors checkpoint (file or directory) or a GGUF file.

    Returns (ModelConfig, weight getter or None for random init, tokenizer or None).
    """
    from ..loaders.safetensors import SafetensorsCheckpoint
    from ..utils.tokenizer import load_tokenizer
    if source in PRESETS:
        from ..utils.tokenizer import ByteTokenizer
        cfg = preset(source)
        return cfg, None, ByteTokenizer(cfg.vocab_size, cfg.eos_token_id)
    if source.endswith(".gguf"):
        from ..loaders.gguf import load_llama_gguf
        cfg, w, f = load_llama_gguf(source, torch.float32, keep_quantized=keep_quantized)
        from ..utils.tokenizer import GGUFTokenizer
        tok = GGUFTokenizer.from_metadata(f.metadata)
        return cfg, w.__getitem__, tok
    if os.path.isdir(source) or source.endswith(".safetensors"):
        d = source if os.path.isdir(source) else os.path.dirname(source)
        import json
        with open(os.path.join(d, "config.json")) as fh:
            cfg = ModelConfig.from_hf(json.load(fh))
        ck = SafetensorsCheckpoint(source)
        from ..quant.int4 import QUANT_METHODS, checkpoint_quant_config, quantized_checkpoint_getter
        qc = checkpoint_quant_config(d)
        getter = ck.get
        if qc.get("quant_method") in QUANT_METHODS:
            getter = quantized_checkpoint_getter(ck, qc)
        return cfg, getter, load_tokenizer(d)
    raise ValueError(f"unknown model source {source!r}")


class LLM:
    """Offline convenience API: ``LLM(model).generate(prompts, SamplingParams(...))``."""

    def __init__(self, model: str = "tiny-llama", **kwargs):
        cfg = EngineConfig.load(**{"model": model, **kwargs})
        self.engine = LLMEngine(cfg)

    def generate(self, prompts, params: Optional[SamplingParams] = None, lora_ids=None) -> List[RequestOutput]:
        return self.engine.generate(prompts, params, lora_ids)

    def beam_search(self, prompt, params=None, lora_id: int = 0):
        return self.engine.beam_search(prompt, params, lora_id)

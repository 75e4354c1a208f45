"""Executes one scheduler step on the device.

Host side: the native ``SeqTables.build_batch`` writes positions, slot mapping, padded block
tables, KV lengths and query offsets for the step straight into pinned int32 buffers; token
ids go into a pinned buffer too. One async H2D copy per buffer, the forward, the sampler,
then one D2H read of the sampled ids (the only synchronisation of the step).

Pure-decode steps of a captured batch size replay a CUDA graph of the whole forward +
greedy argmax (static device buffers, padded rows write no KV and are ignored), which removes
the per-kernel launch cost that dominates small-batch decode.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .. import ops
from ..config import EngineConfig
from ..models.llama import AttnMetadata, LlamaModel
from .kv_cache import KVCacheManager
from .scheduler import SchedulerOutput
from .sequence import Sequence


class _Pinned:
    """Reusable pinned host staging buffers for one step."""

    def __init__(self, max_tokens: int, max_seqs: int, max_blocks: int, pin: bool, max_rows: int = 0):
        kw = dict(pin_memory=pin)
        max_rows = max(max_rows, max_seqs)
        self.input_ids = torch.zeros(max_tokens, dtype=torch.int32, **kw)
        self.positions = torch.zeros(max_tokens, dtype=torch.int32, **kw)
        self.slots = torch.zeros(max_tokens, dtype=torch.int32, **kw)
        self.block_tables = torch.zeros(max_seqs, max_blocks, dtype=torch.int32, **kw)
        self.seq_lens = torch.zeros(max_seqs, dtype=torch.int32, **kw)
        self.query_start = torch.zeros(max_seqs + 1, dtype=torch.int32, **kw)
        self.seq_ids = torch.zeros(max_seqs, dtype=torch.int64)
        self.start = torch.zeros(max_seqs, dtype=torch.int32)
        self.n_new = torch.zeros(max_seqs, dtype=torch.int32)
        self.logits_idx = torch.zeros(max_rows, dtype=torch.int64, **kw)
        self.sampled = torch.zeros(max_rows, dtype=torch.int64, **kw)


class Inflight:
    """A launched step whose sampled ids are still on their way to the host (async scheduling)."""

    def __init__(self, sched, out_dev, host_buf, event, rows):
        self.sched = sched
        self.out_dev = out_dev      # device int64 [ns]: one sampled id per sampled chunk
        self.host_buf = host_buf    # pinned int64 view receiving them
        self.event = event          # recorded after the D2H copy
        self.rows = rows            # seq_id -> row in out_dev
        self.records = []           # (seq, index in output_token_ids) placeholders to fill

    def tokens(self) -> List[int]:
        if self.event is not None:
            self.event.synchronize()
        return self.host_buf.tolist()


class _DecodeGraph:
    def __init__(self, bs: int):
        self.bs = bs
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.input_ids = None
        self.positions = None
        self.slots = None
        self.block_tables = None
        self.seq_lens = None
        self.out_ids = None
        self.logits = None
        self.launches = 0


class ModelRunner:
    def __init__(self, model: LlamaModel, cfg: EngineConfig, kv_cache: Optional[torch.Tensor],
                 kv: KVCacheManager):
        self.model = model
        self.cfg = cfg
        self.kv_cache = kv_cache
        self.kv = kv
        self.device = model.device
        self.is_cuda = self.device.type == "cuda"
        self.block_size = cfg.block_size
        self.max_blocks = (cfg.max_model_len + cfg.block_size - 1) // cfg.block_size
        k_spec = cfg.num_speculative_tokens if cfg.speculative_method != "none" else 0
        max_tokens = cfg.max_num_batched_tokens + cfg.max_num_seqs * (1 + k_spec)
        self.host = _Pinned(max_tokens, cfg.max_num_seqs, self.max_blocks, self.is_cuda,
                            max_rows=cfg.max_num_seqs * (1 + k_spec))
        self.spec_step = 0
        self.greedy_only = False  # draft-model runners: always argmax (deterministic proposals)
        # async scheduling: two pinned receive buffers (step N's D2H is read while step N+1 runs)
        rows = self.host.sampled.numel()
        self.async_bufs = [torch.zeros(rows, dtype=torch.int64, pin_memory=self.is_cuda) for _ in range(2)]
        self.async_flip = 0
        self.graphs: Dict[int, _DecodeGraph] = {}
        self.graph_pool = None
        self.step_counter = 0
        self.num_sms = torch.cuda.get_device_properties(self.device).multi_processor_count if self.is_cuda else 148
        self.timer = None  # optional StepTimer (device span of every step, for benchmarks)
        self.h2d_bytes = 0  # host->device bytes copied by execute() (inputs of every step)
        self.hybrid = getattr(model, "num_gdn_layers", 0) > 0
        if self.hybrid:  # per-sequence recurrent-state slot and reset flag (hybrid GDN models)
            self.gdn_host = torch.zeros(2, cfg.max_num_seqs + 1, dtype=torch.int32, pin_memory=self.is_cuda)
        self.d2h_bytes = 0  # device->host bytes read back (sampled token ids)
        # steps of at least this many tokens run as two halves whose tensor-parallel collectives
        # overlap the other half's compute (0 = never)
        self.split_min_tokens = (cfg.tp_overlap_min_tokens
                                 if cfg.tensor_parallel_size >= max(2, cfg.tp_overlap_min_world) else 0)
        # split-overlap auto-tuning (CUDA, tensor parallel): alternate split / whole on eligible steps,
        # then keep the mode with the lower device time per token
        self.split_auto = bool(self.split_min_tokens) and self.is_cuda and getattr(cfg, "tp_overlap_autotune", False)
        self._tune = {"n": 0, "pending": [], "decided": None, "cur": None, "ms_per_token": None}

    # ------------------------------------------------------------------ batch preparation
    def _fill_host(self, out: SchedulerOutput) -> Tuple[int, int, List[Sequence], List[int]]:
        """Stage the step's inputs. Logits rows: one per sampled chunk, ``verify + 1`` for a
        speculative verify chunk (predictions after the last token and after each draft)."""
        chunks = out.chunks
        n = len(chunks)
        h = self.host
        ids = h.input_ids.numpy()
        self._pending_rows = pending = []
        # per-chunk values are collected in lists and written with one numpy assignment per buffer:
        # an element-wise torch ``__setitem__`` costs microseconds, which at thousands of running
        # sequences per step made this loop the host's largest cost
        seq_ids, starts, n_new = [0] * n, [0] * n, [0] * n
        t = 0
        sample_rows: List[int] = []
        sample_seqs: List[Sequence] = []
        for i, c in enumerate(chunks):
            seq, k, st = c.seq, c.num_tokens, c.start
            seq_ids[i], starts[i], n_new[i] = seq.seq_id, st, k
            if c.tokens is not None:
                toks = c.tokens
            elif k == 1:
                np_ = len(seq.prompt_token_ids)
                toks = (seq.prompt_token_ids[st],) if st < np_ else (seq.output_token_ids[st - np_],)
            else:
                toks = seq.tokens(st, st + k)
            if k == 1:
                ids[t] = toks[0]
            else:
                ids[t:t + k] = toks
            if k and toks[-1] < 0:  # a token still being sampled by the in-flight step
                pending.append((t + k - 1, seq.seq_id))
            t += k
            if c.sample:
                if c.verify:
                    sample_rows.extend(range(t - 1 - c.verify, t))
                else:
                    sample_rows.append(t - 1)
                sample_seqs.append(seq)
        h.seq_ids.numpy()[:n] = seq_ids
        h.start.numpy()[:n] = starts
        h.n_new.numpy()[:n] = n_new
        if self.hybrid:
            g = self.gdn_host.numpy()
            g[0, :n] = [c.seq.state_slot for c in chunks]
            g[1, :n] = [1 if c.start == 0 else 0 for c in chunks]
        T = self.kv.tables.build_batch(h.seq_ids[:n], h.start[:n], h.n_new[:n], h.positions, h.slots,
                                       h.block_tables[:n], h.seq_lens[:n], h.query_start[: n + 1])
        assert T == t
        h.logits_idx.numpy()[: len(sample_rows)] = sample_rows
        return n, T, sample_seqs, sample_rows

    def _half_meta(self, r0: int, r1: int, s0: int, s1: int, nd: int, positions: torch.Tensor, slots: torch.Tensor,
                   bt: torch.Tensor, lens: torch.Tensor, cut: Optional[Tuple[int, int, int]]) -> AttnMetadata:
        """Attention metadata of rows [r0, r1) = sequences [s0, s1) of the step. ``cut`` =
        (sequence, first row, last row + 1) when a prefill sequence is split between the halves:
        the first half sees its KV up to the cut, the second half its rows from the cut on."""
        h = self.host
        dev = self.device
        m = AttnMetadata(positions=positions[r0:r1], slot_mapping=slots[r0:r1], num_decode=max(0, min(s1, nd) - s0))
        ndh = m.num_decode
        if ndh > 0:
            m.decode_block_tables = bt[s0:s0 + ndh]
            m.decode_seq_lens = lens[s0:s0 + ndh]
            m.decode_splits = self._decode_splits(ndh, int(h.seq_lens[s0:s0 + ndh].max()))
        p0 = max(s0, nd)
        if s1 > p0:
            q_lens, seq_lens = [], []
            for i in range(p0, s1):
                a, b = int(h.query_start[i]), int(h.query_start[i + 1])
                L = int(h.seq_lens[i])
                if cut is not None and cut[0] == i:
                    if r0 <= a:      # first half: rows [a, cut) of this sequence, KV up to the cut
                        L -= b - cut[1]
                        b = cut[1]
                    else:            # second half: rows [cut, b), full KV length
                        a = cut[1]
                q_lens.append(b - a)
                seq_lens.append(L)
            qs = [0]
            for q in q_lens:
                qs.append(qs[-1] + q)
            m.num_prefill_tokens = qs[-1]
            m.prefill_block_tables = bt[p0:s1]
            m.prefill_seq_lens = torch.tensor(seq_lens, dtype=torch.int32).to(dev, non_blocking=True)
            m.prefill_query_start = torch.tensor(qs, dtype=torch.int32).to(dev, non_blocking=True)
            if self.is_cuda:
                m.prefill_tiles = ops.prefill_schedule(qs, seq_lens, self.model.H, self.model.Hk,
                                                       self.model.D).to(dev, non_blocking=True)
        return m

    def _split_halves(self, n: int, nd: int, T: int, positions: torch.Tensor, slots: torch.Tensor,
                      bt: torch.Tensor, lens: torch.Tensor) -> tuple:
        """Rows [0, T) in two halves of about T/2 rows (at a sequence boundary, or inside a prefill
        sequence): (rows of the first half, metadata of each half)."""
        qs = self.host.query_start
        tA = T // 2
        c = 0
        while c < n and int(qs[c + 1]) <= tA:
            c += 1
        if c >= n or int(qs[c]) == tA:  # a sequence boundary
            sA, sB, cut = c, c, None
        else:                            # inside prefill sequence c
            sA, sB, cut = c + 1, c, (c, tA, int(qs[c + 1]))
        mA = self._half_meta(0, tA, 0, sA, nd, positions, slots, bt, lens, cut)
        mB = self._half_meta(tA, T, sB, n, nd, positions, slots, bt, lens, cut)
        return tA, mA, mB

    def _mm_meta(self, out: SchedulerOutput, meta: AttnMetadata) -> None:
        """Batch rows of image positions in this step's prompt chunks, with their projected rows."""
        import bisect
        rows, embs = [], []
        r = 0
        for c in out.chunks:
            seq = c.seq
            pos = seq.mm_positions
            if pos is not None and c.start < len(seq.prompt_token_ids):
                lo, hi = c.start, c.start + c.num_tokens
                j0, j1 = bisect.bisect_left(pos, lo), bisect.bisect_left(pos, hi)
                if j1 > j0:
                    rows.extend(r + p - lo for p in pos[j0:j1])
                    embs.append(seq.mm_embeds[j0:j1])
            r += c.num_tokens
        if rows:
            meta.mm_rows = torch.tensor(rows, dtype=torch.int64).to(self.device, non_blocking=True)
            meta.mm_embeds = torch.cat(embs).to(self.device)

    def _decode_splits(self, nd: int, max_len: int) -> int:
        return ops.decode_splits(nd, self.model.Hk, max_len, self.num_sms, self.block_size)

    # ------------------------------------------------------------------ execution
    @torch.inference_mode()
    def execute(self, out: SchedulerOutput) -> List[List[int]]:
        """Run one step; returns, for every chunk with ``sample`` set (in order), its new tokens: one
        sampled token, or for a speculative verify chunk the accepted drafts plus one."""
        self.step_counter += 1
        n, T, sample_seqs, sample_rows = self._fill_host(out)
        if self._pending_rows:
            raise RuntimeError("step inputs contain unresolved tokens: resolve the in-flight step first")
        if self.timer is not None:
            self.timer.begin()
        try:
            return self._timed_execute(out, n, T, sample_seqs, sample_rows)
        finally:
            if self.timer is not None:
                self.timer.end()

    SPLIT_TUNE_STEPS = 12

    def _timed_execute(self, out, n, T, sample_seqs, sample_rows, **kw):
        """``_execute``, with the device time of split-overlap tuning steps recorded."""
        tuning = self.split_auto and self._tune["decided"] is None
        if not tuning:
            return self._execute(out, n, T, sample_seqs, sample_rows, **kw)
        self._tune["cur"] = None
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record()
        res = self._execute(out, n, T, sample_seqs, sample_rows, **kw)
        if self._tune["cur"] is not None:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
            self._tune["pending"].append((self._tune["cur"], T, e0, e1))
            if self._tune["n"] >= self.SPLIT_TUNE_STEPS:
                self._tune_decide()
        return res

    def _split_choice(self, eligible) -> bool:
        """Whether this (eligible) step runs as two overlapped halves."""
        if not eligible:
            return False
        if not self.split_auto:
            return True
        t = self._tune
        if t["decided"] is not None:
            return t["decided"]
        t["cur"] = t["n"] % 2 == 0
        t["n"] += 1
        return t["cur"]

    def _tune_decide(self) -> None:
        """Median device ms per token of the split and the whole tuning steps, summed over the ranks
        (every rank decides at the same eligible step, so all take the same mode)."""
        import statistics
        t = self._tune
        per = {True: [], False: []}
        for use, T, e0, e1 in t["pending"]:
            e1.synchronize()
            per[use].append(e0.elapsed_time(e1) / max(1, T))
        med = torch.tensor([statistics.median(per[True]) if per[True] else float("inf"),
                            statistics.median(per[False]) if per[False] else float("inf")],
                           dtype=torch.float64, device=self.device)
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            dist.all_reduce(med)
        t["ms_per_token"] = (float(med[0]), float(med[1]))
        t["decided"] = bool(med[0] < 0.98 * med[1])
        t["pending"] = []

    @property
    def split_overlap_state(self) -> str:
        """"off", "on", "tuning", or the auto-tuned choice ("auto:on" / "auto:off")."""
        if not self.split_min_tokens:
            return "off"
        if not self.split_auto:
            return "on"
        d = self._tune["decided"]
        return "tuning" if d is None else ("auto:on" if d else "auto:off")

    @torch.inference_mode()
    def launch(self, out: SchedulerOutput, prev: Optional[Inflight]) -> Inflight:
        """Async scheduling: launch a step without waiting for it. Input tokens that the in-flight
        step ``prev`` is still sampling are copied from its device output on the device; the
        sampled ids of this step go to a pinned buffer asynchronously (``Inflight.tokens``)."""
        self.step_counter += 1
        n, T, sample_seqs, sample_rows = self._fill_host(out)
        patch = None
        if self._pending_rows:
            if prev is None:
                raise RuntimeError("unresolved input tokens without an in-flight step")
            in_rows = [r for r, _ in self._pending_rows]
            src = [prev.rows[sid] for _, sid in self._pending_rows]
            patch = (prev.out_dev, in_rows, src)
        if self.timer is not None:
            self.timer.begin()
        try:
            res = self._timed_execute(out, n, T, sample_seqs, sample_rows, patch=patch, sync=False)
        finally:
            if self.timer is not None:
                self.timer.end()
        out_dev = res
        buf = self.async_bufs[self.async_flip][: out_dev.numel()]
        self.async_flip ^= 1
        ev = None
        if self.is_cuda:
            buf.copy_(out_dev, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
        else:
            buf.copy_(out_dev)
        rows = {c.seq.seq_id: i for i, c in enumerate([c for c in out.chunks if c.sample])}
        self.d2h_bytes += 8 * out_dev.numel()
        return Inflight(out, out_dev, buf, ev, rows)

    def _patch_inputs(self, input_ids: torch.Tensor, patch) -> None:
        prev_out, in_rows, src = patch
        dev = input_ids.device
        ir = torch.tensor(in_rows, dtype=torch.int64).to(dev, non_blocking=True)
        sr = torch.tensor(src, dtype=torch.int64).to(dev, non_blocking=True)
        input_ids.index_copy_(0, ir, prev_out.index_select(0, sr).to(input_ids.dtype))
        self.h2d_bytes += 16 * len(in_rows)

    def _execute(self, out: SchedulerOutput, n: int, T: int, sample_seqs: List[Sequence],
                 sample_rows: List[int], patch=None, sync: bool = True):
        nd = len(out.decode)
        h = self.host
        dev = self.device
        lora = self.model.lora
        if lora is not None:
            runs, t = [], 0
            for c in out.chunks:
                runs.append((c.seq.lora_id, t, c.num_tokens))
                t += c.num_tokens
            lora.set_batch_runs(runs)
        lora_active = lora is not None and lora.active
        all_greedy = self.greedy_only or all(s.params.greedy and not s.params.needs_penalties
                                             and not s.params.needs_host_sampling for s in sample_seqs)
        if (self.is_cuda and self.cfg.use_cuda_graphs and nd == n and all_greedy and nd > 0 and not lora_active
                and all(c.verify == 0 for c in out.decode) and self._graph_for(nd) is not None):
            if not sync:
                return self._replay_decode(nd, patch=patch, sync=False)
            return [[t] for t in self._replay_decode(nd)]
        nb = int(max(1, (int(h.seq_lens[:n].max()) + self.block_size - 1) // self.block_size))
        self.h2d_bytes += 4 * (3 * T + n * self.max_blocks + n + (n - nd + 1)) + 8 * max(1, len(sample_rows))
        self.d2h_bytes += 8 * len(sample_rows)
        input_ids = h.input_ids[:T].to(dev, non_blocking=True)
        if patch is not None:
            self._patch_inputs(input_ids, patch)
        positions = h.positions[:T].to(dev, non_blocking=True)
        slots = h.slots[:T].to(dev, non_blocking=True)
        bt = h.block_tables[:n].to(dev, non_blocking=True)[:, :nb]  # contiguous pinned rows; sliced on device
        lens = h.seq_lens[:n].to(dev, non_blocking=True)
        meta = AttnMetadata(positions=positions, slot_mapping=slots, num_decode=nd)
        self._gdn_meta(meta, n)
        if nd > 0:
            meta.decode_block_tables = bt[:nd]
            meta.decode_seq_lens = lens[:nd]
            meta.decode_splits = self._decode_splits(nd, int(h.seq_lens[:nd].max()))
        if n > nd:
            qs = h.query_start[nd: n + 1] - h.query_start[nd]
            meta.num_prefill_tokens = T - nd
            meta.prefill_block_tables = bt[nd:]
            meta.prefill_seq_lens = lens[nd:]
            meta.prefill_query_start = qs.to(dev, non_blocking=True)
            if self.is_cuda:
                meta.prefill_tiles = ops.prefill_schedule(qs.tolist(), h.seq_lens[nd:n].tolist(), self.model.H,
                                                          self.model.Hk, self.model.D).to(dev, non_blocking=True)
        if any(c.seq.mm_positions is not None for c in out.chunks):
            self._mm_meta(out, meta)
        if self._split_choice(self.split_min_tokens and T >= self.split_min_tokens and self.model.can_split_batch()
                              and not lora_active and all(c.verify == 0 for c in out.chunks)):
            meta.halves = self._split_halves(n, nd, T, positions, slots, bt, lens)
        ns = len(sample_rows)
        if ns == 0:
            meta.logits_indices = h.logits_idx[:1].to(dev, non_blocking=True)
            self.model.forward(input_ids, meta, self.kv_cache)
            return [] if sync else torch.zeros(0, dtype=torch.int64, device=dev)
        meta.logits_indices = h.logits_idx[:ns].to(dev, non_blocking=True)
        if all_greedy and all(c.verify == 0 for c in out.chunks):
            # greedy ids straight from the model (under TP: argmax over the vocab shards, no logits gather)
            ids = self.model.forward(input_ids, meta, self.kv_cache, greedy=True)
            if not sync:
                return ids
            if self.is_cuda:
                self.host.sampled[:ns].copy_(ids, non_blocking=True)
                torch.cuda.current_stream().synchronize()
                return [[t] for t in self.host.sampled[:ns].tolist()]
            return [[t] for t in ids.tolist()]
        logits = self.model.forward(input_ids, meta, self.kv_cache)
        if not sync:
            return self._sample_device(logits, sample_seqs)
        sampled = [c for c in out.chunks if c.sample]
        if all(c.verify == 0 for c in sampled):
            return [[t] for t in self.sample(logits, sample_seqs)]
        # speculative verify chunks next to ordinary ones: split the logits rows
        from .speculative import accept_drafts
        plain_rows, ver_rows, plain_seqs, ver_chunks = [], [], [], []
        r = 0
        for c in sampled:
            if c.verify:
                ver_rows.extend(range(r, r + c.verify + 1))
                ver_chunks.append(c)
            else:
                plain_rows.append(r)
                plain_seqs.append(c.seq)
            r += c.verify + 1
        plain = self.sample(logits[plain_rows], plain_seqs) if plain_rows else []
        self.spec_step += 1
        acc = accept_drafts(logits[ver_rows], ver_chunks, [c.seq for c in ver_chunks], self.cfg.seed,
                            self.spec_step)
        res, pi, vi = [], 0, 0
        for c in sampled:
            if c.verify:
                res.append(acc[vi])
                vi += 1
            else:
                res.append([plain[pi]])
                pi += 1
        return res

    @torch.inference_mode()
    def run_hidden(self, out: SchedulerOutput) -> torch.Tensor:
        """Prefill-only forward of ``out`` returning final hidden states [T, hidden] (embeddings)."""
        n, T, _, _ = self._fill_host(out)
        h = self.host
        dev = self.device
        nb = int(max(1, (int(h.seq_lens[:n].max()) + self.block_size - 1) // self.block_size))
        bt = h.block_tables[:n].to(dev)[:, :nb]
        qs = h.query_start[: n + 1].clone()
        meta = AttnMetadata(positions=h.positions[:T].to(dev), slot_mapping=h.slots[:T].to(dev), num_decode=0,
                            num_prefill_tokens=T, prefill_block_tables=bt, prefill_seq_lens=h.seq_lens[:n].to(dev),
                            prefill_query_start=qs.to(dev))
        if self.is_cuda:
            meta.prefill_tiles = ops.prefill_schedule(qs.tolist(), h.seq_lens[:n].tolist(), self.model.H,
                                                      self.model.Hk, self.model.D).to(dev)
        self._gdn_meta(meta, n)
        return self.model.forward(h.input_ids[:T].to(dev), meta, self.kv_cache, hidden_only=True)

    def _gdn_meta(self, meta: AttnMetadata, n: int) -> None:
        """Hybrid GDN models: state slot and reset flag of each sequence, token offsets of all."""
        if not self.hybrid:
            return
        dev = self.device
        meta.gdn_slots = self.gdn_host[0, :n].to(dev, non_blocking=True)
        meta.gdn_reset = self.gdn_host[1, :n].to(dev, non_blocking=True)
        meta.gdn_query_start = self.host.query_start[: n + 1].to(dev, non_blocking=True)
        self.h2d_bytes += 4 * (3 * n + 1)

    def sample(self, logits: torch.Tensor, seqs: List[Sequence]) -> List[int]:
        special = [i for i, s in enumerate(seqs) if s.params.needs_host_sampling]
        if special:
            return self._sample_with_host_modes(logits, seqs, special)
        out = self._sample_device(logits, seqs)
        ns = len(seqs)
        if self.is_cuda:
            self.host.sampled[:ns].copy_(out, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            return self.host.sampled[:ns].tolist()
        return out.tolist()

    def _sample_with_host_modes(self, logits: torch.Tensor, seqs: List[Sequence], special: List[int]) -> List[int]:
        """Rows using typical / mirostat sampling or asking for logprobs: torch per row (after the
        same penalties); the others go through the sampling kernel as usual."""
        from .sampling_modes import sample_row
        plain = [i for i in range(len(seqs)) if i not in set(special)]
        toks = [0] * len(seqs)
        if plain:
            sub = self.sample(logits[plain], [seqs[i] for i in plain])
            for i, t in zip(plain, sub):
                toks[i] = t
        lf = logits.float()
        for i in special:
            s = seqs[i]
            row = lf[i].clone()
            if s.params.needs_penalties:
                pen = self._penalised(row[None], [s])
                row = pen[0]
            toks[i] = sample_row(row, lf[i], s, self.cfg.seed)
        return toks

    def _penalised(self, lf: torch.Tensor, seqs: List[Sequence]) -> torch.Tensor:
        dev = lf.device
        trip = []
        for r, s in enumerate(seqs):
            ou, oc = np.unique(np.asarray([t for t in s.output_token_ids if t >= 0], dtype=np.int64),
                               return_counts=True)
            cnt = dict(zip(ou.tolist(), oc.tolist()))
            toks = set(cnt)
            if s.params.repetition_penalty != 1.0:
                toks |= set(s.prompt_token_ids)
            trip.extend((r, int(tok), int(cnt.get(tok, 0))) for tok in sorted(toks))
        if trip:
            tri = torch.tensor(trip, dtype=torch.int32).to(dev)
            rep = torch.tensor([s.params.repetition_penalty for s in seqs], dtype=torch.float32).to(dev)
            fr = torch.tensor([s.params.frequency_penalty for s in seqs], dtype=torch.float32).to(dev)
            pr = torch.tensor([s.params.presence_penalty for s in seqs], dtype=torch.float32).to(dev)
            ops.apply_penalties(lf, tri, rep, fr, pr)
        return lf

    def _sample_device(self, logits: torch.Tensor, seqs: List[Sequence]) -> torch.Tensor:
        """Sampled ids [ns] (int64, on the logits' device), without synchronising."""
        dev = logits.device
        if self.greedy_only or all(s.params.greedy and not s.params.needs_penalties for s in seqs):
            out = ops.argmax(logits)
        else:
            lf = logits.float()
            if any(s.params.needs_penalties for s in seqs):
                trip = []
                for r, s in enumerate(seqs):
                    if not s.params.needs_penalties:
                        continue
                    ou, oc = np.unique(np.asarray(s.output_token_ids, dtype=np.int64), return_counts=True)
                    cnt = dict(zip(ou.tolist(), oc.tolist()))
                    toks = set(cnt)
                    if s.params.repetition_penalty != 1.0:
                        toks |= set(s.prompt_token_ids)
                    trip.extend((r, int(tok), int(cnt.get(tok, 0))) for tok in sorted(toks))
                if trip:
                    tri = torch.tensor(trip, dtype=torch.int32).to(dev)
                    rep = torch.tensor([s.params.repetition_penalty for s in seqs], dtype=torch.float32).to(dev)
                    fr = torch.tensor([s.params.frequency_penalty for s in seqs], dtype=torch.float32).to(dev)
                    pr = torch.tensor([s.params.presence_penalty for s in seqs], dtype=torch.float32).to(dev)
                    ops.apply_penalties(lf, tri, rep, fr, pr)
            temps = torch.tensor([s.params.temperature for s in seqs], dtype=torch.float32).to(dev)
            tks = torch.tensor([s.params.top_k for s in seqs], dtype=torch.int32).to(dev)
            tps = torch.tensor([s.params.top_p for s in seqs], dtype=torch.float32).to(dev)
            mps = torch.tensor([s.params.min_p for s in seqs], dtype=torch.float32).to(dev)
            seeds = torch.tensor([(s.params.seed if s.params.seed is not None else s.seq_id * 7919 + self.cfg.seed)
                                  for s in seqs], dtype=torch.int64).to(dev)
            offs = torch.tensor([len(s.output_token_ids) for s in seqs], dtype=torch.int64).to(dev)
            out = ops.sample(lf, temps, tks, tps, mps, seeds, offs)
        return out

    # ------------------------------------------------------------------ CUDA graphs
    def _bucket(self, nd: int) -> Optional[int]:
        for b in self.cfg.cuda_graph_batch_sizes:
            if b >= nd and b <= self.cfg.max_num_seqs:
                return b
        return None

    def _graph_for(self, nd: int) -> Optional[_DecodeGraph]:
        b = self._bucket(nd)
        if b is None:
            return None
        g = self.graphs.get(b)
        if g is None:
            g = self._capture(b)
        return g

    def _decode_meta(self, g: _DecodeGraph) -> AttnMetadata:
        splits = self._decode_splits(g.bs, self.cfg.max_model_len)
        meta = AttnMetadata(positions=g.positions, slot_mapping=g.slots, num_decode=g.bs,
                            decode_block_tables=g.block_tables, decode_seq_lens=g.seq_lens,
                            decode_splits=splits)
        if splits > 1:
            meta.decode_workspace = g.workspace
        meta.logits_indices = None
        return meta

    def _capture(self, bs: int) -> _DecodeGraph:
        dev = self.device
        g = _DecodeGraph(bs)
        g.input_ids = torch.zeros(bs, dtype=torch.int32, device=dev)
        g.positions = torch.zeros(bs, dtype=torch.int32, device=dev)
        g.slots = torch.full((bs,), -1, dtype=torch.int32, device=dev)
        g.block_tables = torch.zeros(bs, self.max_blocks, dtype=torch.int32, device=dev)
        g.seq_lens = torch.ones(bs, dtype=torch.int32, device=dev)
        splits = self._decode_splits(bs, self.cfg.max_model_len)
        g.workspace = torch.empty(bs * self.model.H * max(1, splits) * (self.model.D + 2),
                                  dtype=torch.float32, device=dev)
        meta = self._decode_meta(g)
        # warm up (lazy kernel attributes, allocator) outside capture
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self.model.forward(g.input_ids, meta, self.kv_cache, greedy=True)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        if self.graph_pool is None:
            self.graph_pool = torch.cuda.graph_pool_handle()
        n0 = ops.LAUNCHES.n
        with torch.cuda.graph(graph, pool=self.graph_pool):
            g.out_ids = self.model.forward(g.input_ids, meta, self.kv_cache, greedy=True)
        g.launches = ops.LAUNCHES.n - n0
        ops.LAUNCHES.n = n0
        g.graph = graph
        self.graphs[bs] = g
        return g

    def _replay_decode(self, nd: int, patch=None, sync: bool = True):
        g = self._graph_for(nd)
        h = self.host
        bs = g.bs
        self.h2d_bytes += 4 * bs * (4 + self.max_blocks)
        self.d2h_bytes += 8 * bs
        # pad rows: slot -1 (no KV write), length 1, block 0
        if nd < bs:
            h.positions[nd:bs] = 0
            h.slots[nd:bs] = -1
            h.seq_lens[nd:bs] = 1
            h.block_tables[nd:bs] = 0
            h.input_ids[nd:bs] = 0
        g.input_ids.copy_(h.input_ids[:bs], non_blocking=True)
        if patch is not None:
            self._patch_inputs(g.input_ids, patch)
        g.positions.copy_(h.positions[:bs], non_blocking=True)
        g.slots.copy_(h.slots[:bs], non_blocking=True)
        g.seq_lens.copy_(h.seq_lens[:bs], non_blocking=True)
        g.block_tables.copy_(h.block_tables[:bs], non_blocking=True)
        g.graph.replay()
        ops.LAUNCHES.add(g.launches)
        if not sync:
            return g.out_ids[:nd]
        self.host.sampled[:bs].copy_(g.out_ids, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return self.host.sampled[:nd].tolist()

    def capture_all(self, sizes=None) -> None:
        for b in sizes or self.cfg.cuda_graph_batch_sizes:
            if b <= self.cfg.max_num_seqs and b not in self.graphs:
                self._capture(b)

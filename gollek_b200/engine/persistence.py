"""Checkpoint / resume of serving state (no training checkpoints: inference only).

* Prefix-cache snapshot: every cached full KV block (its chain hash and its KV in every layer)
  is written to one safetensors file with a model signature; a restarted engine loads them as
  cached, unowned blocks so prompts sharing those prefixes skip their recomputation. Plays the
  role of the reference's disk prompt-cache store and snapshot reader
  (core/optimization/gollek-plugin-prompt-cache/…/cache/DiskPromptCacheStore.java,
  PromptCacheSnapshotReader.java).
* Request snapshot: queued and running requests (prompt, tokens generated so far, sampling
  parameters) are exported at drain time and re-enqueued after a restart, continuing where they
  stopped (the reference's KV checkpoint on shutdown is a stub, GracefulShutdown.java:269-345).
"""
from __future__ import annotations

import dataclasses
import json
from typing import List

import torch

from .. import ops
from ..loaders.safetensors import SafetensorsFile, save_file
from .sequence import SamplingParams, SeqStatus


def _signature(engine) -> dict:
    m = engine.model
    return {"model": str(engine.cfg.model), "layers": m.cfg.num_hidden_layers, "kv_heads": m.Hk,
            "head_dim": m.D, "block_size": engine.cfg.block_size, "dtype": str(engine.dtype),
            "tp_rank": engine.comm.rank, "tp_size": engine.comm.size, "vocab": m.cfg.vocab_size}


def _tq_save(kv: torch.Tensor, bits: int) -> dict:
    """KV [L, n, 2, Hk, bs, D] -> TurboQuant tensors per (layer, K/V, head): every token's vector of
    that head, the D/4 channels of largest RMS at bits + 1 and the rest at ``bits``."""
    from ..quant.turboquant import quantize_kv
    L, n, _, Hk, bs, D = kv.shape
    out = {}
    for layer in range(L):
        for kvi in range(2):
            for h in range(Hk):
                q = quantize_kv(kv[layer, :, kvi, h].reshape(n * bs, D).float().cpu(), bits, D // 4)
                p = f"tq.{layer}.{kvi}.{h}."
                out[p + "idx"] = q.outlier_idx
                for part, d in (("hi", q.hi), ("lo", q.lo)):
                    out[p + part + "_codes"] = d["codes"]
                    out[p + part + "_norm"] = d["norm"]
    return out


def _tq_load(f, rows, L: int, Hk: int, bs: int, D: int, bits: int, n: int) -> torch.Tensor:
    """Rows ``rows`` of the snapshot's n blocks -> KV [L, len(rows), 2, Hk, bs, D] (fp32)."""
    from ..quant.turboquant import KVQuantized, dequantize_kv
    out = torch.empty(L, len(rows), 2, Hk, bs, D)
    r = torch.tensor(rows)
    for layer in range(L):
        for kvi in range(2):
            for h in range(Hk):
                p = f"tq.{layer}.{kvi}.{h}."
                q = KVQuantized(f.get(p + "idx"), {"codes": f.get(p + "hi_codes"), "norm": f.get(p + "hi_norm")},
                                {"codes": f.get(p + "lo_codes"), "norm": f.get(p + "lo_norm")}, D, bits)
                out[layer, :, kvi, h] = dequantize_kv(q).view(n, bs, D)[r]
    return out


def save_prefix_cache(engine, path: str, max_blocks: int = 0, compress: str = "") -> int:
    """Write the engine's cached prefix blocks to ``path``; returns the number of blocks saved.
    ``compress="turboquant"`` stores the KV at 2.5 bits per value (``quant/turboquant.py``, 6.4x
    smaller than bf16); the blocks restored from it are approximate, so outputs that use them can
    differ slightly from a recomputation."""
    items = engine.kv.pool.cached_items()
    if max_blocks:
        items = items[:max_blocks]
    if not items:
        save_file({"hashes": torch.zeros(0, dtype=torch.int64)}, path, {"signature": json.dumps(_signature(engine))})
        return 0
    hashes = torch.tensor([h for h, _ in items], dtype=torch.int64)
    ids = torch.tensor([b for _, b in items], dtype=torch.int32)
    if getattr(engine.model, "kv_scales", None) is not None:
        raise ValueError("moving KV blocks of an fp8 cache (values + per-token scales) is not supported")
    kv = ops.kv_gather_blocks(engine.kv_cache, ids.to(engine.kv_cache.device))  # [L, n, 2, Hk, bs, D]
    meta = {"signature": json.dumps(_signature(engine))}
    if compress == "turboquant":
        tensors = {"hashes": hashes, **_tq_save(kv, 2)}
        meta.update(compress="turboquant", bits="2", shape=json.dumps(list(kv.shape)))
    elif compress:
        raise ValueError(f"unknown KV compression {compress!r} (turboquant)")
    else:
        tensors = {"hashes": hashes, "kv": kv.transpose(0, 1).contiguous().cpu()}
    save_file(tensors, path, meta)
    return len(items)


def load_prefix_cache(engine, path: str) -> int:
    """Adopt the blocks of a snapshot into the engine's pool as cached prefix blocks (as many as
    fit in free blocks); returns how many were loaded. The model signature must match."""
    f = SafetensorsFile(path)
    try:
        sig = json.loads(f.metadata.get("signature", "{}"))
        if sig != _signature(engine):
            raise ValueError(f"prefix-cache snapshot was written for {sig}, this engine is {_signature(engine)}")
        hashes = f.get("hashes").tolist()
        if not hashes:
            return 0
        compressed = f.metadata.get("compress") == "turboquant"
        kv = None if compressed else f.get("kv")  # [n, L, 2, Hk, bs, D]
        taken, rows = [], []
        for i, h in enumerate(hashes):
            b = engine.kv.pool.adopt_cached(int(h))
            if b < 0:
                if engine.kv.pool.num_free() == 0:
                    break
                continue
            taken.append(b)
            rows.append(i)
        if taken:
            if compressed:
                L, n, _, Hk, bs, D = json.loads(f.metadata["shape"])
                sel = _tq_load(f, rows, L, Hk, bs, D, int(f.metadata["bits"]), n)
            else:
                sel = kv[torch.tensor(rows)].transpose(0, 1).contiguous()  # a copy: the mapping can close
            ops.kv_scatter_blocks(engine.kv_cache, torch.tensor(taken, dtype=torch.int32).to(engine.kv_cache.device),
                                  sel.to(engine.kv_cache.device, engine.kv_cache.dtype))
            del sel
        del kv
        return len(taken)
    finally:
        f.close()


def snapshot_requests(engine) -> List[dict]:
    """Unfinished requests as plain dicts (prompt, generated tokens, sampling parameters)."""
    out = []
    for q in (engine.scheduler.running, engine.scheduler.waiting):
        for s in q:
            if s.status.finished:
                continue
            # a token still in flight (async scheduling placeholder) is not part of the snapshot:
            # it is generated again after the restore
            out.append({"request_id": s.request_id, "prompt_token_ids": list(s.prompt_token_ids),
                        "output_token_ids": [t for t in s.output_token_ids if t >= 0],
                        "params": dataclasses.asdict(s.params),
                        "lora_id": s.lora_id, "priority": getattr(s, "priority", 0)})
    return out


def restore_requests(engine, reqs: List[dict]) -> List[str]:
    """Re-enqueue snapshot requests: generated tokens become part of the prompt (recomputed once,
    or served from a loaded prefix cache) and ``max_tokens`` shrinks by what was already produced."""
    ids = []
    for r in reqs:
        p = SamplingParams(**r["params"])
        done = len(r["output_token_ids"])
        if done >= p.max_tokens:
            continue
        p.max_tokens -= done
        p.min_tokens = max(0, p.min_tokens - done)
        rid = engine.add_request(r["request_id"], list(r["prompt_token_ids"]) + list(r["output_token_ids"]), p,
                                 lora_id=r.get("lora_id", 0), priority=r.get("priority", 0))
        ids.append(rid)
    return ids

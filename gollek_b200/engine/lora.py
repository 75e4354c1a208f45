"""Multi-LoRA serving: adapter registry, GPU slot pool with LRU paging, per-step batching.

Adapters target q/k/v/o (the BASELINE multi-LoRA config: rank 16 on q/k/v/o). Each model layer
holds, per GPU slot, ``A_qkv [3r, hidden]`` (q, k, v shrink matrices stacked), ``B_qkv [qkv_out, r]``,
``A_o [r, q_local]`` and ``B_o [hidden, r]``; slot 0 means "no adapter". Adapters live in host
memory and are copied into a free (or least-recently-used, not in-flight) slot when a request
needs them. Every step, ``set_batch`` groups the step's tokens by slot (CSR segments) and
``apply`` runs the shrink/expand kernels after the base GEMMs (csrc/kernels/lora.cu):

    qkv += scale * (x A_qkv^T) B_qkv^T      (q/k/v column ranges use their own rank block)
    h   += scale * (a A_o^T)   B_o^T

Tensor parallelism: A_qkv and B_o are replicated, B_qkv rows follow the rank's q/k/v heads and
A_o columns follow its o_proj input shard; the o_proj LoRA term is a partial sum like the base
GEMM's, so the layer's single all-reduce covers both.

PEFT format (``adapter_config.json`` with ``r`` / ``lora_alpha`` / ``target_modules``,
``adapter_model.safetensors`` with ``…layers.{i}.self_attn.{q,k,v,o}_proj.lora_{A,B}.weight``) is
read as the reference does (runner/safetensor/gollek-safetensor-engine/…/warmup/LoraAdapterService.java:46-192;
per-request ``adapter_id`` routing …/LoraAdapterRouter.java:262-317).
"""
from __future__ import annotations

import json
import os
from collections import OrderedDict
from dataclasses import dataclass
from typing import Dict, List, Optional

import numpy as np
import torch

from ..native import cuda_ext

MODULES = ("q_proj", "k_proj", "v_proj", "o_proj")


@dataclass
class HostAdapter:
    name: str
    rank: int
    scale: float
    # per layer: {"q_proj": (A [r, in], B [out, r]), ...} full (unsharded) fp32/bf16 tensors on CPU
    layers: List[Dict[str, tuple]]


class LoRAManager:
    def __init__(self, model, max_loras: int = 64, max_rank: int = 16):
        self.model = model
        self.max_loras = max_loras
        self.r = max_rank
        cfg = model.cfg
        dev, dt = model.device, model.dtype
        self.device, self.dtype = dev, dt
        L = cfg.num_hidden_layers
        H, Hk, D = model.H, model.Hk, model.D
        if getattr(model, "D_logical", D) != D:
            raise NotImplementedError("multi-LoRA needs a kernel-native head size (32/64/128/256)")
        S = max_loras + 1
        hidden = cfg.hidden_size
        qkv_out = (H + 2 * Hk) * D
        self.n1, self.n2 = H * D, (H + Hk) * D
        self.A_qkv = [torch.zeros(S, 3 * self.r, hidden, dtype=dt, device=dev) for _ in range(L)]
        self.B_qkv = [torch.zeros(S, qkv_out, self.r, dtype=dt, device=dev) for _ in range(L)]
        self.A_o = [torch.zeros(S, self.r, H * D, dtype=dt, device=dev) for _ in range(L)]
        self.B_o = [torch.zeros(S, hidden, self.r, dtype=dt, device=dev) for _ in range(L)]
        self.scales = torch.zeros(S, dtype=torch.float32, device=dev)
        self.adapters: Dict[int, HostAdapter] = {}
        self.name_to_id: Dict[str, int] = {}
        self.slot_of: "OrderedDict[int, int]" = OrderedDict()  # adapter id -> slot (LRU order)
        self.free_slots = list(range(S - 1, 0, -1))
        self.loads = 0
        self._batch = None
        model.lora = self

    # ------------------------------------------------------------------ registry
    def add_adapter(self, name: str, layers: List[Dict[str, tuple]], rank: int, alpha: float) -> int:
        if rank > self.r:
            raise ValueError(f"adapter rank {rank} exceeds max_lora_rank {self.r}")
        aid = self.name_to_id.get(name) or (max(self.adapters, default=0) + 1)
        self.adapters[aid] = HostAdapter(name, rank, alpha / rank, layers)
        self.name_to_id[name] = aid
        if aid in self.slot_of:  # re-registered: refresh the resident copy
            self._upload(aid, self.slot_of[aid])
        return aid

    def random_adapter(self, name: str, seed: int, rank: int = 16, alpha: Optional[float] = None,
                       std_a: float = 0.02, std_b: float = 0.002) -> int:
        """Adapter with A ~ N(0, std_a), B ~ N(0, std_b) on q/k/v/o (benchmark adapters)."""
        cfg = self.model.cfg
        g = torch.Generator().manual_seed(seed)
        h, q, kv = cfg.hidden_size, cfg.q_size, cfg.kv_size
        dims = {"q_proj": (h, q), "k_proj": (h, kv), "v_proj": (h, kv), "o_proj": (q, h)}
        layers = []
        for _ in range(cfg.num_hidden_layers):
            layers.append({m: (torch.randn(rank, i, generator=g) * std_a, torch.randn(o, rank, generator=g) * std_b)
                           for m, (i, o) in dims.items()})
        return self.add_adapter(name, layers, rank, alpha if alpha is not None else float(rank))

    def load_peft(self, path: str, name: Optional[str] = None) -> int:
        from ..loaders.safetensors import SafetensorsCheckpoint
        with open(os.path.join(path, "adapter_config.json")) as f:
            ac = json.load(f)
        rank, alpha = int(ac["r"]), float(ac.get("lora_alpha", ac["r"]))
        ck = SafetensorsCheckpoint(os.path.join(path, "adapter_model.safetensors"))
        cfg = self.model.cfg
        layers = [dict() for _ in range(cfg.num_hidden_layers)]
        for k in ck.keys():
            parts = k.split(".")
            if "layers" not in parts or "lora_A" not in k and "lora_B" not in k:
                continue
            li = int(parts[parts.index("layers") + 1])
            mod = next((m for m in MODULES if m in parts), None)
            if mod is None:
                continue
            ab = 0 if "lora_A" in k else 1
            cur = list(layers[li].get(mod, (None, None)))
            cur[ab] = ck.get(k).float()
            layers[li][mod] = tuple(cur)
        return self.add_adapter(name or os.path.basename(path.rstrip("/")), layers, rank, alpha)

    # ------------------------------------------------------------------ slots
    def _upload(self, aid: int, slot: int) -> None:
        ad = self.adapters[aid]
        m = self.model
        tp, r = m.comm.size, m.comm.rank
        H, Hk, D = m.H, m.Hk, m.D
        rr = ad.rank
        with torch.no_grad():
            for li, mods in enumerate(ad.layers):
                self.A_qkv[li][slot].zero_()
                self.B_qkv[li][slot].zero_()
                self.A_o[li][slot].zero_()
                self.B_o[li][slot].zero_()
                for j, name in enumerate(("q_proj", "k_proj", "v_proj")):
                    if name not in mods:
                        continue
                    A, B = mods[name]
                    self.A_qkv[li][slot, j * self.r: j * self.r + rr] = A.to(self.device, self.dtype)
                    if name == "q_proj":
                        rows = B[r * H * D:(r + 1) * H * D]
                        self.B_qkv[li][slot, 0:H * D, :rr] = rows.to(self.device, self.dtype)
                    else:
                        kv0 = m.kv_head0 * D
                        rows = B[kv0: kv0 + Hk * D]
                        off = H * D if name == "k_proj" else (H + Hk) * D
                        self.B_qkv[li][slot, off:off + Hk * D, :rr] = rows.to(self.device, self.dtype)
                if "o_proj" in mods:
                    A, B = mods["o_proj"]
                    self.A_o[li][slot, :rr] = A[:, r * H * D:(r + 1) * H * D].to(self.device, self.dtype)
                    self.B_o[li][slot, :, :rr] = B.to(self.device, self.dtype)
        self.scales[slot] = ad.scale
        self.loads += 1

    def acquire(self, aid: int, pinned: set) -> int:
        """Slot holding adapter ``aid`` (loading it, evicting the LRU adapter not in ``pinned``)."""
        if aid in self.slot_of:
            self.slot_of.move_to_end(aid)
            return self.slot_of[aid]
        if aid not in self.adapters:
            raise KeyError(f"unknown adapter id {aid}")
        if self.free_slots:
            slot = self.free_slots.pop()
        else:
            victim = next((a for a in self.slot_of if a not in pinned), None)
            if victim is None:
                raise RuntimeError("all LoRA slots are in use by the current batch")
            slot = self.slot_of.pop(victim)
        self._upload(aid, slot)
        self.slot_of[aid] = slot
        return slot

    # ------------------------------------------------------------------ per step
    def set_batch(self, token_adapter_ids: List[int]) -> None:
        """Group the step's tokens (in model-input order) by adapter slot; 0 = base model."""
        runs, t = [], 0
        for a in token_adapter_ids:  # per-token ids as (adapter, start, length) runs
            if runs and runs[-1][0] == a and runs[-1][1] + runs[-1][2] == t:
                runs[-1][2] += 1
            else:
                runs.append([a, t, 1])
            t += 1
        self.set_batch_runs([tuple(r) for r in runs])

    def set_batch_runs(self, runs: List[tuple]) -> None:
        """Same from (adapter id, first token, token count) runs (one per scheduled chunk): the
        work is per run, not per token."""
        ids = set(a for a, _, n in runs if a and n)
        if not ids:
            self._batch = None
            return
        slots = {a: self.acquire(a, ids) for a in ids}
        groups: Dict[int, List[tuple]] = {}
        for a, t0, n in runs:
            if a and n:
                groups.setdefault(slots[a], []).append((t0, n))
        seg_slot = sorted(groups)
        seg_ptr, parts, tiles = [0], [], []
        total = 0
        for i, s in enumerate(seg_slot):
            cnt = sum(n for _, n in groups[s])
            tiles.extend((i, p) for p in range(total, total + cnt, 64))  # 64-token tiles
            parts.extend(np.arange(t0, t0 + n, dtype=np.int32) for t0, n in groups[s])
            total += cnt
            seg_ptr.append(total)
        tok = np.concatenate(parts)
        dev = self.device
        self._batch = (torch.tensor(seg_ptr, dtype=torch.int32).to(dev, non_blocking=True),
                       torch.from_numpy(tok).to(dev, non_blocking=True),
                       torch.tensor(seg_slot, dtype=torch.int32).to(dev, non_blocking=True),
                       seg_ptr, tok.tolist() if not dev.type == "cuda" else None, seg_slot,
                       torch.tensor(tiles, dtype=torch.int32).view(-1, 2).to(dev, non_blocking=True))

    @property
    def active(self) -> bool:
        return self._batch is not None

    def apply(self, li: int, mod: str, x: torch.Tensor, y: torch.Tensor) -> None:
        """y += LoRA(x) for the tokens of adapter-using sequences (in place)."""
        if self._batch is None:
            return
        seg_ptr, tok, seg_slot, seg_ptr_h, tok_h, seg_slot_h, tiles = self._batch
        if mod == "qkv":
            A, B, n1, n2 = self.A_qkv[li], self.B_qkv[li], self.n1, self.n2
        else:
            A, B, n1, n2 = self.A_o[li], self.B_o[li], y.shape[1], y.shape[1]
        R = A.shape[1]
        if not x.is_cuda:
            self._apply_ref(A, B, n1, n2, x, y, seg_ptr_h, tok_h, seg_slot_h)
            return
        max_seg = max(b - a for a, b in zip(seg_ptr_h[:-1], seg_ptr_h[1:]))
        V = torch.zeros(x.shape[0], R, dtype=torch.float32, device=x.device)  # K chunks accumulate atomically
        ext = cuda_ext()
        ext.lora_shrink(V, x, A, seg_ptr, tok, seg_slot, tiles, max_seg)
        ext.lora_expand(y, V, B, n1, n2, self.scales, seg_ptr, tok, seg_slot, tiles)

    def _apply_ref(self, A, B, n1, n2, x, y, seg_ptr, tok, seg_slot) -> None:
        r = self.r
        for i, s in enumerate(seg_slot):
            idx = torch.tensor(tok[seg_ptr[i]:seg_ptr[i + 1]], dtype=torch.long)
            v = x[idx].float() @ A[s].float().t()
            out = torch.zeros(len(idx), y.shape[1])
            bounds = [(0, n1, 0), (n1, n2, r), (n2, y.shape[1], 2 * r)] if n1 != n2 else [(0, y.shape[1], 0)]
            for lo, hi, ro in bounds:
                if hi > lo:
                    out[:, lo:hi] = v[:, ro:ro + r] @ B[s][lo:hi].float().t()
            y[idx] = (y[idx].float() + float(self.scales[s]) * out).to(y.dtype)


def merged_weights(weights: Dict[str, torch.Tensor], adapter: HostAdapter) -> Dict[str, torch.Tensor]:
    """HF weights with one adapter merged (W + scale * B A): the oracle for LoRA tests."""
    out = dict(weights)
    for li, mods in enumerate(adapter.layers):
        for name, (A, B) in mods.items():
            k = f"model.layers.{li}.self_attn.{name}.weight"
            out[k] = (weights[k].float() + adapter.scale * (B.float() @ A.float())).to(weights[k].dtype)
    return out

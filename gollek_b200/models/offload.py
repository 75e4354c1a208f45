"""Layer weight offload: run a model whose weights do not all fit in device memory.

The weights of the offloaded layers live in pinned host memory. A pool of ``depth`` device slots,
each the size of one layer's weights, is filled on a dedicated copy stream: while layer i
computes, layers i+1 .. i+depth-1 are already being copied host→device. Events order the copy
of a slot after the compute that last used it, and the compute of a layer after its copy.

Replaces the reference's weight-offloading runner (core/optimization/gollek-plugin-weight-offload/
…/WeightOffloadingV2Runner.java: pinned host weights, async H2D prefetch of layer N+1, adaptive
prefetch depth); the prefetch depth here is fixed per engine (``EngineConfig.offload_prefetch``).
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch

# the large matrices move; norms, biases and routers (a few KB) stay resident
OFFLOADED_KEYS = ("w_qkv", "w_o", "w_gate_up", "w_down", "moe_gu", "moe_down")


class LayerOffload:
    def __init__(self, layers: List[dict], offloaded: List[int], device: torch.device, depth: int = 2):
        if depth < 1:
            raise ValueError("prefetch depth must be >= 1")
        self.device = device
        self.offloaded = sorted(set(offloaded))
        self.index = {li: k for k, li in enumerate(self.offloaded)}
        self.depth = min(depth, max(1, len(self.offloaded)))
        self.keys: Dict[int, List[str]] = {}
        self.host: Dict[int, Dict[str, torch.Tensor]] = {}
        # move the offloaded layers' tensors to pinned host memory; remember shapes per key
        for li in self.offloaded:
            L = layers[li]
            self.keys[li] = [k for k, v in L.items() if isinstance(v, torch.Tensor) and k in OFFLOADED_KEYS]
            self.host[li] = {k: L[k].to("cpu").pin_memory() for k in self.keys[li]}
            for k in self.keys[li]:
                L[k] = None  # placeholders until acquired
        self.layers = layers
        # device slots sized for the largest offloaded layer, tensor by tensor
        proto = self.host[self.offloaded[0]] if self.offloaded else {}
        self.slots = [{k: torch.empty_like(v, device=device) for k, v in proto.items()} for _ in range(self.depth)]
        self.slot_of: Dict[int, int] = {}
        self.copy_stream = torch.cuda.Stream(device=device)
        self.copied = [torch.cuda.Event() for _ in range(self.depth)]
        self.released = [torch.cuda.Event() for _ in range(self.depth)]
        self.bytes_copied = 0

    def _issue(self, li: int) -> None:
        if li not in self.index or li in self.slot_of:
            return
        slot = self.index[li] % self.depth
        for other, s in list(self.slot_of.items()):
            if s == slot:
                del self.slot_of[other]
        with torch.cuda.stream(self.copy_stream):
            self.copy_stream.wait_event(self.released[slot])  # the previous user of this slot is done
            for k in self.keys[li]:
                src = self.host[li][k]
                dst = self.slots[slot][k]
                if dst.shape != src.shape:
                    raise ValueError(f"offloaded layer {li} tensor {k} differs in shape from the slot")
                dst.copy_(src, non_blocking=True)
                self.bytes_copied += src.numel() * src.element_size()
            self.copied[slot].record(self.copy_stream)
        self.slot_of[li] = slot

    def begin_forward(self) -> None:
        """Start the copies of the first ``depth`` offloaded layers."""
        for li in self.offloaded[: self.depth]:
            self._issue(li)

    def acquire(self, li: int) -> dict:
        """Layer ``li``'s weights on the device (waits for its copy on the compute stream)."""
        if li not in self.index:
            return self.layers[li]
        self._issue(li)
        slot = self.slot_of[li]
        torch.cuda.current_stream().wait_event(self.copied[slot])
        L = dict(self.layers[li])
        L.update(self.slots[slot])
        return L

    def release(self, li: int) -> None:
        """Layer ``li`` has been enqueued on the compute stream: its slot may be refilled after it
        finishes; prefetch the layer ``depth`` positions ahead."""
        if li not in self.index:
            return
        slot = self.slot_of[li]
        self.released[slot].record(torch.cuda.current_stream())
        k = self.index[li] + self.depth
        if k < len(self.offloaded):
            self._issue(self.offloaded[k])

"""Zero-downtime model hot-swap for the server.

Reference behaviour: runner/safetensor/gollek-safetensor-lifecycle/…/ModelHotSwapManager.java:96-165
(load the new model in the background while the old one serves, promote it atomically, drain the
old one, unload it; refused while another swap of the alias runs or memory is short; lifecycle
events LOADING / WARMING_UP / PROMOTED / DRAINING / UNLOADED / COMPLETE / FAILED).

Here a swap builds a new ``LLMEngine`` on a worker thread, warms it with a one-token generation,
wraps it in its own ``AsyncEngine`` and swaps the server's engine reference; requests that
started on the old engine keep their handle to it and finish there (drain, bounded by
``drain_timeout_s``), after which the old engine is shut down and its device memory released.
"""
from __future__ import annotations

import asyncio
import gc
import time
import uuid
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

PHASES = ("LOADING", "WARMING_UP", "PROMOTED", "DRAINING", "UNLOADED", "COMPLETE", "FAILED")


@dataclass
class SwapState:
    swap_id: str
    model: str
    name: str
    events: List[dict] = field(default_factory=list)
    done: bool = False
    failed: bool = False

    def emit(self, phase: str, message: str) -> None:
        self.events.append({"phase": phase, "message": message, "time": time.time()})

    @property
    def phase(self) -> str:
        return self.events[-1]["phase"] if self.events else "PENDING"

    def as_dict(self) -> dict:
        return {"swapId": self.swap_id, "model": self.model, "name": self.name, "phase": self.phase,
                "done": self.done, "failed": self.failed, "events": list(self.events)}


class HotSwapManager:
    """``build(model)`` returns a ready ``LLMEngine`` for a preset name / checkpoint path."""

    def __init__(self, state, build: Callable[[str], object], drain_timeout_s: float = 30.0,
                 memory_check: Optional[Callable[[str], Optional[str]]] = None):
        self.state = state
        self.build = build
        self.drain_timeout_s = drain_timeout_s
        self.memory_check = memory_check
        self.swaps: Dict[str, SwapState] = {}
        self.active: Optional[SwapState] = None

    def begin(self, model: str, name: Optional[str] = None) -> SwapState:
        if self.active is not None and not self.active.done:
            raise RuntimeError(f"swap {self.active.swap_id} already in progress")
        if self.memory_check is not None:
            problem = self.memory_check(model)
            if problem:
                raise MemoryError(problem)
        sw = SwapState("swap-" + uuid.uuid4().hex[:12], model, name or self.state.model_name)
        self.swaps[sw.swap_id] = sw
        self.active = sw
        sw.emit("LOADING", f"loading {model} while the current model serves")
        asyncio.get_running_loop().create_task(self._run(sw))
        return sw

    async def _run(self, sw: SwapState) -> None:
        from .async_engine import AsyncEngine
        try:
            engine = await asyncio.to_thread(self.build, sw.model)
            sw.emit("WARMING_UP", "one-token warm-up generation")
            from ..engine.sequence import SamplingParams
            await asyncio.to_thread(engine.generate, [[1, 2, 3]],
                                    SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True))
            new_ae = AsyncEngine(engine).start()
            old_ae = self.state.ae
            self.state.ae = new_ae  # atomic for the event loop: every later request sees the new engine
            self.state.model_name = sw.name
            sw.emit("PROMOTED", f"{sw.name} now serves new requests")
            sw.emit("DRAINING", f"old engine finishes its in-flight requests (at most {self.drain_timeout_s:g} s)")
            await asyncio.to_thread(old_ae.shutdown, True, self.drain_timeout_s)
            old_engine = old_ae.engine
            del old_ae
            self._release(old_engine)
            sw.emit("UNLOADED", "old model released")
            sw.emit("COMPLETE", "hot-swap complete")
        except Exception as e:  # the old engine keeps serving
            sw.failed = True
            sw.emit("FAILED", f"swap failed: {e!r}")
        finally:
            sw.done = True

    @staticmethod
    def _release(engine) -> None:
        for attr in ("model", "kv_cache", "runner"):
            if hasattr(engine, attr):
                try:
                    setattr(engine, attr, None)
                except Exception:
                    pass
        gc.collect()
        try:
            import torch
            if torch.cuda.is_available():
                torch.cuda.empty_cache()
        except Exception:
            pass


def default_memory_check(model: str) -> Optional[str]:
    """Refuse a swap when the device cannot hold a second model's weights next to the first
    (both are resident during the swap)."""
    try:
        import torch
        if not torch.cuda.is_available():
            return None
        from ..engine.engine import load_model_source
        cfg, _, _ = load_model_source(model)
        need = 2 * cfg.num_params()
        free, _ = torch.cuda.mem_get_info()
        if free < need:
            return f"{free / 2**30:.1f} GiB free, {need / 2**30:.1f} GiB of weights needed"
    except Exception:
        return None
    return None

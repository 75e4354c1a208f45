"""Engine metrics: request latencies (TTFT, TPOT, end-to-end), throughput, batch and KV usage.

Exported to Prometheus text format by the server's ``/metrics`` route. Covers the reference's
metric surface (core/gollek-observability/…/metrics/PrometheusMetrics.java,
InferenceMetricsCollector.java; inference/gollek-engine/…/engine/inference/InferenceMetrics.java;
llama.cpp runner's gollek.gguf.ttft etc., runner/llamacpp/gollek-runner-llamacpp/README.md:53)
but with true per-token timestamps instead of the reference's chars/4 estimates.
"""
from __future__ import annotations

import threading
import time
from collections import deque
from typing import Deque, Dict, List

import numpy as np


def percentile(xs, q: float) -> float:
    return float(np.percentile(np.asarray(xs, dtype=np.float64), q)) if len(xs) else 0.0


class EngineMetrics:
    def __init__(self, window: int = 10000):
        self.lock = threading.Lock()
        self.start = time.perf_counter()
        self.requests_arrived = 0
        self.requests_finished = 0
        self.prompt_tokens = 0
        self.generation_tokens = 0
        self.steps = 0
        self.preemptions = 0
        self.ttft: Deque[float] = deque(maxlen=window)
        self.tpot: Deque[float] = deque(maxlen=window)
        self.e2e: Deque[float] = deque(maxlen=window)
        self.step_time: Deque[float] = deque(maxlen=window)
        self.num_running = 0
        self.num_waiting = 0
        self.kv_usage = 0.0
        self.per_adapter: Dict[int, int] = {}

    def on_arrival(self) -> None:
        with self.lock:
            self.requests_arrived += 1

    def on_step(self, dt: float, tokens: int, new_tokens: int, running: int, waiting: int, kv_usage: float,
                preempted: int) -> None:
        with self.lock:
            self.steps += 1
            self.step_time.append(dt)
            self.generation_tokens += new_tokens
            self.num_running, self.num_waiting, self.kv_usage = running, waiting, kv_usage
            self.preemptions += preempted

    def on_finish(self, seq) -> None:
        with self.lock:
            self.requests_finished += 1
            self.prompt_tokens += seq.num_prompt_tokens
            self.per_adapter[seq.lora_id] = self.per_adapter.get(seq.lora_id, 0) + 1
            if seq.first_token_time is not None:
                self.ttft.append(seq.first_token_time - seq.arrival_time)
            n = len(seq.output_token_ids)
            if n > 1 and seq.first_token_time is not None and seq.finish_time is not None:
                self.tpot.append((seq.finish_time - seq.first_token_time) / (n - 1))
            if seq.finish_time is not None:
                self.e2e.append(seq.finish_time - seq.arrival_time)

    def snapshot(self) -> dict:
        with self.lock:
            el = time.perf_counter() - self.start
            return {
                "requests_arrived": self.requests_arrived,
                "requests_finished": self.requests_finished,
                "prompt_tokens": self.prompt_tokens,
                "generation_tokens": self.generation_tokens,
                "generation_tok_per_s": self.generation_tokens / el if el > 0 else 0.0,
                "steps": self.steps,
                "preemptions": self.preemptions,
                "ttft_p50_ms": 1e3 * percentile(self.ttft, 50),
                "ttft_p95_ms": 1e3 * percentile(self.ttft, 95),
                "tpot_p50_ms": 1e3 * percentile(self.tpot, 50),
                "tpot_p95_ms": 1e3 * percentile(self.tpot, 95),
                "e2e_p50_ms": 1e3 * percentile(self.e2e, 50),
                "step_p50_ms": 1e3 * percentile(self.step_time, 50),
                "num_running": self.num_running,
                "num_waiting": self.num_waiting,
                "kv_cache_usage": self.kv_usage,
                "per_adapter_requests": dict(self.per_adapter),
            }

    def prometheus(self, prefix: str = "gollek") -> str:
        s = self.snapshot()
        lines: List[str] = []
        for k, v in s.items():
            if isinstance(v, dict):
                for a, c in v.items():
                    lines.append(f'{prefix}_{k}{{adapter="{a}"}} {c}')
            else:
                lines.append(f"{prefix}_{k} {v}")
        return "\n".join(lines) + "\n"

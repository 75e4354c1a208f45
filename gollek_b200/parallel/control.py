"""Control plane of multi-rank serving: step events, heartbeats, failure detection.

Tensor-parallel ranks run identical schedulers: rank 0 (the driver) receives requests, and before
every step publishes that step's events (request adds with their arrival times, aborts) through
the rendezvous key-value store; every rank applies them in order and steps its engine, so all
ranks schedule the same batch and meet in the same collectives. Messages carry a sequence number
and a CRC32; a worker that does not receive step ``n`` within ``timeout_s`` (a dropped message, a
dead driver) or receives a corrupt one raises ``ControlTimeout`` / ``ProtocolError`` instead of
entering a collective its peers never join.

Each rank's watchdog thread refreshes ``hb/<rank>`` every ``heartbeat_s``; the driver checks peers
before publishing a step and raises ``RankFailure`` for a rank whose heartbeat is older than
``stale_s`` (a crashed or hung process), again before any collective could block on it. Failures
are host-side only: no GPU fault, trap or hang is involved in detecting them.

The reference's failure handling is request-level (resilience4j circuit breaker / retry,
inference/gollek-engine/…/resilience/ResilienceManager.java:52-101; health checks
DefaultHealthCheckService.java:124-230); it has no multi-rank runtime to supervise.
"""
from __future__ import annotations

import datetime
import threading
import time
import zlib
from dataclasses import dataclass
from typing import Any, List, Optional

import msgpack


class RankFailure(RuntimeError):
    def __init__(self, rank: int, age: float):
        super().__init__(f"rank {rank} missed its heartbeat for {age:.1f}s")
        self.rank, self.age = rank, age


class ControlTimeout(RuntimeError):
    pass


class ProtocolError(RuntimeError):
    pass


def _encode(seq: int, payload: Any) -> bytes:
    body = msgpack.packb({"seq": seq, "payload": payload}, use_bin_type=True)
    return zlib.crc32(body).to_bytes(4, "little") + body


def _decode(raw: bytes, want_seq: int) -> Any:
    if len(raw) < 4 or zlib.crc32(raw[4:]) != int.from_bytes(raw[:4], "little"):
        raise ProtocolError(f"control message {want_seq}: checksum mismatch")
    try:
        msg = msgpack.unpackb(raw[4:], raw=False)
    except Exception as e:
        raise ProtocolError(f"control message {want_seq}: undecodable ({e})") from e
    if msg.get("seq") != want_seq:
        raise ProtocolError(f"control message out of order: expected {want_seq}, got {msg.get('seq')}")
    return msg["payload"]


class ControlPlane:
    def __init__(self, rank: int, world: int, store, timeout_s: float = 30.0, heartbeat_s: float = 0.5,
                 stale_s: float = 5.0, prefix: str = "gollek/ctl/"):
        import torch.distributed as dist
        self.rank, self.world = rank, world
        self.store = dist.PrefixStore(prefix, store)
        self.timeout_s, self.heartbeat_s, self.stale_s = timeout_s, heartbeat_s, stale_s
        self.seq = 0
        self._stop = threading.Event()
        self._hb: Optional[threading.Thread] = None
        self.started = time.time()

    # ------------------------------------------------------------------ heartbeats
    def start_heartbeat(self) -> "ControlPlane":
        self._beat()
        self._hb = threading.Thread(target=self._hb_loop, daemon=True, name=f"gollek-hb-{self.rank}")
        self._hb.start()
        return self

    def _beat(self) -> None:
        self.store.set(f"hb/{self.rank}", repr(time.time()))

    def _hb_loop(self) -> None:
        while not self._stop.wait(self.heartbeat_s):
            try:
                self._beat()
            except Exception:
                return  # store gone (shutdown): nothing left to supervise

    def heartbeat_age(self, rank: int) -> float:
        try:
            return time.time() - float(self.store.get(f"hb/{rank}").decode())
        except Exception:
            return time.time() - self.started

    def check_peers(self) -> None:
        """Raise RankFailure for the first peer whose heartbeat is stale."""
        for r in range(self.world):
            if r == self.rank:
                continue
            age = self.heartbeat_age(r)
            if age > self.stale_s:
                raise RankFailure(r, age)

    def stop(self) -> None:
        self._stop.set()
        if self._hb is not None:
            self._hb.join(timeout=2 * self.heartbeat_s + 1)

    # ------------------------------------------------------------------ step events
    def publish(self, payload: Any) -> int:
        """Driver: publish the next step's payload (after checking that every peer is alive)."""
        self.check_peers()
        self.seq += 1
        self.store.set(f"step/{self.seq}", _encode(self.seq, payload))
        return self.seq

    def receive(self) -> Any:
        """Worker: the next step's payload, or ControlTimeout / ProtocolError / RankFailure(0)."""
        self.seq += 1
        key = f"step/{self.seq}"
        try:
            self.store.wait([key], datetime.timedelta(seconds=self.timeout_s))
        except Exception as e:
            age = self.heartbeat_age(0)
            if age > self.stale_s:
                raise RankFailure(0, age) from e
            raise ControlTimeout(f"no control message {self.seq} within {self.timeout_s}s") from e
        return _decode(self.store.get(key), self.seq)


@dataclass
class _Event:
    kind: str
    args: dict


class DriverEngine:
    """Rank 0's view of a replicated engine: same API as ``LLMEngine`` for the front end (the
    async server), but every request event is published to the other ranks before the step that
    uses it. Workers run ``follow`` until told to stop."""

    def __init__(self, engine, control: ControlPlane):
        self.engine, self.control = engine, control
        self._events: List[dict] = []

    def __getattr__(self, name):  # metrics, cfg, tokenizer, ... come from the local engine
        return getattr(self.engine, name)

    def add_request(self, request_id, prompt, params=None, lora_id: int = 0, arrival_time=None, priority: int = 0,
                    images=None):
        if images:
            raise ValueError("image inputs are served on a single GPU (tensor-parallel serving takes text only)")
        import dataclasses
        import time as _t
        from ..engine.sequence import SamplingParams
        params = (params or SamplingParams()).validate()
        arrival_time = arrival_time if arrival_time is not None else _t.perf_counter()
        if isinstance(prompt, str):
            prompt = self.engine.tokenizer.encode(prompt)
        rid = self.engine.add_request(request_id, list(prompt), params, lora_id, arrival_time, priority)
        self._events.append({"kind": "add", "request_id": rid, "prompt": list(prompt),
                             "params": dataclasses.asdict(params), "lora_id": lora_id, "arrival": arrival_time,
                             "priority": priority})
        return rid

    def abort_request(self, request_id: str) -> bool:
        self._events.append({"kind": "abort", "request_id": request_id})
        return self.engine.abort_request(request_id)

    def step(self):
        ev, self._events = self._events, []
        self.control.publish({"op": "step", "events": ev})
        return self.engine.step()

    def has_unfinished(self) -> bool:
        return self.engine.has_unfinished()

    def shutdown_workers(self) -> None:
        self.control.publish({"op": "stop", "events": []})


def apply_events(engine, events: List[dict]) -> None:
    from ..engine.sequence import SamplingParams
    for e in events:
        if e["kind"] == "add":
            engine.add_request(e["request_id"], e["prompt"], SamplingParams(**e["params"]), e.get("lora_id", 0),
                               e.get("arrival"), e.get("priority", 0))
        elif e["kind"] == "abort":
            engine.abort_request(e["request_id"])
        else:
            raise ProtocolError(f"unknown control event {e['kind']!r}")


def follow(engine, control: ControlPlane, max_steps: Optional[int] = None) -> int:
    """Worker loop: apply each published step's events and step the engine; returns steps run."""
    n = 0
    while max_steps is None or n < max_steps:
        msg = control.receive()
        if msg["op"] == "stop":
            return n
        apply_events(engine, msg["events"])
        engine.step()
        n += 1
    return n

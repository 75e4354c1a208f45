"""Failure detection of multi-rank serving, exercised on gloo CPU ranks with host-side faults
only: a rank that dies between steps, a dropped or corrupted control message, a slow rank."""
import multiprocessing as mp
import socket

import pytest
import torch

from gollek_b200.models.reference import ReferenceDecoder


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(scenario, world=2, timeout=120):
    from tests.ctl_worker import run
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=run, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, kind, val = q.get(timeout=timeout)
        res.setdefault(rank, []).append((kind, val))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res


def _oracle(cfg, w):
    ref = ReferenceDecoder(cfg, w)
    return {"a": ref.greedy(list(range(1, 20)), 5)[0], "b": ref.greedy(list(range(5, 40)), 5)[0]}


@pytest.mark.parametrize("scenario", ["ok", "slow"])
def test_replicated_driver_serves(tiny_cfg, tiny_weights, scenario):
    """Rank 0 publishes step events; the worker follows; tokens equal the oracle (a slow worker
    within the timeouts changes nothing)."""
    res = _run(scenario)
    kind, outs = res[0][0]
    assert kind == "ok", res
    assert outs == _oracle(tiny_cfg, tiny_weights)
    assert res[1][0][0] == "ok", res


def test_dead_rank_detected_before_next_collective():
    res = _run("rank_dies")
    assert ("RankFailure", 1) in res[0], res


def test_dropped_control_message_times_out():
    res = _run("drop")
    assert res[1][0][0] == "ControlTimeout", res


def test_corrupted_control_message_rejected():
    res = _run("corrupt")
    assert res[1][0][0] == "ProtocolError", res

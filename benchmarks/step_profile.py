"""Steady-state serving steps without the fill phase (for per-kernel attribution).

Builds the Llama-3-8B engine (random init), puts ``--decodes`` sequences directly into the decode
state at contexts uniform in [prompt_min, prompt_max] (their KV blocks allocated, contents random),
and runs ``--steps`` engine steps; every step one new request of ``--prefill-len`` tokens arrives and
one old sequence is retired, which is the composition of a saturated serving step (≈ one prompt
prefill next to ~255 decodes). Prints the mean CUDA-event time of a step.

    python benchmarks/step_profile.py --steps 5
    ncu --metrics gpu__time_duration.sum --clock-control none -s 2000 -c 2000 --csv --log-file l.csv \
        python benchmarks/step_profile.py --steps 5
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--decodes", type=int, default=255)
    ap.add_argument("--prefill-len", type=int, default=1088)
    ap.add_argument("--prompt-min", type=int, default=128)
    ap.add_argument("--prompt-max", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--layers", type=int, default=0)
    a = ap.parse_args()
    from gollek_b200.config import EngineConfig, preset
    from gollek_b200.engine.engine import LLMEngine
    from gollek_b200.engine.sequence import SamplingParams, SeqStatus, Sequence

    cfg = preset(a.model)
    if a.layers:
        cfg.num_hidden_layers = a.layers
    ec = EngineConfig(device="cuda", max_num_seqs=a.decodes + 1, max_num_batched_tokens=8192,
                      max_model_len=a.prompt_max + 512, enable_prefix_caching=False, gpu_memory_utilization=0.9)
    eng = LLMEngine(ec, model_cfg=cfg)
    rng = np.random.default_rng(0)
    sp = SamplingParams(temperature=0.0, max_tokens=10 ** 6, ignore_eos=True)
    for i in range(a.decodes):
        L = int(rng.integers(a.prompt_min, a.prompt_max + 1))
        seq = Sequence(f"d{i}", rng.integers(0, cfg.vocab_size, L).tolist(), SamplingParams(**vars(sp)))
        eng.kv.add(seq)
        assert eng.kv.ensure(seq, L + 1)
        seq.output_token_ids = [int(rng.integers(0, cfg.vocab_size))]
        seq.num_computed_tokens = L
        seq.status = SeqStatus.RUNNING
        eng.scheduler.running.append(seq)
        eng.seqs[seq.request_id] = seq
    times = []
    for s in range(a.steps):
        eng.add_request(f"p{s}", rng.integers(0, cfg.vocab_size, a.prefill_len).tolist(), SamplingParams(**vars(sp)))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        eng.step()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
        old = eng.scheduler.running[0]
        eng.abort_request(old.request_id)
    print(f"step ms: {[round(t, 2) for t in times]}  mean(after first) {np.mean(times[1:]):.2f}")


if __name__ == "__main__":
    main()

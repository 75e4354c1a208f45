"""The end-to-end workload benchmarks (benchmarks/config_bench.py) run on CPU at toy sizes."""
import json
import os
import sys

import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "benchmarks"))
import config_bench  # noqa: E402


@pytest.mark.parametrize("argv,expect", [
    (["--workload", "gguf-lora", "--model", "tiny-llama", "--ffn", "512", "--scale", "0.02"], ["gguf-q4k-multilora"]),
    (["--workload", "llama70b-fp8", "--model", "tiny-llama", "--ffn", "512", "--scale", "0.01"],
     ["llama70b-fp8-decode"] + ["llama70b-fp8-prefill"] * 3),
    (["--workload", "mixtral-ep", "--model", "tiny-mixtral", "--scale", "0.02"],
     ["mixtral-ep-prefill", "mixtral-ep-decode"]),
    (["--workload", "deepseek-ep", "--model", "tiny-deepseek-v3", "--scale", "0.02"],
     ["deepseek-v3-ep-prefill", "deepseek-v3-ep-decode"]),
])
def test_workloads_run(argv, expect, capsys):
    config_bench.main(argv + ["--device", "cpu"])
    recs = [json.loads(ln) for ln in capsys.readouterr().out.splitlines() if ln.startswith("{")]
    assert [r["workload"] for r in recs] == expect
    assert all(r["ms"] > 0 for r in recs)

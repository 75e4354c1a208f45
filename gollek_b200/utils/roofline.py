"""Roofline arithmetic against the peaks measured on this hardware (``MEASURED_PEAKS.json`` at the
repository root: STREAM-style copy bandwidth and cuBLAS bf16 throughput) or the given fallback.

    python -m gollek_b200.utils.roofline --flops 1.9e12 --bytes 3.4e9 --ms 1.2 [--nvlink-bytes 8e6]
"""
from __future__ import annotations

import argparse
import json
import os
from dataclasses import dataclass

FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
NVLINK_GBS = 770.0  # measured peer copy, per direction per GPU


def peaks(path: str = None) -> dict:
    path = path or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                                "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        d["source"] = "measured"
        return d
    return {**FALLBACK, "source": "fallback"}


@dataclass
class Roofline:
    ms: float
    tflops: float
    gbs: float
    frac_compute: float
    frac_hbm: float
    frac_roofline: float  # achieved ÷ the slower of compute, HBM and NVLink bounds
    bound: str

    def as_dict(self) -> dict:
        return dict(self.__dict__)


def analyse(flops: float, nbytes: float, ms: float, nvlink_bytes: float = 0.0, sustained: bool = False,
            pk: dict = None) -> Roofline:
    pk = pk or peaks()
    tf = pk["bf16_tflops_sustained" if sustained and "bf16_tflops_sustained" in pk else "bf16_tflops"]
    t_c = flops / (tf * 1e12)
    t_m = nbytes / (pk["hbm_gbs"] * 1e9)
    t_n = nvlink_bytes / (NVLINK_GBS * 1e9)
    t_roof = max(t_c, t_m, t_n)
    bound = "compute" if t_roof == t_c else ("hbm" if t_roof == t_m else "nvlink")
    s = ms * 1e-3
    return Roofline(ms, flops / s / 1e12 if s else 0.0, nbytes / s / 1e9 if s else 0.0, t_c / s if s else 0.0,
                    t_m / s if s else 0.0, t_roof / s if s else 0.0, bound)


def main(argv=None):
    ap = argparse.ArgumentParser(prog="gollek_b200.utils.roofline")
    ap.add_argument("--flops", type=float, default=0.0)
    ap.add_argument("--bytes", type=float, default=0.0)
    ap.add_argument("--nvlink-bytes", type=float, default=0.0)
    ap.add_argument("--ms", type=float, required=True)
    ap.add_argument("--sustained", action="store_true")
    a = ap.parse_args(argv)
    pk = peaks()
    r = analyse(a.flops, a.bytes, a.ms, a.nvlink_bytes, a.sustained, pk)
    print(json.dumps({**r.as_dict(), "peaks": pk.get("source")}))


if __name__ == "__main__":
    main()

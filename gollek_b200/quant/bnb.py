"""bitsandbytes-serialized checkpoints (QLoRA NF4 / FP4 4-bit, LLM.int8 8-bit).

Layout of a 4-bit linear ``<name>`` as HF writes it (tensor names as in transformers'
quantizers/quantizer_bnb_4bit.py; the reference dequantizes the same tensors on the CPU:
core/quantizer/gollek-quantizer-turboquant/…/turboquant/BnBDequantizer.java:5-45):

* ``<name>.weight``       uint8 [N * K / 2, 1]: the row-major [N, K] codes, two per byte, the first
                          of each pair in the high nibble;
* ``<name>.weight.absmax`` one scale per ``blocksize`` consecutive elements of the flattened matrix
                          (fp32, or uint8 codes when the statistics are themselves quantized);
* ``<name>.weight.quant_map`` the 16 code values (NF4 levels, or the FP4 values);
* ``<name>.weight.nested_absmax`` / ``.nested_quant_map`` (double quantization): absmax =
                          nested_quant_map[code] * nested_absmax[block of nested_blocksize] + offset;
* ``<name>.weight.quant_state.bitsandbytes__<type>``: uint8 bytes of a JSON object with quant_type,
                          blocksize, shape, dtype and, with double quantization, nested_blocksize
                          and nested_offset.

w = quant_map[code] * absmax[block]. NF4 with blocks inside rows (K a multiple of the block size,
block size a multiple of 32) becomes an NF4 ``Int4Weight``, served by the int4 kernels; other code
maps are dequantized to bf16. 8-bit: ``<name>.weight`` int8 [N, K], ``<name>.SCB`` fp32 [N]:
w = q * SCB / 127 (dequantized to bf16).
"""
from __future__ import annotations

import json
from typing import Dict, Optional

import torch

from .int4 import NF4_LEVELS, Int4Weight, _pack


def _state(t: torch.Tensor) -> dict:
    return json.loads(bytes(t.to(torch.uint8).flatten().tolist()).decode("utf-8"))


def from_bnb4(packed: torch.Tensor, absmax: torch.Tensor, quant_map: torch.Tensor, state: dict,
              nested_absmax: Optional[torch.Tensor] = None,
              nested_quant_map: Optional[torch.Tensor] = None) -> "Int4Weight | torch.Tensor":
    N, K = (int(v) for v in state["shape"])
    bs = int(state["blocksize"])
    b = packed.to(torch.uint8).flatten().to(torch.int64)
    codes = torch.stack([b >> 4, b & 0xF], 1).flatten()[: N * K]          # element 2i in the high nibble
    if nested_absmax is not None:
        nbs = int(state.get("nested_blocksize", 256))
        a = absmax.to(torch.int64).flatten()
        am = nested_quant_map.float()[a] * nested_absmax.float().repeat_interleave(nbs)[: a.numel()]
        am = am + float(state.get("nested_offset", 0.0))
    else:
        am = absmax.float().flatten()
    qm = quant_map.float().flatten()
    nf4 = qm.numel() == 16 and torch.allclose(qm, NF4_LEVELS, atol=1e-6)
    if nf4 and K % bs == 0 and bs % 32 == 0:
        return Int4Weight(_pack(codes.view(N, K)), am.view(N, K // bs).to(torch.bfloat16), None, N, K, bs, nf4=True)
    w = qm[codes] * am.repeat_interleave(bs)[: N * K]
    return w.view(N, K).to(torch.bfloat16)


def to_bnb4(w: torch.Tensor, blocksize: int = 64, quant_map: Optional[torch.Tensor] = None,
            double_quant: bool = False, quant_type: str = "nf4") -> Dict[str, torch.Tensor]:
    """Matrix -> the bnb 4-bit tensors above (suffixes relative to ``<name>.weight``); ``quant_map``
    defaults to the NF4 levels. Double quantization codes the absmax with a 256-level map per block
    of 256 after removing their mean."""
    N, K = w.shape
    qm = NF4_LEVELS.clone() if quant_map is None else quant_map.float()
    x = w.float().flatten().view(-1, blocksize)
    am = x.abs().amax(1).clamp_min(1e-12)
    codes = ((x / am[:, None])[..., None] - qm).abs().argmin(-1).flatten()
    if codes.numel() % 2:
        codes = torch.cat([codes, torch.zeros(1, dtype=codes.dtype)])
    packed = ((codes[0::2] << 4) | codes[1::2]).to(torch.uint8).view(-1, 1)
    state = {"quant_type": quant_type, "blocksize": blocksize, "dtype": "bfloat16", "shape": [N, K]}
    out = {"": packed, ".quant_map": qm}
    if double_quant:
        offset = float(am.mean())
        c = am - offset
        nbs = 256
        pad = (-c.numel()) % nbs
        cp = torch.cat([c, torch.zeros(pad)]).view(-1, nbs)
        nab = cp.abs().amax(1).clamp_min(1e-12)
        nmap = torch.linspace(-1, 1, 256)
        q = ((cp / nab[:, None])[..., None] - nmap).abs().argmin(-1).flatten()[: c.numel()]
        out.update({".absmax": q.to(torch.uint8), ".nested_absmax": nab, ".nested_quant_map": nmap})
        state.update(nested_blocksize=nbs, nested_dtype="float32", nested_offset=offset)
    else:
        out[".absmax"] = am
    js = json.dumps(state).encode("utf-8")
    out[f".quant_state.bitsandbytes__{quant_type}"] = torch.tensor(list(js), dtype=torch.uint8)
    return out


def bnb_getter(ck):
    """``get("….weight")`` for a bitsandbytes checkpoint: 4-bit linears as NF4 ``Int4Weight`` (or bf16),
    8-bit ones as bf16, everything else as stored."""
    keys = set(ck.keys())

    def get(name: str):
        if name + ".absmax" in keys:
            st = next(k for k in keys if k.startswith(name + ".quant_state.bitsandbytes__"))
            nested = name + ".nested_absmax" in keys
            return from_bnb4(ck.get(name), ck.get(name + ".absmax"), ck.get(name + ".quant_map"), _state(ck.get(st)),
                             ck.get(name + ".nested_absmax") if nested else None,
                             ck.get(name + ".nested_quant_map") if nested else None)
        if name.endswith(".weight") and name[:-7] + ".SCB" in keys:
            q = ck.get(name).float()
            return (q * ck.get(name[:-7] + ".SCB").float()[:, None] / 127.0).to(torch.bfloat16)
        return ck.get(name)
    return get

"""safetensors reader/writer (own implementation: header parse, mmap, sharded index).

Format: 8-byte little-endian header length N, N bytes of JSON mapping tensor name →
``{"dtype", "shape", "data_offsets": [begin, end]}`` (offsets relative to the byte after
the header), optional ``__metadata__``; raw little-endian tensor bytes follow. Sharded
checkpoints carry ``model.safetensors.index.json`` with a ``weight_map`` name → file.

Covers the reference loader's behaviour (runner/safetensor/gollek-safetensor-loader/…/
SafetensorFFMLoader.java:171,210-227,259-267 mmap with copy fallback; SafetensorShardIndex.java
shard index; SafetensorDType.java dtypes F64/F32/F16/BF16/F8_E4M3/F8_E5M2/ints/bool).
"""
from __future__ import annotations

import json
import mmap
import os
import struct
from typing import Dict, Iterator, Optional

import numpy as np
import torch

DTYPES = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
    "BOOL": torch.bool,
}
NAMES = {v: k for k, v in DTYPES.items()}


class SafetensorsFile:
    """One ``.safetensors`` file, memory-mapped; tensors are zero-copy CPU views."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        if size < 8:
            raise ValueError(f"{path}: not a safetensors file (too small)")
        (n,) = struct.unpack("<Q", self._f.read(8))
        if n > size - 8:
            raise ValueError(f"{path}: header length {n} exceeds file size")
        header = json.loads(self._f.read(n))
        self.metadata = header.pop("__metadata__", {}) or {}
        self.header = header
        self.data_start = 8 + n
        try:
            self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
            self._buf = np.frombuffer(self._mm, dtype=np.uint8)
        except (ValueError, OSError):  # e.g. file systems without mmap: copy fallback
            self._f.seek(0)
            self._mm = None
            self._buf = np.frombuffer(self._f.read(), dtype=np.uint8)
        for name, info in header.items():
            b, e = info["data_offsets"]
            if info["dtype"] not in DTYPES:
                raise ValueError(f"{path}: unsupported dtype {info['dtype']} for {name}")
            if e < b or self.data_start + e > size:
                raise ValueError(f"{path}: bad offsets for {name}")

    def keys(self):
        return self.header.keys()

    def get(self, name: str) -> torch.Tensor:
        info = self.header[name]
        b, e = info["data_offsets"]
        dt = DTYPES[info["dtype"]]
        raw = self._buf[self.data_start + b: self.data_start + e]
        with torch.no_grad():
            t = torch.frombuffer(raw, dtype=torch.uint8) if raw.size else torch.empty(0, dtype=torch.uint8)
            t = t.view(dt) if raw.size else torch.empty(0, dtype=dt)
        return t.view(info["shape"])

    def close(self):
        self._buf = None
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:  # tensors still view the mapping: it is released with them
                pass
        self._f.close()


class SafetensorsCheckpoint:
    """A single file or a sharded directory (``model.safetensors.index.json``)."""

    def __init__(self, path: str):
        self.files: Dict[str, SafetensorsFile] = {}
        self.index: Dict[str, str] = {}
        if os.path.isdir(path):
            idx = os.path.join(path, "model.safetensors.index.json")
            if os.path.exists(idx):
                with open(idx) as f:
                    wm = json.load(f)["weight_map"]
                for name, fn in wm.items():
                    self.index[name] = os.path.join(path, fn)
            else:
                for fn in sorted(os.listdir(path)):
                    if fn.endswith(".safetensors"):
                        self._open(os.path.join(path, fn))
        else:
            self._open(path)

    def _open(self, fp: str) -> SafetensorsFile:
        if fp not in self.files:
            self.files[fp] = SafetensorsFile(fp)
            for k in self.files[fp].keys():
                self.index.setdefault(k, fp)
        return self.files[fp]

    def keys(self):
        return list(self.index.keys())

    def get(self, name: str) -> torch.Tensor:
        return self._open(self.index[name]).get(name)

    def items(self) -> Iterator:
        for k in self.keys():
            yield k, self.get(k)

    def close(self):
        for f in self.files.values():
            f.close()


def save_file(tensors: Dict[str, torch.Tensor], path: str, metadata: Optional[dict] = None) -> None:
    header = {}
    off = 0
    order = sorted(tensors)
    for name in order:
        t = tensors[name]
        nbytes = t.numel() * t.element_size()
        header[name] = {"dtype": NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for name in order:
            t = tensors[name].detach().contiguous().cpu()
            f.write(t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b"")


def save_sharded(tensors: Dict[str, torch.Tensor], directory: str, max_shard_bytes: int = 4 << 30) -> None:
    os.makedirs(directory, exist_ok=True)
    shards, cur, size = [], {}, 0
    for name in sorted(tensors):
        nb = tensors[name].numel() * tensors[name].element_size()
        if cur and size + nb > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[name] = tensors[name]
        size += nb
    if cur:
        shards.append(cur)
    wm = {}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(directory, fn))
        for k in sh:
            wm[k] = fn
    with open(os.path.join(directory, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wm}, f, indent=1)

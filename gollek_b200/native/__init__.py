"""Loading and building of the native extensions.

Two in-tree shared objects are built with ``torch.utils.cpp_extension`` into
``<repo>/build/`` (``build_all()``; ``__graft_entry__.build`` calls it):

* ``gollek_b200_C``    — the sm_100a CUDA kernels (``csrc/kernels/*.cu``), compiled with
  ``-gencode arch=compute_100a,code=sm_100a`` only.
* ``gollek_b200_host`` — host C++ runtime: GGUF quantizers/dequantizers, the KV block
  allocator fast path, the batch-metadata builder and the output-length predictor.

The loaders import the built ``.so`` directly from the build folder, so a GPU process
never JIT-compiles. ``cuda_ext()`` raises if the CUDA extension is missing: GPU code
paths have no silent PyTorch fallback.
"""
from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os
import sys
import threading
from typing import Optional

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
BUILD_DIR = os.path.join(REPO, "build")
CSRC = os.path.join(REPO, "csrc")

_lock = threading.Lock()
_cache: dict = {}

CUDA_SOURCES = [
    "bindings.cpp",
    "kernels/elementwise.cu",
    "kernels/attention.cu",
    "kernels/gemm.cu",
    "kernels/sampling.cu",
    "comm/symm.cu",
    "comm/nvls.cu",
    "comm/ep_a2a.cu",
    "kernels/noalloc.cu",
    "kernels/lora.cu",
    "kernels/gguf.cu",
    "kernels/gemm_fp8.cu", "kernels/gemm_q4k.cu",
    "kernels/attention_tc.cu",
    "kernels/moe.cu",
    "kernels/kv_transfer.cu",
    "kernels/kv_fp8.cu",
    "kernels/int4.cu",
    "kernels/gdn.cu",
]
HOST_SOURCES = [
    "host/host_bindings.cpp",
    "host/gguf_quant.cpp",
    "host/gguf_kquants.cpp",
    "host/block_allocator.cpp",
    "host/forelen.cpp",
    "host/spec_ngram.cpp",
    "host/grammar.cpp",
]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
                           "-Xptxas", "-v" if os.environ.get("GOLLEK_PTXAS_VERBOSE") else "-O3",
                           "-DNDEBUG"]


def _so_path(name: str) -> Optional[str]:
    cands = glob.glob(os.path.join(BUILD_DIR, name, f"{name}*.so"))
    return cands[0] if cands else None


def _import_so(name: str, path: str):
    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[name] = mod
    return mod


def _load(name: str):
    with _lock:
        if name in _cache:
            return _cache[name]
        path = _so_path(name)
        mod = None
        if path is not None:
            import torch  # noqa: F401  (libtorch symbols must be loaded first)
            mod = _import_so(name, path)
        _cache[name] = mod
        return mod


def cuda_ext():
    """The sm_100a kernel module. Raises if it has not been built (no silent fallback)."""
    mod = _load("gollek_b200_C")
    if mod is None:
        raise RuntimeError(
            "gollek_b200 CUDA extension is not built: run `python -c 'import __graft_entry__ as g; g.build()'` "
            "(or gollek_b200.native.build_all()) first")
    return mod


def host_ext(build_if_missing: bool = True):
    """The host C++ runtime module (GGUF quantizers, block allocator, predictor)."""
    mod = _load("gollek_b200_host")
    if mod is None and build_if_missing:
        build_host()
        with _lock:
            _cache.pop("gollek_b200_host", None)
        mod = _load("gollek_b200_host")
    if mod is None:
        raise RuntimeError("gollek_b200 host extension could not be built")
    return mod


def _build(name: str, sources: list, cuda: bool, verbose: bool = False) -> str:
    from torch.utils import cpp_extension
    os.makedirs(os.path.join(BUILD_DIR, name), exist_ok=True)
    os.environ.setdefault("CUDA_HOME", "/usr/local/cuda")
    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 4)))
    srcs = [os.path.join(CSRC, s) for s in sources]
    kwargs = dict(
        name=name,
        sources=srcs,
        build_directory=os.path.join(BUILD_DIR, name),
        # no fused multiply-add contraction: dequantized values must round as the formats define
        extra_cflags=["-O3", "-std=c++17", "-fPIC", "-ffp-contract=off"],
        extra_include_paths=[CSRC],
        verbose=verbose,
        is_python_module=True,
    )
    if cuda:
        kwargs["extra_cuda_cflags"] = NVCC_FLAGS
        kwargs["with_cuda"] = True
    else:
        kwargs["with_cuda"] = False
    cpp_extension.load(**kwargs)
    path = _so_path(name)
    assert path, f"build of {name} produced no shared object"
    with _lock:
        _cache.pop(name, None)
    return path


def build_cuda(verbose: bool = False) -> str:
    return _build("gollek_b200_C", CUDA_SOURCES, cuda=True, verbose=verbose)


def build_host(verbose: bool = False) -> str:
    return _build("gollek_b200_host", HOST_SOURCES, cuda=False, verbose=verbose)


def build_all(verbose: bool = False) -> None:
    build_host(verbose)
    build_cuda(verbose)

"""GGUF conversion service and its REST routes (``/v1/converter/gguf/*``).

Conversions: a safetensors checkpoint directory (``config.json`` + ``*.safetensors``) → GGUF at a
tensor type or a ``*_K_{S,M,L}`` mixture, and GGUF → GGUF requantization. They run in a worker
thread as jobs with progress (per tensor), cancellation, and a server-sent-event stream; paths are
resolved inside an input and an output base directory (``GOLLEK_CONVERTER_INPUT_DIR`` /
``GOLLEK_CONVERTER_OUTPUT_DIR``, default ``$GOLLEK_HOME/models`` and ``$GOLLEK_HOME/converted``),
and a path that resolves outside its base is refused.

Routes and DTO fields follow the reference's resource (inference/gollek-api-rest/…/api/rest/
GGUFConverterResource.java:52-336: health, convert, convert/preview, convert/stream,
convert/{id}/cancel, detect-format, model-info, verify, quantizations, recommend-quantization;
ConversionRequest / ConversionResponse field names). The conversion itself is this package's own
GGUF writer and block quantizers.
"""
from __future__ import annotations

import glob
import json
import os
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

# id, description, quality level, approximate compression vs f32, use case
QUANTIZATIONS = [
    ("F32", "32-bit floating point", "LOSSLESS", 1.0, "reference / debugging"),
    ("F16", "16-bit floating point", "LOSSLESS", 2.0, "full quality, half the size"),
    ("BF16", "16-bit brain floating point", "LOSSLESS", 2.0, "full quality, bf16 training checkpoints"),
    ("Q8_0", "8-bit quantization", "HIGH", 3.8, "near-lossless serving"),
    ("Q6_K", "6-bit K-quant", "HIGH", 4.9, "high quality at a quarter of f16 + 50%"),
    ("Q5_K_M", "5-bit K-quant (medium)", "HIGH", 5.7, "quality-oriented serving"),
    ("Q5_K_S", "5-bit K-quant (small)", "HIGH", 5.8, "quality-oriented serving, smaller"),
    ("Q5_1", "5-bit quantization (higher quality)", "MEDIUM", 5.3, "legacy 5-bit"),
    ("Q5_0", "5-bit quantization (fast)", "MEDIUM", 5.8, "legacy 5-bit"),
    ("Q4_K_M", "4-bit K-quant (medium)", "MEDIUM", 6.8, "recommended default for serving"),
    ("Q4_K_S", "4-bit K-quant (small)", "MEDIUM", 7.1, "memory-constrained serving"),
    ("Q4_1", "4-bit quantization (higher quality)", "MEDIUM", 6.4, "legacy 4-bit"),
    ("Q4_0", "4-bit quantization (fast)", "MEDIUM", 7.1, "legacy 4-bit"),
    ("Q3_K_L", "3-bit K-quant (large)", "LOW", 7.6, "very constrained memory"),
    ("Q3_K_M", "3-bit K-quant (medium)", "LOW", 8.2, "very constrained memory"),
    ("Q3_K_S", "3-bit K-quant (small)", "LOW", 9.1, "very constrained memory"),
    ("Q2_K", "2-bit K-quant", "VERY_LOW", 11.6, "experiments only"),
]
_QUANT_IDS = {q[0] for q in QUANTIZATIONS}


def recommend(model_size_gb: float, prioritize_quality: bool = False) -> str:
    """A quantization for a model of ``model_size_gb`` (f16 size)."""
    if prioritize_quality:
        return "Q8_0" if model_size_gb <= 16 else ("Q6_K" if model_size_gb <= 40 else "Q5_K_M")
    if model_size_gb <= 4:
        return "Q8_0"
    if model_size_gb <= 30:
        return "Q5_K_M" if model_size_gb <= 10 else "Q4_K_M"
    return "Q4_K_M" if model_size_gb <= 150 else "Q3_K_M"


def detect_format(path: str) -> str:
    if os.path.isdir(path):
        if glob.glob(os.path.join(path, "*.safetensors")):
            return "safetensors"
        if glob.glob(os.path.join(path, "*.gguf")):
            return "gguf"
        if glob.glob(os.path.join(path, "*.bin")) or glob.glob(os.path.join(path, "*.pt")):
            return "pytorch"
        return "unknown"
    if not os.path.exists(path):
        return "missing"
    with open(path, "rb") as f:
        head = f.read(8)
    if head[:4] == b"GGUF":
        return "gguf"
    if path.endswith(".safetensors"):
        return "safetensors"
    if path.endswith((".bin", ".pt", ".pth")):
        return "pytorch"
    return "unknown"


def _human(n: int) -> str:
    for unit in ("B", "KB", "MB", "GB", "TB"):
        if n < 1024 or unit == "TB":
            return f"{n:.1f} {unit}" if unit != "B" else f"{n} B"
        n /= 1024.0
    return f"{n} B"


def _size(path: str) -> int:
    if os.path.isdir(path):
        return sum(os.path.getsize(p) for p in glob.glob(os.path.join(path, "*")) if os.path.isfile(p))
    return os.path.getsize(path) if os.path.exists(path) else 0


def model_info(path: str) -> Dict[str, Any]:
    """Format, size and (for GGUF / safetensors) architecture, tensor count and type histogram."""
    fmt = detect_format(path)
    info: Dict[str, Any] = {"path": path, "format": fmt, "sizeBytes": _size(path), "size": _human(_size(path))}
    if fmt == "gguf":
        from ..loaders.gguf import GGML_TYPES, GGUFFile
        gp = path if os.path.isfile(path) else sorted(glob.glob(os.path.join(path, "*.gguf")))[0]
        f = GGUFFile(gp)
        try:
            types: Dict[str, int] = {}
            params = 0
            for ti in f.tensors.values():
                types[GGML_TYPES[ti.ggml_type][0]] = types.get(GGML_TYPES[ti.ggml_type][0], 0) + 1
                params += ti.numel
            arch = f.metadata.get("general.architecture", "unknown")
            info.update(architecture=arch, tensorCount=len(f.tensors), tensorTypes=types, parameters=params,
                        contextLength=f.metadata.get(f"{arch}.context_length"),
                        vocabSize=len(f.metadata.get("tokenizer.ggml.tokens", [])) or None,
                        tokenizer=f.metadata.get("tokenizer.ggml.model"))
        finally:
            f.close()
    elif fmt == "safetensors":
        cfg_path = os.path.join(path, "config.json")
        if os.path.exists(cfg_path):
            with open(cfg_path) as fh:
                c = json.load(fh)
            info.update(architecture=(c.get("architectures") or [c.get("model_type")])[0],
                        hiddenSize=c.get("hidden_size"), layers=c.get("num_hidden_layers"),
                        vocabSize=c.get("vocab_size"))
    return info


def verify_gguf(path: str) -> Dict[str, Any]:
    """Read every tensor of a GGUF file: sizes inside the file, values decodable and finite."""
    from ..loaders.gguf import GGUFFile
    errors: List[str] = []
    checked = 0
    try:
        f = GGUFFile(path)
    except Exception as e:  # noqa: BLE001
        return {"path": path, "valid": False, "errors": [f"header: {e}"], "tensorsChecked": 0}
    try:
        size = os.path.getsize(path)
        for name, ti in f.tensors.items():
            if ti.offset + ti.nbytes > size:
                errors.append(f"{name}: data runs past the end of the file")
                continue
            try:
                t = f.get(name)
                if not bool(t.isfinite().all()):
                    errors.append(f"{name}: non-finite values")
            except Exception as e:  # noqa: BLE001
                errors.append(f"{name}: {e}")
            checked += 1
    finally:
        f.close()
    return {"path": path, "valid": not errors, "errors": errors[:50], "tensorsChecked": checked}


class ConversionCancelled(Exception):
    pass


@dataclass
class ConversionJob:
    conversion_id: int
    request_id: str
    input_path: str
    output_path: str
    quantization: str
    status: str = "PENDING"      # PENDING RUNNING COMPLETED FAILED CANCELLED
    progress: float = 0.0
    current: str = ""
    error: Optional[str] = None
    started: float = field(default_factory=time.time)
    finished: Optional[float] = None
    cancel: threading.Event = field(default_factory=threading.Event)
    events: List[Dict[str, Any]] = field(default_factory=list)
    cond: threading.Condition = field(default_factory=threading.Condition)

    def emit(self, **ev) -> None:
        with self.cond:
            self.events.append(ev)
            self.cond.notify_all()


class ConverterService:
    def __init__(self, input_base: Optional[str] = None, output_base: Optional[str] = None):
        home = os.environ.get("GOLLEK_HOME", os.path.expanduser("~/.gollek"))
        self.input_base = os.path.realpath(input_base or os.environ.get("GOLLEK_CONVERTER_INPUT_DIR",
                                                                       os.path.join(home, "models")))
        self.output_base = os.path.realpath(output_base or os.environ.get("GOLLEK_CONVERTER_OUTPUT_DIR",
                                                                         os.path.join(home, "converted")))
        self.jobs: Dict[int, ConversionJob] = {}
        self._next = 1
        self._lock = threading.Lock()

    # -- paths
    @staticmethod
    def _inside(path: str, base: str) -> str:
        p = os.path.realpath(path if os.path.isabs(path) else os.path.join(base, path))
        if os.path.commonpath([p, base]) != base:
            raise ValueError(f"path {path!r} resolves outside {base}")
        return p

    def resolve_input(self, path: str) -> str:
        if not path:
            raise ValueError("inputPath is required")
        return self._inside(path, self.input_base)

    def derive_output_name(self, input_path: str, quantization: str) -> str:
        base = os.path.basename(os.path.normpath(input_path))
        if base.endswith(".gguf"):
            base = base[:-5]
        return f"{base}-{quantization.lower()}.gguf"

    def resolve_output(self, output_path: Optional[str], input_path: str, quantization: str) -> str:
        name = output_path or self.derive_output_name(input_path, quantization)
        return self._inside(name, self.output_base)

    def plan(self, req: Dict[str, Any], request_id: str = "community") -> Dict[str, Any]:
        q = str(req.get("quantization") or "F16").upper()
        if q not in _QUANT_IDS:
            raise ValueError(f"unknown quantization {q!r}")
        inp = self.resolve_input(req.get("inputPath") or "")
        out = self.resolve_output(req.get("outputPath"), inp, q)
        return {"conversionId": 0, "success": True, "dryRun": True, "requestId": request_id, "inputPath": inp,
                "outputPath": out, "derivedOutputName": self.derive_output_name(inp, q), "quantization": q,
                "inputFormat": detect_format(inp), "inputBasePath": self.input_base,
                "outputBasePath": self.output_base}

    # -- jobs
    def start(self, req: Dict[str, Any], request_id: str = "community") -> ConversionJob:
        p = self.plan(req, request_id)
        if p["inputFormat"] not in ("safetensors", "gguf"):
            raise ValueError(f"cannot convert input of format {p['inputFormat']!r}")
        if os.path.exists(p["outputPath"]) and not req.get("overwriteExisting"):
            raise FileExistsError(f"{p['outputPath']} exists (set overwriteExisting)")
        with self._lock:
            cid = self._next
            self._next += 1
        job = ConversionJob(cid, request_id, p["inputPath"], p["outputPath"], p["quantization"])
        self.jobs[cid] = job
        threading.Thread(target=self._run, args=(job,), daemon=True).start()
        return job

    def _run(self, job: ConversionJob) -> None:
        from ..loaders import gguf as G
        job.status = "RUNNING"
        job.emit(type="started", conversionId=job.conversion_id)

        def progress(i, n, name):
            if job.cancel.is_set():
                raise ConversionCancelled()
            job.progress = i / max(1, n)
            job.current = name
            job.emit(type="progress", progress=round(job.progress, 4), tensor=name)

        try:
            q = job.quantization
            qt = q if q in G.MIXTURES else G.TYPE_BY_NAME[q]
            os.makedirs(os.path.dirname(job.output_path), exist_ok=True)
            tmp = job.output_path + ".part"
            if detect_format(job.input_path) == "gguf":
                src = job.input_path if os.path.isfile(job.input_path) else \
                    sorted(glob.glob(os.path.join(job.input_path, "*.gguf")))[0]
                cfg, w, f = G.load_llama_gguf(src)
                try:
                    G.write_llama_gguf(tmp, cfg, w, qt, progress=progress)
                finally:
                    f.close()
            else:
                from ..config import ModelConfig
                from ..loaders.safetensors import SafetensorsCheckpoint
                with open(os.path.join(job.input_path, "config.json")) as fh:
                    cfg = ModelConfig.from_hf(json.load(fh))
                ck = SafetensorsCheckpoint(job.input_path)

                class _Lazy(dict):  # tensors read one at a time as the writer asks for them
                    def __getitem__(self, k):
                        return ck.get(k).float()

                lazy = _Lazy.fromkeys(ck.keys())
                G.write_llama_gguf(tmp, cfg, lazy, qt, progress=progress)
            os.replace(tmp, job.output_path)
            job.status, job.progress = "COMPLETED", 1.0
        except ConversionCancelled:
            job.status = "CANCELLED"
        except Exception as e:  # noqa: BLE001 - reported in the job
            job.status, job.error = "FAILED", f"{type(e).__name__}: {e}"
        finally:
            part = job.output_path + ".part"
            if job.status != "COMPLETED" and os.path.exists(part):
                os.remove(part)
            job.finished = time.time()
            job.emit(type="done", **self.response(job))

    def response(self, job: ConversionJob) -> Dict[str, Any]:
        dur = (job.finished or time.time()) - job.started
        ins, outs = _size(job.input_path), _size(job.output_path) if job.status == "COMPLETED" else 0
        return {"conversionId": job.conversion_id, "success": job.status == "COMPLETED", "status": job.status,
                "requestId": job.request_id, "inputPath": job.input_path, "outputPath": job.output_path,
                "quantization": job.quantization, "progress": round(job.progress, 4),
                "outputSize": _human(outs) if outs else None, "duration": f"{dur:.2f}s",
                "compressionRatio": round(ins / outs, 3) if outs else None, "errorMessage": job.error,
                "dryRun": False, "inputBasePath": self.input_base, "outputBasePath": self.output_base}

    def wait(self, job: ConversionJob, timeout: Optional[float] = None) -> ConversionJob:
        deadline = None if timeout is None else time.time() + timeout
        with job.cond:
            while job.finished is None:
                left = None if deadline is None else deadline - time.time()
                if left is not None and left <= 0:
                    break
                job.cond.wait(left)
        return job


def register_converter_routes(app, service: Optional[ConverterService] = None) -> ConverterService:
    """Mount ``/v1/converter/gguf/*`` on a FastAPI app."""
    import asyncio

    from fastapi import HTTPException
    from fastapi.responses import StreamingResponse

    svc = service or ConverterService()
    base = "/v1/converter/gguf"

    def bad(e: Exception):
        code = 409 if isinstance(e, FileExistsError) else 400
        raise HTTPException(status_code=code, detail=str(e))

    @app.get(base + "/health")
    async def conv_health():
        return {"status": "UP", "service": "gguf-converter", "inputBasePath": svc.input_base,
                "outputBasePath": svc.output_base, "activeConversions":
                    sum(j.status == "RUNNING" for j in svc.jobs.values())}

    @app.post(base + "/convert")
    async def conv_convert(req: Dict[str, Any]):
        try:
            if req.get("dryRun"):
                return svc.plan(req)
            job = svc.start(req)
        except (ValueError, FileExistsError, OSError) as e:
            bad(e)
        await asyncio.get_running_loop().run_in_executor(None, svc.wait, job)
        return svc.response(job)

    @app.post(base + "/convert/preview")
    async def conv_preview(req: Dict[str, Any]):
        try:
            return svc.plan(req)
        except ValueError as e:
            bad(e)

    @app.post(base + "/convert/stream")
    async def conv_stream(req: Dict[str, Any]):
        try:
            job = svc.start(req)
        except (ValueError, FileExistsError, OSError) as e:
            bad(e)

        async def gen():
            seen = 0
            loop = asyncio.get_running_loop()
            while True:
                def next_events():
                    with job.cond:
                        while len(job.events) <= seen and job.finished is None:
                            job.cond.wait(0.5)
                        return list(job.events[seen:])
                evs = await loop.run_in_executor(None, next_events)
                for ev in evs:
                    yield f"data: {json.dumps(ev)}\n\n"
                seen += len(evs)
                if job.finished is not None and seen >= len(job.events):
                    break
            yield "data: [DONE]\n\n"

        return StreamingResponse(gen(), media_type="text/event-stream")

    @app.post(base + "/convert/{conversion_id}/cancel")
    async def conv_cancel(conversion_id: int):
        job = svc.jobs.get(conversion_id)
        if job is None:
            raise HTTPException(status_code=404, detail=f"no conversion {conversion_id}")
        job.cancel.set()
        return {"conversionId": conversion_id, "cancelled": job.finished is None, "status": job.status}

    @app.get(base + "/convert/{conversion_id}")
    async def conv_status(conversion_id: int):
        job = svc.jobs.get(conversion_id)
        if job is None:
            raise HTTPException(status_code=404, detail=f"no conversion {conversion_id}")
        return svc.response(job)

    @app.get(base + "/detect-format")
    async def conv_detect(path: str):
        try:
            p = svc.resolve_input(path)
        except ValueError as e:
            bad(e)
        return {"path": p, "format": detect_format(p)}

    def existing(path: str) -> str:
        """An existing path inside the output or the input base."""
        for b in (svc.output_base, svc.input_base):
            try:
                p = svc._inside(path, b)
            except ValueError:
                continue
            if os.path.exists(p):
                return p
        raise HTTPException(status_code=404, detail=f"{path} not found inside the converter's directories")

    @app.get(base + "/model-info")
    async def conv_info(path: str):
        return model_info(existing(path))

    @app.get(base + "/verify")
    async def conv_verify(path: str):
        return await asyncio.get_running_loop().run_in_executor(None, verify_gguf, existing(path))

    @app.get(base + "/quantizations")
    async def conv_quants():
        return {"quantizations": [{"id": q.lower(), "name": q, "description": d, "qualityLevel": ql,
                                   "compressionRatio": cr, "useCase": uc} for q, d, ql, cr, uc in QUANTIZATIONS]}

    @app.get(base + "/recommend-quantization")
    async def conv_recommend(modelSizeGb: float, prioritizeQuality: bool = False):
        r = recommend(modelSizeGb, prioritizeQuality)
        q = next(x for x in QUANTIZATIONS if x[0] == r)
        return {"recommended": r.lower(), "name": r, "description": q[1], "qualityLevel": q[2],
                "compressionRatio": q[3],
                "reason": f"Recommended for {modelSizeGb} GB model, "
                          + ("prioritizing quality" if prioritizeQuality else "balanced approach")}

    return svc

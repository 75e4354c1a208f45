"""Error-code catalogue and payloads.

Every error the server returns carries a stable code (``CATEGORY_NNN``), its HTTP status, whether
a retry can succeed, and a suggested action, in the shape of the reference's ``ErrorPayload``
(core/gollek-error-code/…/error/ErrorPayload.java: type, code, message, details, retryable,
timestamp, suggestedAction) so clients that branch on codes keep working. Codes for the same
condition as the reference's catalogue (core/gollek-error-code/…/error/ErrorCode.java) use its
code string (MODEL_001 model not found, MODEL_003 invalid format, MODEL_007 not compatible,
TENSOR_001 shape mismatch); the others are numbered here.

    python -m gollek_b200.errors        # prints the catalogue as a Markdown table
"""
from __future__ import annotations

import enum
import sys
from dataclasses import dataclass, field
from datetime import datetime, timezone
from typing import Any, Dict, Optional


class ErrorCategory(enum.Enum):
    MODEL = "MODEL"
    TENSOR = "TENSOR"
    DEVICE = "DEVICE"
    QUOTA = "QUOTA"
    AUTH = "AUTH"
    INIT = "INIT"
    RUNTIME = "RUNTIME"
    STORAGE = "STORAGE"
    CONVERSION = "CONVERSION"
    VALIDATION = "VALIDATION"
    CIRCUIT = "CIRCUIT"
    ROUTING = "ROUTING"
    CONFIG = "CONFIG"
    NETWORK = "NETWORK"
    STREAM = "STREAM"
    INTERNAL = "INTERNAL"


@dataclass(frozen=True)
class Code:
    name: str
    category: ErrorCategory
    http: int
    code: str
    message: str
    retryable: bool = False
    action: str = ""


_C = ErrorCategory
CODES: Dict[str, Code] = {c.name: c for c in [
    Code("MODEL_NOT_FOUND", _C.MODEL, 404, "MODEL_001", "Model not found", action="list /v1/models"),
    Code("MODEL_INVALID_FORMAT", _C.MODEL, 400, "MODEL_003", "Invalid model format",
         action="provide a safetensors directory, a GGUF file or a preset name"),
    Code("MODEL_NOT_COMPATIBLE", _C.MODEL, 400, "MODEL_007", "Model not compatible with this engine"),
    Code("TENSOR_SHAPE_MISMATCH", _C.TENSOR, 400, "TENSOR_001", "Tensor shape mismatch"),
    Code("DEVICE_OUT_OF_MEMORY", _C.DEVICE, 503, "DEVICE_101", "Device memory exhausted", True,
         "retry later or lower max_num_seqs / max_model_len"),
    Code("DEVICE_FAULT", _C.DEVICE, 500, "DEVICE_102", "Device-side wait timed out or a kernel failed"),
    Code("QUOTA_EXCEEDED", _C.QUOTA, 429, "QUOTA_101", "Tenant quota exceeded", True, "retry after running requests finish"),
    Code("RATE_LIMIT_EXCEEDED", _C.QUOTA, 429, "QUOTA_102", "Rate limit exceeded", True, "back off and retry"),
    Code("AUTH_INVALID_KEY", _C.AUTH, 401, "AUTH_101", "Invalid or missing API key", action="send X-API-Key or Bearer"),
    Code("AUTH_FORBIDDEN", _C.AUTH, 403, "AUTH_102", "Not allowed for this key"),
    Code("INIT_FAILED", _C.INIT, 503, "INIT_101", "Engine failed to initialise"),
    Code("VALIDATION_INVALID_PARAMETER", _C.VALIDATION, 400, "VALIDATION_101", "Invalid request parameter"),
    Code("VALIDATION_PROMPT_TOO_LONG", _C.VALIDATION, 400, "VALIDATION_102", "Prompt exceeds the context length",
         action="shorten the prompt or raise max_model_len"),
    Code("VALIDATION_UNSUPPORTED", _C.VALIDATION, 400, "VALIDATION_103", "Unsupported request option"),
    Code("RUNTIME_TIMEOUT", _C.RUNTIME, 504, "RUNTIME_101", "Request timed out", True),
    Code("RUNTIME_ENGINE_UNAVAILABLE", _C.RUNTIME, 503, "RUNTIME_102", "Engine is not running", True),
    Code("RUNTIME_KV_CACHE_FULL", _C.RUNTIME, 503, "RUNTIME_103", "KV cache full", True, "retry later"),
    Code("RUNTIME_CANCELLED", _C.RUNTIME, 499, "RUNTIME_104", "Request cancelled"),
    Code("RUNTIME_RANK_FAILURE", _C.RUNTIME, 503, "RUNTIME_105", "A tensor-parallel rank failed"),
    Code("STORAGE_SNAPSHOT_INVALID", _C.STORAGE, 400, "STORAGE_101", "Snapshot does not match this engine"),
    Code("CONVERSION_FAILED", _C.CONVERSION, 400, "CONVERSION_101", "Model conversion failed"),
    Code("CIRCUIT_OPEN", _C.CIRCUIT, 503, "CIRCUIT_101", "Circuit breaker open", True, "retry after the cool-down"),
    Code("CIRCUIT_BULKHEAD_FULL", _C.CIRCUIT, 429, "CIRCUIT_102", "Too many concurrent requests", True),
    Code("ROUTING_ADAPTER_NOT_FOUND", _C.ROUTING, 404, "ROUTING_101", "LoRA adapter not found"),
    Code("ROUTING_JOB_NOT_FOUND", _C.ROUTING, 404, "ROUTING_102", "Job not found"),
    Code("CONFIG_INVALID", _C.CONFIG, 400, "CONFIG_101", "Invalid configuration"),
    Code("NETWORK_HANDOFF_FAILED", _C.NETWORK, 502, "NETWORK_101", "KV hand-off to the decode node failed", True),
    Code("STREAM_ERROR", _C.STREAM, 500, "STREAM_101", "Streaming failed"),
    Code("INTERNAL_ERROR", _C.INTERNAL, 500, "INTERNAL_001", "Internal error"),
]}

_BY_HTTP = {400: "VALIDATION_INVALID_PARAMETER", 401: "AUTH_INVALID_KEY", 403: "AUTH_FORBIDDEN",
            404: "MODEL_NOT_FOUND", 429: "RATE_LIMIT_EXCEEDED", 499: "RUNTIME_CANCELLED",
            503: "RUNTIME_ENGINE_UNAVAILABLE", 504: "RUNTIME_TIMEOUT"}


def for_http(status: int) -> Code:
    return CODES[_BY_HTTP.get(status, "INTERNAL_ERROR")]


class GollekError(Exception):
    def __init__(self, name: str, message: Optional[str] = None, **details: Any):
        self.code = CODES[name]
        self.message = message or self.code.message
        self.details = details
        super().__init__(f"{self.code.code}: {self.message}")


def payload(code: Code, message: Optional[str] = None, details: Optional[dict] = None,
            request_id: Optional[str] = None) -> dict:
    p = {"type": code.category.value, "code": code.code, "error": code.name, "message": message or code.message,
         "httpStatus": code.http, "retryable": code.retryable,
         "timestamp": datetime.now(timezone.utc).isoformat(), "details": details or {}}
    if code.action:
        p["suggestedAction"] = code.action
    if request_id:
        p["requestId"] = request_id
    return p


def catalogue_markdown() -> str:
    rows = ["| code | name | HTTP | retryable | meaning |", "|---|---|---|---|---|"]
    for c in sorted(CODES.values(), key=lambda c: c.code):
        rows.append(f"| {c.code} | {c.name} | {c.http} | {'yes' if c.retryable else 'no'} | {c.message} |")
    return "\n".join(rows)


if __name__ == "__main__":
    sys.stdout.write(catalogue_markdown() + "\n")

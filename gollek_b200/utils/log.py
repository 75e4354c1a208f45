"""Library logging switch.

Reference behaviour: runner/llamacpp/gollek-runner-llamacpp/src/main/native/golek_llama_shim.c:3-25
(silences the native runtime's log callback and hands out default parameter structs). Here the
defaults are the ``EngineConfig`` / ``SamplingParams`` dataclass defaults, and this module sets the
level of the ``gollek_b200`` logger tree from ``GOLLEK_LOG_LEVEL`` (``debug`` / ``info`` /
``warning`` / ``error`` / ``off``; default ``warning``).
"""
from __future__ import annotations

import logging
import os
from typing import Optional

_LEVELS = {"debug": logging.DEBUG, "info": logging.INFO, "warning": logging.WARNING, "warn": logging.WARNING,
           "error": logging.ERROR, "off": logging.CRITICAL + 10, "none": logging.CRITICAL + 10}


def configure_logging(level: Optional[str] = None) -> logging.Logger:
    """Set the ``gollek_b200`` loggers' level (argument, else ``GOLLEK_LOG_LEVEL``, else warning);
    ``off`` silences them. Adds one stderr handler the first time."""
    name = (level or os.environ.get("GOLLEK_LOG_LEVEL") or "warning").lower()
    if name not in _LEVELS:
        raise ValueError(f"unknown log level {name!r} (one of {', '.join(_LEVELS)})")
    log = logging.getLogger("gollek_b200")
    log.setLevel(_LEVELS[name])
    if not any(getattr(h, "_gollek", False) for h in log.handlers):
        h = logging.StreamHandler()
        h.setFormatter(logging.Formatter("%(asctime)s %(levelname)s %(name)s: %(message)s"))
        h._gollek = True
        log.addHandler(h)
    return log

"""gollek_b200: an LLM inference and serving framework for NVIDIA B200 (sm_100a).

Public API:
    from gollek_b200 import LLM, LLMEngine, EngineConfig, SamplingParams
    LLM("llama-3-8b").generate(["Hello"], SamplingParams(max_tokens=32))
"""
__version__ = "0.1.0"


def __getattr__(name):
    if name in ("LLM", "LLMEngine"):
        from .engine import engine as _e
        return getattr(_e, name)
    if name == "SamplingParams":
        from .engine.sequence import SamplingParams
        return SamplingParams
    if name in ("EngineConfig", "ModelConfig"):
        from . import config as _c
        return getattr(_c, name)
    raise AttributeError(name)

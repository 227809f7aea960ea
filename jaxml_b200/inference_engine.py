"""``jaxml.inference_engine`` import path: ``Engine``, ``InferenceConfig``, ``SamplingMethod``."""
from .engine import Engine, InferenceConfig
from .sampling import SamplingMethod

__all__ = ["Engine", "InferenceConfig", "SamplingMethod"]

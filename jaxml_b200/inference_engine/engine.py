"""``jaxml.inference_engine.engine`` import path (implementation: ``jaxml_b200.engine``)."""
from ..engine import Engine, InferenceConfig

__all__ = ["Engine", "InferenceConfig"]

"""``jaxml.inference_engine`` import path: ``Engine``, ``InferenceConfig``, ``SamplingMethod``, and the
``engine`` / ``sampling`` submodules (the implementations live in ``jaxml_b200.engine`` and
``jaxml_b200.sampling``)."""
from ..engine import Engine, InferenceConfig
from ..sampling import SamplingMethod

__all__ = ["Engine", "InferenceConfig", "SamplingMethod"]

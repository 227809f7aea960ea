"""B200-native (sm_100a) implementation of jaxml's decode/prefill path.

Public names mirror ``jaxml/__init__.py`` of the reference: ``Engine``, ``InferenceConfig``,
``ModelConfig``, ``SamplingMethod``, ``GenerationConfig``, ``TextGenerationPipeline``, ``KVCache`` (plus
the model classes), and ``jaxml_b200.nn`` mirrors ``jaxml.nn``.  The kernels live in ``libjxb200.so``
(``jaxml_b200/csrc``, C ABI in ``include/jxb200.h``).
"""
from . import nn
from .cache import KVCache
from .config import ModelConfig
from .engine import Engine, InferenceConfig
from .models import (GemmaModel, GemmaModelWithHead, GPTNeoXModel, GPTNeoXModelWithHead, LlamaModel,
                     LlamaModelWithHead)
from .sampling import SamplingMethod
from .text_generation import GenerationConfig, TextGenerationPipeline

__all__ = [
    "Engine",
    "InferenceConfig",
    "ModelConfig",
    "SamplingMethod",
    "GenerationConfig",
    "TextGenerationPipeline",
    "KVCache",
    "LlamaModelWithHead",
    "GPTNeoXModelWithHead",
    "GemmaModelWithHead",
    "LlamaModel",
    "GPTNeoXModel",
    "GemmaModel",
]

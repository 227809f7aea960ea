"""``jaxml.outputs`` import path: the output records of the model, attention and generation calls."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .cache import KVCache
from .models import BaseModelOutputWithCache, CausalLMOutputWithCache
from .nn import AttentionOutput


@dataclass
class DecoderOutput:
    hidden_states: torch.Tensor
    kv_cache: Optional[KVCache] = None
    attention_weight: Optional[torch.Tensor] = None


@dataclass
class GenerationOutput:
    tokens: torch.Tensor
    kv_caches: tuple = ()
    rng: Optional[torch.Tensor] = None


__all__ = ["AttentionOutput", "BaseModelOutputWithCache", "CausalLMOutputWithCache", "DecoderOutput",
           "GenerationOutput"]

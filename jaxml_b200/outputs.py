"""``jaxml.outputs`` import path: the output records of the model, attention and generation calls."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .decoders import DecoderOutput
from .models import BaseModelOutputWithCache, CausalLMOutputWithCache
from .nn import AttentionOutput


@dataclass
class GenerationOutput:
    tokens: torch.Tensor
    kv_caches: tuple = ()
    rng: Optional[torch.Tensor] = None


__all__ = ["AttentionOutput", "BaseModelOutputWithCache", "CausalLMOutputWithCache", "DecoderOutput",
           "GenerationOutput"]

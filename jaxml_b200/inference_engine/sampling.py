"""``jaxml.inference_engine.sampling`` import path (implementation: ``jaxml_b200.sampling``)."""
from ..sampling import (SamplingMethod, SamplingParams, greedy_fn, min_p_filtering, normalize_sampling_params,
                        top_k_filtering, top_p_filtering)

__all__ = ["SamplingMethod", "SamplingParams", "greedy_fn", "min_p_filtering", "normalize_sampling_params",
           "top_k_filtering", "top_p_filtering"]

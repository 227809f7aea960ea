"""``jaxml.utils`` import path: the reference's user-facing helpers (utils.py:179-406).

``torch_to_jax_states`` (the state-dict conversion, ``hf_utils.py`` here) and ``get_default_pos_ids``
(the last valid position of right-padded rows, ``cache.py`` here) are the library's own; ``check_shape``,
``pprint_pytree`` and ``timeit`` are small host-side helpers with the reference's behaviour.  The AOT
executable cache of the reference has no counterpart: a decode step is a captured CUDA graph.
"""
from __future__ import annotations

import functools
import json
import time
from typing import Any

import numpy as np
import torch

from .cache import get_default_pos_ids
from .hf_utils import torch_to_jax_states

__all__ = ["check_shape", "get_default_pos_ids", "pprint_pytree", "timeit", "torch_to_jax_states"]


def check_shape(tensor, *shape):
    """Asserts ``tensor``'s shape: each entry an int, ``None`` (any size) or one ``...`` (any number of
    axes), as ``chex.assert_shape`` takes them (utils.py:179-180)."""
    actual = tuple(tensor.shape)
    expected = tuple(shape[0]) if len(shape) == 1 and isinstance(shape[0], (tuple, list)) else tuple(shape)
    if expected.count(Ellipsis) > 1:
        raise ValueError("check_shape takes at most one Ellipsis.")
    if Ellipsis in expected:
        i = expected.index(Ellipsis)
        head, tail = expected[:i], expected[i + 1:]
        ok = len(actual) >= len(head) + len(tail) and _match(actual[:len(head)], head) and \
            _match(actual[len(actual) - len(tail):], tail)
    else:
        ok = _match(actual, expected)
    if not ok:
        raise AssertionError(f"shape {actual} does not match the expected {expected}.")


def _match(actual: tuple, expected: tuple) -> bool:
    return len(actual) == len(expected) and all(e is None or a == e for a, e in zip(actual, expected))


def pprint_pytree(obj: Any):
    """Prints a nested tree with every array replaced by its shape and dtype (utils.py:374-388)."""

    def fmt(x):
        if isinstance(x, dict):
            return {k: fmt(v) for k, v in x.items()}
        if isinstance(x, (list, tuple)):
            return [fmt(v) for v in x]
        if isinstance(x, (torch.Tensor, np.ndarray)):
            return f"<Array shape={tuple(x.shape)} dtype={x.dtype}>"
        return repr(x)

    print(json.dumps(fmt(obj), indent=2))


def timeit(logger):
    """Decorator factory: the wrapped call logs its wall time at INFO unless called with ``log=False``
    (utils.py:391-406)."""

    def _factory(fn):
        name = fn.__name__

        @functools.wraps(fn)
        def _wrapped(*args, log=True, **kwargs):
            start = time.perf_counter()
            out = fn(*args, **kwargs)
            if log:
                logger.info(f"Execution time for {name}: {time.perf_counter() - start}")
            return out

        return _wrapped

    return _factory

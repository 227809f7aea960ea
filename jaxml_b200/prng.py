"""Host side of the PRNG key flow: ``jax.random.PRNGKey`` and ``jax.random.split`` (threefry2x32).

The reference seeds with ``PRNGKey(seed)`` (inference_engine/engine.py:542) and splits once before the
first sample and once per decode step (_generate.py:130,187,205,348).  The host only builds the first
(key, subkey) pair; every later split runs on the device (csrc/sample.cu).  Threefry-2x32, 20 rounds,
as published by Salmon et al. (SC'11); the split of JAX's partitionable threefry draws element i as
threefry(key, (hi(i), lo(i))).
"""
from __future__ import annotations

import numpy as np

_ROTATIONS = ((13, 15, 26, 6), (17, 29, 16, 24))


def _threefry(k0: int, k1: int, x0: int, x1: int) -> tuple[int, int]:
    m = 0xFFFFFFFF
    ks = (k0 & m, k1 & m, (k0 ^ k1 ^ 0x1BD11BDA) & m)
    x0 = (x0 + ks[0]) & m
    x1 = (x1 + ks[1]) & m
    for g in range(5):
        for r in _ROTATIONS[g % 2]:
            x0 = (x0 + x1) & m
            x1 = ((x1 << r) | (x1 >> (32 - r))) & m
            x1 ^= x0
        x0 = (x0 + ks[(g + 1) % 3]) & m
        x1 = (x1 + ks[(g + 2) % 3] + g + 1) & m
    return x0, x1


def prng_key(seed: int) -> np.ndarray:
    """``jax.random.PRNGKey(seed)`` (32-bit seeds): ``[seed >> 32, seed & 0xFFFFFFFF]``."""
    seed = int(seed)
    return np.array([(seed >> 32) & 0 if -2**31 <= seed < 2**31 else (seed >> 32) & 0xFFFFFFFF,
                     seed & 0xFFFFFFFF], dtype=np.uint32)


def split(key) -> tuple[np.ndarray, np.ndarray]:
    """``jax.random.split(key)`` -> (new key, subkey)."""
    k0, k1 = int(key[0]), int(key[1])
    a = _threefry(k0, k1, 0, 0)
    b = _threefry(k0, k1, 0, 1)
    return np.array(a, dtype=np.uint32), np.array(b, dtype=np.uint32)

"""Oracle (test infrastructure only): JAX's threefry PRNG and categorical sampling, restated in numpy.

Only tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` use this module,
and only to compare against. The product samples on the GPU (``jaxml_b200/csrc/sample.cu``).

What the reference calls (JAX 0.10.1, pinned in ``pyproject.toml:14`` / ``uv.lock:245-246`` of the
reference; JAX itself is not in the reference tree and is not installed here):

* ``jax.random.PRNGKey(seed)``            -- ``inference_engine/engine.py:542``, ``_generate.py:273``
* ``jax.random.split(key)``               -- ``_generate.py:130,187,205,348``
* ``jax.random.categorical(rng, logits/temp)`` -- ``inference_engine/sampling.py:186``

Published algorithm restated here: Threefry-2x32 with 20 rounds (Salmon, Moraes, Dror, Shaw,
"Parallel random numbers: as easy as 1, 2, 3", SC'11), key schedule word ``0x1BD11BDA`` and the
rotation constants (13,15,26,6) / (17,29,16,24).  JAX's documented construction on top of it, with
``jax_threefry_partitionable`` on (the JAX default since 0.5):

* ``PRNGKey(seed)`` = ``[seed >> 32, seed & 0xFFFFFFFF]`` as uint32 (``[0, seed]`` for 32-bit seeds);
* ``split(key, n)``: element ``i`` of the output is ``threefry(key, (hi(i), lo(i)))``;
* ``random_bits(key, width, shape)``: element with flat index ``i`` is
  ``threefry(key, (hi(i), lo(i)))``; 32-bit draws are ``x0 ^ x1`` and narrower draws truncate it;
* ``uniform(dtype)``: a float dtype with fewer than 8 mantissa bits (bfloat16) draws 8 bits, others
  draw as many bits as the dtype is wide; ``bits >> (rng_bits - nmant)`` becomes the mantissa of a
  number in [1, 2), minus 1, then scaled to [tiny, 1) and clamped below at ``tiny``;
* ``gumbel = -log(-log(u))`` and ``categorical = argmax(gumbel + logits)`` (first index on ties).

Parity status: the Threefry block function is pinned against the Random123 known-answer vectors and
the legacy ``split(PRNGKey(0))`` value (``tests/test_oracle_threefry.py``). The partitionable split,
the 8-bit bfloat16 uniform draw and XLA's per-op bfloat16 rounding of the Gumbel chain are NOT
pinned against a running JAX (none is available on either machine): parity of temperature sampling
with the reference is unpinned. GPU-vs-oracle sampling is bit-exact by construction and by test.
"""
from __future__ import annotations

import numpy as np

_ROT = ((13, 15, 26, 6), (17, 29, 16, 24))
_KS_PARITY = np.uint32(0x1BD11BDA)


def _rotl(x: np.ndarray, r: int) -> np.ndarray:
    return (x << np.uint32(r)) | (x >> np.uint32(32 - r))


def threefry2x32(key, x0, x1):
    """Threefry-2x32, 20 rounds, on uint32 arrays ``x0``/``x1`` (broadcast) with key ``(k0, k1)``."""
    k0 = np.uint32(key[0])
    k1 = np.uint32(key[1])
    ks = (k0, k1, np.uint32(k0 ^ k1 ^ _KS_PARITY))
    x0 = np.asarray(x0, dtype=np.uint32).copy()
    x1 = np.asarray(x1, dtype=np.uint32).copy()
    with np.errstate(over="ignore"):
        x0 = x0 + ks[0]
        x1 = x1 + ks[1]
        for group in range(5):
            for r in _ROT[group % 2]:
                x0 = x0 + x1
                x1 = _rotl(x1, r)
                x1 = x1 ^ x0
            x0 = x0 + ks[(group + 1) % 3]
            x1 = x1 + ks[(group + 2) % 3] + np.uint32(group + 1)
    return x0, x1


def prng_key(seed: int) -> np.ndarray:
    """``jax.random.PRNGKey(seed)`` for a 32-bit (x64 disabled) seed."""
    seed = int(seed)
    return np.array([0, seed & 0xFFFFFFFF], dtype=np.uint32)


def split(key, num: int = 2) -> np.ndarray:
    """``jax.random.split`` with ``jax_threefry_partitionable=True``: returns ``[num, 2]`` uint32."""
    idx = np.arange(num, dtype=np.uint64)
    hi = (idx >> np.uint64(32)).astype(np.uint32)
    lo = (idx & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    b0, b1 = threefry2x32(key, hi, lo)
    return np.stack([b0, b1], axis=-1)


def split_legacy(key, num: int = 2) -> np.ndarray:
    """``jax.random.split`` with ``jax_threefry_partitionable=False`` (only used to pin the block function)."""
    counts = np.arange(num * 2, dtype=np.uint32)
    b0, b1 = threefry2x32(key, counts[:num], counts[num:])
    return np.concatenate([b0, b1]).reshape(num, 2)


def random_bits32(key, n: int) -> np.ndarray:
    """Flat 32-bit draws ``x0 ^ x1`` for flat indices ``0..n-1`` (partitionable mode)."""
    idx = np.arange(n, dtype=np.uint64)
    hi = (idx >> np.uint64(32)).astype(np.uint32)
    lo = (idx & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    b0, b1 = threefry2x32(key, hi, lo)
    return b0 ^ b1


def _bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); returned as float32."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounding = ((u >> np.uint64(16)) & np.uint64(1)) + np.uint64(0x7FFF)
    u = ((u + rounding) >> np.uint64(16)) << np.uint64(16)
    return u.astype(np.uint32).view(np.float32)


BF16_TINY = np.float32(2.0 ** -126)


def _bf16_round_from64(x64: np.ndarray) -> np.ndarray:
    """Round float64 values to the nearest bfloat16 (ties to even) with a single rounding.

    Rounding to float32 first only goes wrong when the float32 value lands exactly on a bfloat16
    midpoint; those cases are resolved from the sign of the float64 residual.
    """
    x64 = np.asarray(x64, dtype=np.float64)
    f = x64.astype(np.float32)
    u = f.view(np.uint32)
    out = _bf16_round(f)
    mid = (u & np.uint32(0xFFFF)) == np.uint32(0x8000)
    if np.any(mid):
        resid = x64 - f.astype(np.float64)
        mag_up = np.where(f >= 0, resid > 0, resid < 0)        # true value is farther from zero than f
        mag_down = np.where(f >= 0, resid < 0, resid > 0)
        trunc = (u & np.uint32(0xFFFF0000)).view(np.float32)     # neighbour towards zero
        away = ((u & np.uint32(0xFFFF0000)) + np.uint32(0x10000)).view(np.float32)
        out = np.where(mid & mag_up, away, out)
        out = np.where(mid & mag_down, trunc, out)
    return out.astype(np.float32)


def gumbel_table_bf16() -> np.ndarray:
    """Gumbel noise for each of the 256 possible 8-bit draws of a bfloat16 ``uniform``.

    Draw ``b`` gives ``u = (b >> 1) / 128`` (``u = tiny`` for ``b >> 1 == 0``).  Each op of
    ``-log(-log(u))`` is rounded to bfloat16 as XLA evaluates the bfloat16 program op by op; each log
    is evaluated in float64 and rounded once to bfloat16.  Returned as float32 holding bfloat16 values.
    """
    b = np.arange(256, dtype=np.uint32)
    u = uniform_bits_to_u_bf16(b).astype(np.float64)
    l1 = _bf16_round_from64(np.log(u))
    l2 = _bf16_round_from64(np.log((-l1).astype(np.float64)))
    return (-l2).astype(np.float32)


def uniform_bits_to_u_bf16(bits8: np.ndarray) -> np.ndarray:
    """bfloat16 ``uniform(minval=tiny, maxval=1)`` from 8-bit draws (float32 holding bfloat16 values)."""
    m = (np.asarray(bits8, dtype=np.uint32) & np.uint32(0xFF)) >> np.uint32(1)
    u = m.astype(np.float32) / np.float32(128.0)
    return np.maximum(u, BF16_TINY)


def categorical_bf16(key, logits_bf16: np.ndarray, temperature: float) -> np.ndarray:
    """``jax.random.categorical(key, logits / temperature)`` on bfloat16 logits of shape ``[B, 1, V]``.

    ``logits`` are float32 arrays holding bfloat16 values.  ``temperature`` is converted to bfloat16
    (weak-typed Python scalar meeting a bfloat16 array), the division is evaluated in float32 and
    rounded to bfloat16, the Gumbel draw uses flat index ``b*V + v``, and the sum is rounded to bfloat16
    before the first-index argmax.  Returns int32 ``[B, 1]``.
    """
    logits = np.asarray(logits_bf16, dtype=np.float32)
    shape = logits.shape
    n = int(np.prod(shape))
    temp = _bf16_round(np.array([temperature], dtype=np.float32))[0]
    scaled = _bf16_round(logits / temp)
    bits = random_bits32(key, n).reshape(shape)
    g = gumbel_table_bf16()[bits & np.uint32(0xFF)]
    total = _bf16_round(g + scaled)
    return np.argmax(total, axis=-1).astype(np.int32)


def categorical_f32(key, logits: np.ndarray, temperature: float) -> np.ndarray:
    """``jax.random.categorical`` on float32 logits: 32-bit draws, 23-bit mantissa uniform."""
    logits = np.asarray(logits, dtype=np.float32)
    shape = logits.shape
    n = int(np.prod(shape))
    scaled = (logits / np.float32(temperature)).astype(np.float32)
    bits = random_bits32(key, n).reshape(shape)
    fbits = (bits >> np.uint32(9)) | np.uint32(0x3F800000)
    u = fbits.view(np.float32) - np.float32(1.0)
    tiny = np.float32(np.finfo(np.float32).tiny)
    u = np.maximum(u * (np.float32(1.0) - tiny) + tiny, tiny).astype(np.float32)
    l1 = np.log(u.astype(np.float64)).astype(np.float32)          # each op rounded to float32
    g = (-np.log((-l1).astype(np.float64))).astype(np.float32)
    total = (g + scaled).astype(np.float32)
    return np.argmax(total, axis=-1).astype(np.int32)

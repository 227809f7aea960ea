"""``KVCache``: the reference's functional per-layer KV cache (``cache.py:69-282``) on torch tensors.

Same fields (``k``, ``v`` ``[B, T, H, hd]``, ``max_seq_len``, ``mask`` ``[B, T]`` bool, ``dtype``,
``pos_id`` ``[B, 1]``), constructor (``init``), methods (``update``, ``rollback``, ``resize``,
``validate_state``, ``next_pos_id``, ``next_mask``) and validation messages.  Every method returns a new
cache and leaves its input untouched; the tensors stay on the device they were given on (the decode
update is one scatter on that device).  ``Engine.generate`` does not use this class: its runtime keeps
all layers' caches in one device allocation and appends inside the fused RoPE kernel; the class is for
code that drives the modules itself.
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass
from typing import Any, Optional

import torch

from ._checks import normalize_count, normalize_dtype


def get_default_pos_ids(mask: torch.Tensor) -> torch.Tensor:
    """Index of the last valid position of each right-padded row, ``[B, 1]`` (``utils.py:183-194``)."""
    idx = torch.arange(mask.shape[1], device=mask.device)
    return (mask.to(torch.int64) * idx[None]).argmax(1, keepdim=True).to(torch.int32)


def _as_tensor(x, device=None) -> torch.Tensor:
    return x if isinstance(x, torch.Tensor) else torch.as_tensor(x, device=device)


def _check_binary_int_mask(name: str, mask: torch.Tensor):
    if mask.dtype != torch.bool and bool(((mask != 0) & (mask != 1)).any()):
        raise ValueError(f"{name} integer values must be 0 or 1.")


def _check_right_padded(name: str, mask: torch.Tensor):
    if mask.shape[1] > 1 and bool((mask[:, 1:] & ~mask[:, :-1]).any()):
        raise ValueError(f"{name} must be right padded: valid tokens cannot appear after masked positions.")


def _check_finite(name: str, x: torch.Tensor):
    if not bool(torch.isfinite(x).all()):
        raise ValueError(f"{name} must contain only finite values.")


def _pad_seq(x: torch.Tensor, length: int, value) -> torch.Tensor:
    pad = torch.full((x.shape[0], length - x.shape[1]) + tuple(x.shape[2:]), value, dtype=x.dtype, device=x.device)
    return torch.cat([x, pad], dim=1)


@dataclass(frozen=True)
class KVCache:
    """One layer's KV cache; right-padded rows, ``pos_id`` = last valid position."""

    k: Optional[torch.Tensor]
    v: Optional[torch.Tensor]
    max_seq_len: int
    mask: Optional[torch.Tensor]
    dtype: Any = torch.float32
    pos_id: Optional[torch.Tensor] = None

    def replace(self, **kw) -> "KVCache":
        return dataclasses.replace(self, **kw)

    @classmethod
    def init(cls, max_seq_len: int, k=None, v=None, mask=None, dtype: Any = torch.float32) -> "KVCache":
        max_seq_len = normalize_count("max_seq_len", max_seq_len)
        dtype = normalize_dtype("dtype", dtype)
        if max_seq_len <= 0:
            raise ValueError(f"max_seq_len must be positive, got {max_seq_len}.")
        empty = cls(k=None, v=None, max_seq_len=max_seq_len, mask=None, dtype=dtype)
        if k is None and v is None and mask is None:
            return empty
        if k is None or v is None:
            raise ValueError("Initial KVCache state requires both k and v when either is set.")
        return empty.update(k, v, mask)

    @property
    def next_pos_id(self) -> torch.Tensor:
        if self.pos_id is None:
            raise ValueError("Cannot get next position ids before KV cache initialization.")
        return self.pos_id + 1

    @property
    def next_mask(self):
        return self.mask

    # -- validation --------------------------------------------------------------------------------
    @staticmethod
    def _check_kv(k: torch.Tensor, v: torch.Tensor):
        if k.shape != v.shape:
            raise ValueError(f"k and v must have the same shape, got {tuple(k.shape)} and {tuple(v.shape)}.")
        if k.ndim != 4:
            raise ValueError("k and v must be 4D arrays with batch, sequence, head, and head_dim axes, "
                             f"got shape {tuple(k.shape)}.")
        for axis, size in zip(("batch", "sequence", "head", "head_dim"), k.shape):
            if size <= 0:
                raise ValueError(f"k and v {axis} axis must be non-empty, got shape {tuple(k.shape)}.")
        if not k.dtype.is_floating_point:
            raise TypeError(f"k must contain floating point values, got dtype {k.dtype}.")
        if not v.dtype.is_floating_point:
            raise TypeError(f"v must contain floating point values, got dtype {v.dtype}.")
        _check_finite("k", k)
        _check_finite("v", v)

    def _check_static(self):
        if normalize_count("max_seq_len", self.max_seq_len) <= 0:
            raise ValueError(f"max_seq_len must be positive, got {self.max_seq_len}.")
        normalize_dtype("dtype", self.dtype)

    def _check_populated(self):
        self._check_static()
        if self.k is None:
            if self.v is not None or self.mask is not None or self.pos_id is not None:
                raise ValueError("KVCache has partial state: k is empty but v, mask, or pos_id is populated.")
            return
        if self.v is None or self.mask is None or self.pos_id is None:
            raise ValueError("KVCache has partial state: populated k requires v, mask, and pos_id.")
        k, v, mask, pos = self.k, self.v, self.mask, self.pos_id
        if k.shape != v.shape:
            raise ValueError(f"Cached k and v must have the same shape, got {tuple(k.shape)} and {tuple(v.shape)}.")
        if k.ndim != 4:
            raise ValueError(f"Cached k and v must be 4D arrays, got shape {tuple(k.shape)}.")
        if k.shape[0] <= 0:
            raise ValueError(f"Cached k/v batch axis must be non-empty, got shape {tuple(k.shape)}.")
        if k.shape[1] != self.max_seq_len:
            raise ValueError(f"Cached k/v sequence axis must match max_seq_len={self.max_seq_len}, got {k.shape[1]}.")
        if k.shape[2] <= 0:
            raise ValueError(f"Cached k/v head axis must be non-empty, got shape {tuple(k.shape)}.")
        if k.shape[3] <= 0:
            raise ValueError(f"Cached k/v head_dim axis must be non-empty, got shape {tuple(k.shape)}.")
        for name, x in (("k", k), ("v", v)):
            if not x.dtype.is_floating_point:
                raise TypeError(f"Cached {name} must contain floating point values, got dtype {x.dtype}.")
            if x.dtype != self.dtype:
                raise TypeError(f"Cached {name} dtype must match cache dtype {self.dtype}, got {x.dtype}.")
        _check_finite("Cached k", k)
        _check_finite("Cached v", v)
        if tuple(mask.shape) != tuple(k.shape[:2]):
            raise ValueError(f"Cached mask shape must match cached k/v batch and sequence axes, got {tuple(mask.shape)}.")
        if mask.dtype != torch.bool:
            raise TypeError(f"Cached mask must be boolean, got dtype {mask.dtype}.")
        if not bool(mask.any(dim=1).all()):
            raise ValueError("Cached mask must contain at least one valid token per batch row.")
        _check_right_padded("Cached mask", mask)
        if tuple(pos.shape) != (k.shape[0], 1):
            raise ValueError(f"Cached pos_id shape must be {(k.shape[0], 1)}, got {tuple(pos.shape)}.")
        if pos.dtype.is_floating_point or pos.dtype == torch.bool:
            raise TypeError(f"Cached pos_id must contain integer positions, got dtype {pos.dtype}.")
        if bool(((pos < 0) | (pos >= self.max_seq_len)).any()):
            raise ValueError(f"Cached pos_id values must be within [0, {self.max_seq_len}).")
        if not torch.equal(pos.to(torch.int64), get_default_pos_ids(mask).to(torch.int64)):
            raise ValueError("Cached pos_id must match the last valid token position in cached mask.")

    def validate_state(self) -> "KVCache":
        self._check_populated()
        return self

    # -- updates ---------------------------------------------------------------------------------------
    def update(self, k, v, mask=None) -> "KVCache":
        """First call: the prompt's k/v ``[B, S, H, hd]`` padded to max_seq_len.  Later calls: one token
        per row written at ``pos_id + 1``."""
        self._check_static()
        k, v = _as_tensor(k), _as_tensor(v, device=None)
        self._check_kv(k, v)
        k, v = k.to(self.dtype), v.to(self.dtype)
        if self.k is None:
            if self.v is not None or self.mask is not None or self.pos_id is not None:
                raise ValueError("KVCache has partial state: k is empty but v, mask, or pos_id is populated.")
            if k.shape[1] > self.max_seq_len:
                raise ValueError(f"Cannot cache {k.shape[1]} tokens in max_seq_len={self.max_seq_len}.")
            mask = torch.ones(k.shape[:2], dtype=torch.bool, device=k.device) if mask is None else _as_tensor(mask, k.device)
            if tuple(mask.shape) != tuple(k.shape[:2]):
                raise ValueError(f"mask shape must match k/v batch and sequence axes, got {tuple(mask.shape)} and "
                                 f"{tuple(k.shape[:2])}.")
            if mask.dtype.is_floating_point or mask.dtype.is_complex:
                raise TypeError(f"mask must be boolean or integer, got dtype {mask.dtype}.")
            _check_binary_int_mask("mask", mask)
            mask = mask.to(device=k.device, dtype=torch.bool)
            if not bool(mask.any(dim=1).all()):
                raise ValueError("mask must contain at least one valid token per batch row.")
            _check_right_padded("mask", mask)
            T = self.max_seq_len
            return self.replace(k=_pad_seq(k, T, 0), v=_pad_seq(v, T, 0), mask=_pad_seq(mask, T, False),
                                pos_id=get_default_pos_ids(mask))
        self._check_populated()
        if mask is not None:
            mask = _as_tensor(mask, self.mask.device)
            if tuple(mask.shape) != tuple(self.mask.shape):
                raise ValueError(f"Decode cache mask shape must match cached mask shape, got {tuple(mask.shape)} and "
                                 f"{tuple(self.mask.shape)}.")
            if mask.dtype.is_floating_point or mask.dtype.is_complex:
                raise TypeError(f"Decode cache mask must be boolean or integer, got dtype {mask.dtype}.")
            _check_binary_int_mask("Decode cache mask", mask)
            if not torch.equal(mask.to(torch.bool), self.mask):
                raise ValueError("Decode cache mask must match current cached mask state.")
        if k.shape[0] != self.k.shape[0]:
            raise ValueError(f"Batch size must match cached batch size, got {k.shape[0]} and {self.k.shape[0]}.")
        if k.shape[1] != 1:
            raise ValueError(f"Decode cache updates must contain exactly one token, got sequence length {k.shape[1]}.")
        if tuple(k.shape[2:]) != tuple(self.k.shape[2:]):
            raise ValueError(f"k/v trailing shape must match cached shape, got {tuple(k.shape[2:])} and "
                             f"{tuple(self.k.shape[2:])}.")
        nxt = self.next_pos_id
        if bool((nxt >= self.max_seq_len).any()):
            raise ValueError(f"Cannot decode past max_seq_len={self.max_seq_len}.")
        rows = torch.arange(k.shape[0], device=self.k.device)
        cols = nxt[:, 0].to(device=self.k.device, dtype=torch.int64)
        new_k, new_v, new_mask = self.k.clone(), self.v.clone(), self.mask.clone()
        new_k[rows, cols] = k[:, 0].to(new_k.device)
        new_v[rows, cols] = v[:, 0].to(new_v.device)
        new_mask[rows, cols] = True
        return self.replace(k=new_k, v=new_v, mask=new_mask, pos_id=nxt)

    def rollback(self, n: int) -> "KVCache":
        """Drops the last n tokens of every row (positions > pos_id - n are cleared)."""
        n = normalize_count("n", n)
        if n <= 0:
            raise ValueError("n must be greater than 0.")
        self._check_populated()
        if self.k is None:
            return self
        prev = self.pos_id - n
        if bool((prev < 0).any()):
            raise ValueError("Cannot roll back past the beginning of the KV cache.")
        keep = torch.arange(self.k.shape[1], device=self.k.device)[None] <= prev.to(self.k.device)
        zero = torch.zeros((), dtype=self.k.dtype, device=self.k.device)
        return self.replace(k=torch.where(keep[..., None, None], self.k, zero),
                            v=torch.where(keep[..., None, None], self.v, zero), mask=keep, pos_id=prev)

    def resize(self, new_size: int) -> "KVCache":
        new_size = normalize_count("new_size", new_size)
        if new_size <= 0:
            raise ValueError(f"new_size must be positive, got {new_size}.")
        self._check_populated()
        if self.k is None:
            return self.replace(max_seq_len=new_size)
        if bool((self.pos_id >= new_size).any()):
            raise ValueError("Cannot resize KV cache below the highest cached position.")
        if new_size > self.max_seq_len:
            return self.replace(k=_pad_seq(self.k, new_size, 0), v=_pad_seq(self.v, new_size, 0),
                                mask=_pad_seq(self.mask, new_size, False), max_seq_len=new_size)
        return self.replace(k=self.k[:, :new_size], v=self.v[:, :new_size], mask=self.mask[:, :new_size],
                            max_seq_len=new_size)

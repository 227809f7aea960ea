"""``InferenceConfig`` and ``Engine``: the reference's generation entry point (inference_engine/engine.py).

Argument checks and error messages follow ``engine.py:59-610`` and ``_generate.py:218-330``.  The
difference is where the work runs: ``init_params`` packs the parameter tree into the GPU layout of this
process's tensor-parallel rank, and ``generate`` runs prefill + decode on the GPU (CUDA-graph replay per
token) instead of jit-compiled XLA programs.  One process drives one GPU; with ``tp_size > 1`` the
processes of a ``torch.distributed`` group (NCCL) each hold 1/tp of the heads, FFN columns and
vocabulary.  ``dp_size`` replicas are independent process groups (no cross-replica traffic in
inference), so each Engine instance serves the batch it is given.
"""
from __future__ import annotations

import logging
import os
from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any, Optional

import numpy as np
import torch

from ._checks import normalize_bool, normalize_count, normalize_dtype
from .models import _DecoderWithHead
from .sampling import SamplingMethod, normalize_sampling_params

logger = logging.getLogger(__name__)


@dataclass(frozen=True)
class InferenceConfig:
    tp_size: int = 1
    dp_size: int = 1

    def __post_init__(self):
        tp = normalize_count("tp_size", self.tp_size)
        dp = normalize_count("dp_size", self.dp_size)
        object.__setattr__(self, "tp_size", tp)
        object.__setattr__(self, "dp_size", dp)
        if tp <= 0:
            raise ValueError(f"tp_size must be positive, got {tp}.")
        if dp <= 0:
            raise ValueError(f"dp_size must be positive, got {dp}.")


class _RawF32:
    """Zero-copy view of device memory the library allocated (CUDA array interface); float32 unless
    another typestr is given."""

    def __init__(self, ptr: int, n: int, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


class PeerRegion:
    """This rank's peer-mapped region for tensor parallelism over NVLink (include/jxb200.h,
    jx_comm_layout): a library-allocated device buffer shared with the other ranks through CUDA IPC handles
    exchanged over torch.distributed, and the other ranks' buffers mapped here.

    - `data[0]` and `data[1]`: the two float32 partials buffers of the pull all-reduce (jx_allreduce_f32);
      consecutive all-reduces alternate.
    - push mode (a decode projection with JX_EPI_PUSH_F32 feeding a jx_norm with peer_recv): every rank
      stores its partial into its own receive slot of every region; `bases_dev` is the device table of the
      ranks' region bases the kernels index, `recv_off` / `slot_bytes` / `flag_off` / `seq_off` the byte
      offsets shared by every region."""

    def __init__(self, comm: "TPComm", max_floats: int, device: torch.device):
        import ctypes

        from . import _native as N

        lib = N.load()
        off = (N.LL * 10)()
        N.check(lib.jx_comm_layout(max_floats, comm.size, off), "jx_comm_layout")
        self.max_floats = max_floats
        self._lib, self._N = lib, N
        with torch.cuda.device(device):
            p = N.P()
            N.check(lib.jx_comm_alloc(off[0], ctypes.byref(p)), "jx_comm_alloc")
            self.local = p.value
            torch.cuda.synchronize(device)   # the zeroed flags before any peer can write them
            h = ctypes.create_string_buffer(64)
            N.check(lib.jx_ipc_get_handle(self.local, h), "jx_ipc_get_handle")
            handles = [None] * comm.size
            comm.dist.all_gather_object(handles, h.raw, group=comm.group)
            bases, self._opened = [], []
            for r, hr in enumerate(handles):
                if r == comm.rank:
                    bases.append(self.local)
                    continue
                q = N.P()
                N.check(lib.jx_ipc_open_handle(hr, ctypes.byref(q)), "jx_ipc_open_handle")
                bases.append(q.value)
                self._opened.append(q.value)
            # the bases table the push kernels read, inside this rank's own region
            self.bases_dev = self.local + off[8]
            table = torch.as_tensor(_RawF32(self.bases_dev, comm.size, "<i8"), device=device)
            table.copy_(torch.tensor(bases, dtype=torch.int64))
            torch.cuda.synchronize(device)
        self.bases = (N.P * comm.size)(*bases)
        self._raw = [_RawF32(self.local + o, max_floats) for o in (off[1], off[2])]
        self.data = [torch.as_tensor(r, device=device) for r in self._raw]
        self.rank, self.world = comm.rank, comm.size
        self.recv_off, self.slot_bytes = off[3], off[4]
        self.flag_off, self.seq_off, self.max_units = off[5], off[7], off[9]

    def push_epilogue(self, epi, ldo: int):
        """Fills the JX_EPI_PUSH_F32 fields of a jx_epilogue (rows of `ldo` floats in the slot)."""
        N = self._N
        epi.kind = N.JX_EPI_PUSH_F32
        epi.ldo = ldo
        epi.peer_bases = self.bases_dev
        epi.peer_recv_off = self.recv_off
        epi.peer_slot_bytes = self.slot_bytes
        epi.peer_flag_off = self.flag_off
        epi.peer_seq_off = self.seq_off
        epi.peer_rank, epi.peer_world = self.rank, self.world

    def push_norm(self, args, d: int, lda: int):
        """Fills the push-mode fields of a jx_norm_args (the sum of the last push replaces `a`)."""
        args.a = None
        args.a_f32 = 0
        args.lda = lda
        args.peer_recv = self.local + self.recv_off
        args.peer_stride = self.slot_bytes // 4
        args.peer_flags = self.local + self.flag_off
        args.peer_seq = self.local + self.seq_off
        args.peer_world = self.world
        args.peer_units = d // 64

    def all_reduce(self, which: int, n: int, out: torch.Tensor, status: Optional[torch.Tensor] = None):
        st = None if status is None else status.data_ptr()
        stream = torch.cuda.current_stream(out.device).cuda_stream
        rc = self._lib.jx_allreduce_f32(self.bases, self.rank, self.world, self.max_floats, which, n,
                                        out.data_ptr(), st, 1, stream)
        self._N.check(rc, "jx_allreduce_f32")

    def close(self):
        for q in self._opened:
            self._lib.jx_ipc_close_handle(q)
        self._opened = []
        self.data = None
        if self.local:
            self._lib.jx_comm_free(self.local)
            self.local = 0


class TPComm:
    """Collectives of one tensor-parallel group: decode-sized all-reduces of the row-parallel partial sums
    through the library's NVLink peer kernel (PeerRegion), everything else over NCCL (torch.distributed)."""

    # peer all-reduce capacity in float32 elements: 64 token rows x 8192 hidden
    PEER_MAX_FLOATS = 64 * 8192

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._gather = None
        self.peer: Optional[PeerRegion] = None
        self._peer_tried = False
        self._which = 0

    def prepare_peer(self, device: torch.device) -> Optional[PeerRegion]:
        """Creates the peer region on first call (a collective: every rank makes it, outside any CUDA
        graph capture); None when the peer path does not apply (CPU or non-NCCL group, one rank or more
        than 8)."""
        if not self._peer_tried:
            self._peer_tried = True
            if (device.type == "cuda" and 2 <= self.size <= 8 and self.dist.get_backend(self.group) == "nccl"):
                self.peer = PeerRegion(self, self.PEER_MAX_FLOATS, device)
        return self.peer

    def partial_buffer(self, n_floats: int) -> Optional[torch.Tensor]:
        """The float32 buffer the next peer all-reduce reads (the two buffers alternate call by call), or
        None when the peer path is off or n_floats exceeds PEER_MAX_FLOATS."""
        if self.peer is None or n_floats > self.PEER_MAX_FLOATS:
            return None
        return self.peer.data[self._which][:n_floats]

    def all_reduce_partial(self, src: torch.Tensor, out: torch.Tensor, status: Optional[torch.Tensor] = None):
        """Sum of every rank's `src` (a prefix of partial_buffer()) into this rank's `out`, in rank order."""
        if src.data_ptr() != self.peer.data[self._which].data_ptr() or src.dtype != torch.float32:
            raise ValueError("all_reduce_partial: src must be the buffer partial_buffer() returned")
        if out.dtype != torch.float32 or not out.is_contiguous() or out.numel() < src.numel():
            raise ValueError("all_reduce_partial: out must be a contiguous float32 tensor of src's size")
        self.peer.all_reduce(self._which, src.numel(), out, status)
        self._which ^= 1

    def all_reduce(self, t: torch.Tensor):
        self.dist.all_reduce(t, group=self.group)

    def align(self, status: Optional[torch.Tensor] = None) -> bool:
        """Ends a pass (one decode step, one prefill) on partials buffer 0 by adding a 4-float all-reduce
        when the pass made an odd number of peer all-reduces.  A captured pass then always starts on
        buffer 0, so back-to-back replays keep alternating and no rank rewrites a buffer a peer may still
        be reading.  Every rank makes the same calls.  True when it launched that all-reduce.  (Push-mode
        projections need no alignment: their set follows the device-side epoch.)"""
        if self.peer is not None and self._which == 1:
            if getattr(self, "_align_out", None) is None:
                self._align_out = torch.empty(4, dtype=torch.float32, device=self.peer.data[0].device)
            self.all_reduce_partial(self.partial_buffer(4), self._align_out, status)
            return True
        return False

    def close(self):
        """Releases the peer region (every rank, no kernels in flight)."""
        if self.peer is not None:
            torch.cuda.synchronize()
            self.dist.barrier(group=self.group)
            self.peer.close()
            self.peer = None

    def all_gather_vocab(self, logits: torch.Tensor) -> torch.Tensor:
        """[B, V/size] vocabulary shard per rank -> [B, V] (rank r's shard at columns r*V/size ...)."""
        B, n = logits.shape
        if getattr(self, "_vgather", None) is None or self._vgather.numel() != self.size * B * n:
            self._vgather = torch.empty(self.size * B * n, dtype=logits.dtype, device=logits.device)
        self.dist.all_gather_into_tensor(self._vgather, logits.contiguous().reshape(-1), group=self.group)
        return self._vgather.view(self.size, B, n).permute(1, 0, 2).reshape(B, self.size * n)

    def all_gather_keys(self, keys: torch.Tensor) -> torch.Tensor:
        """[n] per rank -> [size, n] (rank-major), gathered into one flat buffer."""
        n = keys.numel()
        if self._gather is None or self._gather.numel() != self.size * n:
            self._gather = torch.empty(self.size * n, dtype=keys.dtype, device=keys.device)
        self.dist.all_gather_into_tensor(self._gather, keys.reshape(-1), group=self.group)
        return self._gather.view(self.size, n)


def _device_count() -> int:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size()
    return max(torch.cuda.device_count(), 1)


class Engine:
    """Wraps a model class for autoregressive generation on the GPU."""

    def __init__(self, model, config: InferenceConfig, params, dtype: Any = torch.float32, cache_stride: int = 256):
        if not isinstance(config, InferenceConfig):
            raise TypeError(f"config must be an InferenceConfig, got {type(config)}.")
        dtype = normalize_dtype("dtype", dtype)
        cache_stride = normalize_count("cache_stride", cache_stride)
        if cache_stride <= 0:
            raise ValueError(f"cache_stride must be positive, got {cache_stride}.")
        required = config.tp_size * config.dp_size
        available = _device_count()
        if required > available:
            raise ValueError(
                f"InferenceConfig requires {required} devices "
                f"(tp_size={config.tp_size}, dp_size={config.dp_size}), but only {available} are available."
            )
        self.model = model
        self.config = config
        self.params = params
        self.dtype = dtype
        self.cache_stride = cache_stride
        self._weights = None
        self._runtime = None
        self._comm = None

    # -- parameters ------------------------------------------------------------------------------------
    @staticmethod
    def _validate_param_weights(weights):
        if not isinstance(weights, Mapping):
            raise TypeError(f"weights must be a mapping, got {type(weights)}.")
        if "params" not in weights:
            raise ValueError(f"The key 'params' was not found in weights. Got keys: {weights.keys()}.")
        if not isinstance(weights["params"], Mapping):
            raise TypeError(f"weights['params'] must be a mapping, got {type(weights['params'])}.")

    def _device(self) -> torch.device:
        idx = int(os.environ.get("LOCAL_RANK", torch.cuda.current_device() if torch.cuda.is_available() else 0))
        return torch.device("cuda", idx)

    def init_params(self, weights=None, use_tpu: bool = False, reinit_weight: bool = False, tp_group=None):
        """Packs the parameters for this process's GPU (and tensor-parallel rank).

        ``use_tpu`` is accepted for signature compatibility and has no effect: the packed weights always go
        to the GPU of this process.  ``reinit_weight=True`` draws a fresh random tree first.
        """
        normalize_bool("use_tpu", use_tpu)
        reinit_weight = normalize_bool("reinit_weight", reinit_weight)
        if reinit_weight:
            weights = self.model.init(0)
        if weights is None:
            weights = self.params
        self._validate_param_weights(weights)
        from .runtime import ModelWeights

        tp = self.config.tp_size
        rank = 0
        if tp > 1:
            import torch.distributed as dist

            if not (dist.is_available() and dist.is_initialized()):
                raise RuntimeError("tp_size > 1 needs torch.distributed initialised (one process per GPU).")
            self._comm = TPComm(tp_group)
            if self._comm.size != tp:
                raise ValueError(f"tensor-parallel group has {self._comm.size} ranks, expected tp_size={tp}.")
            rank = self._comm.rank
        if not isinstance(self.model, _DecoderWithHead):
            raise TypeError(f"model must be one of the *ModelWithHead classes, got {type(self.model)}.")
        self.params = weights
        self._weights = ModelWeights(self.model.family, self.model.config, weights, self.model.dtype,
                                     self._device(), tp_rank=rank, tp_size=tp)
        self._runtime = None

    # -- inputs ----------------------------------------------------------------------------------------
    @staticmethod
    def _as_int_tensor(x, name: str) -> torch.Tensor:
        if isinstance(x, torch.Tensor):
            t = x.detach()
        else:
            t = torch.as_tensor(np.asarray(x))
        return t

    @staticmethod
    def _prepare_generation_inputs(prompt_tokens, attention_mask):
        """engine.py:379-417: 1D inputs become one row; the prompt and mask checks of ``generate``; integer
        masks become boolean.  Masks must also be right-padded (the kernels attend to key prefixes)."""
        prompt = Engine._as_int_tensor(prompt_tokens, "prompt_tokens")
        if prompt.ndim == 1:
            prompt = prompt[None]
        elif prompt.ndim != 2:
            raise ValueError(f"prompt_tokens must be a 1D or 2D array, got shape {tuple(prompt.shape)}.")
        if prompt.dtype.is_floating_point or prompt.dtype == torch.bool or prompt.dtype.is_complex:
            raise TypeError(f"prompt_tokens must contain integer token ids, got dtype {prompt.dtype}.")
        if prompt.shape[0] == 0:
            raise ValueError("prompt_tokens must contain at least one batch row.")
        if prompt.shape[1] == 0:
            raise ValueError("prompt_tokens must contain at least one token.")
        if attention_mask is None:
            return prompt, None
        mask = Engine._as_int_tensor(attention_mask, "attention_mask")
        if mask.ndim == 1:
            mask = mask[None]
        elif mask.ndim != 2:
            raise ValueError(f"attention_mask must be a 1D or 2D array, got shape {tuple(mask.shape)}.")
        if mask.dtype.is_floating_point or mask.dtype.is_complex:
            raise TypeError(f"attention_mask must be boolean or integer, got dtype {mask.dtype}.")
        if tuple(mask.shape) != tuple(prompt.shape):
            raise ValueError(
                f"attention_mask shape must match prompt_tokens shape; got {tuple(mask.shape)} and {tuple(prompt.shape)}."
            )
        if mask.dtype != torch.bool and bool(((mask != 0) & (mask != 1)).any()):
            raise ValueError("attention_mask integer values must be 0 or 1.")
        mask = mask.to(torch.bool)
        if not bool(mask.any(dim=1).all()):
            raise ValueError("attention_mask must contain at least one valid token per batch row.")
        if mask.shape[1] > 1 and bool((mask[:, :-1].to(torch.int8) < mask[:, 1:].to(torch.int8)).any()):
            raise ValueError("mask must be right padded: valid tokens cannot appear after masked positions.")
        return prompt, mask

    # -- the reference's step-by-step interface ---------------------------------------------------------
    def init_cache(self, max_seq_len: int) -> tuple:
        """``engine.py:110-121``: one empty ``KVCache`` of ``max_seq_len`` slots per layer, in the engine's
        dtype, for driving ``wrapped_apply_fn`` (or the model's ``apply``) step by step."""
        from .cache import KVCache

        max_seq_len = normalize_count("max_seq_len", max_seq_len)
        if max_seq_len <= 0:
            raise ValueError(f"max_seq_len must be positive, got {max_seq_len}.")
        try:
            num_layers = self.model.config.num_layers
        except AttributeError as e:
            raise TypeError("model must expose config.num_layers to initialize KV caches.") from e
        num_layers = normalize_count("model.config.num_layers", num_layers)
        if num_layers <= 0:
            raise ValueError(f"model.config.num_layers must be positive, got {num_layers}.")
        return tuple(KVCache.init(max_seq_len, None, None, dtype=self.dtype) for _ in range(num_layers))

    def prepare_input(self, inputs, dtype: Any = None):
        """``engine.py:320-353``: every leaf of ``inputs`` (an array or a dict / list / tuple of arrays) as a
        2D tensor on this process's GPU (the reference shards them over its data axis; one process drives
        one GPU here), cast to ``dtype`` when given.  Leaves must share the batch size, which must divide
        by ``dp_size``."""
        dtype = None if dtype is None else normalize_dtype("dtype", dtype)
        leaves = []

        def prep(x):
            if isinstance(x, Mapping):
                return type(x)((k, prep(v)) for k, v in x.items())
            if isinstance(x, (list, tuple)):
                return type(x)(prep(v) for v in x)
            try:
                t = x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x))
            except (TypeError, ValueError, RuntimeError) as e:
                raise TypeError(f"prepare_input leaves must be array-like, got {type(x)}.") from e
            if t.ndim != 2:
                raise ValueError(f"prepare_input leaves must be 2D arrays for data/model sharding, got shape "
                                 f"{tuple(t.shape)}.")
            if t.shape[0] == 0:
                raise ValueError("prepare_input leaves must contain at least one batch row.")
            if t.shape[1] == 0:
                raise ValueError("prepare_input leaves must contain at least one token.")
            if t.shape[0] % self.config.dp_size != 0:
                raise ValueError(f"prepare_input batch size must be divisible by dp_size={self.config.dp_size}, "
                                 f"got {t.shape[0]}.")
            if dtype is not None:
                t = t.to(dtype)
            leaves.append(t)
            return t

        out = prep(inputs)
        if not leaves:
            raise ValueError("prepare_input inputs must contain at least one array leaf.")
        for leaf in leaves[1:]:
            if leaf.shape[0] != leaves[0].shape[0]:
                raise ValueError(f"prepare_input leaves must share the same batch size, got {leaves[0].shape[0]} and "
                                 f"{leaf.shape[0]}.")
        if not torch.cuda.is_available():
            return out
        dev = self._device()

        def move(x):
            if isinstance(x, Mapping):
                return type(x)((k, move(v)) for k, v in x.items())
            if isinstance(x, (list, tuple)):
                return type(x)(move(v) for v in x)
            return x.to(dev)

        return move(out)

    def wrapped_apply_fn(self, params, input_token, attention_mask=None, kv_caches=None, use_cache: bool = True):
        """``engine.py:355-377``: one model call for step-by-step decoding, ``(logits of the last position
        [B, 1, V], kv_caches)``: a prompt into empty caches from ``init_cache``, then one token per row into
        the populated caches.  Runs the model's ``apply`` (the decoder blocks on the library's kernels);
        ``generate`` does the same steps on the fused runtime with one CUDA-graph replay per token."""
        out = self.model.apply(params, input_token, position_ids=None, attention_mask=attention_mask,
                               kv_caches=kv_caches, use_cache=use_cache, keep_last_n_logits=1)
        return out.logits, out.kv_caches

    def buffer_length(self, prompt_len: int, max_new_tokens: int) -> int:
        """Cache slots the reference's chunk loop ends with: (P // stride + 1) * stride, grown by stride
        until prompt + new tokens fit (engine.py:543-557)."""
        t = (prompt_len // self.cache_stride + 1) * self.cache_stride
        while t < prompt_len + max_new_tokens:
            t += self.cache_stride
        return t

    def _runtime_for(self, B: int, T: int):
        from .runtime import DecoderRuntime

        if self._weights is None:
            self.init_params()
        rt = self._runtime
        if rt is None or rt.B != B or rt.T < T:
            self._runtime = None
            torch.cuda.empty_cache()
            rt = DecoderRuntime(self._weights, B, T, comm=self._comm)
            self._runtime = rt
        return rt

    def close(self):
        """Releases the decode runtime: its captured CUDA graph, activation buffers and KV cache.

        Under tensor parallelism call it before ``destroy_process_group``: a captured graph that holds NCCL
        calls keeps the communicator alive, and the process-group teardown then waits on it for good."""
        if self._runtime is not None:
            self._runtime.graph = None
        self._runtime = None
        if torch.cuda.is_available():
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
        if self._comm is not None:
            self._comm.close()

    # -- generation ------------------------------------------------------------------------------------
    def generate(self, prompt_tokens, attention_mask=None, seed: int = 0, max_new_tokens: int = 10, top_k: int = 0,
                 top_p: float = 1.0, min_p: float = 0.0, temperature: float = 1.0, fuse_decoding: bool = False,
                 include_prompt: bool = True):
        """Greedy / temperature generation on the GPU; returns int32 tokens ``[B, P*include_prompt + N]``
        on the host.  ``fuse_decoding`` replays the decode loop as CUDA graphs of several steps each (the
        reference compiles it as one scan) instead of one graph replay per step; the tokens are the same."""
        seed = normalize_count("seed", seed)
        max_new_tokens = normalize_count("max_new_tokens", max_new_tokens)
        if max_new_tokens < 0:
            raise ValueError(f"max_new_tokens must be non-negative, got {max_new_tokens}.")
        fuse_decoding = normalize_bool("fuse_decoding", fuse_decoding)
        include_prompt = normalize_bool("include_prompt", include_prompt)
        prompt, mask = self._prepare_generation_inputs(prompt_tokens, attention_mask)
        vocab = self.model.config.vocab_size
        if bool(((prompt < 0) | (prompt >= vocab)).any()):
            raise ValueError(f"prompt_tokens token ids must be within [0, {vocab}).")
        sp = normalize_sampling_params(top_k=top_k, top_p=top_p, min_p=min_p, temp=temperature)
        method = SamplingMethod.from_values(top_k=sp.top_k, top_p=sp.top_p, min_p=sp.min_p, temp=sp.temp)
        logger.info("Given the parameters top_k=%.2f, top_p=%.2f, min_p=%.2f, temperature=%.2f, "
                    "the sampling method is determined as follows: %s.", sp.top_k, sp.top_p, sp.min_p, sp.temp, method)
        prompt = prompt.to(torch.int32)
        B, P = prompt.shape
        if max_new_tokens == 0:
            return prompt.clone() if include_prompt else prompt[:, :0].clone()
        rt = self._runtime_for(B, self.buffer_length(P, max_new_tokens))
        rt.filters = ((sp.top_k if method.use_top_k else 0, sp.top_p if method.use_top_p else 1.0,
                       sp.min_p if method.use_min_p else 0.0) if method.uses_filters else None)
        dev = self._weights.device
        pin = prompt.pin_memory() if not prompt.is_cuda else prompt
        ids_d = pin.to(dev, non_blocking=True)
        mask_d = (torch.ones(B, P, dtype=torch.bool) if mask is None else mask).pin_memory().to(dev, non_blocking=True)
        first_len = (P // self.cache_stride + 1) * self.cache_stride   # the reference's first chunk's cache
        toks = rt.generate(ids_d, mask_d, max_new_tokens, method.use_greedy, sp.temp, seed, fuse=fuse_decoding,
                           first_len=first_len)
        out = toks.to("cpu")
        rt.check_status()
        self.last_rng = rt.rng_key()
        if include_prompt:
            return torch.cat([prompt, out], dim=1)
        return out

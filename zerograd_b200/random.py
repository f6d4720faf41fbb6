"""Device threefry PRNG for loss functions (the subset of jax.random a
candidate loss uses with its per-candidate ``rng``).

Keys are ``torch.uint32`` tensors ``[2]``; every function works on one key
and under ``torch.func.vmap`` over a batch of keys (one launch per call).
"""
from __future__ import annotations

import math

import torch

from . import _ops
from ._keys import key

__all__ = ["key", "fold_in", "split", "bits", "normal"]


def fold_in(k: torch.Tensor, data) -> torch.Tensor:
    """``jax.random.fold_in``: ``threefry(key, (0, data))``."""
    return _ops.fold_in(k, data)


def split(k: torch.Tensor, num: int = 2) -> torch.Tensor:
    """``jax.random.split`` (partitionable): row i = ``threefry(key, (0, i))``."""
    ids = torch.arange(num, dtype=torch.int64, device=k.device)
    return _ops.launch_fold_in(k.reshape(1, 2), ids)


def bits(k: torch.Tensor, shape=()) -> torch.Tensor:
    """32-bit ``jax.random.bits``."""
    shape = tuple(shape)
    return _ops.bits(k, math.prod(shape)).reshape(shape)


def normal(k: torch.Tensor, shape=(), dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """``jax.random.normal`` (float32 draw; bf16 is the float32 draw rounded)."""
    shape = tuple(shape)
    return _ops.normal(k, math.prod(shape), dtype).reshape(shape)

"""Low-rank factors and vector noise (``src/zerograd/_factors.py:30-74``).

Factors are drawn as float32 normals on the device and cast to the leaf
dtype, exactly as the reference draws in float32 and casts afterwards.
"""
from __future__ import annotations

import math
from collections.abc import Sequence
from numbers import Real

import torch

from . import _lib as L
from . import _ops


def _validate_rank(rank: int) -> None:
    if not isinstance(rank, int) or isinstance(rank, bool) or rank < 1:
        raise ValueError(f"rank must be a positive integer, got {rank!r}")


def _validate_shape(shape: Sequence[int], ndim: int, name: str) -> tuple[int, ...]:
    dims = tuple(shape)
    if len(dims) != ndim or any(not isinstance(d, int) or isinstance(d, bool) or d < 1 for d in dims):
        raise ValueError(f"{name} must be a {ndim}-D shape of positive integers, got {shape!r}")
    return dims


def _validate_sigma(sigma) -> None:
    if not isinstance(sigma, Real) or isinstance(sigma, bool) or not math.isfinite(sigma) or sigma <= 0:
        raise ValueError(f"sigma must be a finite positive real, got {sigma!r}")


def scaled_factor(rank: int, sigma: float, dtype: torch.dtype) -> torch.Tensor:
    """``sigma / sqrt(rank)`` as a 0-d tensor of ``dtype`` (``_factors.py:30-40``)."""
    _validate_rank(rank)
    _validate_sigma(sigma)
    return torch.tensor(_ops.round_scalar(sigma / math.sqrt(rank), dtype), dtype=dtype)


def matrix_factors(key: torch.Tensor, shape: Sequence[int], rank: int, *, dtype: torch.dtype):
    """A[in, rank], B[rank, out] for a matrix leaf [in, out] (``_factors.py:43-55``)."""
    dims = _validate_shape(shape, 2, "matrix shape")
    _validate_rank(rank)
    A, B = _ops.launch_factors(key.reshape(1, 2), -1, L.ZG_MATRIX, dims, rank, dtype)
    return A[0], B[0]


def table_factors(key: torch.Tensor, shape: Sequence[int], rank: int, *, dtype: torch.dtype):
    """A[rows, rank], B[cols, rank] for a table leaf (``_factors.py:58-67``)."""
    dims = _validate_shape(shape, 2, "table shape")
    _validate_rank(rank)
    A, B = _ops.launch_factors(key.reshape(1, 2), -1, L.ZG_TABLE, dims, rank, dtype)
    return A[0], B[0]


def vector_noise(key: torch.Tensor, shape: Sequence[int], *, dtype: torch.dtype) -> torch.Tensor:
    """IID normal noise for a 1-D leaf, no split (``_factors.py:70-74``)."""
    (size,) = _validate_shape(shape, 1, "vector shape")
    A, _ = _ops.launch_factors(key.reshape(1, 2), -1, L.ZG_VECTOR, (size,), 1, dtype)
    return A[0]

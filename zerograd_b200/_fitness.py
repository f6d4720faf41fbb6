"""Centred-loss fitness shaping (``src/zerograd/_fitness.py:13-48``)."""
from __future__ import annotations

import math

import torch

from . import _ops


def _check_shape_dtype(losses: torch.Tensor) -> None:
    if losses.ndim != 1:
        raise ValueError(f"losses must be one-dimensional, got shape {tuple(losses.shape)}")
    if losses.shape[0] < 2:
        raise ValueError("at least two candidate losses are required")
    if not losses.is_floating_point():
        raise TypeError(f"losses must be a floating-point array, got dtype {losses.dtype}")


def shape_centered_loss(losses: torch.Tensor, sigma: float) -> torch.Tensor:
    """``-(losses - mean(losses)) / (population_size * sigma)`` in the loss dtype."""
    if losses.ndim != 1:
        raise ValueError(f"losses must be one-dimensional, got shape {tuple(losses.shape)}")
    if losses.shape[0] < 2:
        raise ValueError("at least two candidate losses are required")
    if not isinstance(sigma, float) or not math.isfinite(sigma) or sigma <= 0:
        raise ValueError(f"sigma must be a finite positive float, got {sigma!r}")
    if not losses.is_floating_point():
        raise TypeError(f"losses must be a floating-point array, got dtype {losses.dtype}")
    shaped, _ = _ops.launch_shape_fitness(losses, sigma)
    return shaped.to(losses.dtype)


def validate_losses(losses: torch.Tensor) -> None:
    """Reject non-1-D, too-short, non-float or non-finite losses (one host sync)."""
    _check_shape_dtype(losses)
    if not bool(torch.isfinite(losses).all()):
        raise ValueError("candidate losses must be finite")

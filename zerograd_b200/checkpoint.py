"""Checkpoint, resume and early stopping for long ZeroGrad runs.

A checkpoint holds the step, the parameter tree, the ``ZeroGradState``
(generation and optimizer state) and any extra data (for example the loss
history a late node needs to catch up).  Together with the seed they resume a
run exactly, since every key is derived from (seed, run_id, generation).
Mirrors the reference's helpers (examples/_checkpoint.py:34-55), written with
``torch.save`` so device tensors round-trip.
"""
from __future__ import annotations

import os
from typing import Any

import torch


def save_checkpoint(path: str, step: int, params: Any, state: Any, extra: Any = None) -> None:
    """Write ``{step, params, state, extra}`` to ``path`` atomically: the data
    goes to a temporary file that then replaces ``path``, so a crash during the
    write leaves any earlier checkpoint intact."""
    parent = os.path.dirname(os.path.abspath(path))
    os.makedirs(parent, exist_ok=True)
    tmp = path + ".tmp"
    torch.save({"step": step, "params": params, "state": state, "extra": extra}, tmp)
    os.replace(tmp, path)


def load_checkpoint(path: str, map_location=None) -> dict:
    """Load a checkpoint written by :func:`save_checkpoint`.  It is unpickled,
    so load only checkpoints from sources you trust."""
    return torch.load(path, map_location=map_location, weights_only=False)


class EarlyStopping:
    """Stop once a monitored metric stops improving for ``patience`` calls.

    ``mode='min'`` tracks the lowest value (a loss), ``mode='max'`` the highest
    (an accuracy); an improvement must exceed ``min_delta``.  Calling the
    object with the latest value returns True once patience is exhausted."""

    def __init__(self, patience: int = 50, mode: str = "min", min_delta: float = 0.0) -> None:
        if not isinstance(patience, int) or isinstance(patience, bool) or patience < 1:
            raise ValueError("patience must be a positive integer")
        if mode not in ("min", "max"):
            raise ValueError("mode must be 'min' or 'max'")
        self.patience = patience
        self.mode = mode
        self.min_delta = min_delta
        self.best: float | None = None
        self.wait = 0

    def __call__(self, metric: float) -> bool:
        if self.best is None:
            improved = True
        elif self.mode == "min":
            improved = metric < self.best - self.min_delta
        else:
            improved = metric > self.best + self.min_delta
        if improved:
            self.best = metric
            self.wait = 0
            return False
        self.wait += 1
        return self.wait >= self.patience

"""Checkpoint and resume for long ZeroGrad runs.

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

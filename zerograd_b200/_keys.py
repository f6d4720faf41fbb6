"""Deterministic key derivation (``src/zerograd/_keys.py:20-58``).

A key is a ``torch.uint32`` tensor of shape ``[2]`` (the key data words of
jax.random's threefry keys).  ``step_key`` is host arithmetic (crc32), as in
the reference; ``candidate_key`` / ``group_key`` run the device threefry.
"""
from __future__ import annotations

import zlib

import torch

from . import _ops
from ._manifest import Manifest


def _positive_int(value: int, name: str) -> None:
    if not isinstance(value, int) or isinstance(value, bool) or value < 1:
        raise ValueError(f"{name} must be a positive integer, got {value!r}")


def key(seed: int, device: torch.device | str | None = None) -> torch.Tensor:
    """``jax.random.key(seed)``: key words ``[seed >> 32, seed & 0xFFFFFFFF]``."""
    if not isinstance(seed, int) or isinstance(seed, bool):
        raise TypeError("seed must be an integer")
    seed &= 0xFFFFFFFFFFFFFFFF
    t = torch.tensor([(seed >> 32) & 0xFFFFFFFF, seed & 0xFFFFFFFF], dtype=torch.int64)
    return t.to(torch.uint32).to(device) if device is not None else t.to(torch.uint32)


def step_crc(seed: int, run_id: str, generation: int, manifest_version: int) -> int:
    """The 32-bit seed of one generation: crc32 of ``"seed:run_id:version:generation"``."""
    if not isinstance(seed, int) or isinstance(seed, bool):
        raise TypeError("seed must be an integer")
    if not isinstance(run_id, str) or not run_id:
        raise ValueError("run_id must be a non-empty string")
    if not isinstance(generation, int) or isinstance(generation, bool) or generation < 0:
        raise ValueError("generation must be a non-negative integer")
    _positive_int(manifest_version, "manifest_version")
    payload = f"{seed}:{run_id}:{manifest_version}:{generation}".encode()
    return zlib.crc32(payload) & 0xFFFFFFFF


def step_key(seed: int, run_id: str, generation: int, manifest_version: int,
             device: torch.device | str | None = None) -> torch.Tensor:
    """Stable base key of one generation (``_keys.py:20-30``)."""
    return key(step_crc(seed, run_id, generation, manifest_version), device)


def candidate_key(base_key: torch.Tensor, candidate_id) -> torch.Tensor:
    """``fold_in(base_key, candidate_id)`` (``_keys.py:33-53``)."""
    if isinstance(candidate_id, bool):
        raise TypeError("candidate_id must be a non-negative integer scalar")
    if isinstance(candidate_id, int):
        if candidate_id < 0:
            raise ValueError("candidate_id must be non-negative")
        return _ops.fold_in(base_key, candidate_id)
    if not isinstance(candidate_id, torch.Tensor):
        raise TypeError("candidate_id must be an integer scalar")
    if candidate_id.ndim != 0 or candidate_id.is_floating_point() or candidate_id.dtype == torch.bool:
        raise TypeError("candidate_id must be an integer scalar")
    if not torch._C._functorch.is_batchedtensor(candidate_id):
        if int(candidate_id) < 0:
            raise ValueError("candidate_id must be non-negative")
    return _ops.fold_in(base_key, candidate_id)


def group_key(candidate: torch.Tensor, manifest: Manifest, group: str) -> torch.Tensor:
    """``split(candidate, len(entries))[group_index]`` (``_keys.py:56-58``).

    Under the partitionable threefry the i-th split of a key is
    ``threefry(key, (0, i))``, the same block ``fold_in(key, i)`` computes,
    so the entry count does not change the key.
    """
    return _ops.fold_in(candidate, manifest.group_index(group))

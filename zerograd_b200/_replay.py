"""Factor replay: the pseudo-gradient descent direction rebuilt from the
keys used in the forward pass (``src/zerograd/_replay.py:15-80``).

One launch sequence per manifest entry: factor draw for every candidate,
then one contraction over the (candidate, rank) axis weighted by the shaped
fitness -- a dense perturbation ``[P, *shape]`` is never materialised.
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import _ops
from ._manifest import LAYOUT_CODE, Manifest, ParameterLayout, ParameterPath, ParameterTree


def candidate_keys(base_key: torch.Tensor, candidate_ids: torch.Tensor) -> torch.Tensor:
    """``[len(ids), 2]`` candidate keys ``fold_in(base_key, id)`` in one launch."""
    return _ops.launch_fold_in(base_key.reshape(1, 2), candidate_ids)


def replay_entry_keys(params: ParameterTree, manifest: Manifest, path: ParameterPath, cand_keys: torch.Tensor,
                      shaped_weights: torch.Tensor, rank: int, gen=None) -> torch.Tensor:
    """Descent direction of one entry (float32) from precomputed candidate keys.

    `gen` names the generation whose whole population `cand_keys` are; its
    forward-pass factors are then reused from the factor cache.
    """
    entry = manifest.entry(path)
    parameter = manifest.resolve(params, path)
    layout = LAYOUT_CODE[entry.layout]
    group = manifest.group_index(entry.group)
    r = 1 if entry.layout is ParameterLayout.VECTOR else rank
    return _ops.launch_replay(shaped_weights, cand_keys, group, layout, tuple(parameter.shape), r,
                              parameter.dtype, gen=gen)


def replay_entry_step(params: ParameterTree, manifest: Manifest, path: ParameterPath, cand_keys: torch.Tensor,
                      shaped_weights: torch.Tensor, rank: int, step: dict, gen=None,
                      inplace_guard: torch.Tensor | None = None):
    """Replay of one entry with the optimizer step fused in: (param, mu, nu)
    or None where the fused form does not apply (VECTOR entries, float32
    leaves), in which case the caller replays and steps separately.  With
    `inplace_guard` the step updates the entry in place unless the guard
    (a device float) is non-zero."""
    entry = manifest.entry(path)
    if entry.layout is ParameterLayout.VECTOR:
        return None
    parameter = manifest.resolve(params, path)
    return _ops.launch_replay_step(shaped_weights, cand_keys, manifest.group_index(entry.group),
                                   LAYOUT_CODE[entry.layout], parameter, rank, step, gen=gen,
                                   inplace_guard=inplace_guard)


def replay_entry(params: ParameterTree, manifest: Manifest, path: ParameterPath, base_key: torch.Tensor,
                 candidate_ids: torch.Tensor, shaped_weights: torch.Tensor, rank: int) -> torch.Tensor:
    """``_replay.py:15-54``."""
    parameter = manifest.resolve(params, path)
    ids = torch.as_tensor(candidate_ids, device=parameter.device)
    cks = candidate_keys(base_key, ids)
    return replay_entry_keys(params, manifest, path, cks, shaped_weights.to(parameter.device), rank)


def replay(params: ParameterTree, manifest: Manifest, base_key: torch.Tensor, candidate_ids: torch.Tensor,
           shaped_weights: torch.Tensor, rank: int) -> dict:
    """Descent directions of every manifest entry as a nested dict (``_replay.py:57-80``)."""
    first = manifest.resolve(params, manifest.entries[0].path)
    ids = torch.as_tensor(candidate_ids, device=first.device)
    cks = candidate_keys(base_key, ids)
    w = shaped_weights.to(first.device)
    result: dict = {}
    for entry in manifest.entries:
        leaf = replay_entry_keys(params, manifest, entry.path, cks, w, rank)
        node = result
        for part in entry.path[:-1]:
            node = node.setdefault(part, {})
        node[entry.path[-1]] = leaf
    return result

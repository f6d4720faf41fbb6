"""Optimizer transforms with optax's update rules, fused on the device.

The reference hands the negated replay output to an Optax transform
(``src/zerograd/_optimizer.py:233-234``).  Optax is third-party code absent
from the reference tree; ``adamw`` and ``sgd`` here restate optax 0.2.8's
``adamw`` (scale_by_adam -> add_decayed_weights -> scale(-lr)) and ``sgd``
(scale(-lr), no momentum) and run as one fused kernel per leaf that also
applies the update.  Any object with optax's ``init`` / ``update`` protocol
on torch tensors may be used instead (applied with :func:`apply_updates`).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from . import _ops


def _leaves(tree, prefix=()):
    for k, v in tree.items():
        if isinstance(v, dict):
            yield from _leaves(v, prefix + (k,))
        else:
            yield prefix + (k,), v


def tree_get(tree, path):
    node = tree
    for p in path:
        if not isinstance(node, dict) or p not in node:
            return None
        node = node[p]
    return node


def tree_set(tree, path, value):
    node = tree
    for p in path[:-1]:
        node = node.setdefault(p, {})
    node[path[-1]] = value


@dataclass(frozen=True)
class AdamWState:
    count: int
    mu: dict
    nu: dict
    # Optional device float32 [2]: the bias corrections of step count + 1,
    # read by the kernels instead of deriving them from `count` (a captured
    # generation fills it before each replay).  None: derived from `count`.
    bias_corrections: torch.Tensor | None = None


@dataclass(frozen=True)
class adamw:
    """``optax.adamw(learning_rate, b1, b2, eps, eps_root=0, weight_decay)``."""

    learning_rate: float
    b1: float = 0.9
    b2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 1e-4

    def init(self, params: dict) -> AdamWState:
        mu, nu = {}, {}
        for path, p in _leaves(params):
            if isinstance(p, torch.Tensor):
                tree_set(mu, path, torch.zeros(p.shape, dtype=torch.float32, device=p.device))
                tree_set(nu, path, torch.zeros(p.shape, dtype=torch.float32, device=p.device))
        return AdamWState(count=0, mu=mu, nu=nu)

    def step_spec(self, state: AdamWState, path) -> dict:
        """The step of one leaf, for a replay that applies it in its epilogue."""
        return {"kind": "adamw", "lr": self.learning_rate, "b1": self.b1, "b2": self.b2, "eps": self.eps,
                "weight_decay": self.weight_decay, "count": state.count + 1, "mu": tree_get(state.mu, path),
                "nu": tree_get(state.nu, path), "bc": state.bias_corrections}

    def apply(self, params: dict, descent: dict, state: AdamWState, done: dict | None = None):
        """New params and state from the descent tree (missing leaf: zero
        gradient); `done` maps leaf paths already stepped by a fused replay to
        their (param, mu, nu)."""
        count = state.count + 1
        new_p, mu, nu = {}, {}, {}
        for path, p in _leaves(params):
            if not isinstance(p, torch.Tensor):
                tree_set(new_p, path, p)
                continue
            if done and path in done:
                pn, m, v = done[path]
                tree_set(new_p, path, pn)
                tree_set(mu, path, m)
                tree_set(nu, path, v)
                continue
            d = tree_get(descent, path)
            pn, m, v = _ops.launch_adamw(p, d, tree_get(state.mu, path), tree_get(state.nu, path), count,
                                         self.learning_rate, self.b1, self.b2, self.eps, self.weight_decay,
                                         state.bias_corrections)
            tree_set(new_p, path, pn)
            tree_set(mu, path, m)
            tree_set(nu, path, v)
        return new_p, AdamWState(count=count, mu=mu, nu=nu, bias_corrections=state.bias_corrections)


@dataclass(frozen=True)
class SgdState:
    count: int = 0


@dataclass(frozen=True)
class sgd:
    """``optax.sgd(learning_rate)`` without momentum."""

    learning_rate: float

    def init(self, params: dict) -> SgdState:
        return SgdState()

    def step_spec(self, state: SgdState, path) -> dict:
        return {"kind": "sgd", "lr": self.learning_rate}

    def apply(self, params: dict, descent: dict, state: SgdState, done: dict | None = None):
        new_p = {}
        for path, p in _leaves(params):
            if not isinstance(p, torch.Tensor):
                tree_set(new_p, path, p)
                continue
            if done and path in done:
                tree_set(new_p, path, done[path][0])
                continue
            tree_set(new_p, path, _ops.launch_sgd(p, tree_get(descent, path), self.learning_rate))
        return new_p, SgdState(count=state.count + 1)


def apply_updates(params: dict, updates: dict) -> dict:
    """``optax.apply_updates``: ``p + u`` cast back to the parameter dtype."""
    out = {}
    for path, p in _leaves(params):
        u = tree_get(updates, path)
        if isinstance(p, torch.Tensor) and u is not None:
            tree_set(out, path, (p.to(torch.float32) + u).to(p.dtype))
        else:
            tree_set(out, path, p)
    return out


def is_fused(transform: Any) -> bool:
    return isinstance(transform, (adamw, sgd))

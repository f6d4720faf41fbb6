"""CPU oracle of the ViT-small workload's candidate forward.

TEST INFRASTRUCTURE ONLY (``tests/``, ``bench.py``'s CPU legs); the product
never imports it.

Restates the reference example's candidate forward
(``examples/train_vit_cifar10.py:137-191``: patch embedding, CLS token,
positional table, pre-norm blocks of LayerNorm, q/k/v/o softmax attention,
GELU MLP, residuals; final LayerNorm, head on the CLS token, softmax
cross-entropy) over ``oracle/ref.py``'s perturbed ops, in float64 with the
CUDA path's bf16 storage roundings (each op's output rounded to bf16).
The GELU is the tanh form, ``jax.nn.gelu``'s default.
"""
from __future__ import annotations

import numpy as np

from . import lm, ref


def _bf16(a):
    return ref.round_bf16(np.asarray(a, np.float32)).astype(np.float64)


def candidate_loss(params: dict, entries: list, ck: np.ndarray, cfg: dict, patches: np.ndarray,
                   labels: np.ndarray, rank: int, sigma: float) -> float:
    """Mean cross-entropy of the candidate with key `ck`; `entries` are the
    manifest's paths in order (one group per entry: group index = position)."""
    gi = {tuple(path): i for i, path in enumerate(entries)}
    s = ref.scaled_factor(rank, sigma, "bfloat16")

    def leaf(path):
        node = params
        for k in path:
            node = node[k]
        return node

    def gk(path):
        return ref.fold_in(ck, gi[tuple(path)])

    def vec(*path):
        return _bf16(ref.perturbed_vector(leaf(path), gk(path), sigma, "bfloat16"))

    def linear(path, x, act=None, residual=None):
        W = leaf(path)
        a, b = ref.matrix_factors(gk(path), W.shape, rank, "bfloat16")
        u = _bf16(s * (x @ a.astype(np.float64)))
        y = _bf16(x @ np.asarray(W, np.float64) + u @ b.astype(np.float64))
        if act == "gelu":
            y = _bf16(lm.gelu_tanh(y))
        if residual is not None:
            y = _bf16(residual + y)
        return y

    E, H = cfg["embed"], cfg["heads"]
    B = patches.shape[0]
    x = linear(("patch_embed", "weight"), np.asarray(patches, np.float64))
    cls = np.broadcast_to(vec("cls_token"), (B, 1, E))
    x = np.concatenate([cls, x], axis=1)
    T = x.shape[1]
    pa, pb = ref.table_factors(gk(("pos_embed",)), leaf(("pos_embed",)).shape, rank, "bfloat16")
    pos = _bf16(np.asarray(leaf(("pos_embed",)), np.float64)[:T] + s * (pa[:T].astype(np.float64) @
                                                                      pb.T.astype(np.float64)))
    x = _bf16(x + pos)
    for i in range(cfg["layers"]):
        n = f"layer{i}"
        h = _bf16(ref.layer_norm(x, vec(n, "ln1", "scale"), vec(n, "ln1", "bias")))
        q, k, v = (linear((n, w, "weight"), h).reshape(B, T, H, E // H) for w in ("q", "k", "v"))
        a = _bf16(ref.attention(q, k, v)).reshape(B, T, E)
        x = linear((n, "o", "weight"), a, residual=x)
        h = _bf16(ref.layer_norm(x, vec(n, "ln2", "scale"), vec(n, "ln2", "bias")))
        h = linear((n, "mlp1", "weight"), h, act="gelu")
        x = linear((n, "mlp2", "weight"), h, residual=x)
    x = _bf16(ref.layer_norm(x, vec("ln_f", "scale"), vec("ln_f", "bias")))
    logits = _bf16(linear(("head", "weight"), x[:, 0, :]) + vec("head", "bias"))
    mx = logits.max(axis=-1, keepdims=True)
    lse = mx[:, 0] + np.log(np.exp(logits - mx).sum(axis=-1))
    return float(np.mean(lse - logits[np.arange(B), np.asarray(labels, np.int64)]))


def population_losses(params, entries, base, ids, cfg, patches, labels, rank, sigma) -> np.ndarray:
    cks = ref.candidate_keys(base, ids)
    return np.array([candidate_loss(params, entries, ck, cfg, patches, labels, rank, sigma) for ck in cks])

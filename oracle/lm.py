"""CPU oracle of the decoder-LM workload's candidate forward and replay.

TEST INFRASTRUCTURE ONLY: used by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU legs as the checker (or as the timed CPU
restatement); the product never imports it.

The reference has no language model of its own; its transformer block is
the ViT example's (``examples/train_vit_cifar10.py:137-191``: norm, q/k/v
projections, softmax attention, output projection, residuals, norm, GELU
MLP).  The decoder LM is that block made causal, with RMSNorm (scale a
VECTOR entry), a fused q/k/v projection, the tanh-form GELU, and a tied
embedding TABLE read by ``table_lookup`` (``src/zerograd/_candidate.py:25-30``)
and by ``tied_logits`` (``:33-38``) followed by the next-token softmax
cross-entropy (the examples' loss over logits, ``examples/train_cifar10.py:77-78``).

Every op restates ``oracle/ref.py``'s (factors from the C threefry
restatement) and is rounded to bf16 wherever the CUDA path stores a bf16
tensor, so a comparison measures the kernels' accumulation order, not a
different model.  `dtype` is the arithmetic: float64 for parity checks
(bf16 storage roundings emulated), float32 for the timed CPU baseline (a
plain float32 forward, as a CPU implementation computes it: no emulated
bf16 rounding).
"""
from __future__ import annotations

import math

import numpy as np

from . import ref


def gelu_tanh(x):
    """0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) (Hendrycks & Gimpel), in x's dtype."""
    c = x.dtype.type(math.sqrt(2.0 / math.pi))
    t = x * x
    t *= x.dtype.type(0.044715)
    t += 1
    t *= x
    t *= c
    np.tanh(t, out=t)
    t += 1
    t *= x
    t *= x.dtype.type(0.5)
    return t


def _bf16(a, dtype):
    if dtype == np.float32:
        return np.asarray(a, np.float32)
    return ref.round_bf16(np.asarray(a, np.float32)).astype(dtype, copy=False)


def _attention(q, k, v, dtype):
    """Causal softmax attention in `dtype` (ref.attention's float64 for parity)."""
    if dtype != np.float32:
        return ref.attention(q, k, v, causal=True)
    qh, kh, vh = (np.swapaxes(t, -3, -2) for t in (q, k, v))
    s = qh @ np.swapaxes(kh, -1, -2) * np.float32(1.0 / math.sqrt(q.shape[-1]))
    S = s.shape[-1]
    s = np.where(np.triu(np.ones((S, S), bool), 1), np.float32(-np.inf), s)
    s = np.exp(s - s.max(axis=-1, keepdims=True))
    s /= s.sum(axis=-1, keepdims=True)
    return np.swapaxes(s @ vh, -3, -2)


def candidate_loss(params: dict, entries: list, ck: np.ndarray, cfg: dict, tokens: np.ndarray,
                   labels: np.ndarray, rank: int, sigma: float, dtype=np.float64) -> float:
    """Mean next-token cross-entropy of the candidate with key `ck`.

    `params`: name -> float32 array holding the bf16 values; `entries`: the
    manifest's entry names in order, one group each, so an entry's group
    index is its position (``Manifest.group_index``); `cfg`: layers, heads."""
    gi = {name: i for i, name in enumerate(entries)}
    s = ref.scaled_factor(rank, sigma, "bfloat16")
    P = {k: np.asarray(v, dtype) for k, v in params.items()}

    def gk(name):
        return ref.fold_in(ck, gi[name])

    def vec(name):
        return _bf16(ref.perturbed_vector(params[name], gk(name), sigma, "bfloat16"), dtype)

    def linear(name, x, act=None, residual=None):
        a, b = ref.matrix_factors(gk(name), params[name].shape, rank, "bfloat16")
        u = _bf16(s * (x @ a.astype(dtype)), dtype)  # the low-rank activation, stored in bf16
        y = _bf16(x @ P[name] + u @ b.astype(dtype), dtype)
        if act == "gelu":
            y = _bf16(gelu_tanh(y), dtype)
        if residual is not None:
            y = _bf16(residual + y, dtype)
        return y

    def rms(x, scale):
        return _bf16(x / np.sqrt((x * x).mean(axis=-1, keepdims=True) + 1e-6) * scale, dtype)

    B, T = tokens.shape
    H = cfg["heads"]
    ta, tb = ref.table_factors(gk("emb"), params["emb"].shape, rank, "bfloat16")
    x = _bf16(P["emb"][tokens] + s * (ta[tokens].astype(dtype) @ tb.T.astype(dtype)), dtype)
    E = x.shape[-1]
    D = E // H
    for layer in range(cfg["layers"]):
        p = f"l{layer}."
        h = rms(x, vec(p + "n1"))
        qkv = linear(p + "qkv", h).reshape(B, T, 3, H, D)
        a = _bf16(_attention(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], dtype), dtype)
        x = linear(p + "o", a.reshape(B, T, E), residual=x)
        h = rms(x, vec(p + "n2"))
        m = linear(p + "fc", h, act="gelu")
        x = linear(p + "proj", m, residual=x)
    h = rms(x, vec("nf"))
    # tied logits rounded to bf16 (what tied_logits returns), log-sum-exp over the vocabulary
    u = _bf16(s * (h @ tb.astype(dtype)), dtype)
    logits = _bf16(h @ P["emb"].T + u @ ta.T.astype(dtype), dtype)
    mx = logits.max(axis=-1, keepdims=True)
    lse = mx[..., 0] + np.log(np.exp(logits - mx).sum(axis=-1))
    picked = np.take_along_axis(logits, labels[..., None].astype(np.int64), axis=-1)[..., 0]
    return float(np.mean(lse - picked))


def population_losses(params: dict, entries: list, base: np.ndarray, ids, cfg: dict, tokens: np.ndarray,
                      labels: np.ndarray, rank: int, sigma: float, dtype=np.float64) -> np.ndarray:
    cks = ref.candidate_keys(base, ids)
    return np.array([candidate_loss(params, entries, ck, cfg, tokens, labels, rank, sigma, dtype) for ck in cks],
                    np.float64)


def replay_sample(params: dict, entries: list, layouts: dict, base: np.ndarray, ids, shaped, rank: int,
                  dtype=np.float32) -> dict:
    """The sampled candidates' share of every entry's pseudo-gradient
    (``src/zerograd/_replay.py:15-54``): factors drawn, weighted, contracted
    over the candidates (the CPU restatement's replay, for timing)."""
    cks = ref.candidate_keys(base, ids)
    w = np.asarray(shaped, dtype)
    out = {}
    for g, name in enumerate(entries):
        gks = ref.group_keys(cks, g)
        layout = layouts[name]
        shape = params[name].shape
        if layout == ref.VECTOR:
            n, _ = ref.population_factors(gks, ref.VECTOR, shape, 1, "bfloat16")
            out[name] = (w[:, None] * n.astype(dtype)).sum(0)
            continue
        A, Bf = ref.population_factors(gks, layout, shape, rank, "bfloat16")
        n = A.shape[0]
        wa = (A.astype(dtype) * w[:, None, None]).transpose(1, 0, 2).reshape(shape[0], n * rank)
        bb = Bf.astype(dtype).reshape(n * rank, shape[1]) if layout == ref.MATRIX else \
            Bf.astype(dtype).transpose(0, 2, 1).reshape(n * rank, shape[1])
        out[name] = (wa @ bb) * ref.scaled_factor(rank, 1.0, "bfloat16")
    return out

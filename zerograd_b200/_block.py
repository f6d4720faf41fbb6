"""Transformer-block ops of a candidate's forward, population-batched.

The reference writes a candidate's transformer block as user code around the
perturbed ops (``examples/train_vit_cifar10.py:137-191``): LayerNorm with the
perturbed VECTOR scale and bias, the perturbed q/k/v/o projections, softmax
attention.  Under ``torch.func.vmap`` over candidates, these ops turn the
batched candidate axis into ONE population launch each, like the
``CandidateContext`` ops:

* :func:`layer_norm` / :func:`rms_norm`: ``zg_layer_norm`` / ``zg_rms_norm``,
  statistics in float32, per-candidate scale and bias (what
  ``ctx.vector`` returns for each candidate);
* :func:`attention`: ``zg_attention``, softmax(q kᵀ / √d) v per candidate,
  batch row and head, optionally causal.
"""
from __future__ import annotations

import math

import torch

from . import _lib as L
from ._ops import _NS, _movedim0


def _as(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return t if t.dtype == dtype else t.to(dtype)


def launch_norm(kind: str, x: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None, eps: float,
                x_batched: bool, p_batched: bool, P: int) -> torch.Tensor:
    """Population norm: x [P, ..., C] (x_batched) or [..., C]; scale/bias
    [P, C] (p_batched) or [C].  Returns [P, ..., C] (or [..., C] when
    neither is batched and P == 1)."""
    dev = L.require_cuda(x, scale, bias)
    dt = x.dtype
    L.dtype_code(dt)
    C = int(x.shape[-1])
    x = x.contiguous()
    scale = _as(scale, dt).contiguous()
    bias = None if bias is None else _as(bias, dt).contiguous()
    if scale.shape[-1] != C or (bias is not None and bias.shape[-1] != C):
        raise ValueError(f"scale/bias of width {scale.shape[-1]} do not match the normalised axis {C}")
    rest = tuple(x.shape[1:-1]) if x_batched else tuple(x.shape[:-1])
    M = math.prod(rest)
    out_shape = ((P,) if (x_batched or p_batched) else ()) + rest + (C,)
    y = torch.empty(out_shape, dtype=dt, device=dev)
    if kind == "layer":
        L.call("zg_layer_norm", L.ptr(x), int(x_batched), L.ptr(scale), L.ptr(bias), int(p_batched), P, M, C,
               float(eps), L.dtype_code(dt), L.ptr(y), L.stream_ptr(dev))
    else:
        L.call("zg_rms_norm", L.ptr(x), int(x_batched), L.ptr(scale), int(p_batched), P, M, C, float(eps),
               L.dtype_code(dt), L.ptr(y), L.stream_ptr(dev))
    return y


def _norm_vmap(kind, in_dims, x, scale, bias, eps):
    xd, sd = in_dims[0], in_dims[1]
    bd = in_dims[2] if bias is not None else None
    x, scale = _movedim0(x, xd), _movedim0(scale, sd)
    bias = _movedim0(bias, bd) if bias is not None else None
    sizes = [t.shape[0] for t, d in ((x, xd), (scale, sd), (bias, bd)) if d is not None and t is not None]
    if not sizes:
        return launch_norm(kind, x, scale, bias, eps, False, False, 1), None
    P = sizes[0]
    p_batched = sd is not None or bd is not None
    if p_batched:
        # a scale (or bias) shared while the other is per candidate: both per candidate
        if sd is None:
            scale = scale.expand(P, *scale.shape)
        if bias is not None and bd is None:
            bias = bias.expand(P, *bias.shape)
    return launch_norm(kind, x, scale, bias, eps, xd is not None, p_batched, P), 0


@torch.library.custom_op(f"{_NS}::layer_norm", mutates_args=())
def _layer_norm_op(x: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None, eps: float) -> torch.Tensor:
    return launch_norm("layer", x, scale, bias, eps, False, False, 1)


@torch.library.register_vmap(f"{_NS}::layer_norm")
def _layer_norm_vmap(info, in_dims, x, scale, bias, eps):
    return _norm_vmap("layer", in_dims, x, scale, bias, eps)


@torch.library.custom_op(f"{_NS}::rms_norm", mutates_args=())
def _rms_norm_op(x: torch.Tensor, scale: torch.Tensor, eps: float) -> torch.Tensor:
    return launch_norm("rms", x, scale, None, eps, False, False, 1)


@torch.library.register_vmap(f"{_NS}::rms_norm")
def _rms_norm_vmap(info, in_dims, x, scale, eps):
    return _norm_vmap("rms", (in_dims[0], in_dims[1], None), x, scale, None, eps)


def layer_norm(x: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None = None,
               eps: float = 1e-5) -> torch.Tensor:
    """(x - mean) / sqrt(var + eps) * scale + bias over the last axis
    (``examples/train_vit_cifar10.py:76-79``): float32 statistics, output in
    x's dtype.  Under vmap over candidates, per-candidate x, scale and bias
    are one population launch."""
    return _layer_norm_op(x, scale, bias, float(eps))


def rms_norm(x: torch.Tensor, scale: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x / sqrt(mean(x^2) + eps) * scale over the last axis (float32
    statistics, output in x's dtype)."""
    return _rms_norm_op(x, scale, float(eps))


def _row_pitch(t: torch.Tensor) -> int | None:
    """Elements between consecutive sequence positions of a [..., S, H, D]
    tensor whose heads are contiguous and whose leading axes collapse into
    one axis of S-position blocks (a view into a fused q/k/v projection
    [..., S, 3, H, D] qualifies); None otherwise."""
    S, H, D = (int(d) for d in t.shape[-3:])
    st = t.stride()
    if st[-1] != 1 or (H > 1 and st[-2] != D):
        return None
    ld = st[-3] if S > 1 else H * D
    if ld < H * D:
        return None
    block = S * ld
    for d in range(t.ndim - 4, -1, -1):
        if t.shape[d] > 1 and st[d] != block:
            return None
        block *= t.shape[d]
    return ld


def launch_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool) -> torch.Tensor:
    """softmax(q kᵀ / √D) v over [..., S, H, D] tensors (leading axes: the
    candidates and batch rows), one launch.  q, k and v may be views with a
    common row pitch (three slices of a fused q/k/v projection); the output
    is contiguous."""
    dev = L.require_cuda(q, k, v)
    if q.ndim < 3 or tuple(q.shape) != tuple(k.shape) or tuple(q.shape) != tuple(v.shape):
        raise ValueError("q, k and v must share one [..., S, H, D] shape")
    dt = q.dtype
    L.dtype_code(dt)
    S, H, D = (int(d) for d in q.shape[-3:])
    Z = math.prod(q.shape[:-3])
    k, v = _as(k, dt), _as(v, dt)
    pitches = {_row_pitch(t) for t in (q, k, v)}
    if len(pitches) != 1 or None in pitches:
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        ld = H * D
    else:
        ld = pitches.pop()
    o = torch.empty(q.shape, dtype=dt, device=dev)
    L.call("zg_attention_ex", L.ptr(q), L.ptr(k), L.ptr(v), ld, Z, S, H, D, int(bool(causal)), L.dtype_code(dt),
           L.ptr(o), L.stream_ptr(dev))
    return o


@torch.library.custom_op(f"{_NS}::attention", mutates_args=())
def _attention_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool) -> torch.Tensor:
    return launch_attention(q, k, v, causal)


@torch.library.register_vmap(f"{_NS}::attention")
def _attention_vmap(info, in_dims, q, k, v, causal):
    dims = in_dims[:3]
    ts = [_movedim0(t, d) for t, d in zip((q, k, v), dims)]
    P = next(t.shape[0] for t, d in zip(ts, dims) if d is not None)
    ts = [t if d is not None else t.expand(P, *t.shape) for t, d in zip(ts, dims)]
    return launch_attention(ts[0], ts[1], ts[2], causal), 0


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    """softmax(q kᵀ / sqrt(D)) v per head (``examples/train_vit_cifar10.py:166-172``),
    q, k, v [..., S, H, D] as the projections produce them (no transpose);
    `causal` masks keys after the query.  Under vmap over candidates the
    whole population's attention is one launch."""
    return _attention_op(q, k, v, bool(causal))


__all__ = ["attention", "layer_norm", "rms_norm", "launch_attention", "launch_norm"]

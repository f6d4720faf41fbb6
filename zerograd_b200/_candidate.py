"""Factor-only forward ops of one candidate (``src/zerograd/_candidate.py``).

Each op is a custom op over the C ABI; called per candidate inside
``torch.func.vmap`` (as ``ZeroGrad`` does) it becomes one population-batched
kernel launch.  ``CandidateContext`` passes the CANDIDATE key and the group
index, and the kernel derives the group key itself.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _ops
from ._factors import _validate_rank, _validate_sigma
from ._keys import group_key
from ._manifest import Manifest, ParameterLayout, ParameterPath, ParameterTree


def perturbed_linear(x: torch.Tensor, weight: torch.Tensor, key: torch.Tensor, rank: int,
                     sigma: float) -> torch.Tensor:
    """``x @ weight + sigma/sqrt(rank) * (x @ A) @ B`` for a group key (``_candidate.py:17-22``)."""
    if weight.ndim != 2 or x.shape[-1] != weight.shape[0]:
        raise ValueError("linear input and [in, out] weight shapes are incompatible")
    _validate_rank(rank)
    _validate_sigma(sigma)
    return _ops.linear(x, weight, key, -1, rank, sigma)


def perturbed_table_lookup(table: torch.Tensor, indices: torch.Tensor, key: torch.Tensor, rank: int,
                           sigma: float) -> torch.Tensor:
    """``T[idx] + s * A[idx] @ B^T`` (``_candidate.py:25-30``)."""
    if table.ndim != 2:
        raise ValueError("table weights must be two-dimensional")
    _validate_rank(rank)
    _validate_sigma(sigma)
    return _ops.table_lookup(table, indices, key, -1, rank, sigma)


def perturbed_tied_logits(x: torch.Tensor, table: torch.Tensor, key: torch.Tensor, rank: int,
                          sigma: float) -> torch.Tensor:
    """``x @ T^T + s * (x @ B) @ A^T`` (``_candidate.py:33-38``)."""
    if table.ndim != 2 or x.shape[-1] != table.shape[1]:
        raise ValueError("logit input and [rows, cols] table shapes are incompatible")
    _validate_rank(rank)
    _validate_sigma(sigma)
    return _ops.tied_logits(x, table, key, -1, rank, sigma)


def perturbed_vector(vector: torch.Tensor, key: torch.Tensor, sigma: float) -> torch.Tensor:
    """``v + sigma * noise`` (``_candidate.py:41-45``)."""
    if vector.ndim != 1:
        raise ValueError("vector weights must be one-dimensional")
    _validate_sigma(sigma)
    return _ops.vector(vector, key, -1, sigma)


@dataclass(frozen=True, slots=True)
class CandidateContext:
    """Candidate-local manifest lookup and forward-op facade (``_candidate.py:48-87``)."""

    manifest: Manifest
    candidate_key: torch.Tensor
    rank: int
    sigma: float

    def key_for(self, path: ParameterPath) -> torch.Tensor:
        return group_key(self.candidate_key, self.manifest, self.manifest.entry(path).group)

    def _group(self, path: ParameterPath) -> int:
        return self.manifest.group_index(self.manifest.entry(path).group)

    def linear(self, params: ParameterTree, path: ParameterPath, x: torch.Tensor, *, activation: str | None = None,
               residual: torch.Tensor | None = None) -> torch.Tensor:
        """``x @ W + s (x @ A) @ B`` of the candidate (``_candidate.py:61-66``).

        Keyword additions to the reference's signature: ``activation="gelu"``
        returns ``zerograd_b200.gelu(y)`` and ``residual=r`` returns
        ``r + y`` (after the activation), with the roundings of those
        separate ops; on the tensor-core path for a per-candidate bf16
        input they run in the GEMM's epilogue, so the pre-activation output
        is never written."""
        entry = self.manifest.entry(path)
        if entry.layout is not ParameterLayout.MATRIX:
            raise ValueError(f"{'.'.join(path)} is not a matrix entry")
        weight = self.manifest.resolve(params, path)
        if weight.ndim != 2 or x.shape[-1] != weight.shape[0]:
            raise ValueError("linear input and [in, out] weight shapes are incompatible")
        return _ops.linear(x, weight, self.candidate_key, self._group(path), self.rank, self.sigma,
                           activation=activation, residual=residual)

    def table_lookup(self, params: ParameterTree, path: ParameterPath, indices: torch.Tensor) -> torch.Tensor:
        entry = self.manifest.entry(path)
        if entry.layout is not ParameterLayout.TABLE:
            raise ValueError(f"{'.'.join(path)} is not a table entry")
        table = self.manifest.resolve(params, path)
        if table.ndim != 2:
            raise ValueError("table weights must be two-dimensional")
        return _ops.table_lookup(table, indices, self.candidate_key, self._group(path), self.rank, self.sigma)

    def tied_logits(self, params: ParameterTree, path: ParameterPath, x: torch.Tensor) -> torch.Tensor:
        entry = self.manifest.entry(path)
        if entry.layout is not ParameterLayout.TABLE:
            raise ValueError(f"{'.'.join(path)} is not a table entry")
        table = self.manifest.resolve(params, path)
        if table.ndim != 2 or x.shape[-1] != table.shape[1]:
            raise ValueError("logit input and [rows, cols] table shapes are incompatible")
        return _ops.tied_logits(x, table, self.candidate_key, self._group(path), self.rank, self.sigma)

    def tied_logits_cross_entropy(self, params: ParameterTree, path: ParameterPath, x: torch.Tensor,
                                  labels: torch.Tensor, *, reduction: str = "none") -> torch.Tensor:
        """Per-row softmax cross-entropy of ``tied_logits(params, path, x)``
        against integer ``labels`` (float32, shape of x without its last axis),
        computed without materialising the [rows, vocabulary] logits: the
        logits are the bf16 values tied_logits returns, the log-sum-exp runs
        in float32.  ``reduction="mean"`` returns the mean over the rows
        (float64 accumulation in a fixed order, so a candidate's loss does not
        depend on how many candidates are evaluated with it).  An addition to
        the reference's context (which leaves the cross-entropy to the loss
        function); bf16 tables, rank 8 or 16."""
        entry = self.manifest.entry(path)
        if entry.layout is not ParameterLayout.TABLE:
            raise ValueError(f"{'.'.join(path)} is not a table entry")
        table = self.manifest.resolve(params, path)
        if table.ndim != 2 or x.shape[-1] != table.shape[1]:
            raise ValueError("logit input and [rows, cols] table shapes are incompatible")
        return _ops.tied_logits_ce(x, table, labels, self.candidate_key, self._group(path), self.rank, self.sigma,
                                   reduction)

    def int8_lut_linear(self, params: ParameterTree, path: ParameterPath, x: torch.Tensor, w_q: torch.Tensor,
                        w_scale: torch.Tensor, x_scale: float, y_scale: float, lut: torch.Tensor) -> torch.Tensor:
        """The candidate's integer linear with a 256-entry LUT activation (an
        addition to the reference's context; the reference only has float
        fake quantisation, ``examples/train_qat_xor.py:41-50``):

            acc = x @ w_q                          (int8 x int8 -> int32, exact)
            y   = acc * x_scale * w_scale[n] + s * (x @ A) @ B   (float32; x as integers)
            out = lut[clamp(rint(y / y_scale), -128, 127) + 128]          (int8)

        The low-rank term acts on the integer activations, so a
        perturbation of relative size ``sigma`` in the weights' units needs
        ``sigma`` scaled by ``x_scale``.

        ``path`` names the MATRIX entry whose factors (float32 draws) perturb
        the layer, and whose leaf (a float32 master weight, quantised per
        output channel into ``w_q``/``w_scale``, e.g. by
        :func:`zerograd_b200.quantize_int8_columns`) the replay updates.
        Under ``vmap`` over candidates it is one launch of the tcgen05
        ``kind::i8`` kernel for the population."""
        entry = self.manifest.entry(path)
        if entry.layout is not ParameterLayout.MATRIX:
            raise ValueError(f"{'.'.join(path)} is not a matrix entry")
        weight = self.manifest.resolve(params, path)
        if tuple(weight.shape) != tuple(w_q.shape) or x.shape[-1] != w_q.shape[0]:
            raise ValueError("int8 linear input, quantised weight and [in, out] leaf shapes are incompatible")
        return _ops.int8_lut_linear(x, w_q, w_scale, lut, self.candidate_key, self._group(path), self.rank, self.sigma,
                                    x_scale, y_scale)

    def vector(self, params: ParameterTree, path: ParameterPath) -> torch.Tensor:
        entry = self.manifest.entry(path)
        if entry.layout is not ParameterLayout.VECTOR:
            raise ValueError(f"{'.'.join(path)} is not a vector entry")
        v = self.manifest.resolve(params, path)
        if v.ndim != 1:
            raise ValueError("vector weights must be one-dimensional")
        return _ops.vector(v, self.candidate_key, self._group(path), self.sigma)

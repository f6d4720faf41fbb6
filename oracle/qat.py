"""CPU oracle of the integer QAT MLP workload's candidate forward.

TEST INFRASTRUCTURE ONLY (``tests/``, ``bench.py``'s CPU legs); the product
never imports it.

The reference has no integer path (only float fake quantisation,
``examples/train_qat_xor.py:41-50``); the semantics are this repository's:
float32 master weights quantised per output channel
(``quantize_int8_columns``), each layer ``ref.int8_lut_linear`` (exact int32
accumulation, the float32 low-rank term of the entry's float32 factors, rint,
clamp, 256-entry LUT), tanh LUTs between layers and an identity LUT on the
last, whose int8 output is dequantised for the mean-square loss.
"""
from __future__ import annotations

import numpy as np

from . import ref


def quantize_int8_columns(W: np.ndarray):
    """scale[n] = max_k |W[k, n]| / 127 in float32 (1 for a zero column);
    W_q = clip(rint(W / scale), -127, 127)."""
    W = np.asarray(W, np.float32)
    scale = (np.abs(W).max(axis=0) / np.float32(127.0)).astype(np.float32)
    scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    return np.clip(np.rint(W / scale), -127, 127).astype(np.int8), scale


def candidate_outputs(weights: list, ck: np.ndarray, x_q: np.ndarray, x_scale: float, y_scales: list,
                      luts: list, rank: int, sigma: float) -> np.ndarray:
    """The int8 outputs of the last layer for the candidate with key `ck`
    (entry i = weight i, its group index)."""
    s = ref.scaled_factor(rank, sigma, "float32")
    x = np.asarray(x_q, np.int8)
    xs = x_scale
    for i, W in enumerate(weights):
        wq, ws = quantize_int8_columns(W)
        A, Bf = ref.matrix_factors(ref.fold_in(ck, i), W.shape, rank, "float32")
        x, _ = ref.int8_lut_linear(x, wq, ws, xs, y_scales[i], luts[i], A, Bf, s)
        xs = 1.0 / 127.0
    return x

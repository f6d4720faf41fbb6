"""CPU oracle for the zerograd population-evaluation + factor-replay path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
module; it is used by ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py``, always as the checker.

It restates the reference's algorithm in numpy over the C oracle
(``oracle/zgref.c``, loaded with ctypes) that restates jax.random:

* keys          -- ``src/zerograd/_keys.py:20-58``
* factors       -- ``src/zerograd/_factors.py:30-74``
* forward ops   -- ``src/zerograd/_candidate.py:17-45``
* shaping       -- ``src/zerograd/_fitness.py:13-34``
* replay        -- ``src/zerograd/_replay.py:15-54``
* one step      -- ``src/zerograd/_optimizer.py:213-244,299-326`` with the
  optax 0.2.8 ``adamw``/``sgd`` update rules restated (optax is third-party
  code absent from the reference tree).

Floating-point forward/replay math runs in float64 unless noted, so the
oracle is at least as accurate as the reference's float32 path; tests
compare against it with the tolerances the reference's own tests use.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
import zlib

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libzgoracle.so")
_lib = None

MATRIX, TABLE, VECTOR = 0, 1, 2


def build() -> str:
    """Compile the C oracle in place with its Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        u32p = ctypes.POINTER(ctypes.c_uint32)
        f32p = ctypes.POINTER(ctypes.c_float)
        L.zgo_crc32.restype = ctypes.c_uint32
        L.zgo_crc32.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
        L.zgo_threefry2x32.argtypes = [ctypes.c_uint32] * 4 + [u32p]
        L.zgo_random_bits32.argtypes = [u32p, ctypes.c_int64, u32p]
        L.zgo_normal_f32.argtypes = [u32p, ctypes.c_int64, f32p]
        L.zgo_bits_to_normal.restype = ctypes.c_float
        L.zgo_bits_to_normal.argtypes = [ctypes.c_uint32]
        L.zgo_erfinv_f32.restype = ctypes.c_float
        L.zgo_erfinv_f32.argtypes = [ctypes.c_float]
        L.zgo_population_factors.argtypes = [u32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int64,
                                             ctypes.c_int64, ctypes.c_int, f32p, f32p]
        L.zgo_round_bf16.restype = ctypes.c_float
        L.zgo_round_bf16.argtypes = [ctypes.c_float]
        L.zgo_num_threads.restype = ctypes.c_int
        L.zgo_set_num_threads.argtypes = [ctypes.c_int]
        i8p = ctypes.POINTER(ctypes.c_int8)
        L.zgo_int8_lut_linear.argtypes = [i8p, i8p, f32p, ctypes.c_float, ctypes.c_float, i8p,
                                          f32p, f32p, ctypes.c_int, ctypes.c_float,
                                          ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, i8p,
                                          ctypes.POINTER(ctypes.c_int32)]
        _lib = L
    return _lib


def _p(a, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct))


# --------------------------------------------------------------------------
# keys (src/zerograd/_keys.py)
# --------------------------------------------------------------------------

def crc32(data: bytes) -> int:
    return int(lib().zgo_crc32(data, len(data)))


def key(seed: int) -> np.ndarray:
    """jax.random.key(seed) for a seed that fits 32 bits: words [hi, lo]."""
    seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    return np.array([(seed >> 32) & 0xFFFFFFFF, seed & 0xFFFFFFFF], dtype=np.uint32)


def step_key(seed: int, run_id: str, generation: int, manifest_version: int) -> np.ndarray:
    """``_keys.py:29-30``: key(crc32("seed:run_id:version:generation"))."""
    payload = f"{seed}:{run_id}:{manifest_version}:{generation}".encode()
    c = zlib.crc32(payload) & 0xFFFFFFFF
    assert c == crc32(payload)
    return key(c)


def threefry(k: np.ndarray, c0: int, c1: int) -> np.ndarray:
    out = np.zeros(2, np.uint32)
    lib().zgo_threefry2x32(int(k[0]), int(k[1]), c0 & 0xFFFFFFFF, c1 & 0xFFFFFFFF, _p(out, ctypes.c_uint32))
    return out


def fold_in(k: np.ndarray, d: int) -> np.ndarray:
    return threefry(k, 0, int(d) & 0xFFFFFFFF)


def split(k: np.ndarray, n: int = 2) -> np.ndarray:
    return np.stack([threefry(k, i >> 32, i) for i in range(n)])


def candidate_key(base: np.ndarray, cid: int) -> np.ndarray:
    return fold_in(base, cid)


def group_key(ck: np.ndarray, n_entries: int, group_index: int) -> np.ndarray:
    """``_keys.py:56-58``: split(ck, n_entries)[group_index]."""
    return split(ck, n_entries)[group_index]


def random_bits(k: np.ndarray, n: int) -> np.ndarray:
    k = np.ascontiguousarray(k, np.uint32)
    out = np.zeros(n, np.uint32)
    lib().zgo_random_bits32(_p(k, ctypes.c_uint32), n, _p(out, ctypes.c_uint32))
    return out


def normal(k: np.ndarray, shape) -> np.ndarray:
    """jax.random.normal(k, shape, float32)."""
    n = int(np.prod(shape))
    k = np.ascontiguousarray(k, np.uint32)
    out = np.zeros(n, np.float32)
    lib().zgo_normal_f32(_p(k, ctypes.c_uint32), n, _p(out, ctypes.c_float))
    return out.reshape(shape)


def bits_to_normal(bits: np.ndarray) -> np.ndarray:
    f = lib().zgo_bits_to_normal
    return np.array([f(int(b)) for b in np.asarray(bits, np.uint32).ravel()], np.float32)


# --------------------------------------------------------------------------
# factors (src/zerograd/_factors.py)
# --------------------------------------------------------------------------

def round_bf16(a: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 -> float32 with round-to-nearest-even (uint32
    arithmetic: a finite value's carry runs into the exponent, up to inf)."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32)
    r = (u >> 16) & np.uint32(1)
    r += np.uint32(0x7FFF)
    r += u
    r &= np.uint32(0xFFFF0000)
    out = r.view(np.float32)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.nan
    return out


def cast(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "float32":
        return np.asarray(a, np.float32)
    if dtype == "bfloat16":
        return round_bf16(a)
    raise ValueError(dtype)


def scaled_factor(rank: int, sigma: float, dtype: str) -> float:
    """``_factors.py:30-40``: sigma/sqrt(rank) as a scalar of the weight dtype."""
    return float(cast(np.array([sigma / math.sqrt(rank)], np.float32), dtype)[0])


def matrix_factors(gk, shape, rank, dtype="float32"):
    ka, kb = split(gk)
    return cast(normal(ka, (shape[0], rank)), dtype), cast(normal(kb, (rank, shape[1])), dtype)


def table_factors(gk, shape, rank, dtype="float32"):
    ka, kb = split(gk)
    return cast(normal(ka, (shape[0], rank)), dtype), cast(normal(kb, (shape[1], rank)), dtype)


def vector_noise(gk, shape, dtype="float32"):
    return cast(normal(gk, (shape[0],)), dtype)


def candidate_keys(base: np.ndarray, ids) -> np.ndarray:
    return np.stack([fold_in(base, int(i)) for i in ids]).astype(np.uint32)


def group_keys(cks: np.ndarray, group_index: int) -> np.ndarray:
    return np.stack([fold_in(k, group_index) for k in cks]).astype(np.uint32)


def population_factors(gks: np.ndarray, layout: int, shape, rank: int, dtype="float32"):
    """Factors of every candidate (multi-threaded C), reference layouts + leading P."""
    gks = np.ascontiguousarray(gks, np.uint32)
    P = gks.shape[0]
    rows = shape[0]
    cols = shape[1] if layout != VECTOR else 1
    A = np.zeros((P, rows * (rank if layout != VECTOR else 1)), np.float32)
    B = np.zeros((P, cols * rank if layout != VECTOR else 1), np.float32)
    lib().zgo_population_factors(_p(gks, ctypes.c_uint32), P, layout, rows, cols, rank,
                                 _p(A, ctypes.c_float), _p(B, ctypes.c_float))
    if layout == VECTOR:
        return cast(A.reshape(P, rows), dtype), None
    if layout == MATRIX:
        return cast(A.reshape(P, rows, rank), dtype), cast(B.reshape(P, rank, cols), dtype)
    return cast(A.reshape(P, rows, rank), dtype), cast(B.reshape(P, cols, rank), dtype)


# --------------------------------------------------------------------------
# forward ops (src/zerograd/_candidate.py), float64 math
# --------------------------------------------------------------------------

def perturbed_linear(x, W, gk, rank, sigma, dtype="float32"):
    a, b = matrix_factors(gk, W.shape, rank, dtype)
    s = scaled_factor(rank, sigma, dtype)
    x = np.asarray(x, np.float64)
    return x @ np.asarray(W, np.float64) + s * ((x @ a) @ b)


def perturbed_table_lookup(T, idx, gk, rank, sigma, dtype="float32"):
    a, b = table_factors(gk, T.shape, rank, dtype)
    s = scaled_factor(rank, sigma, dtype)
    return np.asarray(T, np.float64)[idx] + s * np.einsum("...r,cr->...c", a[idx].astype(np.float64), b)


def perturbed_tied_logits(x, T, gk, rank, sigma, dtype="float32"):
    a, b = table_factors(gk, T.shape, rank, dtype)
    s = scaled_factor(rank, sigma, dtype)
    x = np.asarray(x, np.float64)
    return x @ np.asarray(T, np.float64).T + s * np.einsum("...c,cr,vr->...v", x, b, a)


def tied_logits_cross_entropy(x, T, gk, rank, sigma, labels, dtype="bfloat16"):
    """Per-row cross-entropy of the tied logits rounded to the leaf dtype
    (what tied_logits returns), log-sum-exp in float64."""
    logits = perturbed_tied_logits(x, T, gk, rank, sigma, dtype)
    logits = cast(logits, dtype).astype(np.float64)
    mx = logits.max(axis=-1, keepdims=True)
    lse = mx[..., 0] + np.log(np.exp(logits - mx).sum(axis=-1))
    lab = np.asarray(labels, np.int64)
    picked = np.take_along_axis(logits, lab[..., None], axis=-1)[..., 0]
    return lse - picked


def layer_norm(x, scale, bias=None, eps=1e-5):
    """``(x - mean) / sqrt(var + eps) * scale + bias`` over the last axis,
    biased variance, in float64 (``examples/train_vit_cifar10.py:76-79``)."""
    x = np.asarray(x, np.float64)
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    y = (x - mean) / np.sqrt(var + eps) * np.asarray(scale, np.float64)
    return y if bias is None else y + np.asarray(bias, np.float64)


def rms_norm(x, scale, eps=1e-6):
    """``x / sqrt(mean(x^2) + eps) * scale`` over the last axis, in float64."""
    x = np.asarray(x, np.float64)
    return x / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps) * np.asarray(scale, np.float64)


def attention(q, k, v, causal=False):
    """softmax(q kᵀ / sqrt(d)) v per head, in float64, as the reference's ViT
    block computes it (``examples/train_vit_cifar10.py:166-172``); q, k, v
    [..., S, H, D] (the projections' head-interleaved layout), output the same.
    `causal`: key j > query i masked (the decoder LM)."""
    q, k, v = (np.asarray(t, np.float64) for t in (q, k, v))
    qh, kh, vh = (np.swapaxes(t, -3, -2) for t in (q, k, v))      # [..., H, S, D]
    s = qh @ np.swapaxes(kh, -1, -2) / math.sqrt(q.shape[-1])
    if causal:
        S = s.shape[-1]
        s = np.where(np.triu(np.ones((S, S), bool), 1), -np.inf, s)
    s = s - s.max(axis=-1, keepdims=True)
    w = np.exp(s)
    w /= w.sum(axis=-1, keepdims=True)
    return np.swapaxes(w @ vh, -3, -2)


def perturbed_vector(v, gk, sigma, dtype="float32"):
    s = scaled_factor(1, sigma, dtype)
    return np.asarray(v, np.float64) + s * vector_noise(gk, v.shape, dtype)


# --------------------------------------------------------------------------
# shaping + replay (src/zerograd/_fitness.py, _replay.py)
# --------------------------------------------------------------------------

def shape_centered_loss(losses, sigma):
    """``-(l - mean(l)) / (P * sigma)`` in the loss dtype (``_fitness.py:33-34``).

    For float32 losses every step is float32 as in the traced computation:
    the mean rounded to float32 (here the correctly rounded mean), the
    centring subtraction in float32, and P * sigma formed as a Python float
    and rounded to float32 once at the division.
    """
    l = np.asarray(losses)
    if l.dtype == np.float32:
        mean = np.float32(l.astype(np.float64).mean())
        centered = (l - mean).astype(np.float32)
        return ((-centered) / np.float32(l.shape[0] * sigma)).astype(np.float32)
    l = l.astype(np.float64)
    return -(l - l.mean()) / (l.shape[0] * sigma)


def replay_entry(shape, layout, base, ids, shaped, rank, group_index, dtype="float32"):
    """Sum over candidates of shaped_p * A_p B_p / sqrt(rank) (float64)."""
    cks = candidate_keys(base, ids)
    gks = group_keys(cks, group_index)
    w = np.asarray(shaped, np.float64)
    if layout == VECTOR:
        n, _ = population_factors(gks, VECTOR, shape, 1, dtype)
        return (w[:, None] * n).sum(0) * scaled_factor(1, 1.0, dtype)
    A, B = population_factors(gks, layout, shape, rank, dtype)
    P = A.shape[0]
    # sum_p w_p A_p B_p as one [rows, P*r] x [P*r, cols] product (BLAS)
    wa = (A.astype(np.float64) * w[:, None, None]).transpose(1, 0, 2).reshape(shape[0], P * rank)
    sf = scaled_factor(rank, 1.0, dtype)
    if layout == MATRIX:
        bb = B.astype(np.float64).reshape(P * rank, shape[1])
    else:
        bb = B.astype(np.float64).transpose(0, 2, 1).reshape(P * rank, shape[1])
    return (wa @ bb) * sf


# --------------------------------------------------------------------------
# optax update rules (optax 0.2.8, restated)
# --------------------------------------------------------------------------

def adamw_init(params: dict) -> dict:
    return {"count": 0, "mu": {k: np.zeros_like(v, np.float32) for k, v in params.items()},
            "nu": {k: np.zeros_like(v, np.float32) for k, v in params.items()}}


def adamw_update(grads, state, params, lr, b1=0.9, b2=0.999, eps=1e-8, weight_decay=1e-4):
    """scale_by_adam -> add_decayed_weights -> scale(-lr), float32 op order."""
    f = np.float32
    count = state["count"] + 1
    bc1 = f(1) - f(b1) ** f(count)
    bc2 = f(1) - f(b2) ** f(count)
    new_p, mu_o, nu_o = {}, {}, {}
    for k, p in params.items():
        g = np.asarray(grads[k], np.float32)
        mu = f(1 - b1) * g + f(b1) * state["mu"][k]
        nu = f(1 - b2) * (g * g) + f(b2) * state["nu"][k]
        u = (mu / bc1) / (np.sqrt(nu / bc2) + f(eps))
        u = u + f(weight_decay) * np.asarray(p, np.float32)
        u = u * f(-lr)
        new_p[k] = np.asarray(p, np.float32) + u
        mu_o[k], nu_o[k] = mu, nu
    return new_p, {"count": count, "mu": mu_o, "nu": nu_o}


def sgd_update(grads, params, lr):
    return {k: np.asarray(p, np.float32) + np.float32(-lr) * np.asarray(grads[k], np.float32)
            for k, p in params.items()}


# --------------------------------------------------------------------------
# exact int8 GEMM + LUT (no reference counterpart; semantics defined here)
# --------------------------------------------------------------------------

def int8_lut_linear(x, W, w_scale, x_scale, y_scale, lut, A, Bf, s):
    x = np.ascontiguousarray(x, np.int8)
    W = np.ascontiguousarray(W, np.int8)
    w_scale = np.ascontiguousarray(w_scale, np.float32)
    lut = np.ascontiguousarray(lut, np.int8)
    A = np.ascontiguousarray(A, np.float32)
    Bf = np.ascontiguousarray(Bf, np.float32)
    M, K = x.shape
    N = W.shape[1]
    rank = A.shape[1]
    out = np.zeros((M, N), np.int8)
    acc = np.zeros((M, N), np.int32)
    i8 = ctypes.c_int8
    lib().zgo_int8_lut_linear(_p(x, i8), _p(W, i8), _p(w_scale, ctypes.c_float), x_scale, y_scale,
                              _p(lut, i8), _p(A, ctypes.c_float), _p(Bf, ctypes.c_float), rank, s,
                              M, K, N, _p(out, i8), _p(acc, ctypes.c_int32))
    return out, acc


def tanh_lut(scale: float = 32.0) -> np.ndarray:
    """256-entry int8 LUT of a tanh-shaped nonlinearity: lut[q+128] = round(127 tanh(q/scale))."""
    q = np.arange(-128, 128, dtype=np.float64)
    return np.rint(127.0 * np.tanh(q / scale)).astype(np.int8)

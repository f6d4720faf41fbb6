"""The oracle's transformer-block restatements (CPU, float64): properties
that pin them without a reference run."""
import numpy as np

from oracle import ref


def test_layer_norm_properties():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((4, 7, 96)) * 5 + 3
    y = ref.layer_norm(x, np.ones(96), np.zeros(96), eps=0.0)
    np.testing.assert_allclose(y.mean(-1), 0, atol=1e-12)
    np.testing.assert_allclose(y.var(-1), 1, rtol=1e-12)
    s, b = rng.standard_normal(96), rng.standard_normal(96)
    np.testing.assert_allclose(ref.layer_norm(x, s, b, eps=0.0), y * s + b, rtol=1e-12, atol=1e-12)


def test_rms_norm_properties():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 5, 64))
    y = ref.rms_norm(x, np.ones(64), eps=0.0)
    np.testing.assert_allclose((y * y).mean(-1), 1, rtol=1e-12)
    np.testing.assert_allclose(ref.rms_norm(2.5 * x, np.ones(64), eps=0.0), y, rtol=1e-12)


def test_attention_properties():
    rng = np.random.default_rng(2)
    Z, S, H, D = 2, 6, 3, 8
    v = rng.standard_normal((Z, S, H, D))
    k = np.broadcast_to(rng.standard_normal((Z, 1, H, D)), (Z, S, H, D))    # all keys equal
    q = rng.standard_normal((Z, S, H, D))
    o = ref.attention(q, k, v)
    np.testing.assert_allclose(o, np.broadcast_to(v.mean(axis=1, keepdims=True), o.shape), rtol=1e-12)
    oc = ref.attention(q, k, v, causal=True)
    np.testing.assert_allclose(oc[:, 0], v[:, 0], rtol=1e-12)                 # the first query sees one key
    np.testing.assert_allclose(oc[:, 2], v[:, :3].mean(axis=1), rtol=1e-12)   # equal keys: running mean

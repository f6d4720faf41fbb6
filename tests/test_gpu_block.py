"""Transformer-block ops (LayerNorm / RMSNorm with per-candidate scale and
bias, softmax attention) against the float64 oracle, and a ViT block of the
reference's shape run under vmap over candidates.

Tolerances: float32 outputs rtol/atol 1e-5 (norm) and 1e-4 (attention: the
float32 online softmax); bf16 outputs element-wise rel 2e-2 above a stated
floor (bf16_tol.assert_bf16_close: 1e-2 of the output scale for the norms; a
quarter of the values' scale for attention, whose bf16-rounded weights err by
~2^-9 of |v| whatever the output's size).
"""
import numpy as np
import pytest
import torch

import zerograd_b200 as zg
from zerograd_b200 import _block
from zerograd_b200 import _lib as L

from bf16_tol import assert_bf16_close

pytestmark = pytest.mark.gpu


def _np(t):
    return t.float().cpu().numpy().astype(np.float64)


def _close(got, want, dtype):
    if dtype == torch.float32:
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)
    else:
        assert_bf16_close(got, want)


@pytest.mark.parametrize("C", [64, 200, 384, 512, 768, 1536, 3000])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("x_batched,p_batched", [(True, True), (False, True), (True, False)])
def test_layer_norm_matches_oracle(cuda, oracle, C, dtype, x_batched, p_batched):
    P, M = 3, 37
    g = torch.Generator().manual_seed(C)
    x = (torch.randn((P, M, C) if x_batched else (M, C), generator=g) * 3 + 1).to(dtype).to(cuda)
    scale = (1 + 0.1 * torch.randn((P, C) if p_batched else (C,), generator=g)).to(dtype).to(cuda)
    bias = (0.1 * torch.randn((P, C) if p_batched else (C,), generator=g)).to(dtype).to(cuda)
    y = _block.launch_norm("layer", x, scale, bias, 1e-5, x_batched, p_batched, P)
    assert y.shape == (P, M, C)
    for p in range(P):
        xs = _np(x[p] if x_batched else x)
        want = oracle.layer_norm(xs, _np(scale[p] if p_batched else scale), _np(bias[p] if p_batched else bias))
        _close(_np(y[p]), want, dtype)


@pytest.mark.parametrize("C", [128, 768, 2048, 770])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rms_norm_matches_oracle(cuda, oracle, C, dtype):
    P, M = 4, 19
    g = torch.Generator().manual_seed(C + 1)
    x = torch.randn(P, M, C, generator=g).to(dtype).to(cuda)
    scale = (1 + 0.1 * torch.randn(P, C, generator=g)).to(dtype).to(cuda)
    y = _block.launch_norm("rms", x, scale, None, 1e-6, True, True, P)
    for p in range(P):
        _close(_np(y[p]), oracle.rms_norm(_np(x[p]), _np(scale[p])), dtype)


def test_norm_ops_under_vmap(cuda, oracle):
    """Per-candidate scale/bias with a shared or batched input, as ctx.vector
    returns them inside a loss function."""
    P, B, S, C = 5, 2, 9, 384
    g = torch.Generator().manual_seed(0)
    x = torch.randn(B, S, C, generator=g).to(torch.bfloat16).to(cuda)
    xs = torch.randn(P, B, S, C, generator=g).to(torch.bfloat16).to(cuda)
    sc = (1 + 0.1 * torch.randn(P, C, generator=g)).to(torch.bfloat16).to(cuda)
    bi = (0.1 * torch.randn(P, C, generator=g)).to(torch.bfloat16).to(cuda)
    shared = torch.func.vmap(lambda s, b: zg.layer_norm(x, s, b))(sc, bi)
    batched = torch.func.vmap(lambda xx, s: zg.rms_norm(xx, s))(xs, sc)
    for p in range(P):
        assert_bf16_close(_np(shared[p]), oracle.layer_norm(_np(x), _np(sc[p]), _np(bi[p])), what=f"ln {p}")
        assert_bf16_close(_np(batched[p]), oracle.rms_norm(_np(xs[p]), _np(sc[p])), what=f"rms {p}")


@pytest.mark.parametrize("Z,S,H,D,causal,dtype,path", [
    (6, 65, 6, 64, False, torch.bfloat16, "attention"),        # ViT-small: 64 patches + CLS, head dim 64
    (4, 256, 2, 64, True, torch.bfloat16, "attention"),        # decoder LM: seq 256, causal
    (3, 100, 3, 64, True, torch.bfloat16, "attention"),        # ragged causal
    (2, 128, 4, 64, False, torch.bfloat16, "attention"),
    (300, 65, 6, 64, False, torch.bfloat16, "attention"),      # 1800 (z, head) units: many per CTA, one tile each
    (200, 200, 3, 64, True, torch.bfloat16, "attention"),      # 600 units of two tiles, ragged causal
    (5, 65, 4, 16, False, torch.bfloat16, "attention_simt"),   # the reference example's head dim 16
    (3, 50, 2, 64, True, torch.float32, "attention_simt"),
    (2, 300, 2, 64, True, torch.bfloat16, "attention_simt"),   # longer than one score row in TMEM
])
def test_attention_matches_oracle(cuda, oracle, Z, S, H, D, causal, dtype, path):
    g = torch.Generator().manual_seed(Z * S + H)
    q, k, v = (torch.randn(Z, S, H, D, generator=g).to(dtype).to(cuda) for _ in range(3))
    L.profile_begin()
    o = _block.launch_attention(q, k, v, causal)
    prof = L.profile_end()
    assert path in prof, prof
    assert L.load().zg_device_error(1) == 0
    want = oracle.attention(_np(q), _np(k), _np(v), causal)
    if dtype == torch.float32:
        np.testing.assert_allclose(_np(o), want, rtol=1e-4, atol=1e-4)
    else:
        # floor: a quarter of the values' unit scale (see test_attention_lm_size)
        assert_bf16_close(_np(o), want, floor=0.25)


def test_attention_large_scores(cuda, oracle):
    """Scores far from zero (the running max keeps exp2 in range)."""
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(2, 200, 2, 64, generator=g) * 4 for _ in range(3))
    o = _block.launch_attention(*(t.to(torch.bfloat16).to(cuda) for t in (q, k, v)), True)
    want = oracle.attention(*(t.to(torch.bfloat16).double().numpy() for t in (q, k, v)), True)
    assert torch.isfinite(o).all()
    # values of scale 4: the floor a quarter of that
    assert_bf16_close(_np(o), want, floor=1.0)


def _oracle_block_loss(ref, params, ck, x, r, sigma, heads):
    """The block below for the candidate with key `ck`, restated over the
    oracle's perturbed ops in float64 with the CUDA path's bf16 roundings
    (each op's output rounded to bf16), then the mean of squares."""
    from oracle import lm as olm

    s = ref.scaled_factor(r, sigma, "bfloat16")

    def bf(a):
        return ref.round_bf16(np.asarray(a, np.float32)).astype(np.float64)

    def lin(name, gi, h, act=None, residual=None):
        W = params[name]
        a, b = ref.matrix_factors(ref.fold_in(ck, gi), W.shape, r, "bfloat16")
        u = bf(s * (h @ a.astype(np.float64)))
        y = bf(h @ W + u @ b.astype(np.float64))
        if act == "gelu":
            y = bf(olm.gelu_tanh(y))
        return y if residual is None else bf(residual + y)

    B, T, E = x.shape
    sc = bf(ref.perturbed_vector(params["ln_s"], ref.fold_in(ck, 0), sigma, "bfloat16"))
    bi = bf(ref.perturbed_vector(params["ln_b"], ref.fold_in(ck, 1), sigma, "bfloat16"))
    h = bf(ref.layer_norm(x, sc, bi))
    q, k, v = (lin(n, 2 + i, h).reshape(B, T, heads, E // heads) for i, n in enumerate(("q", "k", "v")))
    a = bf(ref.attention(q, k, v)).reshape(B, T, E)
    x1 = lin("o", 5, a, residual=x)
    m = lin("mlp1", 6, x1, act="gelu")
    out = lin("mlp2", 7, m, residual=x1)
    return float(np.mean(out ** 2))


def test_vit_block_under_vmap(cuda, oracle):
    """One pre-norm transformer block of the reference's ViT shape (LayerNorm
    with perturbed scale/bias, perturbed q/k/v/o and MLP projections, softmax
    attention, tanh-form GELU, residuals), every candidate at once under
    vmap, against the oracle's restatement of the same block candidate by
    candidate (losses within 5e-3 relative: bf16 activations, float32
    accumulation)."""
    P, r, sigma, B, T, E, Hh = 6, 8, 0.02, 2, 65, 128, 2
    names = ["q", "k", "v", "o", "mlp1", "mlp2"]
    entries = [zg.ManifestEntry(("ln", "scale"), zg.ParameterLayout.VECTOR, "ln_s"),
               zg.ManifestEntry(("ln", "bias"), zg.ParameterLayout.VECTOR, "ln_b")]
    entries += [zg.ManifestEntry((n,), zg.ParameterLayout.MATRIX, n) for n in names]
    manifest = zg.Manifest(1, tuple(entries))
    g = torch.Generator().manual_seed(1)
    dims = {"q": (E, E), "k": (E, E), "v": (E, E), "o": (E, E), "mlp1": (E, 2 * E), "mlp2": (2 * E, E)}
    params = {n: (torch.randn(*dims[n], generator=g) * 0.05).to(torch.bfloat16).to(cuda) for n in names}
    params["ln"] = {"scale": (1 + 0.1 * torch.randn(E, generator=g)).to(torch.bfloat16).to(cuda),
                    "bias": (0.1 * torch.randn(E, generator=g)).to(torch.bfloat16).to(cuda)}
    x = torch.randn(B, T, E, generator=g).to(torch.bfloat16).to(cuda)

    def loss_fn(p, ctx, batch, rng):
        h = zg.layer_norm(batch, ctx.vector(p, ("ln", "scale")), ctx.vector(p, ("ln", "bias")))
        q, k, v = (ctx.linear(p, (n,), h).reshape(B, T, Hh, E // Hh) for n in ("q", "k", "v"))
        a = zg.attention(q, k, v).reshape(B, T, E)
        x1 = ctx.linear(p, ("o",), a, residual=batch)
        m = ctx.linear(p, ("mlp1",), x1, activation="gelu")
        out = ctx.linear(p, ("mlp2",), m, residual=x1)
        return (out.float() ** 2).mean(), None

    opt = zg.ZeroGrad(manifest, zg.sgd(0.01), P, r, sigma, 0, "vit-block")
    L.profile_begin()
    batched = opt.evaluate_shard(params, 0, loss_fn, x, range(P))
    prof = L.profile_end()
    assert "attention" in prof and "layer_norm" in prof, prof
    assert torch.isfinite(batched).all()
    pn = {n: _np(params[n]) for n in names}
    pn["ln_s"], pn["ln_b"] = _np(params["ln"]["scale"]), _np(params["ln"]["bias"])
    cks = oracle.candidate_keys(oracle.step_key(0, "vit-block", 0, 1), range(P))
    want = [_oracle_block_loss(oracle, pn, cks[i], _np(x), r, sigma, Hh) for i in range(P)]
    np.testing.assert_allclose(batched.cpu().numpy(), np.array(want), rtol=5e-3)
    assert L.load().zg_device_error(1) == 0


def test_attention_lm_size(cuda, oracle):
    """The decoder LM's attention for 16 candidates x 16 sequences (256
    tokens, 12 heads of 64, causal); the first and last z against the oracle."""
    Z, S, H, D = 256, 256, 12, 64
    g = torch.Generator(device=cuda).manual_seed(11)
    q, k, v = (torch.randn(Z, S, H, D, generator=g, device=cuda).to(torch.bfloat16) for _ in range(3))
    o = _block.launch_attention(q, k, v, True)
    assert L.load().zg_device_error(1) == 0
    for z in (0, Z - 1):
        want = oracle.attention(_np(q[z]), _np(k[z]), _np(v[z]), True)
        # floor: a quarter of the values' unit scale (the bf16-rounded softmax
        # weights err by ~2^-9 of |v|, whatever the output's size)
        assert_bf16_close(_np(o[z]), want, floor=0.25, what=f"z {z}")


def test_rms_norm_lm_size(cuda, oracle):
    """RMSNorm of 16 candidates' hidden states [16, 4096, 768] with their own
    scales; rows of the first and last candidate against the oracle."""
    P, M, C = 16, 4096, 768
    g = torch.Generator(device=cuda).manual_seed(12)
    x = torch.randn(P, M, C, generator=g, device=cuda).to(torch.bfloat16)
    sc = (1 + 0.1 * torch.randn(P, C, generator=g, device=cuda)).to(torch.bfloat16)
    y = _block.launch_norm("rms", x, sc, None, 1e-6, True, True, P)
    for p in (0, P - 1):
        assert_bf16_close(_np(y[p, :64]), oracle.rms_norm(_np(x[p, :64]), _np(sc[p])), what=f"candidate {p}")

"""Transformer-block ops (LayerNorm / RMSNorm with per-candidate scale and
bias, softmax attention) against the float64 oracle, and a ViT block of the
reference's shape run under vmap over candidates.

Tolerances: float32 outputs rtol/atol 1e-5 (norm) and 1e-4 (attention: the
float32 online softmax); bf16 outputs 2e-2 (one bf16 step is 2^-8 relative,
and attention's weights are rounded to bf16 before P V).
"""
import numpy as np
import pytest
import torch

import zerograd_b200 as zg
from zerograd_b200 import _block
from zerograd_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _np(t):
    return t.float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("C", [64, 384, 768, 1536, 3000])
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
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    for p in range(P):
        xs = _np(x[p] if x_batched else x)
        want = oracle.layer_norm(xs, _np(scale[p] if p_batched else scale), _np(bias[p] if p_batched else bias))
        np.testing.assert_allclose(_np(y[p]), want, rtol=tol, atol=tol)


@pytest.mark.parametrize("C", [128, 768, 2048, 770])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rms_norm_matches_oracle(cuda, oracle, C, dtype):
    P, M = 4, 19
    g = torch.Generator().manual_seed(C + 1)
    x = torch.randn(P, M, C, generator=g).to(dtype).to(cuda)
    scale = (1 + 0.1 * torch.randn(P, C, generator=g)).to(dtype).to(cuda)
    y = _block.launch_norm("rms", x, scale, None, 1e-6, True, True, P)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    for p in range(P):
        np.testing.assert_allclose(_np(y[p]), oracle.rms_norm(_np(x[p]), _np(scale[p])), rtol=tol, atol=tol)


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
        np.testing.assert_allclose(_np(shared[p]), oracle.layer_norm(_np(x), _np(sc[p]), _np(bi[p])), rtol=2e-2,
                                   atol=2e-2)
        np.testing.assert_allclose(_np(batched[p]), oracle.rms_norm(_np(xs[p]), _np(sc[p])), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("Z,S,H,D,causal,dtype,path", [
    (6, 65, 6, 64, False, torch.bfloat16, "attention"),        # ViT-small: 64 patches + CLS, head dim 64
    (4, 256, 2, 64, True, torch.bfloat16, "attention"),        # decoder LM: seq 256, causal
    (3, 100, 3, 64, True, torch.bfloat16, "attention"),        # ragged causal
    (2, 128, 4, 64, False, torch.bfloat16, "attention"),
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
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    np.testing.assert_allclose(_np(o), want, rtol=tol, atol=tol)


def test_attention_large_scores(cuda, oracle):
    """Scores far from zero (the running max keeps exp2 in range)."""
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(2, 200, 2, 64, generator=g) * 4 for _ in range(3))
    o = _block.launch_attention(*(t.to(torch.bfloat16).to(cuda) for t in (q, k, v)), True)
    want = oracle.attention(*(t.to(torch.bfloat16).double().numpy() for t in (q, k, v)), True)
    assert torch.isfinite(o).all()
    np.testing.assert_allclose(_np(o), want, rtol=3e-2, atol=3e-2)


def test_vit_block_under_vmap(cuda):
    """One pre-norm transformer block of the reference's ViT shape (LayerNorm
    with perturbed scale/bias, perturbed q/k/v/o and MLP projections, softmax
    attention, residuals), every candidate at once under vmap, against the
    same loss evaluated candidate by candidate."""
    P, r, sigma, B, T, E, Hh = 6, 8, 0.02, 2, 65, 128, 2
    names = ["q", "k", "v", "o", "mlp1", "mlp2"]
    entries = [zg.ManifestEntry(("ln", "scale"), zg.ParameterLayout.VECTOR, "ln_s"),
               zg.ManifestEntry(("ln", "bias"), zg.ParameterLayout.VECTOR, "ln_b")]
    entries += [zg.ManifestEntry((n,), zg.ParameterLayout.MATRIX, n) for n in names]
    manifest = zg.Manifest(1, tuple(entries))
    g = torch.Generator().manual_seed(1)
    dims = {"q": (E, E), "k": (E, E), "v": (E, E), "o": (E, E), "mlp1": (E, 2 * E), "mlp2": (2 * E, E)}
    params = {n: (torch.randn(*dims[n], generator=g) * 0.05).to(torch.bfloat16).to(cuda) for n in names}
    params["ln"] = {"scale": torch.ones(E, dtype=torch.bfloat16, device=cuda),
                    "bias": torch.zeros(E, dtype=torch.bfloat16, device=cuda)}
    x = torch.randn(B, T, E, generator=g).to(torch.bfloat16).to(cuda)

    def loss_fn(p, ctx, batch, rng):
        h = zg.layer_norm(batch, ctx.vector(p, ("ln", "scale")), ctx.vector(p, ("ln", "bias")))
        q, k, v = (ctx.linear(p, (n,), h).reshape(B, T, Hh, E // Hh) for n in ("q", "k", "v"))
        a = zg.attention(q, k, v).reshape(B, T, E)
        x1 = batch + ctx.linear(p, ("o",), a)
        m = torch.nn.functional.gelu(ctx.linear(p, ("mlp1",), x1).float()).to(torch.bfloat16)
        out = x1 + ctx.linear(p, ("mlp2",), m)
        return (out.float() ** 2).mean(), None

    opt = zg.ZeroGrad(manifest, zg.sgd(0.01), P, r, sigma, 0, "vit-block")
    L.profile_begin()
    batched = opt.evaluate_shard(params, 0, loss_fn, x, range(P))
    prof = L.profile_end()
    assert "attention" in prof and "layer_norm" in prof, prof
    base = opt.base_key(0)
    from zerograd_b200._candidate import CandidateContext
    from zerograd_b200._replay import candidate_keys
    cks = candidate_keys(base, torch.arange(P, dtype=torch.int32, device=cuda))
    single = torch.stack([loss_fn(params, CandidateContext(manifest, cks[i], r, sigma), x, None)[0]
                          for i in range(P)])
    assert torch.isfinite(batched).all()
    np.testing.assert_allclose(batched.cpu().numpy(), single.cpu().numpy(), rtol=2e-2, atol=1e-3)
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
        np.testing.assert_allclose(_np(o[z]), want, rtol=2e-2, atol=2e-2)


def test_rms_norm_lm_size(cuda, oracle):
    """RMSNorm of 16 candidates' hidden states [16, 4096, 768] with their own
    scales; rows of the first and last candidate against the oracle."""
    P, M, C = 16, 4096, 768
    g = torch.Generator(device=cuda).manual_seed(12)
    x = torch.randn(P, M, C, generator=g, device=cuda).to(torch.bfloat16)
    sc = (1 + 0.1 * torch.randn(P, C, generator=g, device=cuda)).to(torch.bfloat16)
    y = _block.launch_norm("rms", x, sc, None, 1e-6, True, True, P)
    for p in (0, P - 1):
        np.testing.assert_allclose(_np(y[p, :64]), oracle.rms_norm(_np(x[p, :64]), _np(sc[p])), rtol=2e-2, atol=2e-2)

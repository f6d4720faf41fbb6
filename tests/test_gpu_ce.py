"""Tied logits fused with softmax cross-entropy.

loss[p, m] = logsumexp(logits_p[m]) - logits_p[m, label[m]] with logits_p
the bf16 tied logits of candidate p, never materialised.  Against the oracle
(float64 log-sum-exp over the oracle's logits rounded to bf16): rtol 1e-2,
atol 3e-2 (a logit can land one bf16 step away from the oracle's, which moves
the loss by at most that step); against the unfused path (tied_logits, then a
float32 cross-entropy), whose float32 accumulation order differs: at most one
bf16 step of a logit below 16 (1/16) per row, and 2e-3 on average.
"""
import numpy as np
import pytest
import torch

import zerograd_b200 as zg
from zerograd_b200 import _lib as L
from zerograd_b200 import _ops

pytestmark = pytest.mark.gpu


def _u32(a, dev):
    return torch.tensor(np.asarray(a, np.int64)).to(torch.uint32).to(dev)


@pytest.mark.parametrize("P,M,V,C,r,x_batched", [(6, 300, 1000, 256, 8, True),    # ragged rows and vocabulary
                                                  (4, 64, 600, 128, 16, False),   # shared input, rank 16
                                                  (3, 512, 4096, 512, 8, True),   # whole 256-blocks
                                                  (1, 100, 200, 128, 8, False)])  # one tile: one range
def test_tied_ce_matches_oracle(cuda, oracle, P, M, V, C, r, x_batched):
    sigma, group = 0.05, 1
    cks = oracle.candidate_keys(oracle.step_key(2, "ce", 0, 1), range(P))
    g = torch.Generator().manual_seed(P + M + V)
    T = (torch.randn(V, C, generator=g) * 0.1).to(torch.bfloat16).to(cuda)
    x = (torch.randn((P, M, C) if x_batched else (M, C), generator=g)).to(torch.bfloat16).to(cuda)
    labels = torch.randint(0, V, (M,), generator=g).to(cuda)
    L.profile_begin()
    loss = _ops.launch_tied_logits_ce(x, T, labels, _u32(cks, cuda), group, r, sigma, x_batched)
    prof = L.profile_end()
    assert L.load().zg_device_error(1) == 0
    assert "tied_ce" in prof, prof
    xs = x.float().cpu().numpy().astype(np.float64)
    Ts = T.float().cpu().numpy().astype(np.float64)
    lab = labels.cpu().numpy()
    for p in range(P):
        want = oracle.tied_logits_cross_entropy(xs[p] if x_batched else xs, Ts, oracle.fold_in(cks[p], group), r,
                                                sigma, lab)
        np.testing.assert_allclose(loss[p].cpu().numpy(), want, rtol=1e-2, atol=3e-2)


def test_tied_ce_matches_unfused_and_flags_bad_labels(cuda, oracle):
    P, M, V, C, r = 5, 200, 777, 192, 8
    cks = _u32(oracle.candidate_keys(oracle.step_key(4, "ce2", 0, 1), range(P)), cuda)
    g = torch.Generator().manual_seed(4)
    T = (torch.randn(V, C, generator=g) * 0.1).to(torch.bfloat16).to(cuda)
    x = torch.randn(P, M, C, generator=g).to(torch.bfloat16).to(cuda)
    labels = torch.randint(0, V, (M,), generator=g).to(cuda)
    fused = _ops.launch_tied_logits_ce(x, T, labels, cks, 0, r, 0.05, True)
    logits = _ops.launch_tied_logits(x, T, cks, 0, r, 0.05, True)                # [P, M, V] bf16
    ref = torch.nn.functional.cross_entropy(logits.float().reshape(P * M, V), labels.repeat(P),
                                            reduction="none").reshape(P, M)
    diff = (fused - ref).abs()
    assert diff.max().item() <= 1 / 16 and diff.mean().item() <= 2e-3
    bad = labels.clone()
    bad[3], bad[7] = -1, V
    out = _ops.launch_tied_logits_ce(x, T, bad, cks, 0, r, 0.05, True)
    assert torch.isnan(out[:, 3]).all() and torch.isnan(out[:, 7]).all()
    assert torch.isfinite(out[:, 0]).all()
    assert L.load().zg_device_error(1) == 0


def test_step_with_fused_cross_entropy(cuda):
    """A language-model-style loss through the context method under vmap."""
    P, r, B, S, C, V = 16, 8, 2, 96, 128, 500
    manifest = zg.Manifest(1, (zg.ManifestEntry(("emb",), zg.ParameterLayout.TABLE, "emb"),
                               zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w")))
    g = torch.Generator().manual_seed(8)
    params = {"emb": (torch.randn(V, C, generator=g) * 0.1).to(torch.bfloat16).to(cuda),
              "w": (torch.randn(C, C, generator=g) * 0.05).to(torch.bfloat16).to(cuda)}
    tokens = torch.randint(0, V, (B, S + 1), generator=g).to(cuda)

    def loss_fn(p, ctx, batch, rng):
        h = ctx.table_lookup(p, ("emb",), batch[:, :-1])
        h = torch.tanh(ctx.linear(p, ("w",), h).float()).to(torch.bfloat16)
        return ctx.tied_logits_cross_entropy(p, ("emb",), h, batch[:, 1:]).mean(), None

    def loss_unfused(p, ctx, batch, rng):
        h = ctx.table_lookup(p, ("emb",), batch[:, :-1])
        h = torch.tanh(ctx.linear(p, ("w",), h).float()).to(torch.bfloat16)
        logits = ctx.tied_logits(p, ("emb",), h).float()
        return torch.nn.functional.cross_entropy(logits.reshape(-1, V), batch[:, 1:].reshape(-1)), None

    opt = zg.ZeroGrad(manifest, zg.sgd(0.1), P, r, 0.02, 0, "lm-ce")
    a = opt.evaluate_shard(params, 0, loss_fn, tokens, torch.arange(P, device=cuda))
    b = opt.evaluate_shard(params, 0, loss_unfused, tokens, torch.arange(P, device=cuda))
    assert torch.isfinite(a).all()
    assert (a - b).abs().max().item() <= 2e-2
    state = opt.init(params)
    new, _, m = opt.step(state, params, tokens, loss_fn)
    assert np.isfinite(m.mean_loss)
    assert L.load().zg_device_error(1) == 0


def test_tied_ce_lm_slice(cuda, oracle):
    """The decoder LM's output layer (V=32000, C=768, 4096 tokens, rank 16)
    for 16 candidates with their own hidden states; rows 0..7 of candidates 0
    and 15 against the oracle."""
    P, M, V, C, r, sigma = 16, 4096, 32000, 768, 16, 0.01
    cks = oracle.candidate_keys(oracle.step_key(0, "lm", 0, 1), range(P))
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(P, M, C, generator=g, device=cuda).to(torch.bfloat16)
    T = (torch.randn(V, C, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    labels = torch.randint(0, V, (M,), generator=g, device=cuda)
    loss = _ops.launch_tied_logits_ce(x, T, labels, _u32(cks, cuda), 0, r, sigma, True)
    assert L.load().zg_device_error(1) == 0
    Ts = T.float().cpu().numpy().astype(np.float64)
    lab = labels.cpu().numpy()[:8]
    for p in (0, 15):
        xs = x[p, :8].float().cpu().numpy().astype(np.float64)
        want = oracle.tied_logits_cross_entropy(xs, Ts, oracle.fold_in(cks[p], 0), r, sigma, lab)
        np.testing.assert_allclose(loss[p, :8].cpu().numpy(), want, rtol=1e-2, atol=3e-2)
    assert torch.isfinite(loss).all()

"""ZeroGrad lifecycle on the GPU against the oracle and the reference's
relational tests (tests/test_replay_and_optimizer.py, test_coverage_gaps.py,
test_optimizer_validation.py, test_issue_regressions.py of the reference).

Workload of the first config: MLP 784->256->10 float32 (ReLU), population 64,
rank 8, sigma 0.01, adamw 3e-4, MATRIX weights and VECTOR biases, batch 128
of N(0,1) inputs with labels uniform over 0..9, cross-entropy, seed 0.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import zerograd_b200 as zg

pytestmark = pytest.mark.gpu

MANIFEST = zg.Manifest(1, (
    zg.ManifestEntry(("w1",), zg.ParameterLayout.MATRIX, "w1"),
    zg.ManifestEntry(("b1",), zg.ParameterLayout.VECTOR, "b1"),
    zg.ManifestEntry(("w2",), zg.ParameterLayout.MATRIX, "w2"),
    zg.ManifestEntry(("b2",), zg.ParameterLayout.VECTOR, "b2"),
))


def mlp_params(dev, din=784, dh=256, dout=10, seed=0):
    g = torch.Generator().manual_seed(seed)
    return {"w1": (torch.randn(din, dh, generator=g) * (2.0 / din) ** 0.5).to(dev),
            "b1": torch.zeros(dh).to(dev),
            "w2": (torch.randn(dh, dout, generator=g) * (2.0 / dh) ** 0.5).to(dev),
            "b2": torch.zeros(dout).to(dev)}


def mlp_batch(dev, B=128, din=784, seed=0):
    g = torch.Generator().manual_seed(seed + 1)
    return torch.randn(B, din, generator=g).to(dev), torch.randint(0, 10, (B,), generator=g).to(dev)


def mlp_loss(params, ctx, batch, rng):
    x, y = batch
    h = torch.relu(ctx.linear(params, ("w1",), x) + ctx.vector(params, ("b1",)))
    logits = ctx.linear(params, ("w2",), h) + ctx.vector(params, ("b2",))
    return F.cross_entropy(logits, y), None


def oracle_mlp_losses(oracle, params, batch, P, rank, sigma, seed, run_id, gen):
    x, y = (t.cpu().numpy() for t in batch)
    p = {k: v.cpu().numpy() for k, v in params.items()}
    base = oracle.step_key(seed, run_id, gen, 1)
    out = []
    for c in range(P):
        ck = oracle.candidate_key(base, c)
        gk = [oracle.fold_in(ck, g) for g in range(4)]
        h = oracle.perturbed_linear(x, p["w1"], gk[0], rank, sigma) + oracle.perturbed_vector(p["b1"], gk[1], sigma)
        h = np.maximum(h, 0)
        lg = oracle.perturbed_linear(h, p["w2"], gk[2], rank, sigma) + oracle.perturbed_vector(p["b2"], gk[3], sigma)
        lg = lg - lg.max(1, keepdims=True)
        lse = np.log(np.exp(lg).sum(1))
        out.append(float(np.mean(lse - lg[np.arange(len(y)), y])))
    return np.array(out)


def oracle_step(oracle, params, losses, P, rank, sigma, seed, run_id, gen, transform):
    base = oracle.step_key(seed, run_id, gen, 1)
    shaped = oracle.shape_centered_loss(losses.astype(np.float32), sigma)
    grads = {}
    layouts = {"w1": 0, "b1": 2, "w2": 0, "b2": 2}
    for g, name in enumerate(["w1", "b1", "w2", "b2"]):
        r = rank if layouts[name] != 2 else 1
        grads[name] = -oracle.replay_entry(params[name].shape, layouts[name], base, range(P), shaped, r, g)
    pn = {k: v.cpu().numpy() for k, v in params.items()}
    if transform[0] == "adamw":
        new, _ = oracle.adamw_update(grads, oracle.adamw_init(pn), pn, transform[1])
    else:
        new = oracle.sgd_update(grads, pn, transform[1])
    return new


def test_mlp_losses_match_oracle(cuda, oracle):
    params, batch = mlp_params(cuda), mlp_batch(cuda)
    opt = zg.ZeroGrad(MANIFEST, zg.adamw(3e-4), 64, 8, 0.01, 0, "mlp")
    losses = opt.evaluate_shard(params, 0, mlp_loss, batch, torch.arange(64, device=cuda))
    want = oracle_mlp_losses(oracle, params, batch, 64, 8, 0.01, 0, "mlp", 0)
    np.testing.assert_allclose(losses.cpu().numpy(), want, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("transform", [("sgd", 0.05), ("adamw", 3e-4)])
def test_mlp_step_from_losses_matches_oracle(cuda, oracle, transform):
    params, batch = mlp_params(cuda), mlp_batch(cuda)
    tf = zg.sgd(transform[1]) if transform[0] == "sgd" else zg.adamw(transform[1])
    opt = zg.ZeroGrad(MANIFEST, tf, 64, 8, 0.01, 0, "mlp")
    state = opt.init(params)
    losses = opt.evaluate_shard(params, 0, mlp_loss, batch, torch.arange(64, device=cuda))
    new, st, metrics = opt.step_from_losses(state, params, losses)
    want = oracle_step(oracle, params, losses.cpu().numpy(), 64, 8, 0.01, 0, "mlp", 0, transform)
    for k in params:
        got = new[k].cpu().numpy()
        if transform[0] == "sgd":
            np.testing.assert_allclose(got, want[k], rtol=1e-5, atol=1e-7)
        else:
            # adam's first step is lr * g/(|g|+eps): tolerance covers float32 vs float64 only;
            # a sign flip can only occur for |g| within rounding of zero
            bad = ~np.isclose(got, want[k], rtol=1e-5, atol=1e-7)
            assert bad.mean() < 1e-4, (k, bad.sum())
    assert st.generation == 1
    assert metrics.population_size == 64
    assert metrics.mean_loss == pytest.approx(float(losses.mean()), rel=1e-6)
    assert metrics.min_loss == float(losses.min()) and metrics.max_loss == float(losses.max())


def test_step_is_bit_identical_to_evaluate_plus_complete(cuda):
    params, batch = mlp_params(cuda), mlp_batch(cuda)
    opt = zg.ZeroGrad(MANIFEST, zg.adamw(3e-4), 16, 4, 0.01, 3, "bit")
    state = opt.init(params)
    a, sa, ma = opt.step(state, params, batch, mlp_loss)
    losses = opt.evaluate_shard(params, 0, mlp_loss, batch, torch.arange(16, device=cuda))
    b, sb, mb = opt.step_from_losses(state, params, losses)
    for k in params:
        assert torch.equal(a[k], b[k])
    assert ma == mb


def test_subset_evaluation_matches_full(cuda):
    params, batch = mlp_params(cuda), mlp_batch(cuda)
    opt = zg.ZeroGrad(MANIFEST, zg.sgd(0.1), 12, 4, 0.01, 0, "sub")
    full = opt.evaluate_shard(params, 0, mlp_loss, batch, torch.arange(12, device=cuda))
    sub = opt.evaluate_shard(params, 0, mlp_loss, batch, torch.tensor([2, 5, 11], device=cuda))
    np.testing.assert_allclose(sub.cpu().numpy(), full.cpu().numpy()[[2, 5, 11]], rtol=1e-6)


def test_identical_trajectories(cuda):
    outs = []
    for _ in range(2):
        params, batch = mlp_params(cuda), mlp_batch(cuda)
        opt = zg.ZeroGrad(MANIFEST, zg.adamw(1e-3), 8, 2, 0.02, 11, "traj")
        state = opt.init(params)
        for _ in range(3):
            params, state, _ = opt.step(state, params, batch, mlp_loss)
        outs.append(params)
    for k in outs[0]:
        assert torch.equal(outs[0][k], outs[1][k])


def test_equal_losses_sgd_is_noop(cuda):
    params = mlp_params(cuda)
    opt = zg.ZeroGrad(MANIFEST, zg.sgd(0.1), 8, 2, 0.1, 0, "eq")
    state = opt.init(params)
    new, _, _ = opt.step_from_losses(state, params, torch.full((8,), 1.5, device=cuda))
    for k in params:
        assert torch.equal(new[k], params[k])


def test_step_descends_quadratic(cuda):
    params = {"w": torch.ones(4, 4, device=cuda)}
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),))
    opt = zg.ZeroGrad(manifest, zg.sgd(0.05), 64, 4, 0.05, 0, "quad")
    state = opt.init(params)
    eye = torch.eye(4, device=cuda)

    def loss_fn(p, ctx, batch, rng):
        y = ctx.linear(p, ("w",), eye)
        return (y * y).sum(), None

    before = float((params["w"] ** 2).sum())
    for _ in range(5):
        params, state, _ = opt.step(state, params, None, loss_fn)
    assert float((params["w"] ** 2).sum()) < before


def test_non_manifest_leaf(cuda, oracle):
    params = {"w": torch.randn(6, 3, device=cuda), "frozen": torch.randn(5, device=cuda)}
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),))
    losses = torch.randn(8, device=cuda)
    sgd = zg.ZeroGrad(manifest, zg.sgd(0.1), 8, 2, 0.1, 0, "nm")
    new, _, _ = sgd.step_from_losses(sgd.init(params), params, losses)
    assert torch.equal(new["frozen"], params["frozen"])
    aw = zg.ZeroGrad(manifest, zg.adamw(0.1, weight_decay=0.5), 8, 2, 0.1, 0, "nm")
    new, _, _ = aw.step_from_losses(aw.init(params), params, losses)
    fr = params["frozen"].cpu().numpy()
    want, _ = oracle.adamw_update({"f": np.zeros_like(fr)}, oracle.adamw_init({"f": fr}), {"f": fr}, 0.1,
                                  weight_decay=0.5)
    np.testing.assert_allclose(new["frozen"].cpu().numpy(), want["f"], rtol=1e-6)


def test_nonfinite_losses_rejected_before_update(cuda):
    params = mlp_params(cuda)
    opt = zg.ZeroGrad(MANIFEST, zg.sgd(0.1), 4, 2, 0.1, 0, "nf")
    state = opt.init(params)
    with pytest.raises(ValueError):
        opt.step_from_losses(state, params, torch.tensor([1.0, float("nan"), 2.0, 3.0], device=cuda))


def test_per_candidate_rng_differs(cuda):
    params = {"w": torch.zeros(2, 2, device=cuda)}
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),))
    opt = zg.ZeroGrad(manifest, zg.sgd(0.1), 6, 1, 0.1, 0, "rng")

    def loss_fn(p, ctx, batch, rng):
        return zg.random.normal(rng, (1,))[0], None

    losses = opt.evaluate_shard(params, 0, loss_fn, None, torch.arange(6, device=cuda))
    assert len(set(losses.cpu().tolist())) == 6


def test_bf16_mlp_step_runs_close_to_oracle(cuda, oracle):
    params = {k: v.to(torch.bfloat16) for k, v in mlp_params(cuda, 64, 32, 10).items()}
    g = torch.Generator().manual_seed(5)
    batch = (torch.randn(16, 64, generator=g).to(torch.bfloat16).to(cuda), torch.randint(0, 10, (16,), generator=g).to(cuda))
    opt = zg.ZeroGrad(MANIFEST, zg.adamw(1e-3), 8, 4, 0.01, 0, "bf16")
    state = opt.init(params)
    new, _, _ = opt.step(state, params, batch, lambda p, c, b, r: (mlp_loss(p, c, b, r)[0].float(), None))
    for k in params:
        assert new[k].dtype == torch.bfloat16
        assert torch.isfinite(new[k].float()).all()
        # every entry moved by about lr (adam's first step) or less
        assert float((new[k].float() - params[k].float()).abs().max()) < 2e-2


def test_distributed_threads_match_single_device(cuda):
    params, batch = mlp_params(cuda), mlp_batch(cuda)
    opt = zg.ZeroGrad(MANIFEST, zg.adamw(3e-4), 7, 2, 0.01, 0, "dist")
    state = opt.init(params)
    single, _, ms = opt.step(state, params, batch, mlp_loss)
    with zg.DistributedZeroGrad(opt, [cuda, cuda], mlp_loss, weights=[1, 3]) as d:
        assert d.partition_sizes == [2, 5]
        multi, _, md = d.step(state, params, batch)
    for k in params:
        np.testing.assert_allclose(multi[k].cpu().numpy(), single[k].cpu().numpy(), rtol=1e-5, atol=1e-7)
    assert md.mean_loss == pytest.approx(ms.mean_loss, rel=1e-6)

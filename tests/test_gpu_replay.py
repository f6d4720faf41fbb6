"""Replay and shaping against the oracle (reference tests/test_replay_and_optimizer.py:43-99)."""
import numpy as np
import pytest
import torch

import zerograd_b200 as zg
from zerograd_b200 import _ops

pytestmark = pytest.mark.gpu


def _u32(a, dev):
    return torch.tensor(np.asarray(a, np.int64)).to(torch.uint32).to(dev)


def _params(dev, dtype=torch.float32):
    g = torch.Generator().manual_seed(0)
    return {"linear": {"weight": torch.randn(8, 4, generator=g).to(dtype).to(dev)},
            "table": {"embed": torch.randn(16, 4, generator=g).to(dtype).to(dev)},
            "vector": {"scale": torch.randn(4, generator=g).to(dtype).to(dev)}}


def _manifest():
    return zg.Manifest(1, (zg.ManifestEntry(("linear", "weight"), zg.ParameterLayout.MATRIX, "linear"),
                           zg.ManifestEntry(("table", "embed"), zg.ParameterLayout.TABLE, "embed"),
                           zg.ManifestEntry(("vector", "scale"), zg.ParameterLayout.VECTOR, "scale")))


@pytest.mark.parametrize("path,layout,shape,group", [
    (("linear", "weight"), 0, (8, 4), 0), (("table", "embed"), 1, (16, 4), 1), (("vector", "scale"), 2, (4,), 2)])
def test_replay_entry_matches_reference_test(cuda, oracle, path, layout, shape, group):
    params, manifest = _params(cuda), _manifest()
    pop, rank, sigma = 8, 2, 0.1
    base = zg.step_key(42, "test", 0, manifest.version, cuda)
    ids = torch.arange(pop, dtype=torch.int32, device=cuda)
    losses = torch.arange(pop, dtype=torch.float32, device=cuda)
    shaped = zg.shape_centered_loss(losses, sigma)
    got = zg.replay_entry(params, manifest, path, base, ids, shaped, rank)
    ob = oracle.step_key(42, "test", 0, 1)
    osh = oracle.shape_centered_loss(np.arange(pop, dtype=np.float32), sigma)
    want = oracle.replay_entry(shape, layout, ob, range(pop), osh, rank if layout != 2 else 1, group)
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=1e-5)


def test_replay_nested(cuda):
    params, manifest = _params(cuda), _manifest()
    base = zg.step_key(42, "test", 0, 1, cuda)
    shaped = zg.shape_centered_loss(torch.tensor([1.0, 2.0, 3.0, 4.0], device=cuda), 0.1)
    out = zg.replay(params, manifest, base, torch.arange(4, device=cuda), shaped, 2)
    assert out["linear"]["weight"].shape == (8, 4)
    assert out["table"]["embed"].shape == (16, 4)
    assert out["vector"]["scale"].shape == (4,)


def test_shaping_and_metrics(cuda, oracle):
    l = torch.tensor([3.0, -1.0, 2.5, 7.0, 0.0], device=cuda)
    shaped, metrics = _ops.launch_shape_fitness(l, 0.05)
    np.testing.assert_allclose(shaped.cpu().numpy(), oracle.shape_centered_loss(l.cpu().numpy(), 0.05), rtol=1e-6)
    m = metrics.cpu().numpy()
    assert m[0] == pytest.approx(2.3) and m[1] == -1.0 and m[2] == 7.0 and m[3] == 0
    _, metrics = _ops.launch_shape_fitness(torch.tensor([1.0, float("nan"), float("inf")], device=cuda), 0.1)
    assert metrics.cpu()[3].item() == 2


@pytest.mark.parametrize("layout,shape", [(0, (300, 200)), (1, (300, 200)), (2, (5000,))])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_replay_larger_population(cuda, oracle, layout, shape, dtype):
    P, rank = 64, 4
    base = oracle.step_key(0, "bench", 0, 1)
    cks = oracle.candidate_keys(base, range(P))
    w = np.random.default_rng(3).standard_normal(P).astype(np.float32)
    got = _ops.launch_replay(torch.tensor(w, device=cuda), _u32(cks, cuda), 1, layout, shape,
                             rank if layout != 2 else 1, dtype)
    want = oracle.replay_entry(shape, layout, base, range(P), w, rank if layout != 2 else 1, 1,
                               "float32" if dtype == torch.float32 else "bfloat16")
    scale = np.abs(want).max()
    got = got.cpu().numpy()
    if dtype == torch.float32:
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5 * scale)
    else:
        # bf16 leaves: the tensor-core replay rounds w_p * A_p to bf16 (rel 2^-9 per term)
        assert np.abs(got - want).max() <= 2e-2 * scale
        assert np.linalg.norm(got - want) <= 5e-3 * np.linalg.norm(want)

"""Population-batched forward ops against the float64 oracle.

Tolerances: float32 rel 1e-5 (the reference's own tests use rtol/atol 1e-5);
bf16 element-wise rel 2e-2 above a floor of half the output's RMS
(bf16_tol.assert_bf16_close, bf16_tol.rms_floor: the low-rank term's bf16
operands err by ~2^-9 of the terms, not of each element), and the
perturbation (output minus the unperturbed output) within 5% of its own
scale.
"""
import numpy as np
import pytest
import torch

import zerograd_b200 as zg
from zerograd_b200 import _ops

from bf16_tol import assert_bf16_close, assert_perturbation_close, rms_floor

pytestmark = pytest.mark.gpu

DN = {torch.float32: "float32", torch.bfloat16: "bfloat16"}


def _u32(a, dev):
    return torch.tensor(np.asarray(a, np.int64)).to(torch.uint32).to(dev)


def _check(got, want, dtype, base=None, what=""):
    got = got.float().cpu().numpy()
    if dtype == torch.float32:
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)
        return
    assert_bf16_close(got, want, floor=rms_floor(want), what=what)
    if base is not None:
        assert_perturbation_close(got, want, base, what=what)


def _setup(oracle, P, group=1):
    base = oracle.step_key(42, "test", 0, 1)
    cks = oracle.candidate_keys(base, range(P))
    return cks, oracle.group_keys(cks, group)


def _rand(shape, dtype, dev, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype).to(dev)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("x_batched", [False, True])
@pytest.mark.parametrize("dims", [(5, 8, 4, 2), (33, 70, 45, 3), (64, 128, 96, 8)])
def test_perturbed_linear(cuda, oracle, dtype, x_batched, dims):
    M, K, N, rank = dims
    P, sigma = 5, 0.1
    cks, gks = _setup(oracle, P)
    W = _rand((K, N), dtype, cuda, 1)
    x = _rand((P, M, K) if x_batched else (M, K), dtype, cuda, 2)
    y = _ops.launch_linear(x, W, _u32(cks, cuda), 1, rank, sigma, x_batched)
    xs = x.float().cpu().numpy()
    for p in range(P):
        xp, Wn = (xs[p] if x_batched else xs).astype(np.float64), W.float().cpu().numpy().astype(np.float64)
        want = oracle.perturbed_linear(xp, Wn, gks[p], rank, sigma, DN[dtype])
        _check(y[p], want, dtype, base=xp @ Wn, what=f"candidate {p}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("x_batched", [False, True])
def test_tied_logits(cuda, oracle, dtype, x_batched):
    P, M, V, C, rank, sigma = 4, 9, 50, 24, 3, 0.05
    cks, gks = _setup(oracle, P, group=0)
    T = _rand((V, C), dtype, cuda, 3)
    x = _rand((P, M, C) if x_batched else (M, C), dtype, cuda, 4)
    y = _ops.launch_tied_logits(x, T, _u32(cks, cuda), 0, rank, sigma, x_batched)
    xs = x.float().cpu().numpy()
    for p in range(P):
        xp, Tn = (xs[p] if x_batched else xs).astype(np.float64), T.float().cpu().numpy().astype(np.float64)
        want = oracle.perturbed_tied_logits(xp, Tn, gks[p], rank, sigma, DN[dtype])
        _check(y[p], want, dtype, base=xp @ Tn.T, what=f"candidate {p}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("idx_batched", [False, True])
def test_table_lookup(cuda, oracle, dtype, idx_batched):
    P, rows, cols, rank, sigma = 4, 40, 300, 4, 0.2
    cks, gks = _setup(oracle, P, group=2)
    T = _rand((rows, cols), dtype, cuda, 5)
    g = torch.Generator().manual_seed(6)
    idx = torch.randint(0, rows, (P, 3, 5) if idx_batched else (3, 5), generator=g).to(cuda)
    out = _ops.launch_table_lookup(T, idx, _u32(cks, cuda), 2, rank, sigma, idx_batched)
    ii = idx.cpu().numpy()
    for p in range(P):
        Tn, ip = T.float().cpu().numpy().astype(np.float64), ii[p] if idx_batched else ii
        want = oracle.perturbed_table_lookup(Tn, ip, gks[p], rank, sigma, DN[dtype])
        _check(out[p], want, dtype, base=Tn[ip], what=f"candidate {p}")


@pytest.mark.parametrize("rank", [8, 16])
def test_table_lookup_tensor_core_path(cuda, oracle, rank):
    """bf16, ids shared by the candidates, cols a multiple of 8: the lookup
    runs as an expansion on the tensor cores (gathered rows + A rows at the
    ids staged, one K = 16 MMA per candidate and tile); odd P, ragged token
    and column tiles, repeated and negative ids."""
    from zerograd_b200 import _lib as L

    P, rows, cols, sigma = 9, 500, 264, 0.05
    cks, gks = _setup(oracle, P, group=3)
    T = _rand((rows, cols), torch.bfloat16, cuda, 13, scale=0.1)
    g = torch.Generator().manual_seed(14)
    idx = torch.randint(-rows, rows, (3, 101), generator=g).to(torch.int32).to(cuda)
    L.profile_begin()
    out = _ops.launch_table_lookup(T, idx, _u32(cks, cuda), 3, rank, sigma, False)
    prof = L.profile_end()
    assert "lowrank_expand" not in prof and "table_lookup" in prof, prof
    assert L.load().zg_device_error(1) == 0
    ii = idx.cpu().numpy().astype(np.int64)
    eff = np.where(ii < 0, ii + rows, ii)
    Tn = T.float().cpu().numpy().astype(np.float64)
    for p in (0, 4, P - 1):
        want = oracle.perturbed_table_lookup(Tn, eff, gks[p], rank, sigma, "bfloat16")
        _check(out[p], want, torch.bfloat16, base=Tn[eff], what=f"candidate {p}")


def test_table_lookup_negative_and_out_of_range_indices(cuda, oracle):
    """jnp indexing: negative indices wrap, out-of-range gathers clamp."""
    P, rows, cols, rank, sigma = 2, 10, 16, 2, 0.1
    cks, gks = _setup(oracle, P)
    T = _rand((rows, cols), torch.float32, cuda, 7)
    idx = torch.tensor([-1, -10, 0, 9, 12, -13], dtype=torch.int32, device=cuda)
    out = _ops.launch_table_lookup(T, idx, _u32(cks, cuda), 1, rank, sigma, False)
    eff = np.array([9, 0, 0, 9, 9, 0])
    for p in range(P):
        want = oracle.perturbed_table_lookup(T.cpu().numpy(), eff, gks[p], rank, sigma)
        np.testing.assert_allclose(out[p].cpu().numpy(), want, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_vector(cuda, oracle, dtype):
    P, n, sigma = 7, 1000, 0.3
    cks, gks = _setup(oracle, P, group=0)
    v = _rand((n,), dtype, cuda, 8)
    out = _ops.launch_vector(v, _u32(cks, cuda), 0, sigma, False)
    for p in range(P):
        vn = v.float().cpu().numpy().astype(np.float64)
        want = oracle.perturbed_vector(vn, gks[p], sigma, DN[dtype])
        _check(out[p], want, dtype, base=vn, what=f"candidate {p}")


def test_public_ops_take_group_keys(cuda, oracle):
    """perturbed_* take a GROUP key, CandidateContext a candidate key + group."""
    gk = oracle.key(1234)
    x = _rand((3, 8), torch.float32, cuda, 9)
    W = _rand((8, 4), torch.float32, cuda, 10)
    y = zg.perturbed_linear(x, W, _u32(gk, cuda), 2, 0.1)
    want = oracle.perturbed_linear(x.cpu().numpy(), W.cpu().numpy(), gk, 2, 0.1)
    np.testing.assert_allclose(y.cpu().numpy(), want, rtol=1e-5, atol=1e-5)
    A, B = zg.matrix_factors(_u32(gk, cuda), (8, 4), 2, dtype=torch.float32)
    a, b = oracle.matrix_factors(gk, (8, 4), 2)
    np.testing.assert_allclose(A.cpu().numpy(), a, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(B.cpu().numpy(), b, rtol=1e-5, atol=1e-6)


def test_vmap_launches_one_population_op(cuda, oracle):
    """Per-candidate code under torch.func.vmap equals the population launch."""
    P, M, K, N, rank, sigma = 6, 4, 16, 8, 2, 0.1
    cks, gks = _setup(oracle, P, group=0)
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),))
    W = _rand((K, N), torch.float32, cuda, 11)
    x = _rand((M, K), torch.float32, cuda, 12)

    def one(ck):
        ctx = zg.CandidateContext(manifest, ck, rank, sigma)
        return ctx.linear({"w": W}, ("w",), x)

    y = torch.func.vmap(one)(_u32(cks, cuda))
    for p in range(P):
        want = oracle.perturbed_linear(x.cpu().numpy(), W.cpu().numpy(), gks[p], rank, sigma)
        np.testing.assert_allclose(y[p].cpu().numpy(), want, rtol=1e-5, atol=1e-5)
    # and unbatched (a single candidate) matches row 0
    y0 = one(_u32(cks[0], cuda))
    np.testing.assert_allclose(y0.cpu().numpy(), y[0].cpu().numpy(), rtol=0, atol=0)

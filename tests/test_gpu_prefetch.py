"""Replay-factor prefetch for population shards (one process per GPU).

A shard's process replays the whole population, but its forward pass draws
only its own candidates' factors.  With ``prefetch_replay`` the whole
population's replay factors are drawn on a second stream while the shard's
forward runs; the replay then takes them from the factor cache.  The result
must be bit-identical to replaying from fresh draws.
"""
import pytest
import torch

import zerograd_b200 as zg
from zerograd_b200 import _ops

pytestmark = pytest.mark.gpu


def _problem(cuda):
    P, r, B, K, N, V = 64, 8, 32, 256, 128, 300
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),
                               zg.ManifestEntry(("t",), zg.ParameterLayout.TABLE, "t"),
                               zg.ManifestEntry(("b",), zg.ParameterLayout.VECTOR, "b")))
    g = torch.Generator().manual_seed(23)
    params = {"w": (torch.randn(K, N, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
              "t": (torch.randn(V, N, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
              "b": torch.zeros(N, dtype=torch.bfloat16, device=cuda)}
    x = torch.randn(B, K, generator=g).to(torch.bfloat16).to(cuda)

    def loss_fn(p, ctx, batch, rng):
        h = ctx.linear(p, ("w",), batch) + ctx.vector(p, ("b",))
        return (ctx.tied_logits(p, ("t",), h).float() ** 2).mean(), None

    opt = zg.ZeroGrad(manifest, zg.adamw(1e-3), P, r, 0.02, 0, "prefetch")
    return opt, params, x, loss_fn, P


def test_shard_prefetch_feeds_the_replay_bit_identically(cuda):
    opt, params, x, loss_fn, P = _problem(cuda)
    state = opt.init(params)
    _ops.CACHE.clear()
    # this process's shard [16, 48) with prefetch, the rest evaluated plainly
    mid = opt.evaluate_shard(params, 0, loss_fn, x, range(16, 48), prefetch_replay=True)
    base = tuple(int(v) for v in opt.base_key(0))
    full = [k for k in _ops.CACHE._entries if k[0] == base and k[1] == 0 and k[2] == P]
    assert len(full) == 2  # the MATRIX and TABLE entries, whole population
    head = opt.evaluate_shard(params, 0, loss_fn, x, torch.arange(0, 16, device=cuda))
    tail = opt.evaluate_shard(params, 0, loss_fn, x, torch.arange(48, P, device=cuda))
    losses = torch.cat([head, mid, tail])
    h0 = _ops.CACHE.hits
    a, sa, ma = opt.step_from_losses(state, params, losses)
    assert _ops.CACHE.hits - h0 == 2  # both replays used the prefetched factors
    assert not _ops.CACHE._entries

    # the same step from the same losses with nothing cached (fresh draws in
    # the replay).  The losses themselves are compared with nothing: a shard's
    # GEMM tiling, hence its float32 summation order, depends on its size.
    _ops.CACHE.clear()
    b, sb, mb = opt.step_from_losses(state, params, losses)
    for k in params:
        assert torch.equal(a[k], b[k]), k
        assert torch.equal(sa.opt_state.mu[k], sb.opt_state.mu[k]), k
    assert ma == mb


def test_shard_forward_reads_the_whole_population_factors(cuda):
    """With the whole population's factors of a generation already drawn
    (drawn ahead, or prefetched for the replay), a shard's forward reads its
    candidates' columns of them (zg_forward_factors_ld) and draws nothing;
    its outputs are bit for bit those of the shard drawing its own."""
    from zerograd_b200 import _lib as L

    opt, params, x, loss_fn, P = _problem(cuda)
    _ops.CACHE.clear()
    L.profile_begin()
    ref = opt.evaluate_shard(params, 0, loss_fn, x, range(16, 48))  # draws its own factors
    prof_ref = L.profile_end()
    _ops.CACHE.clear()
    opt._prefetch_replay(params, 0, tuple(int(v) for v in opt.base_key(0)), cuda)  # the whole population's
    torch.cuda.synchronize()
    L.profile_begin()
    got = opt.evaluate_shard(params, 0, loss_fn, x, range(16, 48))
    prof = L.profile_end()
    # the linear layer's two operand draws are gone (the tied logits here,
    # V=300, take the path that regenerates its factors in-kernel)
    fills = lambda p: p.get("factor_fill", (0, 0.0))[0]  # noqa: E731
    assert fills(prof) == fills(prof_ref) - 2, (prof_ref, prof)
    assert torch.equal(got, ref)
    _ops.CACHE.clear()
    assert L.load().zg_device_error(1) == 0


def test_strided_factors_rejected_without_the_tensor_core_expansion(cuda):
    """A leading dimension above P*rank needs the rank-8 tensor-core
    expansion: rank 16 is refused with a clear error."""
    from zerograd_b200 import _lib as L

    P, r, M, K, N = 8, 16, 32, 64, 64
    x = torch.zeros(M, K, dtype=torch.bfloat16, device=cuda)
    W = torch.zeros(K, N, dtype=torch.bfloat16, device=cuda)
    F1 = torch.zeros(K, 2 * P * r, dtype=torch.bfloat16, device=cuda)
    F2 = torch.zeros(N, 2 * P * r, dtype=torch.bfloat16, device=cuda)
    y = torch.empty(P, M, N, dtype=torch.bfloat16, device=cuda)
    ws = L.workspace(L.query("zg_forward_factors_workspace_size", P, M, N, r), cuda)
    with pytest.raises(L.ZgLibraryError, match="strided factors"):
        L.call("zg_forward_factors_ld", L.ptr(x), L.ptr(W), 1, L.ptr(F1), 2 * P * r, L.ptr(F2), 2 * P * r, P, M, K, N,
               r, 0.1, L.ptr(y), L.ptr(ws), ws.numel(), L.stream_ptr(cuda))

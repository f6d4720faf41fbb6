"""tcgen05 GEMM and the bf16 tensor-core paths at full config sizes.

The GEMM is checked against a float32 matmul of the same bf16 inputs
(tolerance 1e-3 of the output scale: float32 accumulation in a different
order); the population paths against the oracle (bf16 tolerance 2e-2).
"""
import numpy as np
import pytest
import torch

from zerograd_b200 import _lib as L
from zerograd_b200 import _ops

from bf16_tol import assert_bf16_close, assert_perturbation_close, rms_floor

pytestmark = pytest.mark.gpu


def _u32(a, dev):
    return torch.tensor(np.asarray(a, np.int64)).to(torch.uint32).to(dev)


def _gemm(A, B, b_mn, M, N, K, out_dtype=torch.float32, alpha=1.0):
    dev = A.device
    D = torch.empty((M, N), dtype=out_dtype, device=dev)
    L.call("zg_gemm_bf16", L.ptr(A), A.stride(0), L.ptr(B), B.stride(0), int(b_mn), L.ptr(D), N,
           L.dtype_code(out_dtype), M, N, K, alpha, L.stream_ptr(dev))
    assert L.load().zg_device_error(1) == 0
    return D


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 2048, 4096), (300, 200, 136), (4096, 4096, 2048),
                                   (8, 24, 8), (1000, 520, 1000)])
@pytest.mark.parametrize("b_mn", [False, True])
def test_tc_gemm_matches_fp32(cuda, M, N, K, b_mn):
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16).to(cuda)
    B = torch.randn((K, N) if b_mn else (N, K), generator=g).to(torch.bfloat16).to(cuda)
    D = _gemm(A, B, b_mn, M, N, K, alpha=0.5)
    ref = 0.5 * (A.float() @ (B.float() if b_mn else B.float().t()))
    err = (D - ref).abs().max().item()
    assert err <= 1e-3 * ref.abs().max().item(), err


def test_tc_gemm_bf16_output(cuda):
    g = torch.Generator().manual_seed(1)
    A = torch.randn(256, 512, generator=g).to(torch.bfloat16).to(cuda)
    B = torch.randn(384, 512, generator=g).to(torch.bfloat16).to(cuda)
    D = _gemm(A, B, False, 256, 384, 512, out_dtype=torch.bfloat16)
    ref = (A.float() @ B.float().t()).to(torch.bfloat16).float()
    assert (D.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()


def test_bench_size_perturbed_linear(cuda, oracle):
    """P=256, rank 8, x[256,4096] shared, W[4096,4096] bf16; sampled candidates vs the oracle."""
    P, r, M, K, N, sigma = 256, 8, 256, 4096, 4096, 0.01
    base = oracle.step_key(0, "bench", 0, 1)
    cks = oracle.candidate_keys(base, range(P))
    g = torch.Generator().manual_seed(0)
    x = (torch.randn(M, K, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    W = (torch.randn(K, N, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    y = _ops.launch_linear(x, W, _u32(cks, cuda), 0, r, sigma, False)
    assert L.load().zg_device_error(1) == 0
    xs, Ws = x.float().cpu().numpy(), W.float().cpu().numpy()
    for p in (0, 77, 255):
        gk = oracle.fold_in(cks[p], 0)
        want = oracle.perturbed_linear(xs, Ws, gk, r, sigma, "bfloat16")
        got = y[p].float().cpu().numpy()
        assert_bf16_close(got, want, floor=rms_floor(want), what=f"candidate {p}")
        # the perturbation itself (y - xW) is reproduced, not just the dominant xW
        assert_perturbation_close(got, want, xs.astype(np.float64) @ Ws, what=f"candidate {p}")


def test_bench_size_replay(cuda, oracle):
    P, r, K, N = 256, 8, 4096, 4096
    base = oracle.step_key(0, "bench", 0, 1)
    cks = oracle.candidate_keys(base, range(P))
    fit = np.random.default_rng(0).standard_normal(P).astype(np.float32)
    shaped = oracle.shape_centered_loss(fit, 0.01)
    got = _ops.launch_replay(torch.tensor(shaped, device=cuda), _u32(cks, cuda), 0, L.ZG_MATRIX, (K, N), r,
                             torch.bfloat16)
    assert L.load().zg_device_error(1) == 0
    want = oracle.replay_entry((K, N), oracle.MATRIX, base, range(P), shaped, r, 0, "bfloat16")
    got = got.cpu().numpy()
    scale = np.abs(want).max()
    assert np.abs(got - want).max() <= 2e-2 * scale
    # relative error over the whole matrix, not just the max
    assert np.linalg.norm(got - want) <= 5e-3 * np.linalg.norm(want)


def test_replay_is_linear_in_the_weights(cuda, oracle):
    P, r, K, N = 64, 8, 512, 384
    cks = _u32(oracle.candidate_keys(oracle.step_key(1, "lin", 0, 1), range(P)), cuda)
    g = torch.Generator().manual_seed(3)
    w1 = torch.randn(P, generator=g).to(cuda)
    w2 = torch.randn(P, generator=g).to(cuda)
    rep = lambda w: _ops.launch_replay(w, cks, 2, L.ZG_MATRIX, (K, N), r, torch.bfloat16)
    a, b, ab = rep(w1), rep(w2), rep(w1 + w2)
    assert (ab - (a + b)).abs().max().item() <= 2e-2 * ab.abs().max().item()
    # a one-hot weight replays exactly one candidate's A_p B_p / sqrt(r)
    e = torch.zeros(P, device=cuda)
    e[5] = 1.0
    one = rep(e).cpu().numpy()
    gk = oracle.fold_in(oracle.candidate_keys(oracle.step_key(1, "lin", 0, 1), [5])[0], 2)
    A, B = oracle.matrix_factors(gk, (K, N), r, "bfloat16")
    want = (A.astype(np.float64) @ B) * oracle.scaled_factor(r, 1.0, "bfloat16")
    np.testing.assert_allclose(one, want, rtol=1e-2, atol=1e-2 * np.abs(want).max())


def test_table_replay_and_tied_logits_on_tensor_cores(cuda, oracle):
    P, r, V, C, M, sigma = 32, 8, 1000, 256, 64, 0.02
    base = oracle.step_key(5, "tied", 0, 1)
    cks = oracle.candidate_keys(base, range(P))
    g = torch.Generator().manual_seed(4)
    T = (torch.randn(V, C, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    x = torch.randn(M, C, generator=g).to(torch.bfloat16).to(cuda)
    y = _ops.launch_tied_logits(x, T, _u32(cks, cuda), 1, r, sigma, False)
    xs, Ts = x.float().cpu().numpy().astype(np.float64), T.float().cpu().numpy().astype(np.float64)
    for p in (0, 31):
        want = oracle.perturbed_tied_logits(xs, Ts, oracle.fold_in(cks[p], 1), r, sigma, "bfloat16")
        got = y[p].float().cpu().numpy()
        assert_bf16_close(got, want, floor=rms_floor(want), what=f"candidate {p}")
        assert_perturbation_close(got, want, xs @ Ts.T, what=f"candidate {p}")
    w = np.random.default_rng(1).standard_normal(P).astype(np.float32)
    got = _ops.launch_replay(torch.tensor(w, device=cuda), _u32(cks, cuda), 1, L.ZG_TABLE, (V, C), r,
                             torch.bfloat16).cpu().numpy()
    want = oracle.replay_entry((V, C), oracle.TABLE, base, range(P), w, r, 1, "bfloat16")
    assert np.linalg.norm(got - want) <= 5e-3 * np.linalg.norm(want)
    assert L.load().zg_device_error(1) == 0


def test_cached_factors_give_identical_results(cuda):
    """ZeroGrad.step reuses the forward pass's factors in the replay; the
    result is bit-identical to evaluating without the cache and replaying
    from freshly drawn factors."""
    import zerograd_b200 as zg

    P, r, B, K, N = 32, 8, 64, 256, 128
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),
                               zg.ManifestEntry(("t",), zg.ParameterLayout.TABLE, "t")))
    g = torch.Generator().manual_seed(9)
    params = {"w": (torch.randn(K, N, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
              "t": (torch.randn(200, N, generator=g) * 0.05).to(torch.bfloat16).to(cuda)}
    x = (torch.randn(B, K, generator=g).to(torch.bfloat16).to(cuda), torch.randn(B, N, generator=g).to(torch.bfloat16).to(cuda))

    def loss_fn(p, ctx, batch, rng):
        h = ctx.linear(p, ("w",), batch[0])          # shared input: tensor-core path, factors cached
        logits = ctx.tied_logits(p, ("t",), batch[1])
        return (h.float() ** 2).mean() + (logits.float() ** 2).mean(), None

    opt = zg.ZeroGrad(manifest, zg.sgd(0.1), P, r, 0.02, 0, "cache")
    state = opt.init(params)
    _ops.CACHE.clear()
    h0 = _ops.CACHE.hits
    a, _, ma = opt.step(state, params, x, loss_fn)
    assert _ops.CACHE.hits - h0 == 2  # both entries replayed from the forward's factors
    assert not _ops.CACHE._entries  # dropped after the update
    losses = opt.evaluate_shard(params, 0, loss_fn, x, torch.arange(P, device=cuda))  # device ids: no cache
    b, _, mb = opt.step_from_losses(state, params, losses)
    for k in params:
        assert torch.equal(a[k], b[k]), k
    assert ma == mb


def test_replay_factors_entry_matches_replay(cuda, oracle):
    P, r, K, N = 64, 8, 512, 384
    cks = _u32(oracle.candidate_keys(oracle.step_key(2, "rf", 0, 1), range(P)), cuda)
    w = torch.randn(P, generator=torch.Generator().manual_seed(2)).to(cuda)
    direct = _ops.launch_replay(w, cks, 1, L.ZG_MATRIX, (K, N), r, torch.bfloat16)
    gen = _ops._Generation((7, 7), 0, P, cks)
    A, B = _ops.operand_factors(cks, 1, L.ZG_MATRIX, K, N, r, gen)
    cached = _ops.launch_replay(w, cks, 1, L.ZG_MATRIX, (K, N), r, torch.bfloat16, gen=gen)
    _ops.CACHE.drop_generation((7, 7))
    assert torch.equal(direct, cached)


@pytest.mark.parametrize("rows,cols,P,r", [(1024, 1024, 64, 8),     # 32 tiles: fewer than one wave
                                           (6400, 1024, 32, 8),     # 200 tiles: one wave and a partial one
                                           (4096, 4096, 256, 8),    # 512 tiles: the bench replay
                                           (5504, 1792, 64, 8),     # 301 tiles, ragged rows
                                           (1280, 768, 40, 8),      # 30 tiles, 320-deep contraction
                                           (4096, 2048, 128, 4),    # rank 4: two weights per 8 columns
                                           (4352, 2048, 100, 16),   # rank 16, 1600-deep contraction
                                           (1024, 768, 2048, 16)])  # split over 8 candidate groups
def test_replay_factors_matches_fp32(cuda, rows, cols, P, r):
    """The replay GEMM over P*r matches a float32 matmul of the same weighted
    bf16 operands, is identical from call to call, and is bit for bit the
    plain GEMM of the operands with the smaller side weighted and rounded to
    bf16 on the host."""
    q = P * r
    g = torch.Generator().manual_seed(rows + cols + P)
    A = torch.randn(rows, q, generator=g).to(torch.bfloat16).to(cuda)
    B = torch.randn(cols, q, generator=g).to(torch.bfloat16).to(cuda)
    w = torch.randn(P, generator=g).to(cuda)
    ws = L.workspace(L.query("zg_replay_factors_workspace_size", P, rows, cols, r), cuda)

    def run():
        out = torch.empty((rows, cols), dtype=torch.float32, device=cuda)
        L.call("zg_replay_factors", L.ptr(w), L.ptr(A), L.ptr(B), P, rows, cols, r, 0.5, L.ptr(out), L.ptr(ws),
               ws.numel(), L.stream_ptr(cuda))
        return out

    a = run()
    b = run()
    assert L.load().zg_device_error(1) == 0
    assert torch.equal(a, b)
    wq = w.repeat_interleave(r)[None, :]
    if cols < rows:
        A16, B16 = A, (B.float() * wq).to(torch.bfloat16)
    else:
        A16, B16 = (A.float() * wq).to(torch.bfloat16), B
    if L.load().zg_replay_split_count(P, r) == 1:
        plain = _gemm(A16, B16, False, rows, cols, q, alpha=0.5)
        assert torch.equal(a, plain)
    ref = 0.5 * (A16.float() @ B16.float().t())
    err = (a - ref).abs().max().item()
    assert err <= 1e-3 * ref.abs().max().item(), err

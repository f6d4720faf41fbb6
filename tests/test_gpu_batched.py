"""Per-candidate-input forward (the hidden-layer case: every candidate has its
own input x_p) on the tensor cores, against the oracle.

y_p = x_p @ W + s (x_p @ A_p) @ B_p in bf16 with float32 accumulation; the
oracle computes it in float64 from the same bf16-rounded factors.  Tolerance
element-wise rel 2e-2 above a floor of half the output's RMS on y
(bf16_tol.rms_floor), and
the perturbation y - x W within 5% of its own scale (so the low-rank term is
checked, not only the dominant x W).
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


def _check_candidate(got, want, base):
    assert_bf16_close(got, want, floor=rms_floor(want), what="y_p")
    assert_perturbation_close(got, want, base, what="y_p - x_p W")


def _linear(x, W, cks, group, r, sigma):
    L.profile_begin()
    y = _ops.launch_linear(x, W, cks, group, r, sigma, True)
    prof = L.profile_end()
    assert L.load().zg_device_error(1) == 0
    assert "batched_gemm" in prof and "batched_u_pass" in prof, prof  # the tensor-core path ran
    return y


@pytest.mark.parametrize("P,M,K,N,r", [(8, 128, 256, 256, 8),
                                       (5, 200, 200, 520, 8),     # ragged M, K % 64, N % 256
                                       (4, 64, 512, 384, 16),     # rank 16
                                       (3, 1, 64, 8, 8),          # one row, narrowest N
                                       (17, 130, 136, 264, 8)])   # odd P, tiles straddling every edge
def test_batched_linear_matches_oracle(cuda, oracle, P, M, K, N, r):
    sigma, group = 0.02, 1
    base = oracle.step_key(3, "batched", 0, 1)
    cks = oracle.candidate_keys(base, range(P))
    g = torch.Generator().manual_seed(P * 31 + M + K + N)
    x = torch.randn(P, M, K, generator=g).to(torch.bfloat16).to(cuda)
    W = (torch.randn(K, N, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    y = _linear(x, W, _u32(cks, cuda), group, r, sigma)
    xs, Ws = x.float().cpu().numpy().astype(np.float64), W.float().cpu().numpy().astype(np.float64)
    for p in range(P):
        want = oracle.perturbed_linear(xs[p], Ws, oracle.fold_in(cks[p], group), r, sigma, "bfloat16")
        _check_candidate(y[p].float().cpu().numpy(), want, xs[p] @ Ws)


@pytest.mark.parametrize("act,res", [(0, False), (1, False), (0, True), (1, True)])
def test_pair_kernel_ragged_epilogues(cuda, oracle, act, res):
    """Enough tiles for the CTA-pair kernel (>= 74 pair tiles) with every
    tile edge ragged (M, K, N not multiples of 256 / 64), each epilogue:
    plain and GELU (one staging box per warp, six stages) and with a
    residual (two boxes, five stages)."""
    from oracle.lm import gelu_tanh

    P, M, K, N, r, sigma, group = 40, 300, 200, 600, 8, 0.02, 2
    base = oracle.step_key(5, "pair-edges", 0, 1)
    cks = oracle.candidate_keys(base, range(P))
    g = torch.Generator().manual_seed(act * 2 + int(res))
    x = torch.randn(P, M, K, generator=g).to(torch.bfloat16).to(cuda)
    W = (torch.randn(K, N, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    rs = torch.randn(P, M, N, generator=g).to(torch.bfloat16).to(cuda) if res else None
    L.profile_begin()
    y = _ops.launch_linear(x, W, _u32(cks, cuda), group, r, sigma, True, act, rs)
    prof = L.profile_end()
    assert L.load().zg_device_error(1) == 0
    assert "batched_gemm" in prof, prof
    xs, Ws = x.float().cpu().numpy().astype(np.float64), W.float().cpu().numpy().astype(np.float64)
    for p in range(0, P, 13):
        v = oracle.perturbed_linear(xs[p], Ws, oracle.fold_in(cks[p], group), r, sigma, "bfloat16")
        if act:
            v = gelu_tanh(v)
        got = y[p].float().cpu().numpy()
        if not res:
            assert_bf16_close(got, v, floor=rms_floor(v), what="epilogue output")
            continue
        # the residual is added to the bf16-rounded product (the unfused ops'
        # roundings): the sum keeps that intermediate's rounding error, up to
        # one bf16 ulp of |v| (two half-ulp roundings), which cancellation
        # against the residual does not shrink
        want = v + rs[p].float().cpu().numpy().astype(np.float64)
        bound = 2e-2 * np.maximum(np.abs(want), rms_floor(want)) + 2.0 ** -7 * np.abs(v)
        err = np.abs(got - want)
        assert (err <= bound).all(), (float((err / bound).max()), int((err > bound).sum()))


def test_batched_tied_logits_matches_oracle(cuda, oracle):
    P, M, V, C, r, sigma, group = 6, 100, 1000, 256, 8, 0.02, 2
    base = oracle.step_key(4, "batched-tied", 0, 1)
    cks = oracle.candidate_keys(base, range(P))
    g = torch.Generator().manual_seed(11)
    T = (torch.randn(V, C, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    x = torch.randn(P, M, C, generator=g).to(torch.bfloat16).to(cuda)
    L.profile_begin()
    y = _ops.launch_tied_logits(x, T, _u32(cks, cuda), group, r, sigma, True)
    prof = L.profile_end()
    assert L.load().zg_device_error(1) == 0
    assert "batched_gemm" in prof, prof
    xs, Ts = x.float().cpu().numpy().astype(np.float64), T.float().cpu().numpy().astype(np.float64)
    for p in range(P):
        want = oracle.perturbed_tied_logits(xs[p], Ts, oracle.fold_in(cks[p], group), r, sigma, "bfloat16")
        _check_candidate(y[p].float().cpu().numpy(), want, xs[p] @ Ts.T)


def test_bench_size_batched_linear(cuda, oracle):
    """P=256, rank 8, x_p [256, 4096] per candidate, W [4096, 4096] bf16: sampled candidates vs the oracle."""
    P, r, M, K, N, sigma = 256, 8, 256, 4096, 4096, 0.01
    base = oracle.step_key(0, "bench", 0, 1)
    cks = oracle.candidate_keys(base, range(P))
    g = torch.Generator(device=cuda).manual_seed(0)
    x = (torch.randn(P, M, K, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    W = (torch.randn(K, N, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    y = _linear(x, W, _u32(cks, cuda), 0, r, sigma)
    Ws = W.float().cpu().numpy().astype(np.float64)
    for p in (0, 129, 255):
        xs = x[p].float().cpu().numpy().astype(np.float64)
        want = oracle.perturbed_linear(xs, Ws, oracle.fold_in(cks[p], 0), r, sigma, "bfloat16")
        _check_candidate(y[p].float().cpu().numpy(), want, xs @ Ws)


def test_forward_factors_entry_reuses_drawn_factors(cuda, oracle):
    """zg_batched_forward_factors on the factors zg_batched_forward_operands drew gives the same y."""
    P, M, K, N, r, s = 12, 96, 128, 136, 16, 0.0125
    cks = _u32(oracle.candidate_keys(oracle.step_key(6, "ff", 0, 1), range(P)), cuda)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(P, M, K, generator=g).to(torch.bfloat16).to(cuda)
    W = torch.randn(K, N, generator=g).to(torch.bfloat16).to(cuda)
    F1T = torch.empty((P * r, K), dtype=torch.bfloat16, device=cuda)
    F2 = torch.empty((N, P * r), dtype=torch.bfloat16, device=cuda)
    y1 = torch.empty((P, M, N), dtype=torch.bfloat16, device=cuda)
    y2 = torch.empty_like(y1)
    ws = L.workspace(L.query("zg_batched_forward_workspace_size", P, M, K, N, r), cuda)
    st = L.stream_ptr(cuda)
    L.call("zg_batched_forward_operands", L.ptr(x), L.ptr(W), 1, L.ptr(cks), 0, P, M, K, N, r, s, L.ptr(F1T),
           L.ptr(F2), L.ptr(y1), L.ptr(ws), ws.numel(), st)
    L.call("zg_batched_forward_factors", L.ptr(x), L.ptr(W), 1, L.ptr(F1T), L.ptr(F2), P, M, K, N, r, s, L.ptr(y2),
           L.ptr(ws), ws.numel(), st)
    assert torch.equal(y1, y2)
    # the drawn factors are the operand-layout factors, transposed on the input side
    A_op, B_op = _ops.operand_factors(cks, 0, L.ZG_MATRIX, K, N, r)
    assert torch.equal(F1T, A_op.t().contiguous())
    assert torch.equal(F2, B_op)
    assert L.load().zg_device_error(1) == 0


@pytest.mark.parametrize("layout", ["matrix", "table"])
def test_replay_operands_transposed_matches_replay(cuda, oracle, layout):
    # rows < cols: the direct replay weights A (the smaller side), as the
    # transposed-A one does (it transposes A anyway)
    P, r, rows, cols = 48, 8, 384, 520
    lay = L.ZG_MATRIX if layout == "matrix" else L.ZG_TABLE
    cks = _u32(oracle.candidate_keys(oracle.step_key(8, "rt", 0, 1), range(P)), cuda)
    w = torch.randn(P, generator=torch.Generator().manual_seed(8)).to(cuda)
    direct = _ops.launch_replay(w, cks, 3, lay, (rows, cols), r, torch.bfloat16)
    A_op, B_op = _ops.operand_factors(cks, 3, lay, rows, cols, r)
    a_t, b_t = (1, 0) if lay == L.ZG_MATRIX else (0, 1)
    A = A_op.t().contiguous() if a_t else A_op
    B = B_op.t().contiguous() if b_t else B_op
    out = torch.empty((rows, cols), dtype=torch.float32, device=cuda)
    ws = L.workspace(L.query("zg_replay_operands_workspace_size", P, rows, cols, r), cuda)
    L.call("zg_replay_operands", L.ptr(w), L.ptr(A), a_t, L.ptr(B), b_t, P, rows, cols, r,
           _ops.scaled_factor_value(r, 1.0, torch.bfloat16), L.ptr(out), L.ptr(ws), ws.numel(), L.stream_ptr(cuda))
    assert L.load().zg_device_error(1) == 0
    if a_t:
        assert torch.equal(out, direct)  # same weighted operand, same GEMM
    else:
        scale = direct.abs().max().item()
        assert (out - direct).abs().max().item() <= 1e-5 * scale


def test_step_with_per_candidate_hidden_layer(cuda):
    """A two-layer model whose second layer sees a per-candidate input: the
    step reuses the forward's factors in the replay (cache hits for every
    matrix/table entry) and matches a step replayed from fresh draws."""
    import zerograd_b200 as zg

    P, r, B, K, H, V = 24, 8, 64, 128, 256, 200
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w1",), zg.ParameterLayout.MATRIX, "w1"),
                               zg.ManifestEntry(("w2",), zg.ParameterLayout.MATRIX, "w2"),
                               zg.ManifestEntry(("t",), zg.ParameterLayout.TABLE, "t")))
    g = torch.Generator().manual_seed(21)
    params = {"w1": (torch.randn(K, H, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
              "w2": (torch.randn(H, H, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
              "t": (torch.randn(V, H, generator=g) * 0.05).to(torch.bfloat16).to(cuda)}
    x = torch.randn(B, K, generator=g).to(torch.bfloat16).to(cuda)

    def loss_fn(p, ctx, batch, rng):
        h = torch.relu(ctx.linear(p, ("w1",), batch))   # shared input
        h2 = torch.relu(ctx.linear(p, ("w2",), h))      # per-candidate input
        logits = ctx.tied_logits(p, ("t",), h2)         # per-candidate input, tied table
        return (h2.float() ** 2).mean() + (logits.float() ** 2).mean(), None

    opt = zg.ZeroGrad(manifest, zg.sgd(0.1), P, r, 0.02, 0, "batched-step")
    state = opt.init(params)
    _ops.CACHE.clear()
    h0 = _ops.CACHE.hits
    L.profile_begin()
    a, _, ma = opt.step(state, params, x, loss_fn)
    prof = L.profile_end()
    assert "batched_gemm" in prof, prof
    assert _ops.CACHE.hits - h0 == 3  # every entry replayed from the forward's factors
    losses = opt.evaluate_shard(params, 0, loss_fn, x, torch.arange(P, device=cuda))  # device ids: no cache
    b, _, mb = opt.step_from_losses(state, params, losses)
    assert ma == mb
    assert torch.equal(a["w1"], b["w1"]) and torch.equal(a["w2"], b["w2"])
    torch.testing.assert_close(a["t"].float(), b["t"].float(), rtol=0, atol=1e-2 * b["t"].float().abs().max().item())
    assert L.load().zg_device_error(1) == 0

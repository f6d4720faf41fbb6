"""Optimizer step fused into the replay GEMM's epilogue.

The fused form forms the same float32 descent in the epilogue and applies
the same element-wise optax rule, so it must match replay followed by the
stand-alone update kernel bit for bit (torch.equal), for SGD and AdamW, on the
one-SM and the CTA-pair GEMM, with either operand given transposed.
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


def _unfused(w, A, a_t, B, b_t, P, rows, cols, r, inv, dev):
    out = torch.empty((rows, cols), dtype=torch.float32, device=dev)
    ws = L.workspace(L.query("zg_replay_operands_workspace_size", P, rows, cols, r), dev)
    L.call("zg_replay_operands", L.ptr(w), L.ptr(A), a_t, L.ptr(B), b_t, P, rows, cols, r, inv, L.ptr(out),
           L.ptr(ws), ws.numel(), L.stream_ptr(dev))
    return out


# one-SM GEMM / CTA-pair GEMM / the contraction split over 8 candidate groups (P r = 32768)
@pytest.mark.parametrize("rows,cols,P", [(520, 384, 48), (4096, 4096, 256), (640, 384, 4096)])
@pytest.mark.parametrize("layout,transposed", [("matrix", False), ("matrix", True), ("table", True)])
@pytest.mark.parametrize("opt", ["sgd", "adamw"])
def test_fused_step_matches_replay_then_update(cuda, oracle, rows, cols, P, layout, transposed, opt):
    r = 8
    lay = L.ZG_MATRIX if layout == "matrix" else L.ZG_TABLE
    cks = _u32(oracle.candidate_keys(oracle.step_key(9, "fused", 0, 1), range(P)), cuda)
    g = torch.Generator().manual_seed(rows + P)
    w = torch.randn(P, generator=g).to(cuda)
    param = (torch.randn(rows, cols, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    A_op, B_op = _ops.operand_factors(cks, 1, lay, rows, cols, r)
    a_t = int(transposed and lay == L.ZG_MATRIX)
    b_t = int(transposed and lay == L.ZG_TABLE)
    A = A_op.t().contiguous() if a_t else A_op
    B = B_op.t().contiguous() if b_t else B_op
    inv = _ops.scaled_factor_value(r, 1.0, torch.bfloat16)
    d = _unfused(w, A, a_t, B, b_t, P, rows, cols, r, inv, cuda)
    ws = L.workspace(L.query("zg_replay_operands_workspace_size", P, rows, cols, r), cuda)
    new = torch.empty_like(param)
    d2 = torch.empty_like(d)
    st = L.stream_ptr(cuda)
    if opt == "sgd":
        want = _ops.launch_sgd(param, d, 0.05)
        L.call("zg_replay_sgd", L.ptr(w), L.ptr(A), a_t, L.ptr(B), b_t, P, rows, cols, r, inv, L.ptr(param),
               L.ptr(new), L.ZG_BF16, 0.05, L.ptr(d2), None, L.ptr(ws), ws.numel(), st)
        assert torch.equal(new, want)
    else:
        mu = torch.randn(rows, cols, generator=g).to(cuda) * 1e-3
        nu = torch.rand(rows, cols, generator=g).to(cuda) * 1e-4
        want, wm, wv = _ops.launch_adamw(param, d, mu, nu, 3, 1e-3, 0.9, 0.999, 1e-8, 1e-4)
        mo, vo = torch.empty_like(mu), torch.empty_like(nu)
        L.call("zg_replay_adamw", L.ptr(w), L.ptr(A), a_t, L.ptr(B), b_t, P, rows, cols, r, inv, L.ptr(param),
               L.ptr(new), L.ZG_BF16, L.ptr(mu), L.ptr(nu), L.ptr(mo), L.ptr(vo), 3, 1e-3, 0.9, 0.999, 1e-8, 1e-4,
               L.ptr(d2), None, None, L.ptr(ws), ws.numel(), st)
        assert torch.equal(new, want) and torch.equal(mo, wm) and torch.equal(vo, wv)
    assert torch.equal(d2, d)  # the optional descent output is the unfused replay's
    assert L.load().zg_device_error(1) == 0


@pytest.mark.parametrize("transform", [zg.sgd(0.05), zg.adamw(1e-3)])
def test_step_uses_fused_replay_and_matches_separate_update(cuda, transform):
    """ZeroGrad.step takes the fused path for bf16 MATRIX/TABLE leaves (no
    stand-alone update launch for them) and lands on exactly the parameters
    and optimizer state of replay + separate update."""
    from zerograd_b200._replay import replay_entry_keys
    from zerograd_b200._transforms import tree_set

    P, r, B, K, N, V = 32, 8, 64, 256, 128, 200
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),
                               zg.ManifestEntry(("t",), zg.ParameterLayout.TABLE, "t"),
                               zg.ManifestEntry(("b",), zg.ParameterLayout.VECTOR, "b")))
    g = torch.Generator().manual_seed(17)
    params = {"w": (torch.randn(K, N, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
              "t": (torch.randn(V, N, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
              "b": torch.zeros(N, dtype=torch.bfloat16, device=cuda)}
    x = torch.randn(B, K, generator=g).to(torch.bfloat16).to(cuda)

    def loss_fn(p, ctx, batch, rng):
        h = ctx.linear(p, ("w",), batch) + ctx.vector(p, ("b",))
        logits = ctx.tied_logits(p, ("t",), h)
        return (logits.float() ** 2).mean(), None

    opt = zg.ZeroGrad(manifest, transform, P, r, 0.02, 0, "fused-step")
    state = opt.init(params)
    L.profile_begin()
    a, sa, _ = opt.step(state, params, x, loss_fn)
    prof = L.profile_end()
    # the two bf16 matrix/table leaves were stepped inside their replay GEMMs
    stand_alone = prof.get("sgd_update", (0, 0))[0] + prof.get("adamw_update", (0, 0))[0]
    assert stand_alone == 1, prof  # only the VECTOR leaf

    # the same generation, replayed and updated separately
    losses = opt.evaluate_shard(params, 0, loss_fn, x, torch.arange(P, device=cuda))
    shaped, _ = _ops.launch_shape_fitness(losses, 0.02)
    from zerograd_b200._replay import candidate_keys
    cks = candidate_keys(opt.base_key(0), torch.arange(P, dtype=torch.int32, device=cuda))
    descent: dict = {}
    for entry in manifest.entries:
        tree_set(descent, entry.path, replay_entry_keys(params, manifest, entry.path, cks, shaped, r))
    b, sb = transform.apply(params, descent, state.opt_state)
    for k in params:
        assert torch.equal(a[k], b[k]), k
    if isinstance(transform, zg.adamw):
        for k in params:
            assert torch.equal(sa.opt_state.mu[k], sb.mu[k]) and torch.equal(sa.opt_state.nu[k], sb.nu[k]), k
    assert L.load().zg_device_error(1) == 0


@pytest.mark.parametrize("rows,cols,P", [(520, 384, 48), (4096, 4096, 256)])
@pytest.mark.parametrize("opt", ["sgd", "adamw"])
def test_inplace_guarded_step(cuda, oracle, rows, cols, P, opt):
    """In place with the guard at zero: the out-of-place step's bits; with the
    guard set: nothing written (parameters and moments untouched)."""
    r = 8
    cks = _u32(oracle.candidate_keys(oracle.step_key(5, "guard", 0, 1), range(P)), cuda)
    g = torch.Generator().manual_seed(rows * 3 + P)
    w = torch.randn(P, generator=g).to(cuda)
    param = (torch.randn(rows, cols, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    spec = {"kind": "sgd", "lr": 0.05}
    if opt == "adamw":
        spec = {"kind": "adamw", "lr": 1e-3, "b1": 0.9, "b2": 0.999, "eps": 1e-8, "weight_decay": 1e-4, "count": 2,
                "mu": torch.randn(rows, cols, generator=g).to(cuda) * 1e-3,
                "nu": torch.rand(rows, cols, generator=g).to(cuda) * 1e-4}
    want = _ops.launch_replay_step(w, cks, 0, L.ZG_MATRIX, param, r, spec)
    for flag, writes in ((0.0, True), (3.0, False)):
        p2 = param.clone()
        s2 = dict(spec)
        if opt == "adamw":
            s2["mu"], s2["nu"] = spec["mu"].clone(), spec["nu"].clone()
        got = _ops.launch_replay_step(w, cks, 0, L.ZG_MATRIX, p2, r, s2,
                                      inplace_guard=torch.tensor([flag], device=cuda))
        assert got[0] is p2
        if writes:
            assert torch.equal(p2, want[0])
            if opt == "adamw":
                assert torch.equal(s2["mu"], want[1]) and torch.equal(s2["nu"], want[2])
        else:
            assert torch.equal(p2, param)
            if opt == "adamw":
                assert torch.equal(s2["mu"], spec["mu"]) and torch.equal(s2["nu"], spec["nu"])
    assert L.load().zg_device_error(1) == 0

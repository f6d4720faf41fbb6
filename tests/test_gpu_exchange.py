"""The exchanged update with its ranks emulated on one GPU: every rank's
partial replays from its own candidates' factors (zg_replay_partials), the
all-to-all done by copying chunks, each rank's fixed-order sum and SGD step
(zg_replay_split_sgd), the chunks concatenated as the all-gather would.
The result must be the one-GPU update bit for bit, for 2, 4 and 8 ranks,
from freshly drawn factors and from the factors a per-candidate-input
forward kept (the transposed operand layouts)."""
import ctypes

import pytest
import torch

import zerograd_b200 as zg
from zerograd_b200 import _lib as L
from zerograd_b200 import _ops
from zerograd_b200._exchange import ExchangedReplay

pytestmark = pytest.mark.gpu

P, RANK = 2048, 16  # 8 candidate groups of 4096 contraction columns


def _manifest(names_layouts):
    return zg.Manifest(1, tuple(zg.ManifestEntry((n,), lay, n) for n, lay in names_layouts))


def _emulate(opt, params, losses, world, forward=None):
    """New parameters of the exchanged entries, ranks run in turn.
    `forward(rank_range)`: runs that rank's forward first (its factors stay
    in the cache for its contraction)."""
    dev = losses.device
    state = opt.init(params)
    shaped, _ = _ops.launch_shape_fitness(losses, opt.sigma)
    base = tuple(int(v) for v in opt.base_key(0))
    cks = opt._candidate_keys_range(0, 0, P, dev)
    gen = _ops._Generation(base, 0, P, cks)
    n = P // world
    exs = [ExchangedReplay(r, world, r * n, n) for r in range(world)]
    parts, works, layout, paths = [], [], None, None
    for ex in exs:
        if forward is not None:
            forward(range(ex.start, ex.start + n))
        work = opt._exchange_work(state, params, ex, gen, cks)
        assert work, "the exchanged update does not apply"
        paths = [w[0] for w in work]
        w = [(p, ops, lr) for _, p, ops, lr in work]
        layout, pr = ex.contract(w, shaped, P, RANK)
        parts.append(pr)
        works.append(w)
        _ops.CACHE.drop_generation(base)
    S = exs[0].split_count(P, RANK)
    assert S == 8
    per, c = S // world, layout.chunk
    inv = _ops.scaled_factor_value(RANK, 1.0, torch.bfloat16)
    chunks = []
    for j, ex in enumerate(exs):
        recv = torch.empty_like(parts[0])
        for i in range(per):
            for src in range(world):
                recv[i, src * c:(src + 1) * c] = parts[src][i, j * c:(j + 1) * c]
        chunks.append(ex.step_owned(works[j], layout, recv, S, inv, None))
    gathered = torch.cat(chunks)
    return {p[0]: gathered[off:off + t.numel()].view(t.shape)
            for p, (t, _, _), off in zip(paths, works[0], layout.offsets)}


@pytest.mark.parametrize("world", [2, 4, 8])
def test_exchange_matches_one_gpu_drawn_factors(cuda, world):
    man = _manifest([("w", zg.ParameterLayout.MATRIX), ("t", zg.ParameterLayout.TABLE),
                     ("b", zg.ParameterLayout.VECTOR)])
    g = torch.Generator().manual_seed(world)
    params = {"w": (torch.randn(384, 256, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
              "t": (torch.randn(1024, 128, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
              "b": torch.zeros(256, dtype=torch.bfloat16, device=cuda)}
    opt = zg.ZeroGrad(man, zg.sgd(0.5), P, RANK, 0.02, 1, "exchange")
    losses = torch.randn(P, generator=g).to(cuda)
    whole, _, _ = opt._complete(opt.init(params), params, losses)
    got = _emulate(opt, params, losses, world)
    assert set(got) == {"w", "t"}
    for k, v in got.items():
        assert torch.equal(v, whole[k]), k
        assert not torch.equal(v, params[k]), k  # the step moved it
    assert L.load().zg_device_error(1) == 0


@pytest.mark.parametrize("world", [2, 8])
def test_exchange_matches_one_gpu_forward_factors(cuda, world):
    """A shared-input linear then a per-candidate-input one: the second
    keeps its factors transposed (F1T, F2), the exchange contracts them."""
    man = _manifest([("w1", zg.ParameterLayout.MATRIX), ("w2", zg.ParameterLayout.MATRIX)])
    g = torch.Generator().manual_seed(100 + world)
    params = {"w1": (torch.randn(256, 384, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
              "w2": (torch.randn(384, 128, generator=g) * 0.05).to(torch.bfloat16).to(cuda)}
    x = torch.randn(64, 256, generator=g).to(torch.bfloat16).to(cuda)
    opt = zg.ZeroGrad(man, zg.sgd(0.5), P, RANK, 0.02, 1, "exchange-t")

    def loss_fn(p, ctx, batch, rng):
        h = ctx.linear(p, ("w1",), batch)
        return (ctx.linear(p, ("w2",), h).float() ** 2).mean(), None

    state = opt.init(params)
    losses = opt.evaluate_shard(params, 0, loss_fn, x, range(P))
    whole, _, _ = opt._complete(state, params, losses)
    got = _emulate(opt, params, losses, world,
                   forward=lambda ids: opt.evaluate_shard(params, 0, loss_fn, x, ids))
    for k, v in got.items():
        assert torch.equal(v, whole[k]), k
    assert L.load().zg_device_error(1) == 0


def test_split_sum_gives_the_replay_and_sgd_is_guarded(cuda):
    """zg_replay_split_sum over all groups' partials is zg_replay_operands'
    descent; zg_replay_split_sgd writes nothing when the guard is set."""
    rows, cols = 320, 192
    g = torch.Generator().manual_seed(7)
    keys = _ops.launch_fold_in(torch.tensor([[3, 4]], dtype=torch.uint32).to(cuda),
                               torch.arange(P, dtype=torch.int32, device=cuda))
    A, B = _ops.operand_factors(keys, 0, L.ZG_MATRIX, rows, cols, RANK)
    w = torch.randn(P, generator=g).to(cuda)
    inv = _ops.scaled_factor_value(RANK, 1.0, torch.bfloat16)
    out = torch.empty(rows, cols, dtype=torch.float32, device=cuda)
    ws = L.workspace(L.query("zg_replay_operands_workspace_size", P, rows, cols, RANK), cuda)
    L.call("zg_replay_operands", L.ptr(w), L.ptr(A), 0, L.ptr(B), 0, P, rows, cols, RANK, inv, L.ptr(out), L.ptr(ws),
           ws.numel(), L.stream_ptr(cuda))
    S = int(L.load().zg_replay_split_count(P, RANK))
    parts = torch.empty(S, rows * cols, dtype=torch.float32, device=cuda)
    ws2 = L.workspace(L.query("zg_replay_partials_workspace_size", P, rows, cols, RANK), cuda)
    L.call("zg_replay_partials", L.ptr(w), L.ptr(A), 0, L.ptr(B), 0, P, rows, cols, RANK, S, S, L.ptr(parts),
           rows * cols, L.ptr(ws2), ws2.numel(), L.stream_ptr(cuda))
    offs = (ctypes.c_int64 * S)(*[s * rows * cols for s in range(S)])
    summed = torch.empty_like(out)
    L.call("zg_replay_split_sum", L.ptr(parts), ctypes.addressof(offs), S, rows * cols, inv, L.ptr(summed),
           L.stream_ptr(cuda))
    assert torch.equal(summed, out)
    param = (torch.randn(rows, cols, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    dst = torch.full_like(param, 7.0)
    guard = torch.ones(1, dtype=torch.float32, device=cuda)
    L.call("zg_replay_split_sgd", L.ptr(parts), ctypes.addressof(offs), S, rows * cols, inv, L.ptr(param), L.ptr(dst),
           L.ZG_BF16, 0.5, L.ptr(guard), L.stream_ptr(cuda))
    assert torch.equal(dst, torch.full_like(param, 7.0))
    guard.zero_()
    L.call("zg_replay_split_sgd", L.ptr(parts), ctypes.addressof(offs), S, rows * cols, inv, L.ptr(param), L.ptr(dst),
           L.ZG_BF16, 0.5, L.ptr(guard), L.stream_ptr(cuda))
    want_p = (param.float() + (-0.5) * (-out)).to(torch.bfloat16)
    assert torch.equal(dst, want_p)
    assert L.load().zg_device_error(1) == 0

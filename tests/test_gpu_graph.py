"""A generation captured as a CUDA graph (ZeroGrad.capture) against the eager
ZeroGrad.step of the same generations: bit-identical parameters and equal
metrics; a generation with non-finite losses raises and leaves the captured
parameters untouched."""
import pytest
import torch

import zerograd_b200 as zg
from zerograd_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _small(dev):
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),
                               zg.ManifestEntry(("b",), zg.ParameterLayout.VECTOR, "b")))
    g = torch.Generator().manual_seed(3)
    params = {"w": (torch.randn(256, 128, generator=g) * 0.05).to(torch.bfloat16).to(dev),
              "b": (torch.randn(128, generator=g) * 0.01).to(torch.bfloat16).to(dev)}
    batches = [torch.randn(64, 256, generator=g).to(torch.bfloat16).to(dev) for _ in range(4)]

    def loss_fn(p, ctx, batch, rng):
        y = ctx.linear(p, ("w",), batch) + ctx.vector(p, ("b",))
        return (y.float() ** 2).mean(), None

    return manifest, params, batches, loss_fn


def test_captured_generations_match_eager(cuda):
    manifest, params, batches, loss_fn = _small(cuda)
    opt = zg.ZeroGrad(manifest, zg.sgd(0.05), 48, 8, 0.02, 0, "graph")
    cg = opt.capture(params, loss_fn, batches[0])
    pe, se = params, opt.init(params)
    sc = opt.init(params)
    n0 = L.launch_count()
    for g in range(4):
        pe, se, me = opt.step(se, pe, batches[g], loss_fn)
        pc, sc, mc = cg.step(sc, batches[g])
        assert sc.generation == se.generation == g + 1
        for k in pe:
            assert torch.equal(pc[k], pe[k]), (g, k)
        assert (mc.mean_loss, mc.min_loss, mc.max_loss) == (me.mean_loss, me.min_loss, me.max_loss)
    assert L.load().zg_device_error(1) == 0
    assert L.launch_count() > n0


def test_captured_generation_rejects_nonfinite_losses(cuda):
    manifest, params, batches, loss_fn = _small(cuda)
    opt = zg.ZeroGrad(manifest, zg.sgd(0.05), 32, 8, 0.02, 1, "graph-nan")
    cg = opt.capture(params, loss_fn, batches[0])
    state = opt.init(params)
    _, state, _ = cg.step(state, batches[1])
    before = {k: v.clone() for k, v in cg.params.items()}
    bad = batches[2].clone()
    bad[5, 7] = float("nan")
    with pytest.raises(ValueError, match="finite"):
        cg.step(state, bad)
    for k in before:
        assert torch.equal(cg.params[k], before[k])
    # the next good generation proceeds from the unchanged parameters
    pc, _, m = cg.step(state, batches[3])
    pe, _, me = opt.step(state, before, batches[3], loss_fn)
    for k in pe:
        assert torch.equal(pc[k], pe[k])


def test_captured_bench_generation(cuda):
    """The perturbed-GEMM generation (P=256, rank 8, shared x[256,4096],
    W[4096,4096] bf16, SGD) with a one-element loss per candidate."""
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),))
    g = torch.Generator(device=cuda).manual_seed(0)
    W = (torch.randn(4096, 4096, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    xs = [(torch.randn(256, 4096, generator=g, device=cuda) * 0.02).to(torch.bfloat16) for _ in range(2)]

    def loss_fn(p, ctx, batch, rng):
        y = ctx.linear(p, ("w",), batch)
        return y[0, 0].float(), None

    opt = zg.ZeroGrad(manifest, zg.sgd(1e-3), 256, 8, 0.01, 0, "bench")
    cg = opt.capture({"w": W}, loss_fn, xs[0])
    pe, se = {"w": W}, opt.init({"w": W})
    sc = se
    for i in range(2):
        pe, se, me = opt.step(se, pe, xs[i], loss_fn)
        pc, sc, mc = cg.step(sc, xs[i])
        assert torch.equal(pc["w"], pe["w"])
        assert mc.mean_loss == me.mean_loss
    assert L.load().zg_device_error(1) == 0


def test_enqueued_generations_match_eager(cuda):
    """Generations queued back to back; a non-finite one in the middle is
    rejected (its result raises) and the next starts from unchanged params."""
    manifest, params, batches, loss_fn = _small(cuda)
    opt = zg.ZeroGrad(manifest, zg.sgd(0.05), 48, 8, 0.02, 2, "graph-queue")
    cg = opt.capture(params, loss_fn, batches[0])
    bad = batches[2].clone()
    bad[0, 0] = float("inf")
    seq = [batches[0], batches[1], bad, batches[3]]
    state = opt.init(params)
    pending = []
    for b in seq:
        _, state, p = cg.enqueue(state, b)
        pending.append(p)
    got = cg.params
    pe, se = params, opt.init(params)
    for i, b in enumerate(seq):
        if i == 2:
            with pytest.raises(ValueError, match="finite"):
                pending[i].result()
            se = zg.ZeroGradState(se.generation + 1, se.opt_state)  # the queue moved on a generation
            continue
        pe, se, me = opt.step(se, pe, b, loss_fn)
        assert pending[i].result().mean_loss == me.mean_loss
    for k in pe:
        assert torch.equal(got[k], pe[k])


@pytest.mark.parametrize("nbytes,offset", [(4096 * 4096 * 2, 0), (1001, 0), (4099, 3)])
def test_copy_if_zero(cuda, nbytes, offset):
    from zerograd_b200 import _ops

    src = torch.randint(0, 255, (nbytes + offset,), dtype=torch.uint8, device=cuda)[offset:]
    for flag, copies in ((0.0, True), (2.0, False), (float("nan"), False)):
        dst = torch.zeros(nbytes + offset, dtype=torch.uint8, device=cuda)[offset:]
        _ops.launch_copy_if_zero(dst, src, torch.tensor([flag], device=cuda))
        assert torch.equal(dst, src) == copies
        if not copies:
            assert int(dst.sum()) == 0


def test_captured_adamw_matches_eager(cuda):
    """AdamW: the bias corrections of each step come from a device buffer the
    host fills before the replay; parameters and both moments bit-identical
    to the eager steps, and untouched by a generation with non-finite losses."""
    manifest, params, batches, loss_fn = _small(cuda)
    opt = zg.ZeroGrad(manifest, zg.adamw(3e-3), 48, 8, 0.02, 4, "graph-adamw")
    cg = opt.capture(params, loss_fn, batches[0])
    pe, se = params, opt.init(params)
    sc = opt.init(params)
    for g in range(4):
        pe, se, me = opt.step(se, pe, batches[g], loss_fn)
        pc, sc, mc = cg.step(sc, batches[g])
        assert sc.opt_state.count == se.opt_state.count == g + 1
        for k in pe:
            assert torch.equal(pc[k], pe[k]), (g, k)
            assert torch.equal(cg.opt_state.mu[k], se.opt_state.mu[k]), (g, k)
            assert torch.equal(cg.opt_state.nu[k], se.opt_state.nu[k]), (g, k)
        assert mc.mean_loss == me.mean_loss
    before = ({k: v.clone() for k, v in cg.params.items()}, {k: v.clone() for k, v in cg.opt_state.mu.items()})
    bad = batches[1].clone()
    bad[0, 3] = float("nan")
    with pytest.raises(ValueError, match="finite"):
        cg.step(sc, bad)
    for k in before[0]:
        assert torch.equal(cg.params[k], before[0][k]) and torch.equal(cg.opt_state.mu[k], before[1][k])
    assert L.load().zg_device_error(1) == 0


@pytest.mark.parametrize("slots,transform", [(2, "sgd"), (1, "sgd"), (2, "adamw")])
def test_enqueued_host_batches_match_eager(cuda, slots, transform):
    """Batches from pinned host memory, queued back to back: with two slots
    the copies of generation g+1 run on the copy stream while generation g
    computes; every generation's parameters and metrics are those of the
    eager steps on the same batches."""
    manifest, params, _, loss_fn = _small(cuda)
    g = torch.Generator().manual_seed(17)
    host = [torch.randn(64, 256, generator=g).to(torch.bfloat16).pin_memory() for _ in range(7)]
    tf = zg.sgd(0.05) if transform == "sgd" else zg.adamw(3e-3)
    opt = zg.ZeroGrad(manifest, tf, 48, 8, 0.02, 5, "graph-host")
    cg = opt.capture(params, loss_fn, host[0].to(cuda), slots=slots)
    state = opt.init(params)
    pending, snaps = [], []
    for i, b in enumerate(host):
        _, state, p = cg.enqueue(state, b)
        pending.append(p)
        if i >= 1:
            pending[i - 1].result()  # the previous generation's metrics, read while this one runs
        snaps.append({k: v.clone() for k, v in cg.params.items()})  # ordered after this replay
    pe, se = params, opt.init(params)
    for i, b in enumerate(host):
        pe, se, me = opt.step(se, pe, b.to(cuda), loss_fn)
        assert pending[i].result().mean_loss == me.mean_loss, i
        for k in pe:
            assert torch.equal(snaps[i][k], pe[k]), (i, k)
    assert state.generation == len(host)
    assert L.load().zg_device_error(1) == 0


def test_draw_ahead_out_of_sequence_generations(cuda):
    """Factors drawn one generation ahead are used only for the generation
    they were drawn for: generations called out of sequence (a restart, a
    jump back) draw their own first; every step matches the eager one."""
    manifest, params, batches, loss_fn = _small(cuda)
    opt = zg.ZeroGrad(manifest, zg.sgd(0.05), 48, 8, 0.02, 6, "graph-ahead")
    cg = opt.capture(params, loss_fn, batches[0])
    assert cg._entries, "the bf16 MATRIX leaf is drawn ahead"
    pe = params
    sc = opt.init(params)
    for gen in (0, 1, 2, 7, 8, 3, 3, 9):
        b = batches[gen % 4]
        pe, se, me = opt.step(zg.ZeroGradState(gen, sc.opt_state), pe, b, loss_fn)
        pc, sc, mc = cg.step(zg.ZeroGradState(gen, sc.opt_state), b)
        assert mc.mean_loss == me.mean_loss, gen
        for k in pe:
            assert torch.equal(pc[k], pe[k]), (gen, k)
    assert L.load().zg_device_error(1) == 0


def test_draw_ahead_tied_table(cuda):
    """A tied embedding TABLE (lookup + tied logits) and a MATRIX leaf, both
    drawn ahead, against the eager steps."""
    V, C, B, T = 512, 128, 2, 16
    manifest = zg.Manifest(1, (zg.ManifestEntry(("emb",), zg.ParameterLayout.TABLE, "emb"),
                               zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w")))
    g = torch.Generator().manual_seed(9)
    params = {"emb": (torch.randn(V, C, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
              "w": (torch.randn(C, C, generator=g) * 0.05).to(torch.bfloat16).to(cuda)}
    toks = [torch.randint(0, V, (B, T), generator=g).to(cuda) for _ in range(3)]

    def loss_fn(p, ctx, batch, rng):
        h = ctx.table_lookup(p, ("emb",), batch)
        h = ctx.linear(p, ("w",), h)
        logits = ctx.tied_logits(p, ("emb",), h)
        return (logits.float() ** 2).mean(), None

    opt = zg.ZeroGrad(manifest, zg.sgd(0.02), 32, 8, 0.02, 8, "graph-table")
    cg = opt.capture(params, loss_fn, toks[0])
    assert len(cg._entries) == 2
    pe, se = params, opt.init(params)
    sc = opt.init(params)
    for i in range(3):
        pe, se, me = opt.step(se, pe, toks[i], loss_fn)
        pc, sc, mc = cg.step(sc, toks[i])
        assert mc.mean_loss == me.mean_loss, i
        for k in pe:
            assert torch.equal(pc[k], pe[k]), (i, k)
    assert L.load().zg_device_error(1) == 0

"""DistributedZeroGrad with one process per GPU (NCCL): population shards,
fitness all-gather, replicated replay.  Every rank must end with bit-identical
parameters, equal (float tolerance) to a single-process step.  Needs >= 2 GPUs.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _problem(dev):
    import zerograd_b200 as zg

    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),
                               zg.ManifestEntry(("b",), zg.ParameterLayout.VECTOR, "b")))
    g = torch.Generator().manual_seed(0)
    params = {"w": (torch.randn(256, 128, generator=g) * 0.05).to(torch.bfloat16).to(dev),
              "b": torch.zeros(128, dtype=torch.bfloat16).to(dev)}
    x = torch.randn(64, 256, generator=g).to(torch.bfloat16).to(dev)

    def loss_fn(p, ctx, batch, rng):
        y = ctx.linear(p, ("w",), batch) + ctx.vector(p, ("b",))
        return (y.float() ** 2).mean(), None

    opt = zg.ZeroGrad(manifest, zg.adamw(1e-3), 48, 8, 0.02, 0, "multi")
    return opt, params, x, loss_fn


def _worker(rank, port, q):
    import datetime

    import torch.distributed as dist

    import zerograd_b200 as zg

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        opt, params, x, loss_fn = _problem(dev)
        state = opt.init(params)
        dz = zg.DistributedZeroGrad(opt, None, loss_fn, weights=[1.0, 2.0])
        for _ in range(2):
            params, state, metrics = dz.step(state, params, x)
        q.put((rank, {k: v.float().cpu() for k, v in params.items()}, dz.partition_sizes, metrics.mean_loss))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_process_group_matches_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = sorted([q.get(timeout=300) for _ in procs], key=lambda t: t[0])
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    (_, p0, sizes, m0), (_, p1, _, m1) = out
    assert sizes == [16, 32]
    for k in p0:
        assert torch.equal(p0[k], p1[k]), k  # replicated replay: identical on every rank
    # single process, same generations
    dev = torch.device("cuda", 0)
    opt, params, x, loss_fn = _problem(dev)
    state = opt.init(params)
    for _ in range(2):
        params, state, metrics = opt.step(state, params, x, loss_fn)
    for k in p0:
        torch.testing.assert_close(p0[k], params[k].float().cpu(), rtol=1e-2, atol=1e-2)
    assert m0 == m1


def _worker_captured(rank, port, q):
    import datetime

    import torch.distributed as dist

    import zerograd_b200 as zg

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        opt, params, x, loss_fn = _problem(dev)
        opt = zg.ZeroGrad(opt.manifest, zg.sgd(0.05), 48, 8, 0.02, 0, "multi-graph")
        dz = zg.DistributedZeroGrad(opt, None, loss_fn, weights=[1.0, 2.0])
        cg = dz.capture(params, x)
        pe, se = params, opt.init(params)
        sc = opt.init(params)
        same = True
        for g in range(3):
            xg = x * (1.0 + 0.25 * g)
            pe, se, me = dz.step(se, pe, xg)
            pc, sc, mc = cg.step(sc, xg)
            same = same and all(torch.equal(pc[k], pe[k]) for k in pe) and mc.mean_loss == me.mean_loss
        q.put((rank, same, {k: v.float().cpu() for k, v in pc.items()}))
        del cg  # the graph holds NCCL work: released before the process group
        torch.cuda.synchronize()
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_captured_process_group_generation():
    """Each rank captures its shard's forward, the NCCL fitness all-gather and
    the replicated completion; replays match the eager steps bit for bit."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_captured, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = sorted([q.get(timeout=300) for _ in procs], key=lambda t: t[0])
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    (_, same0, p0), (_, same1, p1) = out
    assert same0 and same1
    for k in p0:
        assert torch.equal(p0[k], p1[k]), k


def _worker_exchanged(rank, port, q):
    import datetime

    import torch.distributed as dist

    import zerograd_b200 as zg

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        opt0, params0, x, loss_fn = _problem(dev)
        # P r = 32768: 8 candidate groups, 4 per rank
        opt = zg.ZeroGrad(opt0.manifest, zg.sgd(0.05), 2048, 16, 0.02, 0, "multi-exchange")
        rep = zg.DistributedZeroGrad(opt, None, loss_fn)
        sh = zg.DistributedZeroGrad(opt, None, loss_fn, replay="sharded")
        cg = sh.capture(params0, x)
        pr, sr = params0, opt.init(params0)
        ps, ss = params0, opt.init(params0)
        sc = opt.init(params0)
        same_graph = True
        for g in range(3):
            xg = x * (1.0 + 0.25 * g)
            pr, sr, mr = rep.step(sr, pr, xg)
            ps, ss, ms = sh.step(ss, ps, xg)
            pc, sc, mc = cg.step(sc, xg)
            same_graph = same_graph and all(torch.equal(pc[k], ps[k]) for k in ps) and mc.mean_loss == ms.mean_loss
        q.put((rank, same_graph, {k: v.float().cpu() for k, v in ps.items()},
               {k: v.float().cpu() for k, v in pr.items()}))
        del cg  # the graph holds NCCL work: released before the process group
        torch.cuda.synchronize()
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_exchanged_update_matches_replicated():
    """Exchanged update (each rank contracts its own candidates' factors,
    partials all-to-all, fixed-order sums, parameters all-gathered): every
    rank ends with the bits of the replicated update, eager and captured."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_exchanged, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = sorted([q.get(timeout=300) for _ in procs], key=lambda t: t[0])
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    (_, g0, s0, r0), (_, g1, s1, r1) = out
    assert g0 and g1
    for k in s0:
        assert torch.equal(s0[k], s1[k]), k
        assert torch.equal(s0[k], r0[k]), k
        assert torch.equal(r0[k], r1[k]), k

"""Host side of the exchanged update, on CPU: the flat layout of the
entries, each rank's owned segments, where every candidate group's partial
lands after the all-to-all (world-size 2 and 4 gloo ranks), and the
all-gather of the new parameters."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from zerograd_b200._exchange import ALIGN, ExchangedReplay, flat_layout, group_offsets, owned_segments

NUMELS = (37, 64, 5, 130, 8)


def test_flat_layout_aligns_and_pads():
    lay = flat_layout(NUMELS, 4)
    assert lay.offsets == (0, 40, 104, 112, 248)
    assert all(o % ALIGN == 0 for o in lay.offsets)
    assert lay.chunk % ALIGN == 0 and lay.total >= lay.offsets[-1] + NUMELS[-1]
    assert lay.chunk == 64  # 256 placed elements over 4 ranks


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_owned_segments_cover_every_element_once(world):
    lay = flat_layout(NUMELS, world)
    seen = {i: [] for i in range(len(NUMELS))}
    for r in range(world):
        for i, a, b in owned_segments(lay, r):
            assert r * lay.chunk <= a < b <= (r + 1) * lay.chunk
            assert (a - r * lay.chunk) % ALIGN == 0 and (a - lay.offsets[i]) % ALIGN == 0
            seen[i].append((a, b))
    for i, segs in seen.items():
        covered = sorted(segs)
        assert covered[0][0] == lay.offsets[i] and covered[-1][1] == lay.offsets[i] + NUMELS[i]
        for (_, b0), (a1, _) in zip(covered, covered[1:]):
            assert b0 == a1


def test_group_offsets_order():
    lay = flat_layout(NUMELS, 2)
    # S = 8 over 2 ranks: groups 0-3 from rank 0 (all-to-alls 0-3), 4-7 from rank 1
    offs = group_offsets(8, lay, 5)
    assert offs == [i * lay.total + 5 for i in range(4)] + [i * lay.total + lay.chunk + 5 for i in range(4)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        S = 8
        per = S // world
        lay = flat_layout(NUMELS, world)
        ex = ExchangedReplay(rank, world, 0, 0)
        # this rank's local groups: global group rank * per + i, value 1000 g + flat index
        parts = torch.empty((per, lay.total), dtype=torch.float32)
        for i in range(per):
            g = rank * per + i
            parts[i] = 1000.0 * g + torch.arange(lay.total, dtype=torch.float32)
        recv = ex.exchange(parts).reshape(-1)
        ok = True
        lo = rank * lay.chunk
        for _, a, b in owned_segments(lay, rank):
            offs = group_offsets(S, lay, a - lo)
            for s in range(S):
                got = recv[offs[s]:offs[s] + (b - a)]
                want = 1000.0 * s + torch.arange(a, b, dtype=torch.float32)
                ok = ok and torch.equal(got, want)
        mine = torch.full((lay.chunk,), float(rank + 1), dtype=torch.bfloat16)
        work = [(torch.empty(n, dtype=torch.bfloat16), None, 0.0) for n in NUMELS]
        views = ex.gather(work, lay, mine)
        owners = []
        for v, off in zip(views, lay.offsets):
            owner = torch.tensor([(off + k) // lay.chunk + 1 for k in range(v.numel())], dtype=torch.bfloat16)
            ok = ok and torch.equal(v, owner)
            owners.append(v.shape == (v.numel(),))
        q.put((rank, ok, all(owners)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_all_to_all_delivers_every_group_in_order(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for rank, ok, shapes in out:
        assert ok and shapes, rank


def test_exchange_applies_only_to_whole_candidate_groups():
    """The exchanged update needs the population split into groups the ranks
    hold whole (zg_replay_split_count(P, r) a multiple of the world size,
    equal consecutive shards); otherwise the replicated update runs."""
    from zerograd_b200 import _lib as L

    lib = L.load()
    assert lib.zg_replay_split_count(2048, 16) == 8
    assert lib.zg_replay_split_count(256, 8) == 1  # 2048 contraction columns: too short to split
    assert lib.zg_replay_split_count(1024, 16) == 4
    for world in (2, 4, 8):
        n = 2048 // world
        assert all(ExchangedReplay(r, world, r * n, n).applies(2048, 16) for r in range(world))
    assert not ExchangedReplay(0, 3, 0, 683).applies(2048, 16)      # 8 groups do not split over 3 ranks
    assert not ExchangedReplay(1, 2, 1000, 1048).applies(2048, 16)  # uneven shards
    assert not ExchangedReplay(0, 2, 0, 128).applies(256, 8)        # one group only
    assert not ExchangedReplay(0, 8, 0, 128).applies(1024, 16)      # 4 groups over 8 ranks
    assert not ExchangedReplay(0, 1, 0, 2048).applies(2048, 16)     # one process: the plain replay

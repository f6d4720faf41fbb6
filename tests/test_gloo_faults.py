"""Rank failures around the collectives of a generation, on CPU gloo ranks
(no GPU is faulted): a rank that dies or raises before the fitness
all-gather, or dies before the exchanged update's all-to-all of partial
replays, makes the survivor's collective end with an error within the
process group's short timeout, instead of hanging; the survivor then leaves
without touching the group again."""
import datetime
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import zerograd_b200 as zg


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _leave(q, code):
    q.close()
    q.join_thread()  # the message is written before the process ends
    os._exit(code)


def _worker(rank, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        if mode in ("exit", "exit_exchange"):
            os._exit(0)  # dies without joining the collective
        try:
            raise RuntimeError("loss function failed on this rank")
        except RuntimeError as e:
            q.put((rank, "raised", str(e)))
            _leave(q, 1)  # a failed rank leaves; it does not join the collective
    t0 = time.monotonic()
    try:
        if mode == "exit_exchange":
            # the exchanged update's partial-replay all-to-all
            from zerograd_b200._exchange import ExchangedReplay

            ExchangedReplay(rank, 2, 0, 0).exchange(torch.ones(1, 16))
        else:
            zg.allgather_losses(torch.ones(3), [3, 3])
        q.put((rank, "completed", time.monotonic() - t0))
    except Exception as e:  # the collective reports the lost peer
        q.put((rank, "error", type(e).__name__, time.monotonic() - t0))
    _leave(q, 0)


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.monotonic() + 90
    while len(out) < (2 if mode == "raise" else 1) and time.monotonic() < deadline:
        try:
            item = q.get(timeout=5)
        except Exception:
            continue
        out[item[0]] = item[1:]
    for p in procs:
        p.join(30)
        if p.is_alive():
            p.kill()
    return out


def test_dead_rank_ends_the_allgather_with_an_error():
    out = _run("exit")
    assert 0 in out and out[0][0] == "error", out
    assert out[0][-1] < 60, out  # bounded by the process group timeout


def test_raising_rank_ends_the_allgather_with_an_error():
    out = _run("raise")
    assert out[1][0] == "raised", out
    assert out[0][0] == "error", out


def test_dead_rank_ends_the_exchange_with_an_error():
    out = _run("exit_exchange")
    assert 0 in out and out[0][0] == "error", out
    assert out[0][-1] < 60, out

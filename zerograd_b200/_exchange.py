"""The exchanged update: one generation's replay spread over the processes
that evaluated its population (one per GPU), for SGD.

The reference all-gathers the fitness and then replays the whole population
on every device (``src/zerograd/_distributed.py:319-366``), so each device
draws every candidate's factors and contracts all of them.  Here the replay
of a bf16 MATRIX/TABLE entry is a fixed-order sum over S candidate groups
(``zg_replay_split_count``): ``d = s * (((G_0 + G_1) + G_2) + ...)`` with
``G_z`` the contraction over group z alone.  Rank j of N evaluates the
candidates of groups ``j S/N .. (j+1) S/N`` and its forward drew their
factors, so it contracts exactly those groups into partials
(``zg_replay_partials``, the kernels and tile schedule of the one-GPU
replay).  The entries are laid out in one flat space cut into N equal
chunks; an all-to-all hands rank j every group's partials of chunk j, rank j
sums them in group order and applies the step there
(``zg_replay_split_sgd``), and an all-gather returns the new parameters to
every rank.  Each element goes through the arithmetic of the one-GPU replay
and update, so every rank ends with the bits one GPU computes.

Collectives per generation: S/N all-to-alls of N chunks of float32 partials
and one all-gather of the bf16 parameters, all on the current stream (they
are captured with the generation's graph).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from . import _lib as L

ALIGN = 8  # elements: segment starts stay 32-byte (float32) / 16-byte (bf16) aligned


@dataclass(frozen=True)
class FlatLayout:
    """Entries placed one after another in a flat element space, each start
    rounded up to ALIGN, cut into `world` chunks of `chunk` elements."""

    offsets: tuple
    numels: tuple
    chunk: int
    world: int

    @property
    def total(self) -> int:
        return self.chunk * self.world


def flat_layout(numels, world: int) -> FlatLayout:
    offsets, off = [], 0
    for n in numels:
        offsets.append(off)
        off += -(-int(n) // ALIGN) * ALIGN
    chunk = -(-off // world) if off else ALIGN
    chunk = -(-chunk // ALIGN) * ALIGN
    return FlatLayout(tuple(offsets), tuple(int(n) for n in numels), chunk, world)


def owned_segments(layout: FlatLayout, rank: int) -> list:
    """(entry index, a, b): the flat ranges [a, b) of entries that fall in
    chunk `rank`, in entry order."""
    lo, hi = rank * layout.chunk, (rank + 1) * layout.chunk
    out = []
    for i, (off, n) in enumerate(zip(layout.offsets, layout.numels)):
        a, b = max(off, lo), min(off + n, hi)
        if a < b:
            out.append((i, a, b))
    return out


def group_offsets(S: int, layout: FlatLayout, pos: int) -> list:
    """Element offsets, in the receive buffer, of the S groups' partials of
    position `pos` of this rank's chunk.  The receive buffer is [S/N,
    total]: all-to-all i brings, from source rank src, that rank's i-th local
    group, whose global index is src * S/N + i."""
    per = S // layout.world
    return [(s % per) * layout.total + (s // per) * layout.chunk + pos for s in range(S)]


@dataclass(frozen=True)
class ExchangedReplay:
    """Rank `rank` of `world`, evaluating candidates start..start+count, in
    process group `group` (None: the default group)."""

    rank: int
    world: int
    start: int
    count: int
    group: Any = None

    def applies(self, population: int, rank: int) -> bool:
        """Whether the population splits into groups that the ranks hold
        whole: S a multiple of the world size, equal consecutive shards."""
        if self.world < 2 or population % self.world:
            return False
        S = int(L.load().zg_replay_split_count(population, rank))
        return (S % self.world == 0 and self.count == population // self.world
                and self.start == self.rank * self.count)

    def split_count(self, population: int, rank: int) -> int:
        return int(L.load().zg_replay_split_count(population, rank))

    def contract(self, work: list, shaped: torch.Tensor, population: int, rank: int):
        """(layout, partials [S/N, total] float32): this rank's groups'
        partial replays of the entries in `work`, each (param [rows, cols]
        bf16, (A, a_t, B, b_t) the local candidates' operand factors, lr),
        at the entries' places in the flat layout."""
        dev = shaped.device
        S = self.split_count(population, rank)
        per = S // self.world
        layout = flat_layout([p.numel() for p, _, _ in work], self.world)
        st = L.stream_ptr(dev)
        w_local = shaped[self.start:self.start + self.count].contiguous()
        parts = torch.empty((per, layout.total), dtype=torch.float32, device=dev)
        base = parts.data_ptr()
        for (param, (A, a_t, B, b_t), _lr), off in zip(work, layout.offsets):
            rows, cols = param.shape
            ws = L.workspace(L.query("zg_replay_partials_workspace_size", self.count, rows, cols, rank), dev)
            L.call("zg_replay_partials", L.ptr(w_local), L.ptr(A), int(a_t), L.ptr(B), int(b_t), self.count, rows,
                   cols, rank, S, per, base + 4 * off, layout.total, L.ptr(ws), ws.numel(), st)
        return layout, parts

    def exchange(self, parts: torch.Tensor) -> torch.Tensor:
        """The receive buffer [S/N, total]: all-to-all i gives chunk
        `rank` of every rank's i-th partial (see group_offsets)."""
        recv = torch.empty_like(parts)
        for i in range(parts.shape[0]):
            dist.all_to_all_single(recv[i], parts[i], group=self.group)
        return recv

    def step_owned(self, work: list, layout: FlatLayout, recv: torch.Tensor, S: int, inv_sqrt_rank: float,
                   guard: torch.Tensor | None) -> torch.Tensor:
        """This rank's chunk of the new parameters (bf16 [chunk]): the
        groups' partials summed in group order, scaled, and the SGD step on
        the parameters' elements in the chunk.  With `guard` non-zero
        nothing is written."""
        dev = recv.device
        st = L.stream_ptr(dev)
        mine = torch.empty(layout.chunk, dtype=torch.bfloat16, device=dev)
        lo = self.rank * layout.chunk
        for i, a, b in owned_segments(layout, self.rank):
            param, _, lr = work[i]
            offs = (ctypes.c_int64 * S)(*group_offsets(S, layout, a - lo))
            L.call("zg_replay_split_sgd", L.ptr(recv), ctypes.addressof(offs), S, b - a, inv_sqrt_rank,
                   param.data_ptr() + 2 * (a - layout.offsets[i]), mine.data_ptr() + 2 * (a - lo), L.ZG_BF16,
                   float(lr), L.ptr(guard), st)
        return mine

    def gather(self, work: list, layout: FlatLayout, mine: torch.Tensor) -> list:
        """Every rank's chunk, all-gathered: the new parameters as views of
        one buffer, in `work` order."""
        gathered = torch.empty(layout.total, dtype=mine.dtype, device=mine.device)
        dist.all_gather_into_tensor(gathered, mine, group=self.group)
        return [gathered[off:off + p.numel()].view(p.shape) for (p, _, _), off in zip(work, layout.offsets)]

    def update(self, work: list, shaped: torch.Tensor, population: int, rank: int, inv_sqrt_rank: float,
               guard: torch.Tensor | None) -> list:
        """New parameters of the entries in `work` (see contract), as views
        of one gathered buffer.  With `guard` (a device float32 count)
        nothing is written when it is non-zero; the caller's copies back
        are guarded the same way."""
        layout, parts = self.contract(work, shaped, population, rank)
        recv = self.exchange(parts)
        mine = self.step_owned(work, layout, recv, self.split_count(population, rank), inv_sqrt_rank, guard)
        return self.gather(work, layout, mine)

"""Population-sharded evaluation (``src/zerograd/_distributed.py``).

The population is the only sharded axis.  Two ways to run it:

* one process per GPU (the B200 layout): ``DistributedZeroGrad`` with
  ``devices=None`` inside an initialised ``torch.distributed`` process group
  (NCCL).  Rank r evaluates its contiguous id range, the 1-D fitness array is
  all-gathered, and every rank replays the identical update -- the
  seed-derived replicated-replay protocol of
  ``src/zerograd/_cluster.py:228-250`` -- so parameters never move.  With
  ``replay="sharded"`` (SGD) each rank contracts only its own candidates'
  factors and the ranks exchange the partial replays and the new parameters
  (``_exchange.py``): the same bits, 1/N of the replay and factor draws.
* one process, several devices (the reference's layout): ``devices`` is a
  list of ``torch.device``; shards run on worker threads, losses are
  gathered to the coordinator device in shard order and the generation is
  completed there (``_distributed.py:241-285``).
"""
from __future__ import annotations

import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from ._exchange import ExchangedReplay
from ._keys import key as make_key
from ._manifest import ParameterTree
from ._optimizer import LossFn, StepMetrics, ZeroGrad, ZeroGradState, _materialize_tree


@dataclass(frozen=True, slots=True)
class ShardResult:
    """One worker's candidate ids and losses (``_distributed.py:36-41``)."""

    candidate_ids: torch.Tensor
    losses: torch.Tensor


@dataclass(frozen=True, slots=True)
class CalibrationResult:
    """Per-device timing from calibration (``_distributed.py:44-52``)."""

    device: Any
    name: str
    num_candidates: int
    elapsed_seconds: float
    per_candidate_seconds: float


def compute_partition_sizes(population: int, weights: list[float]) -> list[int]:
    """Largest-remainder split of ``population`` by ``weights`` (``_distributed.py:55-85``)."""
    if not isinstance(population, int) or isinstance(population, bool) or population < 1:
        raise ValueError(f"population must be a positive integer, got {population!r}")
    if not weights:
        raise ValueError("weights must be non-empty")
    if any(w < 0 for w in weights):
        raise ValueError("weights must be non-negative")
    total = sum(weights)
    if total == 0:
        raise ValueError("at least one weight must be positive")
    quotas = [population * w / total for w in weights]
    sizes = [int(q) for q in quotas]
    remainder = population - sum(sizes)
    order = sorted(range(len(weights)), key=lambda i: quotas[i] - int(quotas[i]), reverse=True)
    for i in range(remainder):
        sizes[order[i]] += 1
    return sizes


def shard_ranges(sizes: list[int]) -> list[tuple[int, int]]:
    """Contiguous ``[start, stop)`` id ranges in shard order (``_distributed.py:225-235``)."""
    out, start = [], 0
    for s in sizes:
        out.append((start, start + s))
        start += s
    return out


def allgather_losses(local: torch.Tensor, sizes: list[int], group=None) -> torch.Tensor:
    """All-gather per-rank loss shards of uneven ``sizes`` into id order.

    Each rank contributes ``local`` (``sizes[rank]`` entries); shards are padded
    to the largest size for a single ``all_gather_into_tensor`` and compacted.
    """
    world = len(sizes)
    width = max(sizes)
    padded = torch.zeros(width, dtype=torch.float32, device=local.device)
    if local.numel():
        padded[: local.numel()] = local.to(torch.float32)
    gathered = torch.empty(world * width, dtype=torch.float32, device=local.device)
    dist.all_gather_into_tensor(gathered, padded, group=group)
    gathered = gathered.view(world, width)
    return torch.cat([gathered[r, : sizes[r]] for r in range(world)])


class DeviceShard:
    """Evaluates a population shard on one device (``_distributed.py:88-139``)."""

    def __init__(self, device, optimizer: ZeroGrad, loss_fn: LossFn, name: str = "") -> None:
        self.device = torch.device(device)
        self._optimizer = optimizer
        self._loss_fn = loss_fn
        self.name = name or f"shard-{self.device.type}"
        self._candidate_ids: torch.Tensor | None = None
        # Draw the whole population's replay factors on a second stream while
        # this shard's forward runs (for a process that also replays).  Off by
        # default: on B200 the integer-bound draws and the forward's GEMMs
        # contend for the same SMs, and drawing after the forward measured
        # faster at 2, 4 and 8 shards.
        self.prefetch_replay = False

    def evaluate(self, params: ParameterTree, batch: Any, candidate_ids: torch.Tensor, generation: int,
                 rng: torch.Tensor | None = None) -> ShardResult:
        if rng is None:
            rng = make_key(0)
        params_d = _to_device(_materialize_tree(params), self.device)
        batch_d = _to_device(batch, self.device)
        # host-side ids: a contiguous range is then known without a device sync,
        # so the forward's factors are kept for this process's replay
        ids_h = torch.as_tensor(candidate_ids)
        ids = ids_h if ids_h.device.type == "cpu" else ids_h.to(self.device)
        with torch.cuda.device(self.device) if self.device.type == "cuda" else _null():
            self._optimizer.manifest.validate(params_d)
            losses = self._optimizer._evaluate_shard(params_d, generation, self._loss_fn, batch_d, ids,
                                                     rng=rng.to(self.device), prefetch_replay=self.prefetch_replay)
        return ShardResult(candidate_ids=candidate_ids, losses=losses)

    @property
    def num_candidates(self) -> int:
        ids = self._candidate_ids
        return int(ids.shape[0]) if ids is not None else 0


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def _to_device(tree, device):
    if isinstance(tree, torch.Tensor):
        return tree.to(device, non_blocking=True)
    if isinstance(tree, dict):
        return {k: _to_device(v, device) for k, v in tree.items()}
    if isinstance(tree, (list, tuple)):
        return type(tree)(_to_device(v, device) for v in tree)
    return tree


class DistributedZeroGrad:
    """Multi-device coordinator with weighted partitioning (``_distributed.py:142-366``)."""

    def __init__(self, optimizer: ZeroGrad, devices: list | None, loss_fn: LossFn, weights: list[float] | None = None,
                 coordinator_device=None, process_group=None, replay: str = "replicated") -> None:
        self._optimizer = optimizer
        self._loss_fn = loss_fn
        self._group = process_group
        self._pg_mode = devices is None
        if replay not in ("replicated", "sharded"):
            raise ValueError("replay must be 'replicated' or 'sharded'")
        if replay == "sharded" and not self._pg_mode:
            raise ValueError("the exchanged update is for process-group mode (one process per GPU)")
        self._replay = replay
        if self._pg_mode:
            if not dist.is_initialized():
                raise ValueError("devices=None requires an initialised torch.distributed process group")
            world = dist.get_world_size(process_group)
            self._rank = dist.get_rank(process_group)
            self._devices = [torch.device("cuda", torch.cuda.current_device())
                             if torch.cuda.is_available() else torch.device("cpu")]
            n = world
        else:
            if not devices:
                raise ValueError("at least one device is required")
            self._devices = [torch.device(d) for d in devices]
            self._rank = 0
            n = len(self._devices)
        if weights is not None and len(weights) != n:
            raise ValueError(f"weights length ({len(weights)}) must match devices ({n})")
        self._n = n
        self._coordinator_device = torch.device(coordinator_device) if coordinator_device else self._devices[0]
        self._weights = list(weights) if weights else [1.0] * n
        if self._pg_mode:
            self._shards = [DeviceShard(self._devices[0], optimizer, loss_fn, name=f"rank-{self._rank}")]
        else:
            self._shards = [DeviceShard(d, optimizer, loss_fn, name=f"worker-{i}-{d.type}")
                            for i, d in enumerate(self._devices)]
        self._partition_sizes = compute_partition_sizes(optimizer.population_size, self._weights)
        self._apply_partition()
        self._exchange = None
        if replay == "sharded":
            a, b = shard_ranges(self._partition_sizes)[self._rank]
            self._exchange = ExchangedReplay(self._rank, n, a, b - a, process_group)
        self._executor = None if self._pg_mode else ThreadPoolExecutor(max_workers=n)
        self._closed = False

    # -- lifecycle ----------------------------------------------------------
    def shutdown(self) -> None:
        ex = self._executor
        if ex is not None:
            ex.shutdown(wait=False)
            self._executor = None
        self._closed = True

    def __enter__(self):
        return self

    def __exit__(self, *exc) -> bool:
        self.shutdown()
        return False

    def __del__(self) -> None:
        try:
            self.shutdown()
        except Exception:
            pass

    def _apply_partition(self) -> None:
        ranges = shard_ranges(self._partition_sizes)
        if self._pg_mode:
            a, b = ranges[self._rank]
            self._shards[0]._candidate_ids = torch.arange(a, b, dtype=torch.int32)
        else:
            for shard, (a, b) in zip(self._shards, ranges):
                shard._candidate_ids = torch.arange(a, b, dtype=torch.int32)

    def init(self, params: ParameterTree) -> ZeroGradState:
        return self._optimizer.init(params)

    # -- one generation -----------------------------------------------------
    def capture(self, params: ParameterTree, batch: Any, *, state: ZeroGradState | None = None,
                rng: torch.Tensor | None = None, warmup: int = 2, slots: int = 2,
                draw_ahead: bool = True):
        """The generation ``step`` runs in process-group mode, captured as a
        CUDA graph: this process's shard of the forward, the fitness
        all-gather (NCCL, in the graph) and the completion (replicated, or
        exchanged, with its collectives in the graph).  Every
        rank must capture together.  Release the returned object before the
        process group is destroyed."""
        from ._graph import CapturedGeneration

        if not self._pg_mode:
            raise NotImplementedError("capture is for process-group mode (one process per GPU)")
        if self._closed:
            raise RuntimeError("coordinator has been shut down")
        a, b = shard_ranges(self._partition_sizes)[self._rank]
        sizes, group = list(self._partition_sizes), self._group
        return CapturedGeneration(self._optimizer, _to_device(_materialize_tree(params), self._devices[0]),
                                  self._loss_fn, batch, state=state, candidate_range=(a, b - a),
                                  gather=lambda local: allgather_losses(local, sizes, group), rng=rng,
                                  warmup=warmup, slots=slots, draw_ahead=draw_ahead, exchange=self._exchange)

    def step(self, state: ZeroGradState, params: ParameterTree, batch: Any, *, rng: torch.Tensor | None = None):
        if rng is None:
            rng = make_key(0)
        if self._closed:
            raise RuntimeError("coordinator has been shut down")
        gen = state.generation
        if self._pg_mode:
            shard = self._shards[0]
            ids = shard._candidate_ids
            if ids.numel():
                local = shard.evaluate(params, batch, ids, gen, rng).losses
            else:
                local = torch.empty(0, dtype=torch.float32, device=shard.device)
            losses = allgather_losses(local.to(torch.float32), self._partition_sizes, self._group)
            params_c = _to_device(_materialize_tree(params), shard.device)
            if self._exchange is not None:
                opt = self._optimizer
                opt._manifest.validate(params_c)
                return opt._step_from_losses(state, params_c, losses, exchange=self._exchange)
            return self._optimizer.step_from_losses(state, params_c, losses)
        futures = []
        for shard in self._shards:
            ids = shard._candidate_ids
            futures.append(self._executor.submit(shard.evaluate, params, batch, ids, gen, rng)
                           if ids is not None and ids.numel() > 0 else None)
        parts = []
        for f in futures:
            if f is None:
                continue
            parts.append(f.result().losses.to(self._coordinator_device))
        losses = torch.cat(parts)
        params_c = _to_device(_materialize_tree(params), self._coordinator_device)
        return self._optimizer.step_from_losses(state, params_c, losses)

    def calibrate(self, params: ParameterTree, batch: Any, *, warmup: int = 1, trials: int = 3,
                  rng: torch.Tensor | None = None) -> list[CalibrationResult]:
        """Weights inversely proportional to per-candidate time (``_distributed.py:287-352``)."""
        if rng is None:
            rng = make_key(0)
        pop = self._optimizer.population_size
        calib_ids = torch.arange(min(pop, 4), dtype=torch.int32)
        results = []
        for shard in self._shards:
            for _ in range(warmup):
                r = shard.evaluate(params, batch, calib_ids, 0, rng)
                _sync(shard.device)
            t0 = time.perf_counter()
            for _ in range(trials):
                r = shard.evaluate(params, batch, calib_ids, 0, rng)
                _sync(shard.device)
            elapsed = (time.perf_counter() - t0) / trials
            results.append(CalibrationResult(device=shard.device, name=shard.name,
                                             num_candidates=len(calib_ids), elapsed_seconds=elapsed,
                                             per_candidate_seconds=elapsed / len(calib_ids)))
            del r
        if self._pg_mode:
            t = torch.tensor([results[0].per_candidate_seconds], dtype=torch.float64,
                             device=self._shards[0].device)
            allt = [torch.empty_like(t) for _ in range(self._n)]
            dist.all_gather(allt, t, group=self._group)
            per = [float(x.item()) for x in allt]
        else:
            per = [r.per_candidate_seconds for r in results]
        self._weights = [1.0 / p for p in per]
        self._partition_sizes = compute_partition_sizes(pop, self._weights)
        self._apply_partition()
        if self._exchange is not None:
            a, b = shard_ranges(self._partition_sizes)[self._rank]
            self._exchange = ExchangedReplay(self._rank, self._n, a, b - a, self._group)
        return results

    @property
    def shards(self) -> list[DeviceShard]:
        return self._shards

    @property
    def weights(self) -> list[float]:
        return list(self._weights)

    @property
    def partition_sizes(self) -> list[int]:
        return list(self._partition_sizes)


def _sync(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)

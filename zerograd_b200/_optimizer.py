"""ZeroGrad optimizer lifecycle (``src/zerograd/_optimizer.py``).

Same surface as the reference: ``init``, ``evaluate_shard``,
``step_from_losses``, ``step`` and the read-only properties.  Candidate
evaluation runs the per-candidate ``loss_fn`` under ``torch.func.vmap`` over
the candidate keys; every ``CandidateContext`` op inside becomes one
population-batched kernel launch.  Completing a generation is one fused
shaping kernel (validation + metrics), one replay per manifest entry and one
fused update kernel per leaf, with a single device-to-host read of the
metrics.
"""
from __future__ import annotations

import collections
import math
from collections.abc import Callable, Mapping
from dataclasses import dataclass
from typing import Any

import torch

from . import _lib as L
from . import _ops
from ._candidate import CandidateContext
from ._fitness import _check_shape_dtype
from ._keys import key as make_key
from ._keys import step_key
from ._manifest import LAYOUT_CODE, Manifest, ParameterLayout, ParameterTree
from ._replay import candidate_keys, replay_entry_keys, replay_entry_step
from ._transforms import _leaves, apply_updates, is_fused, sgd, tree_get, tree_set

LossFn = Callable[[ParameterTree, CandidateContext, Any, torch.Tensor], tuple[torch.Tensor, Any]]


@dataclass(frozen=True, slots=True)
class ZeroGradState:
    """Immutable optimizer state: generation and transform state (``_optimizer.py:25-30``)."""

    generation: int
    opt_state: Any


@dataclass(frozen=True, slots=True)
class StepMetrics:
    """Population diagnostics (``_optimizer.py:33-41``)."""

    generation: int
    mean_loss: float
    min_loss: float
    max_loss: float
    population_size: int


def _device_of(params: ParameterTree) -> torch.device:
    for _, v in _leaves(_materialize_tree(params)):
        if isinstance(v, torch.Tensor):
            return v.device
    raise ValueError("params contain no tensors")


class ZeroGrad:
    """Factor-only ES optimizer (``_optimizer.py:44-277``)."""

    def __init__(self, manifest: Manifest, transform, population_size: int, rank: int, sigma: float, seed: int,
                 run_id: str, *, chunk_size: int | None = None) -> None:
        """``chunk_size`` (an addition to the reference's signature): the
        candidates of one evaluation run through ``loss_fn`` in chunks of at
        most this many, so a large population's activations need not fit at
        once.  Each candidate's factors are still drawn once per generation,
        chunk by chunk, into buffers of the whole evaluated id range that the
        replay reads.  None: all candidates at once (the reference's single
        vmap)."""
        if not isinstance(manifest, Manifest):
            raise TypeError("manifest must be a Manifest")
        if not isinstance(population_size, int) or isinstance(population_size, bool) or population_size < 2:
            raise ValueError("population_size must be an integer >= 2")
        if not isinstance(rank, int) or isinstance(rank, bool) or rank < 1:
            raise ValueError("rank must be a positive integer")
        if not isinstance(sigma, float) or not math.isfinite(sigma) or sigma <= 0:
            raise ValueError("sigma must be a finite positive float")
        if not isinstance(seed, int) or isinstance(seed, bool):
            raise TypeError("seed must be an integer")
        if not isinstance(run_id, str) or not run_id:
            raise ValueError("run_id must be a non-empty string")
        if chunk_size is not None and (not isinstance(chunk_size, int) or isinstance(chunk_size, bool)
                                       or chunk_size < 1):
            raise ValueError("chunk_size must be a positive integer or None")
        self._chunk_size = chunk_size
        self._manifest = manifest
        self._transform = transform
        self._population_size = population_size
        self._rank = rank
        self._sigma = sigma
        self._seed = seed
        self._run_id = run_id
        # Per-generation host and device keys, reused by the calls of one
        # generation (evaluate, prefetch, completion): (tag, device, stream) -> tensor
        self._keys_memo: collections.OrderedDict = collections.OrderedDict()

    def _memo(self, tag, device: torch.device, make):
        """A key tensor of this optimizer, computed once per (tag, device,
        stream): device keys are only read on the stream that wrote them."""
        k = (tag, device, L.stream_ptr(device).value if device.type == "cuda" else None)
        v = self._keys_memo.get(k)
        if v is None:
            v = make()
            self._keys_memo[k] = v
            while len(self._keys_memo) > 16:
                self._keys_memo.popitem(last=False)
        return v

    def _seed_keys(self, generation: int, start: int, count: int, device: torch.device, cks: torch.Tensor) -> None:
        """Use `cks` as the candidate keys of ids [start, start + count) of a
        generation on the current stream (a captured generation derives them
        from its device base-key buffer)."""
        self._keys_memo[(("ck", generation, start, count), device, L.stream_ptr(device).value)] = cks

    def _forget_keys(self, stream_value) -> None:
        """Drop the keys kept for one stream (a finished capture's)."""
        for k in [k for k in self._keys_memo if k[2] == stream_value]:
            del self._keys_memo[k]

    def _candidate_keys_range(self, generation: int, start: int, count: int, device: torch.device):
        """Candidate keys of ids [start, start + count) of a generation."""
        def make():
            ids = torch.arange(start, start + count, dtype=torch.int32, device=device)
            return candidate_keys(self.base_key(generation), ids)
        return self._memo(("ck", generation, start, count), device, make)

    def init(self, params: ParameterTree) -> ZeroGradState:
        self._manifest.validate(params)
        params = _materialize_tree(params)
        return ZeroGradState(generation=0, opt_state=self._transform.init(params))

    @property
    def population_size(self) -> int:
        return self._population_size

    @property
    def rank(self) -> int:
        return self._rank

    @property
    def sigma(self) -> float:
        return self._sigma

    @property
    def manifest(self) -> Manifest:
        return self._manifest

    @property
    def seed(self) -> int:
        return self._seed

    @property
    def run_id(self) -> str:
        return self._run_id

    @property
    def transform(self):
        return self._transform

    @property
    def chunk_size(self) -> int | None:
        return self._chunk_size

    # -- evaluation ---------------------------------------------------------

    def base_key(self, generation: int) -> torch.Tensor:
        """Host-side base key of a generation (passed to kernels by value)."""
        cpu = torch.device("cpu")
        return self._memo(("base", generation, self._manifest.version), cpu,
                          lambda: step_key(self._seed, self._run_id, generation, self._manifest.version)).clone()

    def evaluate_shard(self, params: ParameterTree, generation: int, loss_fn: LossFn, batch: Any,
                       candidate_ids, *, rng: torch.Tensor | None = None,
                       prefetch_replay: bool = False) -> torch.Tensor:
        """Losses of a subset of candidates (``_optimizer.py:126-149``).

        ``prefetch_replay`` (an addition to the reference signature): this
        process will also replay the whole population (one process per GPU),
        so for a contiguous shard the replay's factors are drawn on a second
        stream while the shard's forward runs."""
        self._manifest.validate(params)
        params = _materialize_tree(params)
        return self._evaluate_shard(params, generation, loss_fn, batch, candidate_ids, rng=rng,
                                    prefetch_replay=prefetch_replay)

    def _evaluate_shard(self, params, generation, loss_fn, batch, candidate_ids, *, rng=None, id_range=None,
                        prefetch_replay=False):
        device = _device_of(params)
        if id_range is None:
            id_range = _host_range(candidate_ids)
        base = self.base_key(generation)
        if id_range is not None:
            # keys built on the device (a host-built id tensor would need a
            # copy that synchronises the stream), once per generation and range
            start, count = id_range
            cks = self._candidate_keys_range(generation, start, count, device)
            if rng is None:
                def make_rngs():
                    ids = torch.arange(start, start + count, dtype=torch.int32, device=device)
                    return _ops.launch_fold_in(make_key(0).reshape(1, 2), ids)
                rngs = self._memo(("rng", start, count), device, make_rngs)
            else:
                ids = torch.arange(start, start + count, dtype=torch.int32, device=device)
                rngs = _ops.launch_fold_in(rng.reshape(1, 2), ids)
        else:
            ids = torch.as_tensor(candidate_ids, device=device)
            if ids.ndim != 1:
                raise ValueError("candidate_ids must be one-dimensional")
            cks = candidate_keys(base, ids)
            rngs = _ops.launch_fold_in((make_key(0) if rng is None else rng).reshape(1, 2), ids)
        manifest, rank, sigma = self._manifest, self._rank, self._sigma

        def evaluate_candidate(ck, crng):
            ctx = CandidateContext(manifest, ck, rank, sigma)
            loss, _aux = loss_fn(params, ctx, batch, crng)
            return loss

        if cks.shape[0] == 0:
            return torch.empty(0, dtype=torch.float32, device=device)
        if id_range is None:
            return torch.func.vmap(evaluate_candidate)(cks, rngs)
        base_words = tuple(int(v) for v in base)
        if prefetch_replay and id_range[1] < self._population_size:
            # a shard whose process also replays the whole population: its
            # replay factors are drawn on a second stream while the forward runs
            self._prefetch_replay(params, generation, base_words, device)
        # A contiguous id range known on the host: the factors drawn by the
        # forward ops are kept for this generation's replay.
        start, count = id_range
        chunk = self._chunk_size
        if chunk is None or count <= chunk:
            with _ops.generation_scope(base_words, start, count, cks):
                return torch.func.vmap(evaluate_candidate)(cks, rngs)
        # In chunks: each chunk's ops draw their block of the range's factor
        # buffers (kept for the replay) and read it from there.
        out = []
        for c0 in range(0, count, chunk):
            n = min(chunk, count - c0)
            with _ops.generation_scope(base_words, start + c0, n, cks[c0:c0 + n], pop=(start, count)):
                out.append(torch.func.vmap(evaluate_candidate)(cks[c0:c0 + n], rngs[c0:c0 + n]))
        return torch.cat(out)

    def _factor_entries(self, params) -> list:
        """(group, layout, rows, cols, rank) of every bf16 MATRIX/TABLE leaf:
        the operand factors the replay reads, in the factor cache's key terms."""
        entries = []
        for entry in self._manifest.entries:
            if entry.layout is ParameterLayout.VECTOR:
                continue
            p = self._manifest.resolve(params, entry.path)
            if isinstance(p, torch.Tensor) and p.dtype == torch.bfloat16 and p.ndim == 2:
                e = (self._manifest.group_index(entry.group), LAYOUT_CODE[entry.layout], int(p.shape[0]),
                     int(p.shape[1]), self._rank)
                if e not in entries:
                    entries.append(e)
        return entries

    def _prefetch_replay(self, params, generation, base_words, device) -> None:
        entries = self._factor_entries(params)
        if not entries or torch.cuda.get_device_capability(device) != (10, 0):
            return
        cks = self._candidate_keys_range(generation, 0, self._population_size, device)
        _ops.prefetch_replay_factors(_ops._Generation(base_words, 0, self._population_size, cks), entries)

    # -- completion ---------------------------------------------------------

    def step_from_losses(self, state: ZeroGradState, params: ParameterTree, losses: torch.Tensor):
        """Complete one generation from losses in candidate-id order (``_optimizer.py:183-203``)."""
        if not isinstance(state, ZeroGradState):
            raise TypeError("state must be a ZeroGradState")
        self._manifest.validate(params)
        params = _materialize_tree(params)
        return self._step_from_losses(state, params, losses)

    def _check_losses(self, losses: torch.Tensor) -> None:
        _check_shape_dtype(losses)
        if losses.shape[0] != self._population_size:
            raise ValueError(f"losses must have {self._population_size} entries, got {losses.shape[0]}")

    def _step_from_losses(self, state, params, losses, cand_keys: torch.Tensor | None = None, exchange=None):
        new_params, new_opt_state, metrics = self._complete(state, params, losses, cand_keys, exchange=exchange)
        # The one host sync of a generation, after all its work is queued.  The
        # update wrote new tensors only, so rejecting non-finite losses here
        # leaves params and state exactly as they were.
        return new_params, ZeroGradState(generation=state.generation + 1, opt_state=new_opt_state), \
            self._metrics(state.generation, metrics)

    def _metrics(self, generation: int, metrics: torch.Tensor) -> StepMetrics:
        """Host metrics from the shaping kernel's [mean, min, max, non-finite
        count]; raises on non-finite losses (``_fitness.py:37-48``)."""
        m = metrics.cpu()
        if m[3].item() > 0:
            raise ValueError("candidate losses must be finite")
        return StepMetrics(generation=generation, mean_loss=float(m[0]), min_loss=float(m[1]),
                           max_loss=float(m[2]), population_size=self._population_size)

    def _exchange_work(self, state, params, exchange, gen, cand_keys) -> list:
        """(path, param, operands, lr) of the entries the exchanged update
        takes: bf16 2-D MATRIX/TABLE leaves, their operand factors for this
        rank's candidates (the forward's, from the factor cache, else drawn)."""
        if not isinstance(self._transform, sgd) or not exchange.applies(self._population_size, self._rank):
            return []
        a, n = exchange.start, exchange.count
        local = _ops._Generation(gen.base, a, n, cand_keys[a:a + n])
        work = []
        for entry in self._manifest.entries:
            if entry.layout is ParameterLayout.VECTOR:
                continue
            leaf = self._manifest.resolve(params, entry.path)
            if not (isinstance(leaf, torch.Tensor) and leaf.is_cuda and leaf.dtype == torch.bfloat16
                    and leaf.ndim == 2 and leaf.is_contiguous() and (n * self._rank) % 8 == 0):
                continue
            rows, cols = (int(d) for d in leaf.shape)
            layout = LAYOUT_CODE[entry.layout]
            ops = _ops._replay_operands_for(local.cks, self._manifest.group_index(entry.group), layout, rows, cols,
                                            self._rank, local, _ops.CACHE)
            if ops[3] and cols % 8:
                continue
            work.append((tuple(entry.path), leaf, ops, self._transform.step_spec(state.opt_state, entry.path)["lr"]))
        return work

    def _complete(self, state, params, losses, cand_keys: torch.Tensor | None = None, inplace: bool = False,
                  exchange=None):
        """Device part of a generation's completion, all queued on the
        current stream with no host synchronisation: shaping, replay and the
        optimizer step.  Returns (new params, new optimizer state, device
        metrics [mean, min, max, non-finite count]).  `inplace`: entries whose
        step is fused into the replay are updated in place, and not at all
        when a loss is not finite (the metrics' non-finite count guards the
        writes); the other leaves still come back as new tensors.
        `exchange` (an ExchangedReplay; one process per GPU, SGD): the bf16
        MATRIX/TABLE entries are replayed from this rank's candidates only and
        the partials exchanged (``ExchangedReplay.update``), with the bits of
        the replicated update; their new values come back as new tensors."""
        self._check_losses(losses)
        device = _device_of(params)
        losses = losses.to(device)
        generation = state.generation
        shaped, metrics = _ops.launch_shape_fitness(losses, self._sigma)
        base = self.base_key(generation)
        base_words = tuple(int(v) for v in base)
        if cand_keys is None:
            cand_keys = self._candidate_keys_range(generation, 0, self._population_size, device)
        gen = _ops._Generation(base_words, 0, self._population_size, cand_keys)
        descent: dict = {}
        fused = is_fused(self._transform)
        done: dict = {}
        guard = metrics[3:4] if inplace else None
        if exchange is not None and fused:
            work = self._exchange_work(state, params, exchange, gen, cand_keys)
            if work:
                inv = _ops.scaled_factor_value(self._rank, 1.0, torch.bfloat16)
                new = exchange.update([(p, ops, lr) for _, p, ops, lr in work], shaped, self._population_size,
                                      self._rank, inv, guard)
                for (path, *_), t in zip(work, new):
                    done[path] = (t, None, None)
        for entry in self._manifest.entries:
            if tuple(entry.path) in done:
                continue
            if fused:
                # the optimizer step in the replay GEMM's epilogue (bf16 MATRIX/TABLE)
                spec = self._transform.step_spec(state.opt_state, entry.path)
                res = replay_entry_step(params, self._manifest, entry.path, cand_keys, shaped, self._rank, spec,
                                        gen, inplace_guard=guard)
                if res is not None:
                    done[tuple(entry.path)] = res
                    continue
            tree_set(descent, entry.path,
                     replay_entry_keys(params, self._manifest, entry.path, cand_keys, shaped, self._rank, gen))
        _ops.CACHE.drop_generation(base_words)
        if fused:
            new_params, new_opt_state = self._transform.apply(params, descent, state.opt_state, done)
        else:
            grads = _build_pseudo_grad(descent, params)
            updates, new_opt_state = self._transform.update(grads, state.opt_state, params)
            new_params = apply_updates(params, updates)
        return new_params, new_opt_state, metrics

    def catch_up(self, state: ZeroGradState, params: ParameterTree, loss_history) -> tuple:
        """Replay a loss history: one ``step_from_losses`` per recorded
        generation, from ``state.generation`` on.  No forward pass runs: a
        generation's update needs only its losses and its seed-derived keys,
        so a node that joins late (or restarts from an older checkpoint)
        reaches the cluster's parameters bit for bit (the reference's
        ``add_node`` catch-up, ``_fault_tolerant.py:148-158``).  Returns the
        new (params, state) and the last generation's metrics (None for an
        empty history)."""
        metrics = None
        for losses in loss_history:
            params, state, metrics = self.step_from_losses(state, params, torch.as_tensor(losses))
        return params, state, metrics

    def capture(self, params: ParameterTree, loss_fn: LossFn, batch: Any, *, state: ZeroGradState | None = None,
                rng: torch.Tensor | None = None, warmup: int = 2, slots: int = 2,
                draw_ahead: bool = True):
        """The generation ``step`` runs, captured as a CUDA graph
        (:class:`CapturedGeneration`): replaying it costs one graph launch
        instead of the per-op host work.  `params` and `batch` give the
        shapes and the initial values; the graph keeps its own copies.
        `slots` = 2 captures it over two batch buffers, so the next
        generation's host-to-device copies overlap the current one; with
        `draw_ahead` each generation also draws the next one's factors."""
        from ._graph import CapturedGeneration

        return CapturedGeneration(self, params, loss_fn, batch, state=state, rng=rng, warmup=warmup, slots=slots,
                                  draw_ahead=draw_ahead)

    def step(self, state: ZeroGradState, params: ParameterTree, batch: Any, loss_fn: LossFn, *,
             rng: torch.Tensor | None = None):
        """One generation: evaluate all candidates, then complete (``_optimizer.py:246-277``)."""
        if not isinstance(state, ZeroGradState):
            raise TypeError("state must be a ZeroGradState")
        self._manifest.validate(params)
        params = _materialize_tree(params)
        device = _device_of(params)
        ids = torch.arange(self._population_size, dtype=torch.int32, device=device)
        losses = self._evaluate_shard(params, state.generation, loss_fn, batch, ids, rng=rng,
                                      id_range=(0, self._population_size))
        return self._step_from_losses(state, params, losses)


def _host_range(candidate_ids):
    """(start, count) when the ids are a contiguous ascending range known on
    the host (a range, a list or a CPU tensor); None otherwise (reading a
    device tensor would cost a synchronisation)."""
    if isinstance(candidate_ids, range):
        if len(candidate_ids) == 0 or (candidate_ids.step != 1 and len(candidate_ids) > 1):
            return None
        return candidate_ids.start, len(candidate_ids)
    if isinstance(candidate_ids, (list, tuple)):
        vals = candidate_ids
    elif isinstance(candidate_ids, torch.Tensor) and not candidate_ids.is_cuda and candidate_ids.ndim == 1:
        vals = candidate_ids.tolist()
    else:
        return None
    if len(vals) == 0:
        return None
    start = int(vals[0])
    if any(int(v) != start + i for i, v in enumerate(vals)):
        return None
    return start, len(vals)


def _materialize_tree(params: ParameterTree) -> dict:
    """Plain-dict copy of a Mapping tree (``_optimizer.py:280-296``)."""
    out: dict = {}
    for k, v in params.items():
        out[k] = _materialize_tree(v) if isinstance(v, Mapping) else v
    return out


def _build_pseudo_grad(descent: dict, params: ParameterTree) -> dict:
    """Negated descent, zeros for non-manifest leaves (``_optimizer.py:299-326``)."""
    out: dict = {}
    for path, v in _leaves(_materialize_tree(params)):
        if isinstance(v, torch.Tensor):
            d = tree_get(descent, path)
            tree_set(out, path, -d if isinstance(d, torch.Tensor) else torch.zeros_like(v))
        else:
            tree_set(out, path, v)
    return out

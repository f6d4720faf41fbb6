"""One ES generation captured as a CUDA graph.

``ZeroGrad.step`` issues every kernel of a generation from Python: the
candidate keys, each context op under ``vmap``, the fitness shaping, the
factor replay and the optimizer step, about half a millisecond of host work
for a few hundred microseconds of GPU work at the perturbed-GEMM size.  A
:class:`CapturedGeneration` records that launch sequence once and replays
it for every later generation.  What changes between generations is data,
not launches:

* the base key ``step_key(seed, run_id, generation, version)`` is copied
  into a device buffer before each replay, and the captured candidate keys
  are derived from that buffer in the graph (every factor draw, forward and
  replay kernel reads keys from device memory);
* the batch is copied into the captured batch buffers (from pinned host
  memory, or from the device).  With ``slots=2`` (the default) the
  generation is captured twice, over two batch buffers that share one graph
  memory pool, and successive generations alternate between them: the
  host-to-device copies of generation g+1 (batch, base key, AdamW bias
  corrections) run on a copy stream while generation g computes, ordered
  by events after the last replay that read the same slot;
* with two slots, generation g+1's operand factors (every bf16
  MATRIX/TABLE leaf, the whole population) are drawn on a second stream
  into the other slot's factor buffers while generation g's graph runs:
  those integer-bound draws then share the SMs with g's tensor-core and
  HBM-bound kernels instead of running ahead of g+1's forward.  They are
  launched just before g's graph and joined into the caller's stream just
  after it, so a generation's work includes its draws of the next one.
  Generation g+1's forward and replay read them (they are a function of
  g+1's keys alone).  When a call's generation is not the one drawn ahead
  (the first call, or generations out of sequence), its factors are drawn
  before its replay;
* the parameters live in captured buffers, updated on the device only when
  the shaping kernel counted no non-finite loss: the entries whose step is
  fused into the replay GEMM are updated in place with that count as the
  epilogue's guard, the other leaves are written to the graph's own buffers
  and copied back under the same guard.  A rejected generation leaves the
  parameters as they were, and ``step`` raises as ``step_from_losses`` does.

``step`` reads the metrics back every generation (a synchronisation, as the
reference's ``float(jnp.mean(losses))``); ``enqueue`` queues a generation
and returns a handle whose ``result()`` does that read later, so successive
generations keep the GPU busy.

Each replay gives the same bits as the eager ``evaluate_shard`` +
``step_from_losses`` of the same generation, for ``sgd`` and ``adamw``.
AdamW's bias corrections 1 - b^t change every step: the host computes them
as the eager kernels do (``zg_adam_bias_corrections``) and copies them into
a device buffer before each replay, and the moments live in captured
buffers updated in place like the parameters.

With a process group, ``gather`` (the fitness all-gather) is captured in the
graph as well, and each process captures its own shard of candidates.
"""
from __future__ import annotations

from typing import Any, Callable

import torch
from torch.utils import _pytree as pytree

from . import _lib as L
from . import _ops
from ._manifest import ParameterTree
from ._transforms import _leaves, tree_get


def _clone_tree(tree):
    return pytree.tree_map(lambda t: t.clone() if isinstance(t, torch.Tensor) else t, tree)


class CapturedGeneration:
    """A generation of ``optimizer`` (evaluate + complete) as a CUDA graph.

    Build it with :meth:`ZeroGrad.capture`.  :meth:`step` then runs one
    generation: ``params, state, metrics = cg.step(state, batch)``.  The
    returned parameters are the captured buffers themselves: the next
    ``step`` updates them in place (clone them to keep a generation).
    """

    def __init__(self, optimizer, params: ParameterTree, loss_fn: Callable, batch: Any, *, state=None,
                 candidate_range: tuple[int, int] | None = None,
                 gather: Callable[[torch.Tensor], torch.Tensor] | None = None,
                 rng: torch.Tensor | None = None, prefetch_replay: bool = False, warmup: int = 2,
                 slots: int = 2, draw_ahead: bool = True, exchange=None):
        from ._optimizer import ZeroGradState, _device_of, _materialize_tree
        from ._transforms import AdamWState, adamw, sgd

        if not isinstance(optimizer.transform, (sgd, adamw)):
            raise NotImplementedError("capture supports the library's sgd and adamw transforms")
        optimizer.manifest.validate(params)
        self._opt = optimizer
        self._gather = gather
        self._rng = rng
        P = optimizer.population_size
        self._range = candidate_range if candidate_range is not None else (0, P)
        if gather is None and self._range != (0, P):
            raise ValueError("a shard of the population needs a gather of the losses")
        self.device = _device_of(params)
        dev = self.device
        if dev.type != "cuda":
            raise L.ZgLibraryError("capture runs on CUDA devices only; there is no CPU fallback")
        if slots not in (1, 2):
            raise ValueError("slots must be 1 or 2")
        self._slots = slots
        self._params = _clone_tree(_materialize_tree(params))
        self._batches = [_clone_tree(batch) for _ in range(slots)]
        self._loss_fn = loss_fn
        # prefetch_replay: a shard's replay factors drawn on a second stream
        # (a parallel branch of the graph) during its forward; off by default,
        # since the draws and the forward's GEMMs contend for the same SMs
        self._prefetch = prefetch_replay
        self._exchange = exchange  # the exchanged update (ExchangedReplay), or None: replicated
        # a slot's per-generation inputs, one row of 8 words copied in by one
        # host-to-device copy: the base key (words 0-1), the next
        # generation's base key (2-3), AdamW's bias corrections (float32, 4-5)
        self._inputs = torch.zeros((slots, 8), dtype=torch.uint32, device=dev)
        self._ids = torch.arange(P, dtype=torch.int32, device=dev)
        # the candidates whose factors this process draws ahead: all of them
        # for a replicated replay, its own shard for the exchanged update
        self._draw_range = (0, P)
        if exchange is not None and isinstance(optimizer.transform, sgd) and \
                exchange.applies(P, optimizer.rank):
            self._draw_range = (exchange.start, exchange.count)
        g0 = state.generation if state is not None else 0
        opt_state0 = state.opt_state if state is not None else optimizer.init(self._params).opt_state
        self._state_cls = ZeroGradState
        self._adam = isinstance(optimizer.transform, adamw)
        if self._adam:
            # the moments in captured buffers; the bias corrections of each
            # step in the slot's inputs, filled before the replay
            self._adam_cls = AdamWState
            opt_state0 = AdamWState(opt_state0.count, _clone_tree(opt_state0.mu), _clone_tree(opt_state0.nu))
        self._opt_state = opt_state0

        # warm-up outside the graph: first-call setup (kernel attributes, the
        # factor-cache budget, the communicator) must not happen in a capture.
        # The warm-up also shows which factor layout the forward draws for
        # each entry (a shared-input op's operand layout, or a per-candidate
        # input's, "t"): the layout drawn ahead below.
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        _ops.CACHE.log = []
        try:
            with torch.cuda.stream(side):
                for i in range(max(1, warmup)):
                    self._set_inputs(g0 + i, opt_state0, 0, False)
                    self._generation(g0 + i, self._slot_state(opt_state0, 0), 0, copy_back=False)
            forward_keys = list(_ops.CACHE.log)
        finally:
            _ops.CACHE.log = None
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        t_entries = {k[3:8] for k in forward_keys if len(k) == 9 and k[8] == _ops._T_TAG}

        # factors drawn one generation ahead (two slots): per slot, one
        # buffer pair per bf16 MATRIX/TABLE leaf, in the layout its forward
        # reads ((A_op, B_op), or the per-candidate-input (F1T, F2) pair)
        self._entries = []
        if slots == 2 and draw_ahead and torch.cuda.get_device_capability(dev) == (10, 0):
            self._entries = [e + ((_ops._T_TAG,) if e in t_entries and e[4] in (8, 16) else ())
                             for e in optimizer._factor_entries(self._params)]
            need = sum((e[2] + e[3]) * self._draw_range[1] * e[4] * 2 for e in self._entries)
            if need > _ops.CACHE._budget(dev):
                self._entries = []  # over the factor-cache budget: drawn in the generation, as eagerly
        self._fbuf = [[self._factor_buffers(e) for e in self._entries] for _ in range(slots)]
        self._draw_stream = torch.cuda.Stream(dev)
        self._drawn: list = [None] * slots  # generation whose factors each slot's buffers hold
        self._draw_done = [torch.cuda.Event() for _ in range(slots)]  # draws into the slot's buffers done

        # one graph per batch slot, all in one memory pool: replays never
        # overlap (one stream), so their intermediates may share memory
        pool = torch.cuda.graph_pool_handle()
        self._graphs, self._outs = [], []
        base0 = tuple(int(v) for v in optimizer.base_key(g0))
        d0, dn = self._draw_range
        for slot in range(slots):
            graph = torch.cuda.CUDAGraph()
            self._set_inputs(g0, opt_state0, slot, False)
            for e, bufs in zip(self._entries, self._fbuf[slot]):
                # the forward and the replay read the slot's factor buffers
                _ops.CACHE.put((base0, d0, dn) + e, bufs, dev)
                _ops.CACHE.mark_drawn((base0, d0, dn) + e)
            n0 = L.launch_count()
            with torch.cuda.graph(graph, pool=pool):
                capture_stream = L.stream_ptr(dev).value
                out = self._generation(g0, self._slot_state(opt_state0, slot), slot, copy_back=True)
            torch.cuda.synchronize(dev)
            optimizer._forget_keys(capture_stream)
            _ops.CACHE.drop_generation(base0)
            self._graphs.append(graph)
            self._outs.append(out)
        #: this library's kernels in one generation: the graph's, and the draws
        #: of the next generation's factors
        self.kernels_per_generation = L.launch_count() - n0
        self._draw_graphs = []
        if self._entries:
            # g0's factors into slot 0 (the first call's), eagerly; then per
            # slot a graph of the draws from the slot's next base key into the
            # other slot's buffers (each in its own memory pool: it runs beside
            # the generation's graph)
            self._draw(self._opt.base_key(g0), self._fbuf[0])
            self._drawn[0] = g0
            torch.cuda.synchronize(dev)
            for slot in range(slots):
                dg = torch.cuda.CUDAGraph()
                n0 = L.launch_count()
                with torch.cuda.graph(dg):
                    self._draw(self._inputs[slot, 2:4], self._fbuf[1 - slot])
                self._draw_graphs.append(dg)
            self.kernels_per_generation += L.launch_count() - n0
            torch.cuda.synchronize(dev)
        self._copy_stream = torch.cuda.Stream(dev)
        self._ready = [torch.cuda.Event() for _ in range(slots)]  # slot's inputs copied
        self._free = [torch.cuda.Event() for _ in range(slots)]  # slot's last replay done
        self._next = 0

    def _factor_buffers(self, e):
        """A buffer pair for entry `e` = (group, layout, rows, cols, rank[,
        "t"]) of the candidates drawn ahead, in the factor cache's (A, B) order."""
        P, dev = self._draw_range[1], self.device
        _, layout, rows, cols, rank = e[:5]
        if len(e) == 6:  # per-candidate-input layout
            k_rows, n_rows = (rows, cols) if layout == L.ZG_MATRIX else (cols, rows)
            F1T = torch.empty((P * rank, k_rows), dtype=torch.bfloat16, device=dev)
            F2 = torch.empty((n_rows, P * rank), dtype=torch.bfloat16, device=dev)
            return (F1T, F2) if layout == L.ZG_MATRIX else (F2, F1T)
        return (torch.empty((rows, P * rank), dtype=torch.bfloat16, device=dev),
                torch.empty((cols, P * rank), dtype=torch.bfloat16, device=dev))

    def _draw(self, base: torch.Tensor, bufs) -> None:
        """Every entry's factors, for the candidates drawn ahead of the
        generation with base key `base`, into `bufs` (current stream)."""
        d0, P = self._draw_range
        cks = _ops.launch_fold_in(base, self._ids[d0:d0 + P])
        for e, (A, B) in zip(self._entries, bufs):
            group, layout, rows, cols, rank = e[:5]
            if len(e) == 6:
                F1T, F2 = (A, B) if layout == L.ZG_MATRIX else (B, A)
                L.call("zg_factor_operands_t", L.ptr(cks), group, P, layout, rows, cols, rank, L.ptr(F1T), L.ptr(F2),
                       0, L.stream_ptr(self.device))
            else:
                L.call("zg_factor_operands", L.ptr(cks), group, P, layout, rows, cols, rank, L.ZG_BF16, L.ptr(A),
                       L.ptr(B), L.stream_ptr(self.device))

    def _slot_state(self, opt_state, slot: int):
        """The optimizer state a slot's graph reads: AdamW's bias corrections
        from that slot's inputs."""
        if not self._adam:
            return opt_state
        bc = self._inputs[slot, 4:6].view(torch.float32)
        return self._adam_cls(opt_state.count, opt_state.mu, opt_state.nu, bias_corrections=bc)

    def _set_inputs(self, generation: int, opt_state, slot: int, ahead: bool) -> None:
        """The slot's inputs for `generation` (current stream): its base key,
        the next generation's when drawing ahead, AdamW's bias corrections of
        step count + 1."""
        # a fresh pinned buffer per call: the pinned allocator reuses it only
        # after this copy has run, so queued generations never race on it
        host = torch.zeros(8, dtype=torch.uint32, pin_memory=True)
        h = host.numpy()
        h[0:2] = self._opt.base_key(generation).numpy()
        if ahead:
            h[2:4] = self._opt.base_key(generation + 1).numpy()
        if self._adam:
            t = self._opt.transform
            L.call("zg_adam_bias_corrections", int(opt_state.count) + 1, float(t.b1), float(t.b2),
                   host.data_ptr() + 16)
        self._inputs[slot].copy_(host, non_blocking=True)

    def _generation(self, generation: int, opt_state, slot: int, copy_back: bool):
        """The launch sequence of one generation over batch slot `slot`, keys
        read from the slot's device base-key buffer."""
        opt, dev, (start, count) = self._opt, self.device, self._range
        P = opt.population_size
        cks_all = _ops.launch_fold_in(self._inputs[slot, 0:2], self._ids)
        opt._seed_keys(generation, 0, P, dev, cks_all)
        if (start, count) != (0, P):
            opt._seed_keys(generation, start, count, dev, cks_all[start:start + count])
        losses = opt._evaluate_shard(self._params, generation, self._loss_fn, self._batches[slot],
                                     range(start, start + count), rng=self._rng,
                                     prefetch_replay=self._prefetch)
        if self._gather is not None:
            losses = self._gather(losses.to(torch.float32))
        state = self._state_cls(generation, opt_state)
        # in the graph, fused steps update the captured parameters in place,
        # guarded by the non-finite count; the other leaves are copied back
        new_params, new_opt_state, metrics = opt._complete(state, self._params, losses, cand_keys=cks_all,
                                                           inplace=copy_back, exchange=self._exchange)
        if copy_back:
            flag = metrics[3:4]  # non-finite loss count
            pairs = [(t, tree_get(new_params, path)) for path, t in _leaves(self._params)]
            if self._adam:
                for which in ("mu", "nu"):
                    old, new = getattr(opt_state, which), getattr(new_opt_state, which)
                    pairs += [(t, tree_get(new, path)) for path, t in _leaves(old)]
            for t, new in pairs:
                if new is not t:
                    _ops.launch_copy_if_zero(t, new.contiguous(), flag)
        return new_params, new_opt_state, metrics

    @property
    def params(self) -> ParameterTree:
        """The captured parameter buffers (the current parameters)."""
        return self._params

    def load_params(self, params: ParameterTree) -> None:
        """Copy `params` (same tree and shapes) into the captured buffers."""
        for path, t in _leaves(self._params):
            t.copy_(tree_get(params, path), non_blocking=True)

    def _queue(self, state, batch) -> int:
        """Copy one generation's inputs into the next slot and replay that
        slot's graph; returns the slot."""
        if not isinstance(state, self._state_cls):
            raise TypeError("state must be a ZeroGradState")
        slot = self._next
        pairs = []
        if batch is not None:
            dst = pytree.tree_leaves(self._batches[slot])
            src = pytree.tree_leaves(batch)
            if len(dst) != len(src):
                raise ValueError("batch does not match the captured batch's structure")
            for d, s in zip(dst, src):
                if isinstance(d, torch.Tensor):
                    if tuple(s.shape) != tuple(d.shape):
                        raise ValueError(f"batch leaf of shape {tuple(s.shape)}; captured {tuple(d.shape)}")
                    pairs.append((d, s))
        self._next = (slot + 1) % self._slots
        cur = torch.cuda.current_stream(self.device)
        cs = self._copy_stream
        # host-side inputs on the copy stream, once the slot's last replay is
        # done; it overlaps the generation queued before this one
        with torch.cuda.stream(cs):
            cs.wait_event(self._free[slot])
            for d, s in pairs:
                if not s.is_cuda:
                    d.copy_(s, non_blocking=True)
            self._set_inputs(state.generation, state.opt_state, slot, bool(self._entries))
            self._ready[slot].record(cs)
        cur.wait_event(self._ready[slot])
        for d, s in pairs:
            if s.is_cuda:  # produced on the current stream: copied there
                d.copy_(s, non_blocking=True)
        if self._entries and self._drawn[slot] != state.generation:
            # not drawn ahead with the previous generation: draw this one's now
            self._draw(self._opt.base_key(state.generation), self._fbuf[slot])
        if self._entries:
            # the next generation's factors, beside this one: the other slot's
            # buffers were last read by the replay before this one (done on
            # this stream), and its base key is in with this slot's inputs
            ds = self._draw_stream
            ds.wait_stream(cur)
            with torch.cuda.stream(ds):
                self._draw_graphs[slot].replay()
                self._draw_done[1 - slot].record(ds)
        self._graphs[slot].replay()
        if self._entries:
            cur.wait_event(self._draw_done[1 - slot])
            self._drawn[slot] = state.generation
            self._drawn[1 - slot] = state.generation + 1
        self._free[slot].record(cur)  # the slot's inputs (batch, keys) are read by now
        return slot

    @property
    def opt_state(self):
        """The captured optimizer state (AdamW's moments live here)."""
        return self._opt_state

    def _next_state(self, state, slot: int):
        """The state after one replay: the generation and the step count
        advance; AdamW's moments are the captured buffers."""
        if self._adam:
            nxt = self._adam_cls(int(state.opt_state.count) + 1, self._opt_state.mu, self._opt_state.nu)
        else:
            nxt = _advance_state(state.opt_state, self._outs[slot][1])
        return self._state_cls(state.generation + 1, nxt)

    def step(self, state, batch: Any = None):
        """One generation: copy `batch` (if given) into the captured batch,
        replay the graph and read its metrics.  Returns (params, new state,
        metrics) like ``ZeroGrad.step``; raises ValueError, with the
        parameters unchanged, when a loss is not finite."""
        slot = self._queue(state, batch)
        m = self._opt._metrics(state.generation, self._outs[slot][2])
        return self._params, self._next_state(state, slot), m

    def enqueue(self, state, batch: Any = None):
        """Queue one generation without waiting for it.  Returns (params, new
        state, pending); ``pending.result()`` waits and returns the metrics,
        or raises ValueError if that generation's losses were not all finite
        (its update was then not applied; generations queued after it start
        from the unchanged parameters)."""
        slot = self._queue(state, batch)
        host = torch.empty(4, dtype=torch.float32, pin_memory=True)
        host.copy_(self._outs[slot][2], non_blocking=True)
        done = torch.cuda.Event()
        done.record(torch.cuda.current_stream(self.device))
        return self._params, self._next_state(state, slot), PendingGeneration(self._opt, state.generation, host,
                                                                               done)


class PendingGeneration:
    """Metrics of a queued generation, read when asked for."""

    def __init__(self, optimizer, generation: int, host: torch.Tensor, done: torch.cuda.Event):
        self._opt, self.generation, self._host, self._done = optimizer, generation, host, done

    def result(self):
        self._done.synchronize()
        return self._opt._metrics(self.generation, self._host)


def _advance_state(old, captured):
    """The optimizer state after one replay: the captured generation's host
    fields advanced from `old` (sgd keeps only a counter)."""
    from ._transforms import SgdState

    if isinstance(old, SgdState):
        return SgdState(count=old.count + 1)
    return captured


__all__ = ["CapturedGeneration", "PendingGeneration"]

"""Torch custom ops over the libzgb200 C ABI, with population vmap rules.

The reference calls its forward ops per candidate inside ``jax.vmap`` over
candidate ids (``src/zerograd/_optimizer.py:173-181``).  Here the same
per-candidate code runs under ``torch.func.vmap``; each op below has a vmap
rule that turns the batched candidate key into ONE population-batched
kernel launch (an unbatched activation stays shared across candidates, the
way vmap leaves an unbatched ``x @ W`` unbatched).

Launchers (``launch_*``) are the population-form entry points: keys
``[P, 2]`` uint32, outputs with a leading population axis.
"""
from __future__ import annotations

import ctypes
import math
import struct

import torch

from . import _lib as L

# ---------------------------------------------------------------------------
# scalars
# ---------------------------------------------------------------------------


def round_scalar(value: float, dtype: torch.dtype) -> float:
    """A Python float converted to a scalar of ``dtype`` (float32 or bf16).

    bf16 goes through float32 first, as numpy/ml_dtypes scalar conversion does.
    """
    f32 = struct.unpack("<f", struct.pack("<f", value))[0]
    if dtype == torch.float32:
        return f32
    if dtype == torch.bfloat16:
        u = struct.unpack("<I", struct.pack("<f", f32))[0]
        if (u & 0x7F800000) != 0x7F800000:
            u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
        return struct.unpack("<f", struct.pack("<I", u & 0xFFFFFFFF))[0]
    raise TypeError(f"unsupported dtype {dtype}")


def scaled_factor_value(rank: int, sigma: float, dtype: torch.dtype) -> float:
    return round_scalar(sigma / math.sqrt(rank), dtype)


def _keys2d(keys: torch.Tensor) -> torch.Tensor:
    if keys.dtype != torch.uint32:
        raise TypeError(f"keys must be uint32 key data, got {keys.dtype}")
    if keys.shape[-1] != 2:
        raise ValueError(f"keys must have a trailing dimension of 2, got {tuple(keys.shape)}")
    return keys.reshape(-1, 2).contiguous()


def _compute_dtype(*ts: torch.Tensor) -> torch.dtype:
    dt = ts[0].dtype
    for t in ts[1:]:
        dt = torch.promote_types(dt, t.dtype)
    L.dtype_code(dt)
    return dt


# ---------------------------------------------------------------------------
# launchers (population form)
# ---------------------------------------------------------------------------


def _as_u32(data: torch.Tensor) -> torch.Tensor:
    d = data.reshape(-1)
    if d.dtype in (torch.int32, torch.uint32):
        return d.contiguous().view(torch.uint32)
    return d.to(torch.int64).to(torch.uint32).contiguous()


def launch_fold_in(keys: torch.Tensor, data: torch.Tensor) -> torch.Tensor:
    """out[i] = fold_in(keys[i] (or the single key), data[i]).

    A single key held on the host is passed by value (no host-to-device copy).
    """
    if not keys.is_cuda and keys.numel() == 2 and data.is_cuda:
        k = _keys2d(keys)
        d = _as_u32(data)
        out = torch.empty((d.numel(), 2), dtype=torch.uint32, device=data.device)
        L.call("zg_candidate_keys", int(k[0, 0]), int(k[0, 1]), L.ptr(d), L.ptr(out), d.numel(),
               L.stream_ptr(data.device))
        return out
    dev = L.require_cuda(keys, data)
    k = _keys2d(keys)
    d = _as_u32(data)
    n = max(d.numel(), k.shape[0])
    if k.shape[0] not in (1, n) or d.numel() not in (1, n):
        raise ValueError("fold_in: keys and data counts do not broadcast")
    if d.numel() == 1 and n > 1:
        d = d.expand(n).contiguous()
    out = torch.empty((n, 2), dtype=torch.uint32, device=dev)
    L.call("zg_fold_in", L.ptr(k), int(k.shape[0] != 1), L.ptr(d), L.ptr(out), n, L.stream_ptr(dev))
    return out


def launch_copy_if_zero(dst: torch.Tensor, src: torch.Tensor, flag: torch.Tensor) -> None:
    """dst <- src on the device when flag[0] == 0 (contiguous, same bytes)."""
    dev = L.require_cuda(dst, src, flag)
    if not (dst.is_contiguous() and src.is_contiguous()) or dst.nbytes != src.nbytes:
        raise ValueError("copy_if_zero needs contiguous tensors of the same size")
    if flag.dtype != torch.float32:
        raise TypeError("the flag is a float32 count")
    L.call("zg_copy_if_zero", L.ptr(dst), L.ptr(src), dst.nbytes, L.ptr(flag), L.stream_ptr(dev))


def launch_normal(keys: torch.Tensor, n: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    dev = L.require_cuda(keys)
    k = _keys2d(keys)
    out = torch.empty((k.shape[0], n), dtype=dtype, device=dev)
    L.call("zg_normal", L.ptr(k), k.shape[0], n, L.dtype_code(dtype), L.ptr(out), L.stream_ptr(dev))
    return out


def launch_bits(keys: torch.Tensor, n: int) -> torch.Tensor:
    dev = L.require_cuda(keys)
    k = _keys2d(keys)
    out = torch.empty((k.shape[0], n), dtype=torch.uint32, device=dev)
    L.call("zg_random_bits", L.ptr(k), k.shape[0], n, L.ptr(out), L.stream_ptr(dev))
    return out


def launch_factors(keys: torch.Tensor, group: int, layout: int, shape, rank: int,
                   dtype: torch.dtype):
    """Population factors in the reference layouts (leading P axis)."""
    dev = L.require_cuda(keys)
    k = _keys2d(keys)
    P = k.shape[0]
    rows = int(shape[0])
    if layout == L.ZG_VECTOR:
        A = torch.empty((P, rows), dtype=dtype, device=dev)
        L.call("zg_population_factors", L.ptr(k), group, P, layout, rows, 1, 1, L.dtype_code(dtype),
               L.ptr(A), None, L.stream_ptr(dev))
        return A, None
    cols = int(shape[1])
    A = torch.empty((P, rows, rank), dtype=dtype, device=dev)
    B = torch.empty((P, rank, cols) if layout == L.ZG_MATRIX else (P, cols, rank), dtype=dtype, device=dev)
    L.call("zg_population_factors", L.ptr(k), group, P, layout, rows, cols, rank, L.dtype_code(dtype),
           L.ptr(A), L.ptr(B), L.stream_ptr(dev))
    return A, B


# ---------------------------------------------------------------------------
# generation-scoped factor cache
# ---------------------------------------------------------------------------


class _Generation:
    """The candidate keys of one generation being evaluated by ZeroGrad.

    `pop` = (start, count) of the id range whose factors are kept for the
    replay; a chunk of that range (ids start..start+count) draws its block
    of the range's factor buffers and reads it from there.  By default the
    range is the chunk itself."""

    def __init__(self, base: tuple, start: int, count: int, cks: torch.Tensor, pop: tuple | None = None):
        self.base, self.start, self.count, self.cks = base, start, count, cks
        self.pop_start, self.pop_count = pop if pop is not None else (start, count)


def _capturing() -> bool:
    """True while the current CUDA stream is being captured into a graph."""
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


class _AllChunks(set):
    """The drawn-chunk record of buffers drawn whole (every chunk is in)."""

    def __contains__(self, item) -> bool:
        return True


ALL_DRAWN = _AllChunks()


class FactorCache:
    """Operand-layout factors drawn during a generation's forward pass, kept
    (within a byte budget) for that generation's replay, so every factor
    element is drawn once per generation.  Entries are a pure function of
    (base key, candidate ids, group, layout, shape, rank), so reuse is exact.
    """

    def __init__(self, budget_bytes: int | None = None):
        self.budget_bytes = budget_bytes
        self._entries: dict = {}
        self._ready: dict = {}  # key -> event: entry drawn on another stream, not yet waited for
        self._drawn: dict = {}  # key -> set of (start, count) chunks of an id range's buffers drawn so far
        self._bytes = 0
        self.log: list | None = None  # when a list: every key put is appended (a capture learns the layouts)
        self.hits = 0
        self.misses = 0
        self._active: _Generation | None = None

    def _budget(self, device) -> int:
        if self.budget_bytes is None:
            free, total = torch.cuda.mem_get_info(device)
            self.budget_bytes = int(min(0.5 * free, 0.25 * total))
        return self.budget_bytes

    def active_for(self, keys: torch.Tensor) -> _Generation | None:
        g = self._active
        if g is not None and keys.data_ptr() == g.cks.data_ptr() and keys.shape[0] == g.count:
            return g
        return None

    def get(self, key):
        hit = self._entries.get(key)
        if hit is not None:
            self._entries[key] = self._entries.pop(key)  # most recent last
            self.hits += 1
            ev = self._ready.pop(key, None)
            if ev is not None:
                # drawn on a second stream: order this stream after the draws
                cur = torch.cuda.current_stream(hit[0].device)
                cur.wait_event(ev)
                for t in hit:
                    t.record_stream(cur)
        else:
            self.misses += 1
        return hit

    def find(self, *keys):
        """(key, value) of the first of `keys` present, counted as one hit or
        one miss; (None, None) when none is."""
        for key in keys:
            if key in self._entries:
                return key, self.get(key)
        self.misses += 1
        return None, None

    def covering(self, base: tuple, start: int, count: int, tail: tuple):
        """(count of its population, value) of an entry drawn for candidates
        0..n of the generation `base` that covers candidates start..start+count
        (same group, layout, shape and rank: `tail`), or None.  A shard's
        forward reads its candidates' columns from it."""
        for key in list(self._entries):
            if (len(key) == 3 + len(tail) and key[0] == base and key[1] == 0 and key[2] >= start + count
                    and key[3:] == tail):
                ev = self._ready.get(key)
                if ev is not None and not _capturing() and not ev.query():
                    # still being drawn on another stream (a replay prefetch
                    # that overlaps this forward): look for one that is
                    # ready; without one the shard draws its own rather
                    # than wait for the whole population's
                    continue
                return key[2], self.get(key)
        return None

    def __contains__(self, key) -> bool:
        return key in self._entries

    def put(self, key, value, device, ready=None) -> bool:
        """Keep `value` under `key` within the budget (oldest entries go
        first); False when it alone exceeds the budget and is not kept."""
        nbytes = sum(t.numel() * t.element_size() for t in value)
        budget = self._budget(device)
        while self._entries and self._bytes + nbytes > budget:
            self._pop(next(iter(self._entries)))
        if self.log is not None:
            self.log.append(key)
        if nbytes <= budget:
            self._entries[key] = value
            self._bytes += nbytes
            if ready is not None:
                self._ready[key] = ready
            return True
        return False

    def _pop(self, key):
        old = self._entries.pop(key)
        self._ready.pop(key, None)
        self._drawn.pop(key, None)
        self._bytes -= sum(t.numel() * t.element_size() for t in old)
        return old

    def range_buffers(self, key, make, device):
        """(value, drawn chunks) of the factor buffers of an id range, made
        by `make()` and kept on first use; the caller records the chunks it
        draws into them in the returned set."""
        hit = self.get(key)
        if hit is None:
            hit = make()
            if not self.put(key, hit, device):
                return hit, set()
        return hit, self._drawn.setdefault(key, set())

    def mark_drawn(self, key) -> None:
        """Record that the buffers under `key` hold every candidate's factors."""
        if key in self._entries:
            self._drawn[key] = ALL_DRAWN

    def covering_drawn(self, base: tuple, start: int, count: int, tail: tuple):
        """(n, value) of buffers of candidates 0..n of the generation `base`,
        drawn whole, that cover candidates start..start+count (same `tail`),
        or None.  A shard's (or chunk's) forward reads its block of them."""
        for key in list(self._entries):
            if (len(key) == 3 + len(tail) and key[0] == base and key[1] == 0 and key[2] >= start + count
                    and key[3:] == tail and self._drawn.get(key) is ALL_DRAWN):
                return key[2], self.get(key)
        return None

    def drop_generation(self, base: tuple) -> None:
        for key in [k for k in self._entries if k[0] == base]:
            self._pop(key)

    def clear(self) -> None:
        self._entries.clear()
        self._ready.clear()
        self._drawn.clear()
        self._bytes = 0


CACHE = FactorCache()


class generation_scope:
    """Context manager marking `cks` as the keys of candidates start..start+count
    of the generation with base key words `base` (used by ZeroGrad)."""

    def __init__(self, base: tuple, start: int, count: int, cks: torch.Tensor, cache: FactorCache = CACHE,
                 pop: tuple | None = None):
        self.gen = _Generation(base, start, count, cks, pop)
        self.cache = cache

    def __enter__(self):
        self._prev = self.cache._active
        self.cache._active = self.gen
        return self.gen

    def __exit__(self, *exc):
        self.cache._active = self._prev
        return False


def _tc_ok(dev: torch.device, P: int, K: int, N: int, rank: int) -> bool:
    return (torch.cuda.get_device_capability(dev) == (10, 0) and (P * rank) % 8 == 0 and K % 8 == 0
            and N % 8 == 0 and rank <= 32)


_PREFETCH_STREAMS: dict = {}


def _prefetch_stream(dev: torch.device) -> torch.cuda.Stream:
    s = _PREFETCH_STREAMS.get(dev)
    if s is None:
        s = torch.cuda.Stream(device=dev)
        _PREFETCH_STREAMS[dev] = s
    return s


def prefetch_replay_factors(gen: _Generation, entries, cache: FactorCache = CACHE) -> None:
    """Draw, on a second stream, the operand factors of `entries` -- (group,
    layout, rows, cols, rank) of bf16 MATRIX/TABLE entries -- for the whole
    population whose candidate keys are ``gen.cks``, and keep them in the
    cache under gen's key.  A shard's replay needs every candidate's factors
    but its forward pass draws only its own; started with the generation,
    these draws (integer-ALU work) overlap the forward's GEMMs, and the
    replay waits for them only when it uses them."""
    dev = gen.cks.device
    side = _prefetch_stream(dev)
    main = torch.cuda.current_stream(dev)
    side.wait_stream(main)  # the candidate keys come from this stream
    k = _keys2d(gen.cks)
    k.record_stream(side)
    P = k.shape[0]
    for group, layout, rows, cols, rank in entries:
        key = (gen.base, gen.start, gen.count, group, layout, rows, cols, rank)
        if key in cache or group < 0:
            continue
        with torch.cuda.stream(side):
            A = torch.empty((rows, P * rank), dtype=torch.bfloat16, device=dev)
            B = torch.empty((cols, P * rank), dtype=torch.bfloat16, device=dev)
            L.call("zg_factor_operands", L.ptr(k), group, P, layout, rows, cols, rank, L.ZG_BF16, L.ptr(A),
                   L.ptr(B), ctypes.c_void_p(side.cuda_stream))
            ev = torch.cuda.Event()
            ev.record(side)
        cache.put(key, (A, B), dev, ready=ev)


def operand_factors(keys: torch.Tensor, group: int, layout: int, rows: int, cols: int, rank: int,
                    gen: _Generation | None = None, cache: FactorCache = CACHE):
    """(A_op [rows, P r], B_op [cols, P r]) bf16, from the cache when the keys are
    a generation's candidate keys."""
    dev = keys.device
    k = _keys2d(keys)
    P = k.shape[0]
    ckey = None
    if gen is not None and group >= 0:
        ckey = (gen.base, gen.start, gen.count, group, layout, rows, cols, rank)
        hit = cache.get(ckey)
        if hit is not None:
            return hit
    A = torch.empty((rows, P * rank), dtype=torch.bfloat16, device=dev)
    B = torch.empty((cols, P * rank), dtype=torch.bfloat16, device=dev)
    L.call("zg_factor_operands", L.ptr(k), group, P, layout, rows, cols, rank, L.ZG_BF16, L.ptr(A), L.ptr(B),
           L.stream_ptr(dev))
    if ckey is not None:
        cache.put(ckey, (A, B), dev)
    return A, B


def _forward_factors(x, W, w_is_kn: bool, F1, F2, P, M, K, N, rank, s, y):
    dev = x.device
    ws = L.workspace(L.query("zg_forward_factors_workspace_size", P, M, N, rank), dev)
    L.call("zg_forward_factors", L.ptr(x), L.ptr(W), int(w_is_kn), L.ptr(F1), L.ptr(F2), P, M, K, N, rank, s,
           L.ptr(y), L.ptr(ws), ws.numel(), L.stream_ptr(dev))


def _forward_cached(x, W, w_is_kn: bool, keys, group, layout, rows, cols, P, M, K, N, rank, s, y, gen,
                    cache: FactorCache = CACHE):
    """Shared-input forward whose operand factors (A_op [rows, P r], B_op
    [cols, P r]) are kept in the cache for the generation's replay."""
    dev = x.device
    ckey = (gen.base, gen.start, gen.count, group, layout, rows, cols, rank)
    hit = cache.get(ckey)
    if hit is not None:
        A_op, B_op = hit
        F1, F2 = (A_op, B_op) if w_is_kn else (B_op, A_op)
        _forward_factors(x, W, w_is_kn, F1, F2, P, M, K, N, rank, s, y)
        return
    cover = cache.covering(gen.base, gen.start, gen.count, ckey[3:]) if (rank == 8 and gen.count == P) else None
    if cover is not None:
        # a shard of a population whose factors are drawn already (for the
        # replay): its candidates' columns, rows P_all*rank apart
        _, (A_all, B_all) = cover
        c0 = gen.start * rank
        A_v, B_v = A_all[:, c0:c0 + P * rank], B_all[:, c0:c0 + P * rank]
        F1, F2 = (A_v, B_v) if w_is_kn else (B_v, A_v)
        ld = int(A_all.shape[1])
        ws = L.workspace(L.query("zg_forward_factors_workspace_size", P, M, N, rank), dev)
        L.call("zg_forward_factors_ld", L.ptr(x), L.ptr(W), int(w_is_kn), L.ptr(F1), ld, L.ptr(F2), ld, P, M, K, N,
               rank, s, L.ptr(y), L.ptr(ws), ws.numel(), L.stream_ptr(dev))
        return
    A_op = torch.empty((rows, P * rank), dtype=torch.bfloat16, device=dev)
    B_op = torch.empty((cols, P * rank), dtype=torch.bfloat16, device=dev)
    F1, F2 = (A_op, B_op) if w_is_kn else (B_op, A_op)
    ws = L.workspace(L.query("zg_forward_factors_workspace_size", P, M, N, rank), dev)
    L.call("zg_forward_operands", L.ptr(x), L.ptr(W), int(w_is_kn), L.ptr(_keys2d(keys)), group, P, M, K, N, rank,
           s, L.ptr(F1), L.ptr(F2), L.ptr(y), L.ptr(ws), ws.numel(), L.stream_ptr(dev))
    cache.put(ckey, (A_op, B_op), dev)


# Cache keys of per-candidate-input forwards end with this tag: their input-side
# factor is kept K-major ([P r, K]), so the replay reads it transposed.
_T_TAG = "t"


def _batched_ok(dev: torch.device, P: int, K: int, N: int, rank: int) -> bool:
    return torch.cuda.get_device_capability(dev) == (10, 0) and rank in (8, 16) and K % 8 == 0 and N % 8 == 0


def _range_factors(gen: _Generation, key_tail: tuple, q_rows: int, n_rows: int, rank: int, dev,
                   cache: FactorCache = CACHE):
    """(F1T, F2, ld2, draw) for the candidates of `gen` in the per-candidate-
    input layout: F1T [count r, q_rows] rows and F2 [n_rows, count r] columns
    of the factor buffers of gen's id range (F1T [Pp r, q_rows], F2 [n_rows,
    Pp r], kept in the cache in the replay's (A, B) order: MATRIX (F1T, F2),
    tied TABLE (F2, F1T)), and whether this chunk still has to draw them."""
    Pp = gen.pop_count
    key = (gen.base, gen.pop_start, gen.pop_count) + key_tail
    if key not in cache:
        # the whole population's buffers, drawn already (a generation drawn
        # ahead): read this chunk's block of them
        cover = cache.covering_drawn(gen.base, gen.start, gen.count, key_tail)
        if cover is not None:
            n, val = cover
            F1T_all, F2_all = val if key_tail[1] == L.ZG_MATRIX else (val[1], val[0])
            return (F1T_all[gen.start * rank:(gen.start + gen.count) * rank], F2_all[:, gen.start * rank:],
                    n * rank, False)

    def make():
        F1T = torch.empty((Pp * rank, q_rows), dtype=torch.bfloat16, device=dev)
        F2 = torch.empty((n_rows, Pp * rank), dtype=torch.bfloat16, device=dev)
        return (F1T, F2) if key_tail[1] == L.ZG_MATRIX else (F2, F1T)

    val, drawn = cache.range_buffers(key, make, dev)
    F1T_all, F2_all = val if key_tail[1] == L.ZG_MATRIX else (val[1], val[0])
    off = gen.start - gen.pop_start
    F1T = F1T_all[off * rank:(off + gen.count) * rank]
    F2 = F2_all[:, off * rank:]
    chunk = (gen.start, gen.count)
    draw = chunk not in drawn
    drawn.add(chunk)
    return F1T, F2, Pp * rank, draw


def _forward_batched(x, W, w_is_kn: bool, keys, group, layout, rows, cols, P, M, K, N, rank, s, y, gen,
                     cache: FactorCache = CACHE, act: int = 0, res: torch.Tensor | None = None):
    """Per-candidate-input forward (x [P, M, K]) on the tensor cores.  Its
    factors (F1T [P r, K] K-major, F2 [N, P r]) are the candidates' block of
    the buffers of gen's id range, drawn by the first op of each chunk that
    uses them and kept in the cache for the generation's replay, in the
    replay's (A, B) order.  `act` / `res`: the epilogue's activation and
    residual (zg_batched_forward_ex)."""
    dev = x.device
    ws = L.workspace(L.query("zg_batched_forward_workspace_size", P, M, K, N, rank), dev)
    F1T, F2, ld2, draw = _range_factors(gen, (group, layout, rows, cols, rank, _T_TAG), K, N, rank, dev, cache)
    L.call("zg_batched_forward_ex", L.ptr(x), L.ptr(W), int(w_is_kn), L.ptr(_keys2d(keys)), group, P, M, K, N, rank,
           s, L.ptr(F1T), L.ptr(F2), ld2, int(draw), int(act), L.ptr(res), L.ptr(y), L.ptr(ws), ws.numel(),
           L.stream_ptr(dev))


ACTIVATIONS = {None: L.ZG_ACT_NONE, "none": L.ZG_ACT_NONE, "gelu": L.ZG_ACT_GELU}


def launch_gelu(x: torch.Tensor) -> torch.Tensor:
    """Element-wise GELU (tanh form) of a float32 or bf16 tensor."""
    dev = L.require_cuda(x)
    xc = x.contiguous()
    y = torch.empty_like(xc)
    L.call("zg_gelu", L.ptr(xc), L.ptr(y), xc.numel(), L.dtype_code(xc.dtype), L.stream_ptr(dev))
    return y


def _epilogue_unfused(y: torch.Tensor, act: int, res: torch.Tensor | None) -> torch.Tensor:
    """The activation and residual of a linear whose kernel has no fused
    epilogue: the same roundings as the fused one (bf16 / float32 result,
    element-wise GELU, then the residual add in the result's dtype)."""
    if act == L.ZG_ACT_GELU:
        y = launch_gelu(y)
    if res is not None:
        y = res.to(y.dtype) + y
    return y


def launch_linear(x: torch.Tensor, weight: torch.Tensor, keys: torch.Tensor, group: int, rank: int,
                  sigma: float, x_batched: bool, act: int = 0, residual: torch.Tensor | None = None) -> torch.Tensor:
    """y[p] = x_p @ W + s (x_p @ A_p) @ B_p; x [*M, K] shared or [P, *M, K].
    `act` (ZG_ACT_*) and `residual` ([P, *M, N]): y = act(y) + residual with
    the unfused ops' roundings, fused into the GEMM's epilogue on the
    per-candidate-input tensor-core path."""
    dev = L.require_cuda(x, weight, keys, residual)
    k = _keys2d(keys)
    P = k.shape[0]
    if weight.ndim != 2 or x.ndim < 1 or x.shape[-1] != weight.shape[0]:
        raise ValueError("linear input and [in, out] weight shapes are incompatible")
    if x_batched and (x.ndim < 2 or x.shape[0] != P):
        raise ValueError("batched linear input must lead with the population axis")
    dt = _compute_dtype(x, weight)
    x = x.to(dt).contiguous()
    W = weight.to(dt).contiguous()
    K, N = W.shape
    mshape = tuple(x.shape[1:-1] if x_batched else x.shape[:-1])
    M = math.prod(mshape)
    y = torch.empty((P, *mshape, N), dtype=dt, device=dev)
    if residual is not None and tuple(residual.shape) != tuple(y.shape):
        raise ValueError(f"residual of shape {tuple(residual.shape)} does not match the output {tuple(y.shape)}")
    if M == 0:
        return y
    s = scaled_factor_value(rank, sigma, weight.dtype)
    code = L.dtype_code(dt)
    gen = CACHE.active_for(keys)
    if x_batched and dt == torch.bfloat16 and _batched_ok(dev, P, K, N, rank):
        res = None if residual is None else residual.to(dt).contiguous()
        if gen is None:
            # outside a generation (a direct call): a one-off range of these candidates
            _forward_batched(x, W, True, k, group, L.ZG_MATRIX, K, N, P, M, K, N, rank, s, y,
                             _Generation((-1, -1, id(k)), 0, P, k), cache=FactorCache(budget_bytes=0), act=act,
                             res=res)
        else:
            _forward_batched(x, W, True, k, group, L.ZG_MATRIX, K, N, P, M, K, N, rank, s, y, gen, act=act,
                             res=res)
        return y
    if gen is not None and dt == torch.bfloat16 and not x_batched and _tc_ok(dev, P, K, N, rank):
        _forward_cached(x, W, True, k, group, L.ZG_MATRIX, K, N, P, M, K, N, rank, s, y, gen)
        return _epilogue_unfused(y, act, residual)
    ws = L.workspace(L.query("zg_perturbed_linear_workspace_size", P, M, K, N, rank, code, int(x_batched)), dev)
    L.call("zg_perturbed_linear", L.ptr(x), int(x_batched), L.ptr(W), L.ptr(k), group, P, M, K, N, rank, s,
           code, L.ptr(y), L.ptr(ws), ws.numel(), L.stream_ptr(dev))
    return _epilogue_unfused(y, act, residual)


def launch_tied_logits(x: torch.Tensor, table: torch.Tensor, keys: torch.Tensor, group: int, rank: int,
                       sigma: float, x_batched: bool) -> torch.Tensor:
    dev = L.require_cuda(x, table, keys)
    k = _keys2d(keys)
    P = k.shape[0]
    if table.ndim != 2 or x.ndim < 1 or x.shape[-1] != table.shape[1]:
        raise ValueError("logit input and [rows, cols] table shapes are incompatible")
    dt = _compute_dtype(x, table)
    x = x.to(dt).contiguous()
    T = table.to(dt).contiguous()
    V, C = T.shape
    mshape = tuple(x.shape[1:-1] if x_batched else x.shape[:-1])
    M = math.prod(mshape)
    y = torch.empty((P, *mshape, V), dtype=dt, device=dev)
    if M == 0:
        return y
    s = scaled_factor_value(rank, sigma, table.dtype)
    code = L.dtype_code(dt)
    gen = CACHE.active_for(keys)
    if gen is not None and dt == torch.bfloat16 and not x_batched and _tc_ok(dev, P, C, V, rank):
        # table factors: A_t [V, q] (rows), B_t [C, q] (cols)
        _forward_cached(x, T, False, k, group, L.ZG_TABLE, V, C, P, M, C, V, rank, s, y, gen)
        return y
    if gen is not None and dt == torch.bfloat16 and x_batched and _batched_ok(dev, P, C, V, rank):
        _forward_batched(x, T, False, k, group, L.ZG_TABLE, V, C, P, M, C, V, rank, s, y, gen)
        return y
    ws = L.workspace(L.query("zg_tied_logits_workspace_size", P, M, V, C, rank, code, int(x_batched)), dev)
    L.call("zg_tied_logits", L.ptr(x), int(x_batched), L.ptr(T), L.ptr(k), group, P, M, V, C, rank, s, code,
           L.ptr(y), L.ptr(ws), ws.numel(), L.stream_ptr(dev))
    return y


def launch_tied_logits_ce(x: torch.Tensor, table: torch.Tensor, labels: torch.Tensor, keys: torch.Tensor,
                          group: int, rank: int, sigma: float, x_batched: bool) -> torch.Tensor:
    """Per-row cross-entropy of the tied logits, [P, *rows] float32, without
    materialising the logits (bf16 table and input, rank 8 or 16)."""
    dev = L.require_cuda(x, table, labels, keys)
    k = _keys2d(keys)
    P = k.shape[0]
    if table.ndim != 2 or x.shape[-1] != table.shape[1]:
        raise ValueError("logit input and [rows, cols] table shapes are incompatible")
    if x_batched and (x.ndim < 2 or x.shape[0] != P):
        raise ValueError("batched logit input must lead with the population axis")
    mshape = tuple(x.shape[1:-1] if x_batched else x.shape[:-1])
    if tuple(labels.shape) != mshape:
        raise ValueError(f"labels of shape {tuple(labels.shape)} do not match the rows {mshape}")
    if labels.dtype not in (torch.int32, torch.int64):
        raise TypeError("labels must be integer class indices")
    if table.dtype != torch.bfloat16 or x.dtype != torch.bfloat16:
        raise TypeError("the fused tied-logits cross-entropy takes bf16 tables and inputs")
    x = x.contiguous()
    T = table.contiguous()
    V, C = T.shape
    M = math.prod(mshape)
    loss = torch.empty((P, *mshape), dtype=torch.float32, device=dev)
    if M == 0:
        return loss
    s = scaled_factor_value(rank, sigma, table.dtype)
    lab = labels.to(torch.int32).contiguous()
    gen = CACHE.active_for(keys)
    if gen is not None and group >= 0:
        # the table's factors in the per-candidate-input layout (F2 = A_op,
        # F1T = B^T): this chunk's block of its id range's buffers, kept for
        # the replay like a batched tied_logits'
        F1T, F2, ld2, draw = _range_factors(gen, (group, L.ZG_TABLE, V, C, rank, _T_TAG), C, V, rank, dev)
        ws = L.workspace(L.query("zg_tied_logits_ce_ex_workspace_size", P, M, V, C, rank), dev)
        L.call("zg_tied_logits_ce_ex", L.ptr(x), int(x_batched), L.ptr(T), L.ptr(k), group, L.ptr(lab), P, M, V, C,
               rank, s, L.ptr(F1T), L.ptr(F2), ld2, int(draw), L.ptr(loss), L.ptr(ws), ws.numel(), L.stream_ptr(dev))
        return loss
    ws = L.workspace(L.query("zg_tied_logits_ce_workspace_size", P, M, V, C, rank), dev)
    L.call("zg_tied_logits_ce", L.ptr(x), int(x_batched), L.ptr(T), L.ptr(k), group, L.ptr(lab), P, M, V, C, rank,
           s, L.ptr(loss), L.ptr(ws), ws.numel(), L.stream_ptr(dev))
    return loss


def launch_table_lookup(table: torch.Tensor, indices: torch.Tensor, keys: torch.Tensor, group: int,
                        rank: int, sigma: float, idx_batched: bool) -> torch.Tensor:
    dev = L.require_cuda(table, indices, keys)
    k = _keys2d(keys)
    P = k.shape[0]
    if table.ndim != 2:
        raise ValueError("table weights must be two-dimensional")
    if indices.is_floating_point() or indices.dtype == torch.bool:
        raise TypeError("table indices must be integers")
    T = table.contiguous()
    rows, cols = T.shape
    ishape = tuple(indices.shape[1:] if idx_batched else indices.shape)
    n_idx = math.prod(ishape)
    idx = indices.to(torch.int32).contiguous()
    out = torch.empty((P, *ishape, cols), dtype=T.dtype, device=dev)
    if n_idx == 0:
        return out
    s = scaled_factor_value(rank, sigma, T.dtype)
    code = L.dtype_code(T.dtype)
    ws = L.workspace(L.query("zg_table_lookup_workspace_size", P, n_idx, rows, cols, rank, code), dev)
    L.call("zg_table_lookup", L.ptr(T), L.ptr(idx), int(idx_batched), n_idx, L.ptr(k), group, P, rows, cols,
           rank, s, code, L.ptr(out), L.ptr(ws), ws.numel(), L.stream_ptr(dev))
    return out


def launch_vector(v: torch.Tensor, keys: torch.Tensor, group: int, sigma: float, v_batched: bool) -> torch.Tensor:
    dev = L.require_cuda(v, keys)
    k = _keys2d(keys)
    P = k.shape[0]
    n = v.shape[-1]
    if (v.ndim != 1 and not v_batched) or (v_batched and v.ndim != 2):
        raise ValueError("vector weights must be one-dimensional")
    vv = v.contiguous()
    out = torch.empty((P, n), dtype=v.dtype, device=dev)
    if n == 0:
        return out
    s = scaled_factor_value(1, sigma, v.dtype)
    L.call("zg_perturbed_vector", L.ptr(vv), int(v_batched), L.ptr(k), group, P, n, s, L.dtype_code(v.dtype),
           L.ptr(out), L.stream_ptr(dev))
    return out


def launch_shape_fitness(losses: torch.Tensor, sigma: float):
    """Returns (shaped [P] float32, metrics [4] float32 = mean, min, max, #non-finite)."""
    dev = L.require_cuda(losses)
    l32 = losses.to(torch.float32).contiguous()
    P = l32.shape[0]
    shaped = torch.empty(P, dtype=torch.float32, device=dev)
    metrics = torch.empty(4, dtype=torch.float32, device=dev)
    L.call("zg_shape_fitness", L.ptr(l32), P, float(sigma), L.ptr(shaped), L.ptr(metrics), L.stream_ptr(dev))
    return shaped, metrics


def launch_replay(shaped: torch.Tensor, cand_keys: torch.Tensor, group: int, layout: int, shape, rank: int,
                  dtype: torch.dtype, out: torch.Tensor | None = None, gen: _Generation | None = None,
                  cache: FactorCache = CACHE) -> torch.Tensor:
    """Descent direction [*shape] float32 of one entry (``_replay.py:15-54``).

    With `gen` (the generation whose full population the keys are), factors
    its forward pass left in the cache are reused instead of redrawn.
    """
    dev = L.require_cuda(shaped, cand_keys)
    k = _keys2d(cand_keys)
    P = k.shape[0]
    w = shaped.to(torch.float32).contiguous()
    if w.numel() != P:
        raise ValueError("shaped weights and candidate keys differ in length")
    rows = int(shape[0])
    cols = int(shape[1]) if layout != L.ZG_VECTOR else 1
    r = rank if layout != L.ZG_VECTOR else 1
    code = L.dtype_code(dtype)
    if out is None:
        out = torch.empty(tuple(int(d) for d in shape), dtype=torch.float32, device=dev)
    inv = scaled_factor_value(r, 1.0, dtype)
    if gen is not None and layout != L.ZG_VECTOR and dtype == torch.bfloat16 and group >= 0:
        key = (gen.base, gen.start, gen.count, group, layout, rows, cols, r)
        found, hit = cache.find(key, key + (_T_TAG,))
        if hit is not None:
            A, B = hit
            # factors of a per-candidate-input forward: MATRIX keeps A^T, TABLE keeps B^T
            a_t = int(found[-1] == _T_TAG and layout == L.ZG_MATRIX)
            b_t = int(found[-1] == _T_TAG and layout == L.ZG_TABLE)
            ws = L.workspace(L.query("zg_replay_operands_workspace_size", P, rows, cols, r), dev)
            L.call("zg_replay_operands", L.ptr(w), L.ptr(A), a_t, L.ptr(B), b_t, P, rows, cols, r, inv, L.ptr(out),
                   L.ptr(ws), ws.numel(), L.stream_ptr(dev))
            return out
    ws = L.workspace(L.query("zg_replay_workspace_size", P, layout, rows, cols, r, code), dev)
    L.call("zg_replay", L.ptr(w), L.ptr(k), group, P, layout, rows, cols, r, inv, code, L.ptr(out), L.ptr(ws),
           ws.numel(), L.stream_ptr(dev))
    return out


def _replay_operands_for(cand_keys, group, layout, rows, cols, rank, gen, cache):
    """(A, a_transposed, B, b_transposed) bf16 replay operands of one entry:
    the forward's cached factors when present, else freshly drawn."""
    if gen is not None and group >= 0:
        key = (gen.base, gen.start, gen.count, group, layout, rows, cols, rank)
        found, hit = cache.find(key, key + (_T_TAG,))
        if hit is not None:
            t = found[-1] == _T_TAG
            return hit[0], int(t and layout == L.ZG_MATRIX), hit[1], int(t and layout == L.ZG_TABLE)
    A, B = operand_factors(cand_keys, group, layout, rows, cols, rank)
    return A, 0, B, 0


def launch_replay_step(shaped: torch.Tensor, cand_keys: torch.Tensor, group: int, layout: int, param: torch.Tensor,
                       rank: int, step: dict, gen: _Generation | None = None, cache: FactorCache = CACHE,
                       inplace_guard: torch.Tensor | None = None):
    """Replay of one MATRIX/TABLE entry with the optimizer step fused into the
    replay GEMM's epilogue (bf16 parameters on the tensor cores).  `step`:
    {"kind": "sgd", "lr"} or {"kind": "adamw", "lr", "b1", "b2", "eps",
    "weight_decay", "count", "mu", "nu"}.  Returns (new param, new mu, new nu)
    -- the moments None for SGD -- or None when the fused path does not apply
    (the caller then replays and updates separately, with identical results).
    With `inplace_guard` (a device float32 scalar) the step updates param and
    the moments in place and writes nothing when the guard is non-zero."""
    dev = L.require_cuda(shaped, cand_keys, param)
    k = _keys2d(cand_keys)
    P = k.shape[0]
    if (layout == L.ZG_VECTOR or param.dtype != torch.bfloat16 or param.ndim != 2 or not param.is_contiguous()
            or torch.cuda.get_device_capability(dev) != (10, 0) or (P * rank) % 8 != 0):
        return None
    rows, cols = (int(d) for d in param.shape)
    w = shaped.to(torch.float32).contiguous()
    if w.numel() != P:
        raise ValueError("shaped weights and candidate keys differ in length")
    A, a_t, B, b_t = _replay_operands_for(k, group, layout, rows, cols, rank, gen, cache)
    if b_t and cols % 8:
        return None
    inv = scaled_factor_value(rank, 1.0, param.dtype)
    ws = L.workspace(L.query("zg_replay_operands_workspace_size", P, rows, cols, rank), dev)
    inplace = inplace_guard is not None
    if inplace and (inplace_guard.dtype != torch.float32 or inplace_guard.device != dev):
        raise TypeError("the guard is a float32 scalar on the parameter's device")
    guard = L.ptr(inplace_guard) if inplace else None
    out = param if inplace else torch.empty_like(param)
    st = L.stream_ptr(dev)
    if step["kind"] == "sgd":
        L.call("zg_replay_sgd", L.ptr(w), L.ptr(A), a_t, L.ptr(B), b_t, P, rows, cols, rank, inv, L.ptr(param),
               L.ptr(out), L.ZG_BF16, float(step["lr"]), None, guard, L.ptr(ws), ws.numel(), st)
        return out, None, None
    mu, nu = step["mu"].contiguous(), step["nu"].contiguous()
    if inplace and (mu is not step["mu"] or nu is not step["nu"]):
        raise ValueError("an in-place step needs contiguous moments")
    mu_out = mu if inplace else torch.empty_like(mu)
    nu_out = nu if inplace else torch.empty_like(nu)
    L.call("zg_replay_adamw", L.ptr(w), L.ptr(A), a_t, L.ptr(B), b_t, P, rows, cols, rank, inv, L.ptr(param),
           L.ptr(out), L.ZG_BF16, L.ptr(mu), L.ptr(nu), L.ptr(mu_out), L.ptr(nu_out), int(step["count"]),
           float(step["lr"]), float(step["b1"]), float(step["b2"]), float(step["eps"]), float(step["weight_decay"]),
           None, guard, L.ptr(step.get("bc")), L.ptr(ws), ws.numel(), st)
    return out, mu_out, nu_out


def launch_adamw(param: torch.Tensor, descent: torch.Tensor | None, mu: torch.Tensor, nu: torch.Tensor,
                 count: int, lr: float, b1: float, b2: float, eps: float, weight_decay: float,
                 bias_corrections: torch.Tensor | None = None):
    dev = L.require_cuda(param, descent, mu, nu)
    p_out = torch.empty_like(param)
    mu_out = torch.empty_like(mu)
    nu_out = torch.empty_like(nu)
    d = None if descent is None else descent.to(torch.float32).contiguous()
    L.call("zg_adamw_update", L.ptr(param.contiguous()), L.ptr(p_out), L.dtype_code(param.dtype), L.ptr(d),
           L.ptr(mu), L.ptr(nu), L.ptr(mu_out), L.ptr(nu_out), param.numel(), count, lr, b1, b2, eps,
           weight_decay, L.ptr(bias_corrections), L.stream_ptr(dev))
    return p_out, mu_out, nu_out


def launch_sgd(param: torch.Tensor, descent: torch.Tensor | None, lr: float) -> torch.Tensor:
    dev = L.require_cuda(param, descent)
    p_out = torch.empty_like(param)
    d = None if descent is None else descent.to(torch.float32).contiguous()
    L.call("zg_sgd_update", L.ptr(param.contiguous()), L.ptr(p_out), L.dtype_code(param.dtype), L.ptr(d),
           param.numel(), lr, L.stream_ptr(dev))
    return p_out


def launch_int8_lut_linear(x: torch.Tensor, weight: torch.Tensor, w_scale: torch.Tensor, x_scale: float,
                           y_scale: float, lut: torch.Tensor, keys: torch.Tensor, group: int, rank: int,
                           sigma: float, x_batched: bool, return_acc: bool = False):
    dev = L.require_cuda(x, weight, w_scale, lut, keys)
    k = _keys2d(keys)
    P = k.shape[0]
    if x.dtype != torch.int8 or weight.dtype != torch.int8 or lut.dtype != torch.int8:
        raise TypeError("int8 linear takes int8 activations, weights and LUT")
    if weight.ndim != 2 or x.shape[-1] != weight.shape[0] or lut.numel() != 256:
        raise ValueError("int8 linear shapes are incompatible")
    K, N = weight.shape
    mshape = tuple(x.shape[1:-1] if x_batched else x.shape[:-1])
    M = math.prod(mshape)
    out = torch.empty((P, *mshape, N), dtype=torch.int8, device=dev)
    acc = torch.empty((P, *mshape, N), dtype=torch.int32, device=dev) if return_acc else None
    s = round_scalar(sigma / math.sqrt(rank), torch.float32)
    ws = L.workspace(L.query("zg_int8_lut_linear_workspace_size", P, M, K, N, rank, int(x_batched)), dev)
    L.call("zg_int8_lut_linear", L.ptr(x.contiguous()), int(x_batched), L.ptr(weight.contiguous()),
           L.ptr(w_scale.to(torch.float32).contiguous()), float(x_scale), float(y_scale), L.ptr(lut.contiguous()),
           L.ptr(k), group, P, M, K, N, rank, s, L.ptr(out), L.ptr(acc), L.ptr(ws), ws.numel(), L.stream_ptr(dev))
    return (out, acc) if return_acc else out


# ---------------------------------------------------------------------------
# custom ops (single-candidate semantics) + vmap rules (population launch)
# ---------------------------------------------------------------------------

_NS = "zerograd_b200"


def _movedim0(t, d):
    return t if d is None or d == 0 else t.movedim(d, 0)


@torch.library.custom_op(f"{_NS}::fold_in", mutates_args=())
def _fold_in_op(key: torch.Tensor, data: torch.Tensor) -> torch.Tensor:
    return launch_fold_in(key, data).reshape(2)


@torch.library.register_vmap(f"{_NS}::fold_in")
def _fold_in_vmap(info, in_dims, key, data):
    kd, dd = in_dims
    key = _movedim0(key, kd)
    data = _movedim0(data, dd)
    return launch_fold_in(key, data), 0


def fold_in(key: torch.Tensor, data) -> torch.Tensor:
    if isinstance(data, int):
        data = torch.tensor(data & 0xFFFFFFFF, dtype=torch.int64, device=key.device)
    return _fold_in_op(key, data)


@torch.library.custom_op(f"{_NS}::linear", mutates_args=())
def _linear_op(x: torch.Tensor, weight: torch.Tensor, key: torch.Tensor, group: int, rank: int,
               sigma: float, act: int, residual: torch.Tensor | None) -> torch.Tensor:
    res = None if residual is None else residual.unsqueeze(0)
    return launch_linear(x, weight, key.reshape(1, 2), group, rank, sigma, False, act, res)[0]


@torch.library.register_vmap(f"{_NS}::linear")
def _linear_vmap(info, in_dims, x, weight, key, group, rank, sigma, act, residual):
    xd, wd, kd = in_dims[:3]
    rd = in_dims[7]
    if wd is not None:
        raise NotImplementedError("weights batched over candidates are not supported")
    x = _movedim0(x, xd)
    if kd is None:
        # one key for every batch row: a single candidate's op over the rows
        y = _epilogue_unfused(launch_linear(x, weight, key.reshape(1, 2), group, rank, sigma, False)[0], act, None)
        if residual is not None:
            y = _movedim0(residual, rd).to(y.dtype) + y if rd is not None else residual.to(y.dtype) + y
        return y, 0
    keys = _movedim0(key, kd)
    P = keys.shape[0]
    res = None
    if residual is not None:
        res = _movedim0(residual, rd) if rd is not None else residual.unsqueeze(0).expand(P, *residual.shape)
    return launch_linear(x, weight, keys, group, rank, sigma, xd is not None, act, res), 0


@torch.library.custom_op(f"{_NS}::tied_logits", mutates_args=())
def _tied_op(x: torch.Tensor, table: torch.Tensor, key: torch.Tensor, group: int, rank: int,
             sigma: float) -> torch.Tensor:
    return launch_tied_logits(x, table, key.reshape(1, 2), group, rank, sigma, False)[0]


@torch.library.register_vmap(f"{_NS}::tied_logits")
def _tied_vmap(info, in_dims, x, table, key, group, rank, sigma):
    xd, td, kd = in_dims[:3]
    if td is not None:
        raise NotImplementedError("tables batched over candidates are not supported")
    x = _movedim0(x, xd)
    if kd is None:
        return launch_tied_logits(x, table, key.reshape(1, 2), group, rank, sigma, False)[0], 0
    return launch_tied_logits(x, table, _movedim0(key, kd), group, rank, sigma, xd is not None), 0


def launch_row_mean(x: torch.Tensor) -> torch.Tensor:
    """[P, ...] float32 -> [P]: each leading row's mean, float64 accumulation
    in a fixed order (independent of P)."""
    dev = L.require_cuda(x)
    x2 = x.to(torch.float32).reshape(x.shape[0], -1).contiguous()
    out = torch.empty(x.shape[0], dtype=torch.float32, device=dev)
    L.call("zg_row_mean", L.ptr(x2), x2.shape[0], x2.shape[1], L.ptr(out), L.stream_ptr(dev))
    return out


def _ce_reduce(loss: torch.Tensor, mean: bool) -> torch.Tensor:
    return launch_row_mean(loss) if mean else loss


@torch.library.custom_op(f"{_NS}::tied_logits_ce", mutates_args=())
def _tied_ce_op(x: torch.Tensor, table: torch.Tensor, labels: torch.Tensor, key: torch.Tensor, group: int,
                rank: int, sigma: float, mean: bool) -> torch.Tensor:
    return _ce_reduce(launch_tied_logits_ce(x, table, labels, key.reshape(1, 2), group, rank, sigma, False), mean)[0]


@torch.library.register_vmap(f"{_NS}::tied_logits_ce")
def _tied_ce_vmap(info, in_dims, x, table, labels, key, group, rank, sigma, mean):
    xd, td, ld, kd = in_dims[:4]
    if td is not None or ld is not None:
        raise NotImplementedError("tables and labels batched over candidates are not supported")
    x = _movedim0(x, xd)
    if kd is None:
        out = _ce_reduce(launch_tied_logits_ce(x, table, labels, key.reshape(1, 2), group, rank, sigma, False), mean)
        return out[0], None
    return _ce_reduce(launch_tied_logits_ce(x, table, labels, _movedim0(key, kd), group, rank, sigma, xd is not None),
                      mean), 0


@torch.library.custom_op(f"{_NS}::table_lookup", mutates_args=())
def _lookup_op(table: torch.Tensor, indices: torch.Tensor, key: torch.Tensor, group: int, rank: int,
               sigma: float) -> torch.Tensor:
    return launch_table_lookup(table, indices, key.reshape(1, 2), group, rank, sigma, False)[0]


@torch.library.register_vmap(f"{_NS}::table_lookup")
def _lookup_vmap(info, in_dims, table, indices, key, group, rank, sigma):
    td, idd, kd = in_dims[:3]
    if td is not None:
        raise NotImplementedError("tables batched over candidates are not supported")
    indices = _movedim0(indices, idd)
    if kd is None:
        return launch_table_lookup(table, indices, key.reshape(1, 2), group, rank, sigma, False)[0], 0
    return launch_table_lookup(table, indices, _movedim0(key, kd), group, rank, sigma, idd is not None), 0


@torch.library.custom_op(f"{_NS}::vector", mutates_args=())
def _vector_op(v: torch.Tensor, key: torch.Tensor, group: int, sigma: float) -> torch.Tensor:
    return launch_vector(v, key.reshape(1, 2), group, sigma, False)[0]


@torch.library.register_vmap(f"{_NS}::vector")
def _vector_vmap(info, in_dims, v, key, group, sigma):
    vd, kd = in_dims[:2]
    v = _movedim0(v, vd)
    if kd is None:
        # shared key, batched leaf: each row gets the same noise
        return launch_vector(v.reshape(-1, v.shape[-1]), key.reshape(1, 2).expand(v.shape[0], 2), group, sigma,
                             True), 0
    return launch_vector(v, _movedim0(key, kd), group, sigma, vd is not None), 0


@torch.library.custom_op(f"{_NS}::normal", mutates_args=())
def _normal_op(key: torch.Tensor, n: int, dtype_code: int) -> torch.Tensor:
    return launch_normal(key.reshape(1, 2), n, torch.bfloat16 if dtype_code == L.ZG_BF16 else torch.float32)[0]


@torch.library.register_vmap(f"{_NS}::normal")
def _normal_vmap(info, in_dims, key, n, dtype_code):
    key = _movedim0(key, in_dims[0])
    return launch_normal(key, n, torch.bfloat16 if dtype_code == L.ZG_BF16 else torch.float32), 0


@torch.library.custom_op(f"{_NS}::bits", mutates_args=())
def _bits_op(key: torch.Tensor, n: int) -> torch.Tensor:
    return launch_bits(key.reshape(1, 2), n)[0]


@torch.library.register_vmap(f"{_NS}::bits")
def _bits_vmap(info, in_dims, key, n):
    return launch_bits(_movedim0(key, in_dims[0]), n), 0


@torch.library.custom_op(f"{_NS}::int8_lut_linear", mutates_args=())
def _int8_op(x: torch.Tensor, w_q: torch.Tensor, w_scale: torch.Tensor, lut: torch.Tensor, key: torch.Tensor,
             group: int, rank: int, sigma: float, x_scale: float, y_scale: float) -> torch.Tensor:
    return launch_int8_lut_linear(x, w_q, w_scale, x_scale, y_scale, lut, key.reshape(1, 2), group, rank, sigma,
                                  False)[0]


@torch.library.register_vmap(f"{_NS}::int8_lut_linear")
def _int8_vmap(info, in_dims, x, w_q, w_scale, lut, key, group, rank, sigma, x_scale, y_scale):
    xd, wd, sd, ld, kd = in_dims[:5]
    if wd is not None or sd is not None or ld is not None:
        raise NotImplementedError("int8 weights, scales and LUTs batched over candidates are not supported")
    x = _movedim0(x, xd)
    if kd is None:
        return launch_int8_lut_linear(x, w_q, w_scale, x_scale, y_scale, lut, key.reshape(1, 2), group, rank, sigma,
                                      False)[0], 0
    return launch_int8_lut_linear(x, w_q, w_scale, x_scale, y_scale, lut, _movedim0(key, kd), group, rank, sigma,
                                  xd is not None), 0


def int8_lut_linear(x, w_q, w_scale, lut, key, group, rank, sigma, x_scale, y_scale):
    return _int8_op(x, w_q, w_scale, lut, key, int(group), int(rank), float(sigma), float(x_scale), float(y_scale))


def quantize_int8_columns(weight: torch.Tensor):
    """Per-output-channel symmetric int8 quantisation of a [K, N] weight:
    scale[n] = max_k |W[k, n]| / 127 (float32; 1 for an all-zero column),
    W_q = clamp(rint(W / scale), -127, 127) (int8)."""
    W = weight.to(torch.float32)
    scale = W.abs().amax(dim=0) / 127.0
    scale = torch.where(scale > 0, scale, torch.ones_like(scale))
    return torch.clamp(torch.round(W / scale), -127, 127).to(torch.int8), scale


def linear(x, weight, key, group, rank, sigma, activation=None, residual=None):
    if activation not in ACTIVATIONS:
        raise ValueError(f"unknown activation {activation!r}: expected one of None, 'gelu'")
    return _linear_op(x, weight, key, int(group), int(rank), float(sigma), ACTIVATIONS[activation], residual)


@torch.library.custom_op(f"{_NS}::gelu", mutates_args=())
def _gelu_op(x: torch.Tensor) -> torch.Tensor:
    return launch_gelu(x)


@torch.library.register_vmap(f"{_NS}::gelu")
def _gelu_vmap(info, in_dims, x):
    return launch_gelu(x), in_dims[0]


def gelu(x: torch.Tensor) -> torch.Tensor:
    """GELU in its tanh form, 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
    (the form GPT-2 uses), element-wise in float32, rounded to x's dtype;
    the same values as ``CandidateContext.linear(..., activation="gelu")``
    produces in its epilogue."""
    return _gelu_op(x)


def tied_logits(x, table, key, group, rank, sigma):
    return _tied_op(x, table, key, int(group), int(rank), float(sigma))


def tied_logits_ce(x, table, labels, key, group, rank, sigma, reduction="none"):
    if reduction not in ("none", "mean"):
        raise ValueError(f"reduction must be 'none' or 'mean', got {reduction!r}")
    return _tied_ce_op(x, table, labels, key, int(group), int(rank), float(sigma), reduction == "mean")


def table_lookup(table, indices, key, group, rank, sigma):
    return _lookup_op(table, indices, key, int(group), int(rank), float(sigma))


def vector(v, key, group, sigma):
    return _vector_op(v, key, int(group), float(sigma))


def normal(key, n: int, dtype: torch.dtype = torch.float32):
    return _normal_op(key, int(n), L.dtype_code(dtype))


def bits(key, n: int):
    return _bits_op(key, int(n))

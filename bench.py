#!/usr/bin/env python
"""Throughput of one ES generation of the decoder-LM workload under zerograd's API.

Workload (the reference's decoder-LM configuration): a decoder-only
transformer with tied embeddings -- vocabulary 32000 (a TABLE entry read by
``table_lookup`` and by the tied logits), width 768, 12 layers of causal
12-head attention and a GELU MLP of width 3072 (the configuration leaves the
MLP width open: 4x width, as GPT-2), RMSNorm scales as VECTOR entries, bf16
-- evaluated for a population of 2048 candidates at rank 16, sigma 0.01, on
a batch of 16 sequences of 256 tokens uniform over the vocabulary, loss the
next-token cross-entropy; then the fitness shaping (the reference's
centred-loss rule), the factor replay of all 74 entries and the SGD update.
One step = one generation, run as the public API runs it: ``ZeroGrad`` with
``chunk_size`` (the population evaluated 128 candidates at a time),
``ZeroGrad.capture`` (the generation as one CUDA graph, the next
generation's factors drawn beside it).  Synthetic seeded data and weights.

`python bench.py [--gpus N --steps K --warmup W]` prints one JSON line.  With
N > 1 (one process per GPU under torch.distributed.run) the population is
sharded across ranks, the fitness array is all-gathered (the only
collective) and every rank replays the identical update; the line carries
a hash of every rank's parameters after the timed generations.
`--impl reference` times the CPU restatement of the reference's algorithm
(the reference is JAX code that cannot be installed here) on this host's
cores, on a sample of candidates per step.

Secondary sections (one GPU, `--sections all`, the default): the
perturbed-GEMM microbench (shared and per-candidate input, with the replay
GEMM), the f32 MLP configuration's whole generation on the GPU and on the
host, and the int8 QAT layer.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "candidate forward evals/sec"
UNIT = "evals/s"
LM = dict(vocab=32000, width=768, layers=12, heads=12, mlp=3072, seq=256, batch=16, P=2048, rank=16, sigma=0.01,
          seed=0, run_id="lm", lr=1e-3, chunk=128)
CPU_SAMPLE = 1  # candidates per step in both CPU legs (the same sample)


def lm_workload_name(cfg=LM) -> str:
    return (f"decoder LM, tied vocab {cfg['vocab']} TABLE, d {cfg['width']}, {cfg['layers']} layers, {cfg['heads']} "
            f"heads causal, GELU MLP {cfg['mlp']}, RMSNorm VECTOR scales, bf16; P={cfg['P']}, rank {cfg['rank']}, "
            f"sigma {cfg['sigma']}, batch {cfg['batch']}x{cfg['seq']} tokens, next-token CE; centred-loss shaping, "
            f"replay + SGD of every entry")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    # "headline": the decoder-LM generation alone; "all" adds the secondary
    # workloads and the CPU baseline on one GPU; "profile": small cases for
    # ncu captures (two evaluations of a 2-layer decoder-LM chunk of 16
    # candidates at the LM's shapes, then that model's replay for 2048
    # candidates), no JSON line
    ap.add_argument("--sections", choices=["all", "headline", "profile"], default="all")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count()


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock and clock-event reasons sampled through NVML every 5 ms
    while the timed region runs (read-only queries)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, device):
        self.device = device
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = None
        self._thread = None

    def _handle(self, nv):
        import torch

        props = torch.cuda.get_device_properties(self.device)
        bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        return nv.nvmlDeviceGetHandleByPciBusId(bus)

    def __enter__(self):
        import threading

        try:
            import pynvml as nv

            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception:
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                    bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    for b, name in self.REASONS.items():
                        if bits & b:
                            self.reasons.add(name)
                except Exception:
                    pass
                self._stop.wait(0.005)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(2)
        return False

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}




def traffic_for(name: str):
    """DRAM bytes per launch of a kernel from the committed ncu summary, or None."""
    tpath = os.path.join(ROOT, "profiles", "traffic.txt")
    if os.path.exists(tpath):
        for tl in open(tpath):
            parts = tl.split()
            if len(parts) == 2 and not tl.startswith("#") and parts[0] == name:
                return int(parts[1])
    return None


# ---------------------------------------------------------------------------
# the decoder-LM workload
# ---------------------------------------------------------------------------
def lm_entries(cfg=LM) -> list:
    names = ["emb"]
    for layer in range(cfg["layers"]):
        names += [f"l{layer}.{n}" for n in ("n1", "qkv", "o", "n2", "fc", "proj")]
    return names + ["nf"]


def lm_layouts(cfg=LM) -> dict:
    """Entry name -> layout code (0 MATRIX, 1 TABLE, 2 VECTOR)."""
    out = {}
    for n in lm_entries(cfg):
        tail = n.rsplit(".", 1)[-1]
        out[n] = 1 if n == "emb" else 2 if tail in ("n1", "n2", "nf") else 0
    return out


def lm_manifest(cfg=LM):
    import zerograd_b200 as zg

    kinds = {0: zg.ParameterLayout.MATRIX, 1: zg.ParameterLayout.TABLE, 2: zg.ParameterLayout.VECTOR}
    lay = lm_layouts(cfg)
    return zg.Manifest(1, tuple(zg.ManifestEntry((n,), kinds[lay[n]], n) for n in lm_entries(cfg)))


def lm_shapes(cfg=LM) -> dict:
    E, F, V = cfg["width"], cfg["mlp"], cfg["vocab"]
    out = {"emb": (V, E), "nf": (E,)}
    for layer in range(cfg["layers"]):
        p = f"l{layer}."
        out.update({p + "n1": (E,), p + "qkv": (E, 3 * E), p + "o": (E, E), p + "n2": (E,), p + "fc": (E, F),
                    p + "proj": (F, E)})
    return out


def lm_params_host(cfg=LM, seed=0) -> dict:
    """Seeded synthetic weights (bf16): N(0, 0.02) matrices and table, unit norm scales."""
    import torch

    g = torch.Generator().manual_seed(seed)
    out = {}
    for n, shape in lm_shapes(cfg).items():
        if len(shape) == 1:
            out[n] = torch.ones(shape, dtype=torch.bfloat16)
        else:
            out[n] = (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16)
    return out


def lm_batch_host(cfg=LM, seed=0):
    """Tokens uniform over the vocabulary: inputs [B, T] and their next tokens [B, T] (int32)."""
    import torch

    g = torch.Generator().manual_seed(seed + 1)
    t = torch.randint(0, cfg["vocab"], (cfg["batch"], cfg["seq"] + 1), generator=g, dtype=torch.int64)
    return t[:, :-1].to(torch.int32).contiguous(), t[:, 1:].to(torch.int32).contiguous()


def make_lm_loss(cfg=LM):
    import zerograd_b200 as zg

    B, T, E, H = cfg["batch"], cfg["seq"], cfg["width"], cfg["heads"]
    D = E // H

    def loss_fn(p, ctx, batch, rng):
        tokens, labels = batch
        x = ctx.table_lookup(p, ("emb",), tokens)
        for layer in range(cfg["layers"]):
            n = f"l{layer}."
            h = zg.rms_norm(x, ctx.vector(p, (n + "n1",)))
            qkv = ctx.linear(p, (n + "qkv",), h).view(B, T, 3, H, D)
            a = zg.attention(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], causal=True)
            x = ctx.linear(p, (n + "o",), a.reshape(B, T, E), residual=x)
            h = zg.rms_norm(x, ctx.vector(p, (n + "n2",)))
            m = ctx.linear(p, (n + "fc",), h, activation="gelu")
            x = ctx.linear(p, (n + "proj",), m, residual=x)
        h = zg.rms_norm(x, ctx.vector(p, ("nf",)))
        return ctx.tied_logits_cross_entropy(p, ("emb",), h, labels, reduction="mean"), None

    return loss_fn


def lm_work(cfg=LM, P=None):
    """Algorithmic work of P candidates' forward, by kernel family: FLOPs of
    the projections (dense x W plus the rank-r term U F2^T), of attention
    (the causal pairs only: q.k and p.v over the S(S+1)/2 visible pairs),
    of the tied logits (dense + rank-r) and of the replay GEMMs; bytes of
    the norms, the lookup, the low-rank u passes and attention (q, k, v read,
    o written)."""
    P = cfg["P"] if P is None else P
    tok = cfg["batch"] * cfg["seq"]
    E, F, L, V, r, S, H = cfg["width"], cfg["mlp"], cfg["layers"], cfg["vocab"], cfg["rank"], cfg["seq"], cfg["heads"]
    projs = [(E, 3 * E), (E, E), (E, F), (F, E)]
    dense = sum(K * N for K, N in projs)
    lowrank = sum(r * N for K, N in projs)
    work = {
        "batched_gemm": 2.0 * tok * P * L * (dense + lowrank),
        "attention": 4.0 * cfg["batch"] * H * (S * (S + 1) / 2) * (E // H) * P * L,
        "tied_ce": 2.0 * tok * V * (E + r) * P,
        "batched_u_pass": float(P * L * sum(tok * K * 2 + tok * 16 * 2 for K, N in projs)) + P * tok * E * 2.0,
        "rms_norm": float(P * (2 * L + 1) * tok * E * 2 * 2),
        "table_lookup": float(P * tok * E * 2 * 2),
        # this rank's candidates: the exchanged update contracts only those
        "replay_gemm": 2.0 * (L * dense + V * E) * P * r,
        # attention's HBM bytes: q, k and v read, o written
        "attention_bytes": float(4 * P * L * tok * E * 2),
    }
    bound = {"batched_gemm": "tensor", "attention": "tensor", "tied_ce": "tensor", "replay_gemm": "tensor",
             "batched_u_pass": "hbm", "rms_norm": "hbm", "table_lookup": "hbm"}
    return work, bound


# ---------------------------------------------------------------------------
# CPU legs: the oracle restatement on a bounded sample of candidates
# ---------------------------------------------------------------------------
def lm_cpu_sample(n_cand: int, step: int = 0):
    """Forward of `n_cand` candidates of generation `step` of the decoder-LM
    workload plus their share of the replay of every entry, on the host
    cores in float32 numpy (BLAS) over the C threefry restatement.  Returns
    seconds."""
    import numpy as np

    from oracle import lm as olm
    from oracle import ref

    cfg = LM
    params = {k: v.float().numpy() for k, v in lm_params_host(cfg, cfg["seed"]).items()}
    tokens, labels = (t.numpy() for t in lm_batch_host(cfg, cfg["seed"]))
    entries = lm_entries(cfg)
    base = ref.step_key(cfg["seed"], cfg["run_id"], step, 1)
    ids = range(n_cand)
    t0 = time.perf_counter()
    losses = olm.population_losses(params, entries, base, ids, {"layers": cfg["layers"], "heads": cfg["heads"]},
                                   tokens, labels, cfg["rank"], cfg["sigma"], np.float32)
    shaped = ref.shape_centered_loss(losses.astype(np.float32), cfg["sigma"])
    olm.replay_sample(params, entries, lm_layouts(cfg), base, ids, shaped, cfg["rank"])
    return time.perf_counter() - t0


CPU_SAMPLE_TEXT = (f"{CPU_SAMPLE} of {LM['P']} candidates per step (their forward through all {LM['layers']} layers "
                   "and the tied CE, plus their share of the replay of every entry); float32 numpy/BLAS on all host "
                   "threads + the C threefry restatement; per-candidate rate, extrapolated to the population")


def lm_cpu_baseline(steps: int):
    from oracle import ref

    ref.lib()
    times = [lm_cpu_sample(CPU_SAMPLE, s) for s in range(steps)]
    total = sum(times)
    return {"value": CPU_SAMPLE * steps / total, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
            "sample": CPU_SAMPLE_TEXT, "steps": steps, "ms_per_step": 1e3 * total / steps}


def lm_config(world: int) -> dict:
    return {"workload": lm_workload_name(), "population": LM["P"], "rank": LM["rank"], "layers": LM["layers"],
            "width": LM["width"], "vocab": LM["vocab"], "batch": f"{LM['batch']}x{LM['seq']} tokens",
            "chunk_size": LM["chunk"],
            "parallelism": (f"population shards x{world}, fitness all-gather, exchanged update (each rank "
                            "contracts its own candidates' factors; partial replays all-to-all, fixed-order sums, "
                            "parameters all-gathered)" if world > 1 else "1 GPU"),
            "l2": "inputs larger than L2 (each chunk's activations are GBs); 256 MiB flush between generations",
            "sample_cpu": f"{CPU_SAMPLE} candidate(s) per step"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import ref

    ref.lib()
    for w in range(max(1, min(args.warmup, 1))):
        lm_cpu_sample(CPU_SAMPLE, 1000 + w)
    times = [lm_cpu_sample(CPU_SAMPLE, s) for s in range(args.steps)]
    total = sum(times)
    value = CPU_SAMPLE * args.steps / total
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
        "config": lm_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
                         "sample": CPU_SAMPLE_TEXT},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
class Ranks:
    """Rank, world size, barrier and max-over-ranks for the timed regions."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist

        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != args.gpus:
            raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={self.world}")
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.dist = dist
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=self.dev)

    def barrier(self):
        import torch

        if self.world > 1:
            self.dist.barrier(device_ids=[self.local])
        torch.cuda.synchronize()

    def max(self, v: float) -> float:
        import torch

        if self.world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather_ints(self, v: int) -> list:
        import torch

        if self.world == 1:
            return [v]
        t = torch.tensor([v], dtype=torch.int64, device=self.dev)
        out = torch.empty(self.world, dtype=torch.int64, device=self.dev)
        self.dist.all_gather_into_tensor(out, t)
        return [int(x) for x in out.tolist()]


def params_hash(params: dict) -> int:
    """A position-weighted checksum of every parameter's bits (ranks that
    replayed the same update hold the same value)."""
    import torch

    h = 0
    for i, name in enumerate(sorted(params)):
        t = params[name].contiguous().view(-1).view(torch.int16).to(torch.int64)
        w = torch.arange(1, t.numel() + 1, device=t.device, dtype=torch.int64) % 65521
        h = (h * 1000003 + int((t * w).sum().item()) + i) % (1 << 61)
    return h


def lm_section(args, R):
    """The headline: the decoder-LM generation on this rank's shard."""
    import torch

    import zerograd_b200 as zg
    from zerograd_b200 import _lib as L

    cfg = LM
    dev, world, rank = R.dev, R.world, R.rank
    P, r = cfg["P"], cfg["rank"]
    sizes = zg.compute_partition_sizes(P, [1.0] * world)
    a = sum(sizes[:rank])
    P_local = sizes[rank]
    manifest = lm_manifest(cfg)
    params = {k: v.to(dev) for k, v in lm_params_host(cfg, cfg["seed"]).items()}
    tok_h, lab_h = (t.pin_memory() for t in lm_batch_host(cfg, cfg["seed"]))
    batch = (tok_h.to(dev), lab_h.to(dev))
    loss_fn = make_lm_loss(cfg)
    opt = zg.ZeroGrad(manifest, zg.sgd(cfg["lr"]), P, r, cfg["sigma"], cfg["seed"], cfg["run_id"],
                      chunk_size=cfg["chunk"])
    gather = (lambda l: zg.allgather_losses(l, sizes)) if world > 1 else None
    exchange = zg.ExchangedReplay(rank, world, a, P_local) if world > 1 else None
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    cg = zg.CapturedGeneration(opt, params, loss_fn, batch, state=opt.init(params),
                               candidate_range=(a, P_local) if world > 1 else None, gather=gather,
                               exchange=exchange)
    cstate = opt.init(params)
    pending = []

    def enqueue(gen, host_batch=None):
        nonlocal cstate
        _, cstate, pend = cg.enqueue(zg.ZeroGradState(gen, cstate.opt_state), host_batch)
        pending.append(pend)

    for i in range(args.warmup):
        enqueue(i)
    R.barrier()
    # timed: inputs resident, generations queued back to back, metrics read after
    ev = []
    with ClockSampler(dev) as clk:
        R.barrier()
        for i in range(args.steps):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            enqueue(args.warmup + i)
            e.record()
            ev.append((s, e))
        torch.cuda.synchronize()
        R.barrier()
    ms = R.max(sum(s.elapsed_time(e) for s, e in ev))
    clocks = clk.summary()
    launches = cg.kernels_per_generation * args.steps
    metrics = [p.result() for p in pending]
    pending.clear()

    # end to end through the public API: the batch (tokens + labels) copied in
    # from pinned host memory every generation on the copy stream while the
    # previous generation runs, generation g-1's metrics read on the host
    # before g+1 is queued; one device interval, flushes subtracted
    e2e_steps = max(1, min(args.steps, 6))

    def pipelined(steps, first):
        pend, flushes = [], []
        mk = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
        start, end = mk(), mk()
        start.record()
        for i in range(steps):
            f0, f1 = mk(), mk()
            f0.record()
            flush.zero_()
            f1.record()
            flushes.append((f0, f1))
            enqueue(first + i, (tok_h, lab_h))
            pend.append(pending.pop())
            if i >= 1:
                pend[i - 1].result()
        pend[-1].result()
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) - sum(x.elapsed_time(y) for x, y in flushes)

    pipelined(2, 100)
    R.barrier()
    e2e_ms = R.max(pipelined(e2e_steps, 200))
    R.barrier()
    hashes = R.gather_ints(params_hash(cg.params))
    del cg  # holds NCCL work with more than one rank: released before the process group
    torch.cuda.synchronize()

    # per-kernel device times: one eager generation (this rank's shard, the
    # all-gather, the completion) with events around every launch
    R.barrier()
    L.profile_begin(1 << 16)
    losses = opt.evaluate_shard(params, 300, loss_fn, batch, range(a, a + P_local))
    if world > 1:
        losses = zg.allgather_losses(losses, sizes)
    opt._step_from_losses(zg.ZeroGradState(300, opt.init(params).opt_state), params, losses, exchange=exchange)
    kernels = L.profile_end()
    R.barrier()
    return {"ms": ms, "e2e_ms": e2e_ms, "e2e_steps": e2e_steps, "clocks": clocks, "launches": launches,
            "kernels": kernels, "P_local": P_local, "hashes": hashes, "mean_loss": metrics[-1].mean_loss,
            "h2d": tok_h.nbytes + lab_h.nbytes + 32, "d2h": 16}


def lm_roofline(kern: dict, P_local: int) -> dict:
    """Roofline of the kernel family that takes the most time in one
    generation: its algorithmic work over its event-timed launches."""
    pk = peaks()
    work, bound = lm_work(LM, P_local)
    known = {k: v for k, v in kern.items() if k in work}
    name, (n, tot) = max(known.items(), key=lambda kv: kv[1][1])
    sec = tot / 1e3
    if bound[name] == "hbm":
        ach, peak, unit, src = work[name] / sec / 1e9, pk["hbm_gbs"], "GB/s", pk["source"]
    else:
        # a generation keeps the tensor cores busy for seconds: the sustained (power-capped) peak
        ach, peak, unit = work[name] / sec / 1e12, pk["bf16_tflops_sustained"], "TFLOP/s"
        src = pk["source"] + " (sustained)"
    return {"kernel": name, "bound": bound[name], "achieved": ach, "peak": peak, "unit": unit, "frac": ach / peak,
            "traffic": traffic_for(f"lm_{name}"), "peak_source": src, "launches": n, "launch_ms": tot / n,
            "frac_of_burst_peak": (ach / pk["bf16_tflops"]) if bound[name] == "tensor" else None}


def family_rates(kern: dict, P_local: int) -> dict:
    """Achieved rate of every kernel family with a work figure."""
    pk = peaks()
    work, bound = lm_work(LM, P_local)
    out = {}
    for name, (n, tot) in kern.items():
        if name not in work or tot <= 0:
            continue
        sec = tot / 1e3
        if bound[name] == "hbm":
            out[name] = {"GB/s": work[name] / sec / 1e9, "frac_hbm": work[name] / sec / 1e9 / pk["hbm_gbs"],
                         "ms": tot}
        else:
            out[name] = {"TFLOP/s": work[name] / sec / 1e12,
                         "frac_sustained": work[name] / sec / 1e12 / pk["bf16_tflops_sustained"], "ms": tot}
        if name == "attention":  # bound by its loads and softmax latency more than by the tensor cores
            gbs = work["attention_bytes"] / sec / 1e9
            out[name].update({"GB/s": gbs, "frac_hbm": gbs / pk["hbm_gbs"]})
    return out


def profile_case(dev):
    """Small cases for ncu captures, at the decoder LM's shapes: two
    evaluations of a 2-layer chunk of 16 candidates (every forward kernel of
    the headline), then the replay and SGD step of the same 2-layer model for
    the headline's population (2048 candidates, rank 16: the replay split
    over candidate groups) from synthetic losses."""
    import torch

    import zerograd_b200 as zg

    cfg = dict(LM, layers=2, P=16, chunk=16)
    params = {k: v.to(dev) for k, v in lm_params_host(cfg, 0).items()}
    batch = tuple(t.to(dev) for t in lm_batch_host(cfg, 0))
    opt = zg.ZeroGrad(lm_manifest(cfg), zg.sgd(1e-3), cfg["P"], cfg["rank"], cfg["sigma"], 0, "profile",
                      chunk_size=cfg["chunk"])
    loss = make_lm_loss(cfg)
    for gen in range(2):
        losses = opt.evaluate_shard(params, gen, loss, batch, range(cfg["P"]))
        torch.cuda.synchronize()
    print("profile case done, mean loss", float(losses.mean()))
    P = LM["P"]
    ropt = zg.ZeroGrad(lm_manifest(cfg), zg.sgd(1e-3), P, cfg["rank"], cfg["sigma"], 0, "profile-replay")
    g = torch.Generator(device=dev).manual_seed(1)
    rlosses = torch.randn(P, generator=g, device=dev)
    ropt.step_from_losses(ropt.init(params), params, rlosses)
    torch.cuda.synchronize()
    print("replay case done")


def run_ours(args):
    import torch

    from zerograd_b200 import _lib as L

    R = Ranks(args)
    L.load()
    if args.sections == "profile":
        profile_case(R.dev)
        return
    lm = lm_section(args, R)
    P = LM["P"]
    value = P * args.steps / (lm["ms"] / 1e3)
    e2e_value = P * lm["e2e_steps"] / (lm["e2e_ms"] / 1e3)
    secondary = {}
    if R.world == 1 and args.sections == "all":
        secondary["perturbed_gemm"] = perturbed_gemm_section(R.dev, args)
        secondary["mlp_f32"] = mlp_section(R.dev, args)
        secondary["vit_small"] = vit_section(R.dev, args)
        secondary["int8_qat_mlp"] = qat_section(R.dev, args)
        secondary["int8_qat_layer"] = int8_layer_section(R.dev, args)
    if R.rank == 0:
        kern = lm["kernels"]
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": R.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": lm["ms"] / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "generations_per_sec": args.steps / (lm["ms"] / 1e3),
            "timed": "CapturedGeneration.enqueue back to back (one CUDA graph per generation, population "
                     f"evaluated in chunks of {LM['chunk']}), inputs resident",
            "config": lm_config(R.world),
            "roofline": lm_roofline(kern, lm["P_local"]),
            "kernel_rates": family_rates(kern, lm["P_local"]),
            "kernels_ms_per_generation": {k: v[1] for k, v in sorted(kern.items())},
            "gpu_launches": lm["launches"],
            "clocks": lm["clocks"],
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": lm["h2d"],
                    "d2h_bytes_per_step": lm["d2h"], "ms_per_step": lm["e2e_ms"] / lm["e2e_steps"],
                    "steps": lm["e2e_steps"],
                    "api": "ZeroGrad.capture -> CapturedGeneration.enqueue, tokens and labels copied from pinned "
                           "host memory every generation (during the previous one), metrics read back one "
                           "generation behind"},
            "ranks_identical": len(set(lm["hashes"])) == 1,
            "params_hash": lm["hashes"][0],
            "last_mean_loss": lm["mean_loss"],
        }
        line.update(secondary)
        if R.world == 1 and args.sections == "all":
            line["cpu_baseline"] = lm_cpu_baseline(2)
        print(json.dumps(line), flush=True)
    if R.world > 1:
        R.dist.barrier(device_ids=[R.local])
        R.dist.destroy_process_group()
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------
# the ViT-small workload (the reference example's model at the configuration's size)
# ---------------------------------------------------------------------------
VIT = dict(embed=384, layers=6, heads=6, mlp=1536, classes=10, patch=4, img=32, batch=128, P=1024, rank=8,
           sigma=0.01, seed=0, run_id="vit", lr=1e-3, chunk=128)


def vit_tokens(cfg=VIT) -> int:
    return (cfg["img"] // cfg["patch"]) ** 2 + 1


def vit_manifest(cfg=VIT):
    """The reference example's manifest (``examples/train_vit_cifar10.py:109-133``): one group per entry."""
    import zerograd_b200 as zg

    M, T, V = zg.ParameterLayout.MATRIX, zg.ParameterLayout.TABLE, zg.ParameterLayout.VECTOR
    e = [(("patch_embed", "weight"), M, "patch_embed"), (("cls_token",), V, "cls_token"),
         (("pos_embed",), T, "pos_embed"), (("ln_f", "scale"), V, "ln_f_scale"), (("ln_f", "bias"), V, "ln_f_bias"),
         (("head", "weight"), M, "head_w"), (("head", "bias"), V, "head_b")]
    for i in range(cfg["layers"]):
        p = f"layer{i}"
        e += [((p, n, "weight"), M, f"{p}_{n}") for n in ("q", "k", "v", "o", "mlp1", "mlp2")]
        e += [((p, ln, w), V, f"{p}_{ln}_{w[0]}") for ln in ("ln1", "ln2") for w in ("scale", "bias")]
    return zg.Manifest(1, tuple(zg.ManifestEntry(path, lay, g) for path, lay, g in e))


def vit_params_host(cfg=VIT, seed=0) -> dict:
    """Seeded synthetic weights in the example's tree: N(0, 0.02) matrices,
    CLS token and positional table; unit LayerNorm scales, zero biases (bf16)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    E, F, C = cfg["embed"], cfg["mlp"], cfg["classes"]
    pd = cfg["patch"] ** 2 * 3

    def n(*shape):
        return (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16)

    def ln():
        return {"scale": torch.ones(E, dtype=torch.bfloat16), "bias": torch.zeros(E, dtype=torch.bfloat16)}

    p = {"patch_embed": {"weight": n(pd, E)}, "cls_token": n(E), "pos_embed": n(vit_tokens(cfg), E),
         "ln_f": ln(), "head": {"weight": n(E, C), "bias": torch.zeros(C, dtype=torch.bfloat16)}}
    for i in range(cfg["layers"]):
        p[f"layer{i}"] = {"q": {"weight": n(E, E)}, "k": {"weight": n(E, E)}, "v": {"weight": n(E, E)},
                          "o": {"weight": n(E, E)}, "mlp1": {"weight": n(E, F)}, "mlp2": {"weight": n(F, E)},
                          "ln1": ln(), "ln2": ln()}
    return p


def vit_batch_host(cfg=VIT, seed=0):
    """Images U[0, 1] [B, 32, 32, 3] cut into patches [B, 64, 48] (bf16, the
    example's extract_patches order) and labels uniform over the classes."""
    import torch

    g = torch.Generator().manual_seed(seed + 1)
    B, I, ps = cfg["batch"], cfg["img"], cfg["patch"]
    img = torch.rand(B, I, I, 3, generator=g)
    patches = img.reshape(B, I // ps, ps, I // ps, ps, 3).permute(0, 1, 3, 2, 4, 5).reshape(B, (I // ps) ** 2, -1)
    labels = torch.randint(0, cfg["classes"], (B,), generator=g)
    return patches.to(torch.bfloat16).contiguous(), labels


def make_vit_loss(cfg=VIT):
    """The reference example's candidate forward (``examples/train_vit_cifar10.py:137-191``)
    with its residual adds and GELU in the projections' epilogues, and the
    mean softmax cross-entropy over the CLS logits."""
    import torch.nn.functional as F_

    import zerograd_b200 as zg

    E, H, T, B = cfg["embed"], cfg["heads"], vit_tokens(cfg), cfg["batch"]
    D = E // H

    def loss_fn(p, ctx, batch, rng):
        patches, labels = batch
        x = ctx.linear(p, ("patch_embed", "weight"), patches)                       # [B, 64, E]
        cls = ctx.vector(p, ("cls_token",)).reshape(1, 1, E).expand(B, 1, E)
        x = torch_cat((cls, x), 1)
        x = x + ctx.table_lookup(p, ("pos_embed",), pos_ids(x.device))              # [T, E] broadcast
        for i in range(cfg["layers"]):
            n = f"layer{i}"
            h = zg.layer_norm(x, ctx.vector(p, (n, "ln1", "scale")), ctx.vector(p, (n, "ln1", "bias")))
            q, k, v = (ctx.linear(p, (n, w, "weight"), h).reshape(B, T, H, D) for w in ("q", "k", "v"))
            a = zg.attention(q, k, v).reshape(B, T, E)
            x = ctx.linear(p, (n, "o", "weight"), a, residual=x)
            h = zg.layer_norm(x, ctx.vector(p, (n, "ln2", "scale")), ctx.vector(p, (n, "ln2", "bias")))
            h = ctx.linear(p, (n, "mlp1", "weight"), h, activation="gelu")
            x = ctx.linear(p, (n, "mlp2", "weight"), h, residual=x)
        x = zg.layer_norm(x, ctx.vector(p, ("ln_f", "scale")), ctx.vector(p, ("ln_f", "bias")))
        logits = ctx.linear(p, ("head", "weight"), x[:, 0, :]) + ctx.vector(p, ("head", "bias"))
        return F_.cross_entropy(logits.float(), labels), None

    _ids = {}

    def pos_ids(dev):
        if dev not in _ids:
            import torch

            _ids[dev] = torch.arange(T, dtype=torch.int32, device=dev)
        return _ids[dev]

    def torch_cat(ts, dim):
        import torch

        return torch.cat(ts, dim)

    return loss_fn


def tree_to(tree, dev):
    """A nested dict of tensors moved to `dev`."""
    return {k: tree_to(v, dev) if isinstance(v, dict) else v.to(dev) for k, v in tree.items()}


def vit_flops(cfg=VIT) -> float:
    """Forward FLOPs of one candidate: projections (dense + rank-r) and attention."""
    E, F, L, r, T, B = cfg["embed"], cfg["mlp"], cfg["layers"], cfg["rank"], vit_tokens(cfg), cfg["batch"]
    tok = B * T
    per_layer = 2.0 * tok * (4 * E * E + 2 * E * F) + 2.0 * tok * r * (4 * E + F + E)
    attn = 4.0 * B * cfg["heads"] * T * T * (E // cfg["heads"])
    patch = 2.0 * B * (T - 1) * (cfg["patch"] ** 2 * 3) * E
    return L * (per_layer + attn) + patch


def vit_section(dev, args):
    """The ViT-small configuration's whole generation (P=1024, rank 8, batch
    128, 6 layers, width 384, 65 tokens) through ZeroGrad.capture, chunks of 128."""
    import torch

    import zerograd_b200 as zg
    from zerograd_b200 import _lib as L

    cfg = VIT
    params = tree_to(vit_params_host(cfg), dev)
    batch = tuple(t.to(dev) for t in vit_batch_host(cfg))
    opt = zg.ZeroGrad(vit_manifest(cfg), zg.sgd(cfg["lr"]), cfg["P"], cfg["rank"], cfg["sigma"], cfg["seed"],
                      cfg["run_id"], chunk_size=cfg["chunk"])
    loss = make_vit_loss(cfg)
    cg = opt.capture(params, loss, batch)
    st = opt.init(params)
    pend = []

    def step(i):
        nonlocal st
        _, st, pe = cg.enqueue(zg.ZeroGradState(i, st.opt_state))
        pend.append(pe)

    for i in range(3):
        step(i)
    steps = max(1, min(args.steps, 10))
    with ClockSampler(dev) as clk:
        ms = _timed_events(lambda i: step(10 + i), steps)
    m = [pe.result() for pe in pend][-1]
    del cg
    L.profile_begin(1 << 15)
    losses = opt.evaluate_shard(params, 100, loss, batch, range(cfg["P"]))
    opt.step_from_losses(zg.ZeroGradState(100, st.opt_state), params, losses)
    kern = L.profile_end()
    pk = peaks()
    gemm = kern.get("batched_gemm", (1, 0.0))[1]
    proj = vit_flops(cfg) - cfg["layers"] * 4.0 * cfg["batch"] * cfg["heads"] * vit_tokens(cfg) ** 2 * 64 - \
        2.0 * cfg["batch"] * (vit_tokens(cfg) - 1) * 48 * cfg["embed"]
    return {"workload": "ViT-small generation: 32x32x3 images U[0,1], patch 4 (64 tokens + CLS), d 384, 6 layers, 6 "
                        "heads, MLP 1536, 10 classes, bf16; P=1024, rank 8, batch 128, CE; chunks of 128, captured",
            "ms_per_generation": ms / steps, "generations_per_sec": steps / (ms / 1e3),
            "candidate_evals_per_sec": cfg["P"] * steps / (ms / 1e3), "steps": steps, "clocks": clk.summary(),
            "forward_tflops_per_generation": cfg["P"] * vit_flops(cfg) / 1e12, "last_mean_loss": m.mean_loss,
            "kernels_ms_per_generation": {k: v[1] for k, v in sorted(kern.items())},
            "batched_gemm_rate": {"TFLOP/s": cfg["P"] * proj / (gemm / 1e3) / 1e12 if gemm else None,
                                  "frac_sustained": (cfg["P"] * proj / (gemm / 1e3) / 1e12 /
                                                     pk["bf16_tflops_sustained"]) if gemm else None}}


# ---------------------------------------------------------------------------
# the integer QAT MLP workload
# ---------------------------------------------------------------------------
QAT = dict(dims=(1024, 4096, 4096, 1024), batch=512, P=512, rank=4, sigma=2.5e-5, seed=0, run_id="qat", lr=1e-2,
           chunk=128)
# Activations are int8 with scale 1/127 (inputs uniform in [-127, 127]; the
# tanh LUT's outputs 127 tanh(q / 32)); every layer quantises its output
# at 1/32.  The low-rank term acts on the integer activations, so sigma is
# the weights' relative perturbation times the activations' scale 1/127.
QAT_X_SCALE, QAT_Y_SCALE = 1.0 / 127.0, 1.0 / 32.0


def qat_luts():
    """The hidden layers' tanh LUT (lut[q + 128] = round(127 tanh(q / 32)))
    and the last layer's identity LUT, int8 [256] each."""
    import torch

    q = torch.arange(-128, 128, dtype=torch.float64)
    return torch.round(127 * torch.tanh(q / 32)).to(torch.int8), q.to(torch.int8)


def qat_manifest(cfg=QAT):
    import zerograd_b200 as zg

    n = len(cfg["dims"]) - 1
    return zg.Manifest(1, tuple(zg.ManifestEntry((f"w{i}",), zg.ParameterLayout.MATRIX, f"w{i}") for i in range(n)))


def qat_params_host(cfg=QAT, seed=0) -> dict:
    """float32 master weights N(0, 1/fan_in), quantised per output channel by the forward."""
    import torch

    g = torch.Generator().manual_seed(seed)
    d = cfg["dims"]
    return {f"w{i}": torch.randn(d[i], d[i + 1], generator=g) / d[i] ** 0.5 for i in range(len(d) - 1)}


def qat_batch_host(cfg=QAT, seed=0):
    """int8 inputs uniform in [-127, 127] [B, d0] and N(0, 1) targets [B, d_last]."""
    import torch

    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randint(-127, 128, (cfg["batch"], cfg["dims"][0]), generator=g, dtype=torch.int8)
    t = torch.randn(cfg["batch"], cfg["dims"][-1], generator=g)
    return x, t


def make_qat_loss(cfg=QAT, luts=None):
    """Quantise the master weights (once per launch: they are shared by the
    candidates), three integer LUT layers, the last with the identity LUT,
    dequantised output, mean-square error against the targets."""
    import zerograd_b200 as zg

    n = len(cfg["dims"]) - 1
    tanh_lut, ident_lut = luts

    def loss_fn(p, ctx, batch, rng):
        x, target = batch
        for i in range(n):
            wq, ws = zg.quantize_int8_columns(p[f"w{i}"])
            x = ctx.int8_lut_linear(p, (f"w{i}",), x, wq, ws, QAT_X_SCALE, QAT_Y_SCALE,
                                    ident_lut if i == n - 1 else tanh_lut)
        y = x.float() * QAT_Y_SCALE
        return ((y - target) ** 2).mean(), None

    return loss_fn


def qat_section(dev, args):
    """The integer QAT MLP's whole generation (1024 -> 4096 -> 4096 -> 1024,
    P=512, rank 4, batch 512, MSE) through ZeroGrad.capture, chunks of 128."""
    import zerograd_b200 as zg
    from zerograd_b200 import _lib as L

    cfg = QAT
    params = tree_to(qat_params_host(cfg), dev)
    batch = tuple(t.to(dev) for t in qat_batch_host(cfg))
    luts = tuple(t.to(dev) for t in qat_luts())
    opt = zg.ZeroGrad(qat_manifest(cfg), zg.sgd(cfg["lr"]), cfg["P"], cfg["rank"], cfg["sigma"], cfg["seed"],
                      cfg["run_id"], chunk_size=cfg["chunk"])
    loss = make_qat_loss(cfg, luts)
    cg = opt.capture(params, loss, batch)
    st = opt.init(params)
    pend = []

    def step(i):
        nonlocal st
        _, st, pe = cg.enqueue(zg.ZeroGradState(i, st.opt_state))
        pend.append(pe)

    for i in range(2):
        step(i)
    steps = max(1, min(args.steps, 3))
    with ClockSampler(dev) as clk:
        ms = _timed_events(lambda i: step(10 + i), steps)
    m = [pe.result() for pe in pend][-1]
    del cg
    L.profile_begin(1 << 14)
    losses = opt.evaluate_shard(params, 100, loss, batch, range(cfg["P"]))
    opt.step_from_losses(zg.ZeroGradState(100, st.opt_state), params, losses)
    kern = L.profile_end()
    d, B, P = cfg["dims"], cfg["batch"], cfg["P"]
    ops = 2.0 * B * d[0] * d[1] + P * 2.0 * B * sum(d[i] * d[i + 1] for i in range(1, len(d) - 1))
    gm = kern.get("int8_lut_gemm", (1, 0.0))[1]
    ip = int8_library_peak(dev)
    return {"workload": "integer QAT MLP generation 1024->4096->4096->1024: int8 weights quantised per output "
                        "channel from float32 masters, int8 activations through a 256-entry tanh LUT, identity LUT "
                        "on the last layer, MSE vs N(0,1) targets; P=512, rank 4, batch 512; chunks of 128, captured",
            "ms_per_generation": ms / steps, "generations_per_sec": steps / (ms / 1e3),
            "candidate_evals_per_sec": P * steps / (ms / 1e3), "steps": steps, "clocks": clk.summary(),
            "int8_tera_ops_per_generation": ops / 1e12, "last_mean_loss": m.mean_loss,
            "kernels_ms_per_generation": {k: v[1] for k, v in sorted(kern.items())},
            "int8_gemm_rate": {"TOP/s": ops / (gm / 1e3) / 1e12 if gm else None,
                               "frac_of_int8_peak": ops / (gm / 1e3) / 1e12 / ip["value"] if gm else None,
                               "int8_peak": ip}}


# ---------------------------------------------------------------------------
# secondary sections (one GPU)
# ---------------------------------------------------------------------------
PG = dict(P=256, rank=8, M=256, K=4096, N=4096, sigma=0.01, seed=0, run_id="bench", lr=1e-3)


def _timed_events(fn, steps, flush=None):
    import torch

    ev = []
    for i in range(steps):
        if flush is not None:
            flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn(i)
        e.record()
        ev.append((s, e))
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in ev)


def perturbed_gemm_section(dev, args):
    """The perturbed-GEMM microbench (population 256, rank 8, x[256,4096] and
    W[4096,4096] N(0,0.02) bf16, sigma 0.01): (i) one shared input, every
    candidate's [256,4096] output materialised, loss one output element,
    the generation captured (ZeroGrad.capture); (ii) a per-candidate input
    x_p (the hidden-layer form) through the population tensor-core GEMM;
    both with the replay of W and the SGD step fused into the replay GEMM."""
    import torch

    import zerograd_b200 as zg
    from zerograd_b200 import _lib as L
    from zerograd_b200 import _ops

    P, r, M, K, N, sigma = PG["P"], PG["rank"], PG["M"], PG["K"], PG["N"], PG["sigma"]
    pk = peaks()
    g = torch.Generator().manual_seed(PG["seed"])
    x = (torch.randn(M, K, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    W0 = (torch.randn(K, N, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),))
    opt = zg.ZeroGrad(manifest, zg.sgd(PG["lr"]), P, r, sigma, PG["seed"], PG["run_id"])

    def fwd_loss(p, ctx, batch, rng):
        return ctx.linear(p, ("w",), batch)[0, 0].float(), None

    cg = opt.capture({"w": W0}, fwd_loss, x)
    st = opt.init({"w": W0})
    pend = []

    def step(i):
        nonlocal st
        _, st, pe = cg.enqueue(zg.ZeroGradState(1000 + i, st.opt_state))
        pend.append(pe)

    for i in range(5):
        step(i)
    steps = max(1, min(args.steps, 20))
    with ClockSampler(dev) as clk:
        ms = _timed_events(lambda i: step(10 + i), steps, flush)
    for pe in pend:
        pe.result()
    del cg
    # per-kernel times of the same generation, eager
    L.profile_begin(1 << 14)
    for i in range(3):
        losses = opt.evaluate_shard({"w": W0}, 2000 + i, fwd_loss, x, range(P))
        opt.step_from_losses(zg.ZeroGradState(2000 + i, st.opt_state), {"w": W0}, losses)
    kern = L.profile_end()
    exp_ms = kern["lowrank_expand"][1] / kern["lowrank_expand"][0]
    exp_bytes = P * M * N * 2 + M * N * 4 + P * M * r * 2 + P * r * N * 2
    rep_ms = kern["replay_gemm"][1] / kern["replay_gemm"][0]
    rep_flops = 2.0 * K * N * P * r
    shared = {"workload": "shared x[256,4096], every candidate's output written, captured generation",
              "value": P * steps / (ms / 1e3), "unit": UNIT, "ms_per_generation": ms / steps, "steps": steps,
              "clocks": clk.summary(),
              "kernels_ms_per_generation": {k: v[1] / 3 for k, v in sorted(kern.items())},
              "roofline": {"kernel": "lowrank_expand", "bound": "hbm", "achieved": exp_bytes / (exp_ms / 1e3) / 1e9,
                           "peak": pk["hbm_gbs"], "unit": "GB/s",
                           "frac": exp_bytes / (exp_ms / 1e3) / 1e9 / pk["hbm_gbs"], "launch_ms": exp_ms,
                           "traffic": traffic_for("lowrank_expand")},
              "replay_roofline": {"kernel": "replay_gemm", "bound": "tensor",
                                  "achieved": rep_flops / (rep_ms / 1e3) / 1e12, "peak": pk["bf16_tflops"],
                                  "unit": "TFLOP/s", "frac": rep_flops / (rep_ms / 1e3) / 1e12 / pk["bf16_tflops"],
                                  "launch_ms": rep_ms, "peak_source": pk["source"] + " (burst)",
                                  "traffic": traffic_for("replay_gemm")}}

    # (ii) per-candidate inputs
    gx = torch.Generator(device=dev).manual_seed(PG["seed"] + 1)
    xb = (torch.randn(P, M, K, generator=gx, device=dev) * 0.02).to(torch.bfloat16)
    ids = torch.arange(P, dtype=torch.int32, device=dev)
    fitness = torch.randn(P, generator=gx, device=dev)

    def hidden_step(gen):
        base = tuple(int(v) for v in opt.base_key(gen))
        cks = _ops.launch_fold_in(opt.base_key(gen), ids)
        with _ops.generation_scope(base, 0, P, cks):
            y = _ops.launch_linear(xb, W0, cks, 0, r, sigma, True)
        shaped, _ = _ops.launch_shape_fitness(fitness, sigma)
        _ops.launch_replay_step(shaped, cks, 0, L.ZG_MATRIX, W0.clone(), r, {"kind": "sgd", "lr": PG["lr"]},
                                gen=_ops._Generation(base, 0, P, cks))
        _ops.CACHE.drop_generation(base)
        del y

    for i in range(3):
        hidden_step(3000 + i)
    h_steps = max(1, min(args.steps, 30))
    with ClockSampler(dev) as hclk:
        h_ms = _timed_events(lambda i: hidden_step(3100 + i), h_steps)
    L.profile_begin(1 << 14)
    for i in range(5):
        hidden_step(3200 + i)
    hk = L.profile_end()
    bg = hk["batched_gemm"][1] / hk["batched_gemm"][0]
    bg_flops = 2.0 * P * M * K * N + 2.0 * P * M * r * N
    del xb
    hidden = {"workload": "per-candidate x_p[256,4096] (hidden-layer form), population tensor-core GEMM, replay + "
                          "SGD", "value": P * h_steps / (h_ms / 1e3), "unit": UNIT,
              "ms_per_generation": h_ms / h_steps, "clocks": hclk.summary(),
              "kernels_ms_per_generation": {k: v[1] / 5 for k, v in sorted(hk.items())},
              "roofline": {"kernel": "batched_gemm", "bound": "tensor", "achieved": bg_flops / (bg / 1e3) / 1e12,
                           "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                           "frac": bg_flops / (bg / 1e3) / 1e12 / pk["bf16_tflops_sustained"],
                           "frac_of_burst_peak": bg_flops / (bg / 1e3) / 1e12 / pk["bf16_tflops"],
                           "launch_ms": bg, "traffic": traffic_for("batched_gemm")}}
    return {"shared_input": shared, "per_candidate_input": hidden}


def _mlp_parts():
    import torch
    import torch.nn.functional as F

    import zerograd_b200 as zg

    manifest = zg.Manifest(1, (zg.ManifestEntry(("w1",), zg.ParameterLayout.MATRIX, "w1"),
                               zg.ManifestEntry(("b1",), zg.ParameterLayout.VECTOR, "b1"),
                               zg.ManifestEntry(("w2",), zg.ParameterLayout.MATRIX, "w2"),
                               zg.ManifestEntry(("b2",), zg.ParameterLayout.VECTOR, "b2")))
    g = torch.Generator().manual_seed(0)
    params = {"w1": torch.randn(784, 256, generator=g) * (2.0 / 784) ** 0.5, "b1": torch.zeros(256),
              "w2": torch.randn(256, 10, generator=g) * (2.0 / 256) ** 0.5, "b2": torch.zeros(10)}
    g = torch.Generator().manual_seed(1)
    batch = (torch.randn(128, 784, generator=g), torch.randint(0, 10, (128,), generator=g))

    def loss(p, ctx, b, rng):
        x, y = b
        h = torch.relu(ctx.linear(p, ("w1",), x) + ctx.vector(p, ("b1",)))
        logits = ctx.linear(p, ("w2",), h) + ctx.vector(p, ("b2",))
        return F.cross_entropy(logits, y), None

    return manifest, params, batch, loss


def mlp_cpu_generation(params, batch, gen: int) -> float:
    """The f32 MLP configuration's whole generation on the host cores (the
    oracle: 64 candidates' losses, the replay of all four entries, adamw)."""
    import numpy as np

    from oracle import ref

    x, y = (t.numpy() for t in batch)
    p = {k: v.numpy() for k, v in params.items()}
    t0 = time.perf_counter()
    base = ref.step_key(0, "mlp", gen, 1)
    losses = []
    for c in range(64):
        ck = ref.candidate_key(base, c)
        gk = [ref.fold_in(ck, i) for i in range(4)]
        h = np.maximum(ref.perturbed_linear(x, p["w1"], gk[0], 8, 0.01) + ref.perturbed_vector(p["b1"], gk[1], 0.01),
                       0)
        lg = ref.perturbed_linear(h, p["w2"], gk[2], 8, 0.01) + ref.perturbed_vector(p["b2"], gk[3], 0.01)
        lg = lg - lg.max(1, keepdims=True)
        losses.append(float(np.mean(np.log(np.exp(lg).sum(1)) - lg[np.arange(len(y)), y])))
    shaped = ref.shape_centered_loss(np.array(losses, np.float32), 0.01)
    grads = {}
    for i, (name, lay) in enumerate([("w1", 0), ("b1", 2), ("w2", 0), ("b2", 2)]):
        grads[name] = -ref.replay_entry(p[name].shape, lay, base, range(64), shaped, 8 if lay == 0 else 1, i)
    ref.adamw_update(grads, ref.adamw_init(p), p, 3e-4)
    return time.perf_counter() - t0


def mlp_section(dev, args):
    """The f32 MLP configuration (784 -> 256 -> 10, ReLU, P=64, rank 8, sigma
    0.01, adamw 3e-4, batch 128, cross-entropy) as whole generations: on the
    GPU captured, and on the host cores through the oracle, timed in full."""
    import zerograd_b200 as zg

    manifest, params, batch, loss = _mlp_parts()
    opt = zg.ZeroGrad(manifest, zg.adamw(3e-4), 64, 8, 0.01, 0, "mlp")
    dparams = {k: v.to(dev) for k, v in params.items()}
    dbatch = tuple(t.to(dev) for t in batch)
    cg = opt.capture(dparams, loss, dbatch)
    st = opt.init(dparams)
    pend = []

    def step(i):
        nonlocal st
        _, st, pe = cg.enqueue(zg.ZeroGradState(i, st.opt_state))
        pend.append(pe)

    for i in range(5):
        step(i)
    steps = max(5, min(args.steps * 5, 100))
    ms = _timed_events(lambda i: step(10 + i), steps)
    for pe in pend:
        pe.result()
    del cg
    mlp_cpu_generation(params, batch, 0)
    cpu_s = statistics.median(mlp_cpu_generation(params, batch, 1 + i) for i in range(3))
    return {"workload": "MLP 784->256->10 f32 (ReLU), P=64, rank 8, sigma 0.01, adamw 3e-4, batch 128, CE; whole "
                        "generation", "gpu_generations_per_sec": steps / (ms / 1e3), "gpu_ms_per_generation": ms / steps,
            "gpu_evals_per_sec": 64 * steps / (ms / 1e3), "steps": steps,
            "cpu_generations_per_sec": 1.0 / cpu_s, "cpu_ms_per_generation": 1e3 * cpu_s,
            "cpu_evals_per_sec": 64 / cpu_s, "cpu_cores": cpu_threads(),
            "cpu_kind": "port (oracle restatement, float64 numpy + C threefry), timed in full"}


_INT8_PEAK: dict = {}


def int8_library_peak(dev) -> dict:
    """Dense int8 tensor-core throughput of a library GEMM on this GPU, the
    int8 roofline's denominator: torch._int_mm (cuBLASLt, int8 x int8 ->
    int32) on 8192 x 8192 x 8192, event-timed after warm-up."""
    import torch

    if "value" in _INT8_PEAK:
        return _INT8_PEAK
    n = 8192
    g = torch.Generator(device=dev).manual_seed(5)
    a = torch.randint(-127, 128, (n, n), generator=g, device=dev, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, n), generator=g, device=dev, dtype=torch.int8).t()  # column-major operand
    try:
        for _ in range(3):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        reps = 20
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            torch._int_mm(a, b)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / reps
        _INT8_PEAK.update(value=2.0 * n ** 3 / (ms / 1e3) / 1e12, unit="TOP/s", ms=ms,
                          source="measured live: torch._int_mm (cuBLASLt) 8192^3 int8")
    except RuntimeError as exc:  # no int8 library GEMM on this build: fall back to 2x the bf16 figure
        _INT8_PEAK.update(value=2.0 * peaks()["bf16_tflops"], unit="TOP/s", ms=None,
                          source=f"2x measured bf16 dense (torch._int_mm unavailable: {str(exc)[:80]})")
    del a, b
    return _INT8_PEAK


def int8_layer_section(dev, args):
    """The integer QAT MLP's 4096 -> 4096 layer (batch 512 int8 inputs per
    candidate, P=512, rank 4): int8 x int8 -> int32 on the tensor cores, the
    float32 low-rank term, rint and the 256-entry tanh LUT in the epilogue.
    Seeded synthetic int8 inputs/weights (U[-127,127]), per-channel scales
    U[0.5,1.5]/127.  Inputs (1 GiB) exceed L2."""
    import torch

    import zerograd_b200 as zg
    from zerograd_b200 import _lib as L
    from zerograd_b200 import _ops

    P8, M8, K8, N8, r8 = 512, 512, 4096, 4096, 4
    g = torch.Generator(device=dev).manual_seed(3)
    x8 = torch.randint(-127, 128, (P8, M8, K8), generator=g, device=dev, dtype=torch.int8)
    W8 = torch.randint(-127, 128, (K8, N8), generator=g, device=dev, dtype=torch.int8)
    ws8 = (torch.rand(N8, generator=g, device=dev) + 0.5) / 127
    q = torch.arange(-128, 128, dtype=torch.float64, device=dev)
    lut = torch.round(127 * torch.tanh(q / 32)).to(torch.int8)
    keys8 = _ops.launch_fold_in(zg.step_key(0, "qat", 0, 1), torch.arange(P8, dtype=torch.int32, device=dev))

    def run(_=None):
        return _ops.launch_int8_lut_linear(x8, W8, ws8, 1 / 127, 1 / 32, lut, keys8, 1, r8, 0.01, True)

    for _ in range(3):
        run()
    steps = max(1, min(args.steps, 20))
    with ClockSampler(dev) as clk:
        ms = _timed_events(run, steps)
    L.profile_begin()
    for _ in range(steps):
        run()
    kern = L.profile_end()
    ops = 2.0 * P8 * M8 * K8 * N8
    gm = kern["int8_lut_gemm"][1] / kern["int8_lut_gemm"][0]
    ip = int8_library_peak(dev)
    peak = ip["value"]
    return {"workload": "int8 QAT layer 4096->4096, P=512, batch 512 per candidate, rank 4, tanh LUT",
            "ms_per_layer": ms / steps, "candidate_layers_per_sec": P8 / (ms / steps / 1e3), "clocks": clk.summary(),
            "kernels_ms": {k: v[1] / v[0] for k, v in sorted(kern.items())},
            "roofline": {"kernel": "int8_lut_gemm", "bound": "tensor", "achieved": ops / (gm / 1e3) / 1e12,
                         "peak": peak, "unit": "TOP/s", "frac": ops / (gm / 1e3) / 1e12 / peak,
                         "peak_source": ip["source"], "launch_ms": gm}}


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

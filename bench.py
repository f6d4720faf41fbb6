#!/usr/bin/env python
"""Throughput of one ES generation of the batched perturbed GEMM + factor replay.

Workload (the reference's perturbed-GEMM microbench config): population 256,
rank 8, a shared bf16 input x[256,4096] (N(0, 0.02)) through W[4096,4096]
(N(0, 0.02)) plus sigma*(x A_i) B_i^T per candidate (sigma 0.01, factors from
the threefry keys of seed 0, generation 0 onwards), every candidate's output
[256,4096] materialised in HBM and its loss one element of that output; then
the fitness shaping (the reference's centred-loss rule), factor replay of W's
pseudo-gradient with the SGD update applied in the replay GEMM's epilogue.
One step = one generation, run as the public API runs it (ZeroGrad.capture:
the generation as one CUDA graph, the per-generation key copied in before
each replay).  Synthetic data, fixed seeds.

`python bench.py [--gpus N --steps K --warmup W]` prints one JSON line.  With
N > 1 (one process per GPU under torch.distributed.run) the population is
sharded across ranks, the fitness array is all-gathered (the only
collective) and every rank replays the identical update.
`--impl reference` times the CPU restatement of the reference's algorithm
(the reference itself is JAX code that cannot be installed here) on this
host's cores.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WL = dict(P=256, rank=8, M=256, K=4096, N=4096, sigma=0.01, seed=0, run_id="bench", lr=1e-3)
METRIC = "candidate forward evals/sec"
UNIT = "evals/s"
WORKLOAD_NAME = ("batched perturbed GEMM + factor replay: P=256, rank=8, shared x[256,4096] bf16, "
                 "W[4096,4096] bf16, sigma=0.01, seed 0; loss = one output element per candidate, centred-loss "
                 "shaped; SGD update")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    # with more than one GPU: every rank replays the whole update (the
    # reference's protocol) or its block of W's rows, then W is all-gathered
    ap.add_argument("--replay", choices=["replicated", "sharded"], default="replicated")
    # "headline": the shared-input generation alone (value, e2e, the eager
    # launch sequence and its per-kernel times), for profiler runs; the
    # default also runs the secondary workloads and the CPU baseline
    ap.add_argument("--sections", choices=["all", "headline"], default="all")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


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


# ---------------------------------------------------------------------------
# algorithmic work per launch of each kernel (this workload)
# ---------------------------------------------------------------------------
def kernel_work(name: str, P_local: int, world: int = 1, row_blocks: int = 1):
    P, r, M, K, N = WL["P"], WL["rank"], WL["M"], WL["K"], WL["N"]
    if name == "factor_fill":
        # bf16 operand bytes written per launch: the forward draws A_op and B_op
        # for this rank's candidates; with more than one rank the replay draws
        # both for the whole population (only the local ones are cached)
        fills = [P_local * r * K * 2, P_local * r * N * 2]
        if world > 1:
            fills += [P * r * K * 2, P * r * N * 2]
        return "hbm", sum(fills) / len(fills)
    if name == "lowrank_expand":      # y = xW + s (xA) B : write y bf16, read xW f32, U f32, B bf16
        return "hbm", P_local * M * N * 2 + M * N * 4 + P_local * M * r * 4 + P_local * r * N * 2
    if name == "replay_gemm":         # [K, P r] x [P r, N] (this rank's block of the K rows)
        return "tensor", 2.0 * (K // row_blocks) * N * P * r
    if name in ("forward_xw_gemm", "shared_xw"):
        return "tensor", 2.0 * M * K * N
    if name in ("forward_u_gemm", "lowrank_u"):
        return "tensor", 2.0 * P_local * M * K * r
    if name == "forward_factor_fill":  # bf16 operand written per launch (K = N here)
        return "hbm", P_local * r * K * 2
    if name == "replay_factor_fill":
        return "hbm", P * r * K * 2
    if name == "sgd_update":          # read W bf16 + descent f32, write W bf16
        return "hbm", K * N * (2 + 4 + 2)
    if name == "batched_gemm":        # per-candidate x_p W + the low-rank correction U_p B_p^T
        return "tensor", 2.0 * P_local * M * K * N + 2.0 * P_local * M * r * N
    if name == "batched_u_pass":      # reads every x_p once (bf16), writes U (bf16, 16 columns)
        return "hbm", P_local * M * K * 2 + P_local * M * 16 * 2
    return None, None


def traffic_for(name: str):
    """DRAM bytes per launch of a kernel from the committed ncu summary, or None."""
    tpath = os.path.join(ROOT, "profiles", "traffic.txt")
    if os.path.exists(tpath):
        for tl in open(tpath):
            parts = tl.split()
            if len(parts) == 2 and not tl.startswith("#") and parts[0] == name:
                return int(parts[1])
    return None


def int8_layer_section(dev, args):
    """The integer QAT MLP's 4096 -> 4096 layer (batch 512 int8 inputs per
    candidate, P=512, rank 4): int8 x int8 -> int32 on the tensor cores, the
    float32 low-rank term, rint and the 256-entry tanh LUT in the epilogue.
    Seeded synthetic int8 inputs/weights (U[-127,127]), per-channel scales
    U[0.5,1.5]/127.  Inputs (1 GiB) exceed L2, so no flush is needed."""
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

    def run():
        return _ops.launch_int8_lut_linear(x8, W8, ws8, 1 / 127, 1 / 32, lut, keys8, 1, r8, 0.01, True)

    for _ in range(max(3, min(args.warmup, 5))):
        run()
    torch.cuda.synchronize()
    steps = max(1, min(args.steps, 20))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        e0.record()
        for _ in range(steps):
            run()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    L.profile_begin()
    for _ in range(steps):
        run()
    kern = L.profile_end()
    pk = peaks()
    ops = 2.0 * P8 * M8 * K8 * N8
    gm = kern["int8_lut_gemm"][1] / kern["int8_lut_gemm"][0]
    peak = 2.0 * pk["bf16_tflops"]  # dense int8 issues at twice the bf16 rate
    return {"workload": "int8 QAT layer 4096->4096, P=512, batch 512 per candidate, rank 4, tanh LUT",
            "ms_per_layer": ms, "candidate_layers_per_sec": P8 / (ms / 1e3), "clocks": clk.summary(),
            "kernels_ms": {k: v[1] / v[0] for k, v in sorted(kern.items())},
            "roofline": {"kernel": "int8_lut_gemm", "bound": "tensor", "achieved": ops / (gm / 1e3) / 1e12,
                         "peak": peak, "unit": "TOP/s", "frac": ops / (gm / 1e3) / 1e12 / peak,
                         "peak_source": "2x measured bf16 dense (no measured int8 figure)",
                         "traffic": (traffic_for("int8_lut_gemm_p64") * P8 // 64
                                     if traffic_for("int8_lut_gemm_p64") else None),
                         "launch_ms": gm}}


def tied_ce_section(dev, args):
    """The decoder LM's tied output layer with its cross-entropy (vocabulary
    32000, width 768, 16 sequences x 256 tokens per candidate, rank 16): 16
    candidates of the population, each with its own hidden states (seeded
    N(0,1) bf16, table N(0, 0.02)), logits never materialised."""
    import torch

    import zerograd_b200 as zg
    from zerograd_b200 import _lib as L
    from zerograd_b200 import _ops

    P, M, V, C, r = 16, 16 * 256, 32000, 768, 16
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn(P, M, C, generator=g, device=dev).to(torch.bfloat16)
    T = (torch.randn(V, C, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    labels = torch.randint(0, V, (M,), generator=g, device=dev)
    keys = _ops.launch_fold_in(zg.step_key(0, "lm", 0, 1), torch.arange(P, dtype=torch.int32, device=dev))

    def run():
        return _ops.launch_tied_logits_ce(x, T, labels, keys, 0, r, 0.01, True)

    for _ in range(3):
        run()
    torch.cuda.synchronize()
    steps = max(1, min(args.steps, 10))
    with ClockSampler(dev) as clk:
        L.profile_begin()
        for _ in range(steps):
            run()
        kern = L.profile_end()
    pk = peaks()
    ce = kern["tied_ce"][1] / kern["tied_ce"][0]
    flops = 2.0 * P * M * V * C + 2.0 * P * M * r * V  # x . T^T and the low-rank term
    return {"workload": "tied logits + softmax cross-entropy, V=32000, C=768, 4096 tokens per candidate, "
                        "rank 16, 16 candidates, per-candidate hidden states",
            "kernels_ms": {k: v[1] / v[0] for k, v in sorted(kern.items())}, "clocks": clk.summary(),
            "candidates_per_sec": P / (sum(v[1] / v[0] for v in kern.values()) / 1e3),
            "roofline": {"kernel": "tied_ce", "bound": "tensor", "achieved": flops / (ce / 1e3) / 1e12,
                         "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": flops / (ce / 1e3) / 1e12 / pk["bf16_tflops"], "peak_source": pk["source"],
                         "traffic": traffic_for("tied_ce"), "launch_ms": ce}}


def lm_block_section(dev, args):
    """One decoder-LM block for 16 candidates through the public API
    (evaluate_shard under vmap): embedding lookup of the tied TABLE (vocab
    32000, width 768) with each candidate's perturbation, RMSNorm with the
    perturbed VECTOR scale, perturbed q/k/v/o projections, causal softmax
    attention (12 heads of 64), RMSNorm, perturbed MLP 768 -> 3072 -> 768
    (GELU), residuals; 16 sequences x 256 tokens per candidate, rank 16.
    Seeded synthetic tokens (uniform over the vocabulary) and weights
    (N(0, 0.02)); loss = mean square of the block's output."""
    import torch

    import zerograd_b200 as zg
    from zerograd_b200 import _lib as L

    P, B, T, E, Hh, F, V, r = 16, 16, 256, 768, 12, 3072, 32000, 16
    mats = {"q": (E, E), "k": (E, E), "v": (E, E), "o": (E, E), "mlp1": (E, F), "mlp2": (F, E)}
    entries = [zg.ManifestEntry(("emb",), zg.ParameterLayout.TABLE, "emb"),
               zg.ManifestEntry(("n1",), zg.ParameterLayout.VECTOR, "n1"),
               zg.ManifestEntry(("n2",), zg.ParameterLayout.VECTOR, "n2")]
    entries += [zg.ManifestEntry((n,), zg.ParameterLayout.MATRIX, n) for n in mats]
    manifest = zg.Manifest(1, tuple(entries))
    g = torch.Generator(device=dev).manual_seed(7)
    params = {n: (torch.randn(*d, generator=g, device=dev) * 0.02).to(torch.bfloat16) for n, d in mats.items()}
    params["emb"] = (torch.randn(V, E, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    params["n1"] = torch.ones(E, dtype=torch.bfloat16, device=dev)
    params["n2"] = torch.ones(E, dtype=torch.bfloat16, device=dev)
    tokens = torch.randint(0, V, (B, T), generator=g, device=dev)

    def loss_fn(p, ctx, batch, rng):
        x = ctx.table_lookup(p, ("emb",), batch)
        h = zg.rms_norm(x, ctx.vector(p, ("n1",)))
        q, k, v = (ctx.linear(p, (n,), h).reshape(B, T, Hh, E // Hh) for n in ("q", "k", "v"))
        x = x + ctx.linear(p, ("o",), zg.attention(q, k, v, causal=True).reshape(B, T, E))
        h = zg.rms_norm(x, ctx.vector(p, ("n2",)))
        m = torch.nn.functional.gelu(ctx.linear(p, ("mlp1",), h))
        x = x + ctx.linear(p, ("mlp2",), m)
        return (x.float() ** 2).mean(), None

    opt = zg.ZeroGrad(manifest, zg.sgd(1e-3), P, r, 0.01, 0, "lm-block")
    # one generation (forward of every candidate, shaping, replay and SGD of
    # all nine entries) as the public API's captured graph, queued back to back
    cg = opt.capture(params, loss_fn, tokens)
    state = opt.init(params)
    pending = []

    def run(gen):
        nonlocal state
        _, state, pend = cg.enqueue(zg.ZeroGradState(gen, state.opt_state))
        pending.append(pend)

    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    steps = max(1, min(args.steps, 10))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        e0.record()
        for i in range(steps):
            run(10 + i)
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    for pend in pending:
        pend.result()
    del cg
    # per-kernel device times: the same generation launched eagerly under the profiler
    eager_state = opt.init(params)
    L.profile_begin()
    for i in range(steps):
        _, eager_state, _ = opt.step(zg.ZeroGradState(40 + i, eager_state.opt_state), params, tokens, loss_fn)
    kern = L.profile_end()
    pk = peaks()
    per = {k: v[1] / steps for k, v in sorted(kern.items())}
    tokens_all = P * B * T
    # dense x W of q, k, v, o, mlp1, mlp2 plus their rank-r terms 2 tokens r (K + N)
    lin_flops = 2.0 * tokens_all * (4 * E * E + 2 * E * F) + 2.0 * tokens_all * r * (10 * E + 2 * F)
    attn_flops = 4.0 * P * B * Hh * T * T * (E // Hh)  # q k^T and p v, all T x T scores (causal half masked)
    out = {"workload": "decoder-LM block (vocab 32000 tied table lookup, d 768, 12 heads, MLP 3072, RMSNorm, "
                       "causal attention), 16 candidates x 16 sequences x 256 tokens, rank 16, bf16; one "
                       "generation = forward + shaping + replay and SGD of all entries, captured",
           "ms_per_generation": ms, "candidate_evals_per_sec": P / (ms / 1e3), "clocks": clk.summary(),
           "kernels_ms_per_generation": per}
    at = kern.get("attention")
    if at:
        a_ms = at[1] / at[0]
        out["attention_roofline"] = {"kernel": "attention", "bound": "tensor",
                                     "achieved": attn_flops / (a_ms / 1e3) / 1e12, "peak": pk["bf16_tflops"],
                                     "unit": "TFLOP/s", "frac": attn_flops / (a_ms / 1e3) / 1e12 / pk["bf16_tflops"],
                                     "launch_ms": a_ms, "peak_source": pk["source"]}
    gemm_ms = sum(v for k, v in per.items() if k in ("batched_gemm", "batched_u_pass"))
    if gemm_ms:
        out["projection_tflops"] = lin_flops / (gemm_ms / 1e3) / 1e12
    return out


# ---------------------------------------------------------------------------
# CPU arm: the oracle restatement of the reference on a bounded sample
# ---------------------------------------------------------------------------
def cpu_generation_sample(n_cand: int, seed: int = 0):
    """Forward of n_cand candidates + their replay contribution, on the host.

    Follows the reference's computation per generation: the shared x @ W once
    (jax.vmap leaves it unbatched), then per candidate (x A) B added, then the
    replay contraction over the sampled candidates.  Returns seconds.
    """
    import numpy as np

    from oracle import ref

    P, r, M, K, N = WL["P"], WL["rank"], WL["M"], WL["K"], WL["N"]
    rng = np.random.default_rng(seed)
    x = ref.round_bf16((rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    W = ref.round_bf16((rng.standard_normal((K, N)) * 0.02).astype(np.float32))
    losses = rng.standard_normal(P).astype(np.float32)  # candidates outside the sample
    base = ref.step_key(WL["seed"], WL["run_id"], 0, 1)
    t0 = time.perf_counter()
    cks = ref.candidate_keys(base, range(n_cand))
    gks = ref.group_keys(cks, 0)
    A, B = ref.population_factors(gks, ref.MATRIX, (K, N), r, "bfloat16")
    xw = x @ W
    s = ref.scaled_factor(r, WL["sigma"], "bfloat16")
    for p in range(n_cand):
        y = xw + s * ((x @ A[p]) @ B[p])
        y = ref.round_bf16(y)
        losses[p] = y[0, 0]
    shaped = ref.shape_centered_loss(losses, WL["sigma"])[:n_cand]
    wa = (A * shaped[:, None, None].astype(np.float32)).transpose(1, 0, 2).reshape(K, n_cand * r)
    g = (wa @ B.reshape(n_cand * r, N)) * ref.scaled_factor(r, 1.0, "bfloat16")
    del y, g
    return time.perf_counter() - t0


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count()


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import ref

    ref.lib()
    n_cand = 8
    for _ in range(max(1, min(args.warmup, 2))):
        cpu_generation_sample(n_cand)
    times = [cpu_generation_sample(n_cand, seed=i) for i in range(args.steps)]
    total = sum(times)
    value = n_cand * args.steps / total
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD_NAME, "population": WL["P"], "rank": WL["rank"], "batch": WL["M"],
                   "d_in": WL["K"], "d_out": WL["N"], "sample": f"{n_cand} candidates per step"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
                         "sample": f"{n_cand} of {WL['P']} candidates per step: shared x@W, per-candidate "
                                   "low-rank forward, replay contraction; numpy/BLAS + C threefry"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    import zerograd_b200 as zg
    from zerograd_b200 import _lib as L
    from zerograd_b200 import _ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    L.load()

    P, r, M, K, N, sigma = WL["P"], WL["rank"], WL["M"], WL["K"], WL["N"], WL["sigma"]
    sizes = zg.compute_partition_sizes(P, [1.0] * world)
    a = sum(sizes[:rank])
    b = a + sizes[rank]
    P_local = b - a

    g = torch.Generator().manual_seed(WL["seed"])
    x_host = (torch.randn(M, K, generator=g) * 0.02).to(torch.bfloat16).pin_memory()
    W0 = (torch.randn(K, N, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    fit_host = torch.randn(P, generator=g).pin_memory()
    x = x_host.to(dev)
    fitness = fit_host.to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),))
    ids_all = torch.arange(P, dtype=torch.int32, device=dev)
    total_steps = args.warmup + args.steps

    # per-generation candidate keys, derived up front (inputs resident)
    keys, bases = [], []
    for gen in range(total_steps):
        base = zg.step_key(WL["seed"], WL["run_id"], gen, manifest.version)
        bases.append(tuple(int(v) for v in base))
        cks = _ops.launch_fold_in(base, ids_all)
        keys.append((cks, cks[a:b]))

    def gather(local_losses):
        if world == 1:
            return local_losses
        return zg.allgather_losses(local_losses, sizes)

    replay_entries = [(0, L.ZG_MATRIX, K, N, r)]

    def prefetch(gen):
        # A shard's replay draws the whole population's factors after the
        # forward (on the same stream): drawing them concurrently on a second
        # stream contends with the forward's GEMMs for the SMs and measured
        # slower.  Kept as a no-op hook for that alternative.
        return None

    row_shard = zg.RowShard(rank, world) if (world > 1 and args.replay == "sharded") else None
    row_blocks = world if row_shard is not None else 1

    def replay_update(shaped, cks, W, gen):
        # replay with the SGD step in the replay GEMM's epilogue (what
        # ZeroGrad.step runs): the whole of W, or this rank's block of rows
        # followed by the all-gather of W
        g = _ops._Generation(bases[gen], 0, P, cks)
        spec = {"kind": "sgd", "lr": WL["lr"]}
        if row_shard is not None:
            blk = K // world
            W, _, _ = _ops.launch_replay_step(shaped, cks, 0, L.ZG_MATRIX, W, r, spec, gen=g,
                                              row_range=(rank * blk, (rank + 1) * blk))
            row_shard.gather(W, rank * blk, (rank + 1) * blk)
            return W
        W, _, _ = _ops.launch_replay_step(shaped, cks, 0, L.ZG_MATRIX, W, r, spec, gen=g)
        return W

    def device_step(W, gen):
        # the same sequence ZeroGrad.step runs: forward (factors kept for the
        # generation), fitness exchange, shaping, replay (cached factors when
        # this rank drew the whole population), update
        cks, cks_local = keys[gen]
        prefetch(gen)
        with _ops.generation_scope(bases[gen], a, P_local, cks_local):
            y = _ops.launch_linear(x, W, cks_local, 0, r, sigma, False)
        losses = gather(fitness[a:b])
        shaped, metrics = _ops.launch_shape_fitness(losses, sigma)
        W = replay_update(shaped, cks, W, gen)
        _ops.CACHE.drop_generation(bases[gen])
        del y
        return W

    def timed(step_fn, steps, W):
        times = []
        for i in range(steps):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            W = step_fn(W, args.warmup + i)
            e.record()
            times.append((s, e))
        torch.cuda.synchronize()
        return sum(s.elapsed_time(e) for s, e in times), W

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # The generation as the public API runs it (ZeroGrad.capture ->
    # CapturedGeneration): one CUDA graph holding every candidate's forward
    # (its output [256, 4096] materialised; its loss one element of that
    # output), the fitness all-gather with more than one rank, shaping,
    # replay with the SGD step in the replay GEMM's epilogue, and the guarded
    # write-back of W.  The per-generation base key is copied in before each
    # replay, so every generation draws its own factors.
    opt = zg.ZeroGrad(manifest, zg.sgd(WL["lr"]), P, r, sigma, WL["seed"], WL["run_id"])

    def fwd_loss(p, ctx, batch, rng):
        return ctx.linear(p, ("w",), batch)[0, 0].float(), None

    cg = zg.CapturedGeneration(opt, {"w": W0}, fwd_loss, x, state=opt.init({"w": W0}),
                               candidate_range=(a, P_local) if world > 1 else None,
                               gather=(lambda l: zg.allgather_losses(l, sizes)) if world > 1 else None,
                               row_shard=row_shard)
    cstate = opt.init({"w": W0})
    pending = []

    def resident_step(_, gen):
        # inputs resident in HBM: generations queued back to back, metrics read after the timed region
        nonlocal cstate
        _, cstate, pend = cg.enqueue(zg.ZeroGradState(gen, cstate.opt_state))
        pending.append(pend)

    for i in range(args.warmup):
        resident_step(None, i)
    barrier()

    # timed (device-resident inputs)
    with ClockSampler(dev) as clk:
        barrier()
        ms, _ = timed(resident_step, args.steps, None)
        barrier()
    launches = cg.kernels_per_generation * args.steps
    ms = max_over_ranks(ms)
    clocks = clk.summary()
    for pend in pending:
        pend.result()  # every generation's losses were finite
    pending.clear()

    # the eager launch sequence of the same generation (Python issues every
    # kernel; fitness N(0,1) resident), for comparison and for the per-kernel
    # profile below
    W = W0
    for i in range(args.warmup):
        W = device_step(W, i)
    barrier()
    eager_dev_ms, W = timed(device_step, args.steps, W0)
    eager_dev_ms = max_over_ranks(eager_dev_ms)
    barrier()

    # per-kernel device times (same steps, events around each launch)
    barrier()
    L.profile_begin(1 << 14)
    prof_ms, _ = timed(device_step, args.steps, W0)
    kernels = L.profile_end()
    barrier()

    # end to end through the public API: the batch copied in from pinned host
    # memory every generation, the step's metrics read back.  Eager form:
    # evaluate_shard + (all-gather) + step_from_losses, the fitness from the host.
    params = {"w": W0}
    state = opt.init(params)
    ids_local = range(a, b)  # host-side ids: the public API keeps this range's factors for the replay

    def fwd(p, ctx, batch, rng):
        return ctx.linear(p, ("w",), batch), None

    def e2e_step(Wcur, gen):
        nonlocal state
        xb = x_host.to(dev, non_blocking=True)
        fl = fit_host[a:b].to(dev, non_blocking=True)
        y = opt.evaluate_shard({"w": Wcur}, gen, fwd, xb, ids_local)
        losses = gather(fl)
        newp, state, m = opt.step_from_losses(zg.ZeroGradState(gen, state.opt_state), {"w": Wcur}, losses)
        del y
        return newp["w"]

    Wc = W0
    for i in range(min(args.warmup, 3)):
        Wc = e2e_step(Wc, i)
    barrier()
    eager_ms, _ = timed(e2e_step, args.steps, W0)
    eager_ms = max_over_ranks(eager_ms)
    barrier()

    # Captured form, synchronous: CapturedGeneration.step with the batch
    # copied in from pinned host memory and the metrics read back (a host
    # synchronisation) before the next generation is queued.
    def captured_step(Wcur, gen):
        nonlocal cstate
        _, cstate, _ = cg.step(zg.ZeroGradState(gen, cstate.opt_state), x_host)
        return Wcur

    for i in range(min(args.warmup, 3)):
        captured_step(None, i)
    barrier()
    sync_ms, _ = timed(captured_step, args.steps, None)
    sync_ms = max_over_ranks(sync_ms)
    barrier()

    # Captured form, pipelined, the headline: CapturedGeneration.enqueue with
    # the batch copied from pinned host memory every generation (on the copy
    # stream, into the batch slot the previous-but-one generation used, while
    # the previous generation computes) and generation g-1's metrics read
    # back on the host before generation g+1 is queued.  Timed as one
    # interval on the device from before the first copy to after the last
    # metrics read, less the L2 flushes queued between generations (each
    # bracketed by its own events on the compute stream).  The copy of
    # generation g+1 is issued when generation g-1 ends, so it runs during
    # generation g, not during a flush.
    def pipelined(steps, first):
        nonlocal cstate
        pend, flushes = [], []
        ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
        start, end = ev(), ev()
        start.record()
        for i in range(steps):
            f0, f1 = ev(), ev()
            f0.record()
            flush.zero_()
            f1.record()
            flushes.append((f0, f1))
            _, cstate, p = cg.enqueue(zg.ZeroGradState(first + i, cstate.opt_state), x_host)
            pend.append(p)
            if i >= 1:
                pend[i - 1].result()
        pend[-1].result()
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) - sum(a.elapsed_time(b) for a, b in flushes)

    pipelined(max(3, args.warmup), 0)
    barrier()
    e2e_ms = max_over_ranks(pipelined(args.steps, args.warmup))
    barrier()
    del cg  # holds NCCL work with more than one rank: released before the process group
    torch.cuda.synchronize()

    # "--sections headline" stops here: no secondary workloads
    secondary = args.sections == "all"
    h_kernels, h_ms, h_steps, h_clocks = {}, None, 0, None
    if secondary:
        # the hidden-layer form of the same generation: every candidate has its own
        # input x_p [256, 4096] (seeded N(0, 0.02)), so x_p W is a batched GEMM on
        # the tensor cores; replay reuses the forward's factors; SGD update
        gx = torch.Generator(device=dev).manual_seed(WL["seed"] + a)
        xb_all = (torch.randn(P_local, M, K, generator=gx, device=dev) * 0.02).to(torch.bfloat16)

        def hidden_step(W, gen):
            cks, cks_local = keys[gen]
            prefetch(gen)
            with _ops.generation_scope(bases[gen], a, P_local, cks_local):
                y = _ops.launch_linear(xb_all, W, cks_local, 0, r, sigma, True)
            losses = gather(fitness[a:b])
            shaped, metrics = _ops.launch_shape_fitness(losses, sigma)
            W = replay_update(shaped, cks, W, gen)
            _ops.CACHE.drop_generation(bases[gen])
            del y
            return W

        h_steps = max(1, min(args.steps, 50))
        Wh = W0
        for i in range(args.warmup):
            Wh = hidden_step(Wh, i)
        barrier()
        with ClockSampler(dev) as h_clk:
            barrier()
            h_ms, _ = timed(hidden_step, h_steps, W0)
            barrier()
        h_ms = max_over_ranks(h_ms)
        h_clocks = h_clk.summary()
        L.profile_begin(1 << 14)
        timed(hidden_step, h_steps, W0)
        h_kernels = L.profile_end()
        barrier()
        del xb_all

    value = P * args.steps / (ms / 1e3)
    e2e_value = P * args.steps / (e2e_ms / 1e3)
    sync_value = P * args.steps / (sync_ms / 1e3)
    eager_value = P * args.steps / (eager_ms / 1e3)
    eager_dev_value = P * args.steps / (eager_dev_ms / 1e3)
    if rank == 0:
        pk = peaks()
        known = {k: v for k, v in kernels.items() if kernel_work(k, P_local, world, row_blocks)[0] is not None}
        top = max(known.items(), key=lambda kv: kv[1][1]) if known else None
        roof = None
        if top:
            name, (n, tot) = top
            bound, work = kernel_work(name, P_local, world, row_blocks)
            per = tot / n / 1e3
            if bound == "hbm":
                ach, peak, unit = work / per / 1e9, pk["hbm_gbs"], "GB/s"
            else:
                ach, peak, unit = work / per / 1e12, pk["bf16_tflops"], "TFLOP/s"
            traffic = traffic_for(name)
            roof = {"kernel": name, "bound": bound, "achieved": ach, "peak": peak, "unit": unit,
                    "frac": ach / peak, "traffic": traffic, "peak_source": pk["source"],
                    "launch_ms": tot / n, "launches": n}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "generations_per_sec": args.steps / (ms / 1e3),
            "timed": "CapturedGeneration.enqueue back to back (one CUDA graph per generation), inputs resident",
            "eager_launch_value": {"value": eager_dev_value, "ms_per_step": eager_dev_ms / args.steps,
                                   "what": "the same kernels issued one by one from Python, fitness N(0,1)"},
            "config": {"workload": WORKLOAD_NAME, "population": P, "rank": r, "batch": M, "d_in": K, "d_out": N,
                       "parallelism": (f"population shards x{world}, fitness allgather, "
                                       + ("row-sharded update + W allgather" if row_shard is not None
                                          else "replicated update")) if world > 1 else "1 GPU",
                       "l2": "flushed between steps (256 MiB write outside the timed events)",
                       "update": ("row-sharded" if row_shard is not None else "replicated") if world > 1 else "whole"},
            "roofline": roof,
            "kernels_ms_per_step": {k: v[1] / args.steps for k, v in sorted(kernels.items())},
            "profiled_ms_per_step": prof_ms / args.steps,
            "gpu_launches": launches,
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": M * K * 2 + 8,
                    "d2h_bytes_per_step": 16, "ms_per_step": e2e_ms / args.steps,
                    "api": "ZeroGrad.capture -> CapturedGeneration.enqueue, pinned host batch every generation "
                           "(copied during the previous generation), metrics read back one generation behind",
                    "l2": "flushed before every generation (256 MiB write on the compute stream); "
                          "the flushes' own event time subtracted from the loop's interval"},
            "e2e_sync": {"value": sync_value, "unit": UNIT, "h2d_bytes_per_step": M * K * 2 + 8,
                         "d2h_bytes_per_step": 16, "ms_per_step": sync_ms / args.steps,
                         "api": "CapturedGeneration.step: copy, replay, metrics read before the next generation"},
            "e2e_eager": {"value": eager_value, "unit": UNIT, "h2d_bytes_per_step": M * K * 2 + 4 * P_local,
                          "d2h_bytes_per_step": 16, "ms_per_step": eager_ms / args.steps,
                          "api": "evaluate_shard + step_from_losses (fitness from the host)"},
        }
        hg = h_kernels.get("batched_gemm")
        hidden = None if not secondary else {"workload": "same generation with a per-candidate input x_p[256,4096] (seeded N(0,0.02)): "
                              "batched perturbed GEMM on the tensor cores, replay from the forward's factors, SGD",
                  "value": P * h_steps / (h_ms / 1e3), "unit": UNIT, "steps": h_steps,
                  "ms_per_step": h_ms / h_steps, "clocks": h_clocks,
                  "kernels_ms_per_step": {k: v[1] / h_steps for k, v in sorted(h_kernels.items())}}
        if hidden is not None and hg:
            per = hg[1] / hg[0] / 1e3
            ach = kernel_work("batched_gemm", P_local, world)[1] / per / 1e12
            # the loop keeps the tensor cores busy for ~0.1 s, so the sustained
            # (power-capped) peak is the matching denominator; the burst one is shown too
            hidden["roofline"] = {"kernel": "batched_gemm", "bound": "tensor", "achieved": ach,
                                  "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                                  "frac": ach / pk["bf16_tflops_sustained"],
                                  "frac_of_burst_peak": ach / pk["bf16_tflops"],
                                  "traffic": traffic_for("batched_gemm"),
                                  "peak_source": pk["source"] + " (sustained)", "launch_ms": hg[1] / hg[0]}
            # the whole forward (factor draws + u pass + GEMM) against the same peak
            fwd_ms = sum(h_kernels[k][1] for k in ("batched_gemm", "batched_u_pass") if k in h_kernels) / h_steps
            flops = 2.0 * P_local * M * K * N + 2.0 * P_local * M * r * (K + N)
            hidden["forward_tflops"] = flops / (fwd_ms / 1e3) / 1e12
        if hidden is not None:
            line["hidden_layer"] = hidden
        if world == 1 and secondary:
            line["int8_qat_layer"] = int8_layer_section(dev, args)
            line["lm_tied_ce"] = tied_ce_section(dev, args)
            line["lm_block"] = lm_block_section(dev, args)
        if world == 1 and secondary:
            secs = cpu_generation_sample(8)
            n_cand = max(1, min(64, int(8 * 15.0 / max(secs, 1e-3))))
            secs = cpu_generation_sample(n_cand)
            line["cpu_baseline"] = {"value": n_cand / secs, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
                                    "sample": f"{n_cand} of {P} candidates of one generation (shared x@W, "
                                              "per-candidate low-rank forward, replay contraction), numpy/BLAS "
                                              "+ C threefry"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

"""Benchmark of the NVFP4 hot paths on B200; the last JSON line (rank 0) is the headline.

    python bench.py [--gpus N] [--steps K] [--warmup W]            # the default suite
    python bench.py --config C [--impl ours|reference]              # one configuration
    python bench.py --suite task     # the reference's task.yml shapes vs its published geomeans

Default suite, one JSON line each, headline last:
  N = 1: configurations 2, 3 and 4, the task.yml benchmark geomeans (dual and
         grouped), then configuration 1 (dual GEMM M=8192 N=14336 K=4096, the
         compute-bound SiLU-gated FFN shape) -- the headline.
  N > 1: configurations 2 and 4 (strong scaling), configuration 1 weak-scaled
         (an extra, labelled line), then configuration 1 strong-scaled -- the
         headline.
A step is one call of the hot path over one batch of synthetic input (seeded
N(0,1) operands quantised to NVFP4).

* value: device time of the K timed calls (CUDA events on the launching
  stream; L2 flushed between calls outside the events by a 512 MiB write
  followed by a 512 MiB read, so no dirty flush lines are written back inside
  the next call), max over ranks; whole-job effective TFLOP/s = the FLOP all
  ranks did / that time.
* sustained (headline): the same calls back to back for at least 2 s of
  kernel time, with the SM clock sampled over them; both figures also as
  cycles per call (us x median SM MHz).
* e2e: the same metric through the public drop-in ``custom_kernel`` with the
  step's inputs copied from pinned host memory and the output copied back,
  inside the timed region.
* roofline: dominant kernel's achieved FLOP/s (or GB/s) against the NVFP4
  dense peak (4x the measured bf16 peak) or the measured HBM copy bandwidth.
* cpu_baseline / --impl reference: the CPU oracle (dequantise + fp32 matmul,
  the reference's ref_kernel restated), timed by one protocol for both arms
  in a spawned process that holds no CUDA context: W warm-up steps, then K
  steps, each a 2048 x 2048 output block (all of K) of the configuration,
  with every BLAS thread of the host; plus configuration 0 in full.

Multi-GPU (torchrun, one rank per GPU, no collective on the data path): the
dual GEMM is sharded along N in contiguous 128-row shards of the
configuration's N (shard.n_shard: strong scaling; the rank shards
concatenated are the single-GPU problem); grouped configurations assign
experts by LPT (strong scaling).
"""
from __future__ import annotations

import argparse
import contextlib
import gc
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT / "blackwell-nvfp4-kernels_b200"), str(ROOT)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


@contextlib.contextmanager
def gc_paused():
    """Python's cyclic garbage collector collected before and paused over a
    timed region (as `timeit` does): a collection triggered by allocation
    counts inside the region stalls the launch loop for up to milliseconds,
    idling the GPU inside a timed batch."""
    gc.collect()
    was = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if was:
            gc.enable()
L2_FLUSH_BYTES = 512 << 20


class L2Flush:
    """Evicts L2 between timed calls: a write over one 512 MiB buffer, then a
    read over another.  The read pass evicts the written lines (their
    write-back happens here, not inside the next timed call) and leaves L2
    holding clean lines of a buffer no kernel reads."""

    def __init__(self, device):
        self.w = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
        self.r = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=device)
        self.sink = torch.empty((), dtype=torch.int32, device=device)

    def __call__(self):
        self.w.zero_()
        torch.amax(self.r, dim=0, out=self.sink)

    describe = "flushed (512 MiB write + 512 MiB read) between timed calls"


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def dual_workload(cfg: int, rank: int, world: int, device, scaling: str = "strong"):
    """Rank's share of dual configuration `cfg`, A replicated (same seed
    everywhere).  strong: B1/B2 rows [n0, n1) = shard.n_shard(N, world, rank)
    of the configuration's own operands, so the rank outputs side by side are
    the single-GPU C; weak: every rank a full-N problem (rank 0's is the
    single-GPU configuration, the others draw their own B1/B2)."""
    from nvfp4_b200 import inputs as I
    from nvfp4_b200.shard import n_shard
    spec = I.DUAL_CONFIGS[cfg]
    m, n, k = spec["m"], spec["n"], spec["k"]
    g = torch.Generator().manual_seed(spec["seed"])
    a = torch.randn(m, k, generator=g)
    if scaling == "weak" and rank > 0:
        g = torch.Generator().manual_seed(spec["seed"] * 1000 + rank)
    b1 = torch.randn(n, k, generator=g)
    b2 = torch.randn(n, k, generator=g)
    n0, n1 = n_shard(n, world, rank) if scaling == "strong" else (0, n)
    data = I.dual_from_fp32(a, b1[n0:n1], b2[n0:n1], device=device)
    nr = n1 - n0
    flop = 4.0 * m * nr * k
    nbytes = m * k // 2 + 2 * nr * k // 2 + (m + 2 * nr) * k // 16 + 2 * m * nr
    desc = dict(workload=f"dual_gemm_cfg{cfg}", m=m, n_global=n if scaling == "strong" else n * world,
                n_this_rank=nr, n_rows_this_rank=[n0, n1], k=k, l=1)
    return data, flop, nbytes, desc


def group_workload(cfg: int, rank: int, world: int, device):
    from nvfp4_b200 import inputs as I
    from nvfp4_b200.shard import imbalance, lpt_assign
    spec = I.GROUP_CONFIGS[cfg]
    ms = I.config3_m_sizes(spec["seed"], spec["groups"]) if cfg == 3 else \
        I.config4_m_sizes(spec["seed"], spec["experts"], spec["tokens"], spec["zipf_s"])
    n, k = spec["n"], spec["k"]
    costs = [float(m) * n * k for m in ms]
    bins = lpt_assign(costs, world)
    mine = bins[rank]
    g = torch.Generator().manual_seed(1000 + spec["seed"])
    pairs = []
    for i, m in enumerate(ms):   # draw every group so data is identical for any world size
        a = torch.randn(m, k, generator=g)
        b = torch.randn(n, k, generator=g)
        if i in mine:
            pairs.append((a, b))
    data = I.group_from_fp32(pairs, device=device)
    mr = [ms[i] for i in mine]
    flop = sum(2.0 * m * n * k for m in mr)
    nbytes = sum(m * k // 2 + m * k // 16 + 2 * m * n + n * k // 2 + n * k // 16 for m in mr)
    desc = dict(workload=f"grouped_gemm_cfg{cfg}", groups=len(ms), groups_this_rank=len(mine),
                sum_m=sum(ms), n=n, k=k, lpt_imbalance=round(imbalance(costs, bins), 4))
    return data, flop, nbytes, desc


def quant_workload(rank, world, device):
    """Configuration 5: quantise configuration 1's fp32 operands (A, B1, B2)
    to NVFP4 on the device (the producer step in front of both GEMMs); HBM-bound."""
    from nvfp4_b200 import inputs as I
    spec = I.DUAL_CONFIGS[1]
    m, n, k = spec["m"], spec["n"], spec["k"]
    g = torch.Generator().manual_seed(spec["seed"] * 1000 + rank)
    from nvfp4_b200.quantize import quantize
    xs = [torch.randn(r, k, generator=g).to(device) for r in (m, n, n)]
    xs = [(x, quantize(x)) for x in xs]            # outputs allocated once, reused per step
    elems = sum(x.numel() for x, _ in xs)
    nbytes = elems * 4 + elems // 2 + elems // 16 * 2      # fp32 in, e2m1 + two scale layouts out
    desc = dict(workload="quantize_cfg1_operands", rows=[m, n, n], k=k)
    return xs, 0.0, nbytes, desc


def moe_workload(rank, world, device, tokens=32768):
    """Configuration 6: MoE dispatch of configuration 4's routing (32768 tokens,
    Zipf over 64 experts, top-1) at its K = 7168: fp32 tokens -> per-expert
    NVFP4 A operands + scale atoms + permutation; HBM-bound."""
    from nvfp4_b200 import inputs as I
    from nvfp4_b200 import moe
    spec = I.GROUP_CONFIGS[4]
    k, experts = spec["k"], 64
    g = torch.Generator().manual_seed(4000 + rank)
    x = torch.randn(tokens, k, generator=g).to(device)
    ids = I.config4_expert_ids(seed=4 + rank, tokens=tokens).to(device)
    d = moe.dispatch(x, ids, experts)                  # buffers allocated once, reused per step
    torch.cuda.synchronize()
    blocks = int(d.atom_offsets[-1].item())
    rows = int(d.row_offsets[-1].item())
    nbytes = (tokens * k * 4 + tokens * 4 + rows * k // 2 + blocks * (k // 64) * 512
              + 2 * rows * 4 + 3 * (experts + 1) * 4)
    desc = dict(workload="moe_dispatch_cfg4" if tokens == 32768 else f"moe_dispatch_{tokens}x{k}",
                tokens=tokens, k=k, experts=experts, topk=1)
    return (x, ids, experts, d), 0.0, nbytes, desc


def moe_layer_workload(rank, world, device, tokens=32768):
    """Configuration 7: the MoE expert layer around configuration 4's grouped
    GEMM -- dispatch of 32768 fp32 tokens (Zipf top-1 over 64 experts),
    device-routed grouped GEMM against 64 NVFP4 experts [2048 x 7168], weighted
    combine -- with no host round trip inside the step.  Metric: the grouped
    GEMM's FLOP over the whole layer's time."""
    from nvfp4_b200 import inputs as I
    from nvfp4_b200 import moe
    from nvfp4_b200.quantize import quantize
    spec = I.GROUP_CONFIGS[4]
    k, n, experts = spec["k"], spec["n"], spec["experts"]
    g = torch.Generator().manual_seed(7000 + rank)
    weights = []
    for _ in range(experts):
        packed, _, sfp = quantize(torch.randn(n, k, generator=g).to(device))
        weights.append((packed, sfp))
    w = moe.ExpertWeights(weights)
    x = torch.randn(tokens, k, generator=g).to(device)
    ids = I.config4_expert_ids(seed=4 + rank, tokens=tokens).to(device)
    rw = torch.rand(tokens, generator=g).to(device)
    d = moe.dispatch(x, ids, experts)
    c_all = torch.empty(tokens, n, dtype=torch.float16, device=device)
    out = torch.empty(tokens, n, dtype=torch.float32, device=device)
    torch.cuda.synchronize()
    flop = 2.0 * tokens * n * k
    nbytes = (tokens * k * 4 + tokens * 4 + experts * n * (k // 2 + k // 16)
              + tokens * n * 4 + tokens * 4)          # tokens in, weights, out (the layer's I/O)
    desc = dict(workload="moe_layer_cfg4", tokens=tokens, k=k, n=n, experts=experts, topk=1,
                stages="dispatch + device-routed grouped GEMM + combine")
    return (x, ids, rw, w, d, c_all, out), flop, nbytes, desc


def shape_workload(args, device):
    """--shape M,N,K (dual) or --group-shape M1:M2:..,N,K (grouped): a seeded
    N(0,1) workload of any size for kernel-only profiling runs."""
    from nvfp4_b200 import inputs as I
    g = torch.Generator().manual_seed(11)
    if args.shape:
        m, n, k = (int(v) for v in args.shape.split(","))
        data = I.dual_from_fp32(torch.randn(m, k, generator=g), torch.randn(n, k, generator=g),
                                torch.randn(n, k, generator=g), device=device)
        nbytes = m * k // 2 + 2 * n * k // 2 + (m + 2 * n) * k // 16 + 2 * m * n
        return 1, data, 4.0 * m * n * k, nbytes, dict(workload=f"dual_gemm_{m}x{n}x{k}", m=m, n=n, k=k)
    ms_s, n_s, k_s = args.group_shape.split(",")
    ms, n, k = [int(v) for v in ms_s.split(":")], int(n_s), int(k_s)
    data = I.group_from_fp32([(torch.randn(m, k, generator=g), torch.randn(n, k, generator=g))
                              for m in ms], device=device)
    nbytes = sum(m * k // 2 + m * k // 16 + 2 * m * n + n * k // 2 + n * k // 16 for m in ms)
    return 3, data, sum(2.0 * m * n * k for m in ms), nbytes, \
        dict(workload=f"grouped_gemm_{'+'.join(map(str, ms))}x{n}x{k}", groups=ms, n=n, k=k)


def make_workload(cfg, rank, world, device, tokens=32768, scaling="strong"):
    if cfg == 5:
        return quant_workload(rank, world, device)
    if cfg == 6:
        return moe_workload(rank, world, device, tokens)
    if cfg == 7:
        return moe_layer_workload(rank, world, device, tokens)
    return dual_workload(cfg, rank, world, device, scaling) if cfg in (0, 1, 2) else \
        group_workload(cfg, rank, world, device)


def call(cfg, data):
    if cfg == 5:
        from nvfp4_b200.quantize import quantize
        return [quantize(x, out=o) for x, o in data]
    if cfg == 6:
        from nvfp4_b200 import moe
        x, ids, experts, d = data
        return moe.dispatch(x, ids, experts, out=d)
    if cfg == 7:
        from nvfp4_b200 import moe
        x, ids, rw, w, d, c_all, out = data
        moe.dispatch(x, ids, len(w), out=d)
        moe.grouped_gemm(d, w, c_all)
        return moe.combine(c_all, d, rw, out=out)
    if cfg in (0, 1, 2):
        from nvfp4_b200.dual_gemm import custom_kernel
    else:
        from nvfp4_b200.group_gemm import custom_kernel
    return custom_kernel(data)


def device_tensors(cfg, data):
    """(input tensors a user would ship each step, output tensors)."""
    if cfg == 5:
        return [x for x, _ in data], [t for _, o in data for t in o]
    if cfg == 6:
        x, ids, _, d = data
        return [x, ids], [d.packed, d.sf, d.counts, d.row_offsets, d.atom_offsets, d.src, d.dst]
    if cfg == 7:
        x, ids, rw, _, _, _, out = data
        return [x, ids, rw], [out]
    if cfg in (0, 1, 2):
        return [data[0], data[1], data[2], data[6], data[7], data[8]], [data[9]]
    abc, _, perm, sizes = data
    ins, outs = [], []
    for (a, b, c), (sa, sb), s in zip(abc, perm, sizes):
        if s[0] > 0:
            ins += [a, sa]
            outs.append(c)
        ins += [b, sb]
    return ins, outs


def nbytes_of(ts):
    return sum(t.numel() * t.element_size() for t in ts)


# ---------------------------------------------------------------------------
# clocks (NVML, read-only)
# ---------------------------------------------------------------------------
# The sampler loop runs in a child process (a sampling thread here would
# compete with the launch loop for the GIL); NVML queries also go through the
# driver like the launches, so the period is a few milliseconds, not one.
_SAMPLER_SRC = r"""
import select, sys
import pynvml
pynvml.nvmlInit()
bus, index, period = sys.argv[1], int(sys.argv[2]), float(sys.argv[3])
try:
    h = pynvml.nvmlDeviceGetHandleByPciBusId_v2(bus)
except Exception:
    h = pynvml.nvmlDeviceGetHandleByIndex(index)
reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
    pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
print("ready", pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), flush=True)
out = []
while not select.select([sys.stdin], [], [], period)[0]:   # until the parent closes stdin
    try:
        out.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), reasons(h)))
    except Exception:
        pass
print("\n".join(f"{m} {r}" for m, r in out), flush=True)
"""


class ClockSampler:
    """SM clock and clock-event reasons of one GPU, sampled every `period_s`
    by NVML in a child process while the `with` block runs."""
    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples, self.reasons = [], set()
        self.ok = False
        self.err = None
        self.max_mhz = None
        self.proc = None
        try:
            pr = torch.cuda.get_device_properties(device_index)
            self.bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        except Exception:  # noqa: BLE001
            self.bus = ""
        self.index = device_index
        self.period = period_s

    def __enter__(self):
        import subprocess
        try:
            self.proc = subprocess.Popen(
                [sys.executable, "-c", _SAMPLER_SRC, self.bus, str(self.index), str(self.period)],
                stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
            first = self.proc.stdout.readline().split()
            if len(first) != 2 or first[0] != "ready":
                raise RuntimeError("sampler did not start: " + self.proc.stderr.read()[-300:])
            self.max_mhz = int(first[1])
            self.ok = True
        except Exception as e:  # noqa: BLE001
            self.err = repr(e)
            if self.proc is not None and self.proc.poll() is None:
                self.proc.kill()
                self.proc.wait()
        return self

    def __exit__(self, *exc):
        if not self.ok:
            return
        try:
            out, _ = self.proc.communicate(input="", timeout=30)
        except Exception as e:  # noqa: BLE001
            self.proc.kill()
            self.proc.wait()
            self.ok, self.err = False, repr(e)
            return
        for line in out.split("\n"):
            f = line.split()
            if len(f) != 2:
                continue
            self.samples.append(int(f[0]))
            bits = int(f[1])
            for name, b in self.REASONS.items():
                if bits & b:
                    self.reasons.add(name)

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": self.err}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU oracle timing
# ---------------------------------------------------------------------------
CPU_SAMPLE = 2048   # output rows and columns of one CPU oracle step (all of K)


def _cpu_step(cfg: int, rows: int = CPU_SAMPLE, cols: int = CPU_SAMPLE):
    """(step function, FLOP per step, description) of one CPU oracle step of
    configuration `cfg`: a rows x cols output block over the configuration's
    whole K, seeded N(0,1) operands quantised to NVFP4 on the host
    (the dual GEMM: both GEMMs and the SiLU gate; grouped: one group's GEMM,
    as many rows as the largest group has, at most `rows`)."""
    from nvfp4_b200 import inputs as I
    from nvfp4_b200.formats import quantize_nvfp4
    from oracle import nvfp4_oracle as O
    g = torch.Generator().manual_seed(100 + cfg)
    if cfg in (0, 1, 2):
        spec = I.DUAL_CONFIGS[cfg]
        k = spec["k"]
        rows, cols = min(rows, spec["m"]), min(cols, spec["n"])
        (a, sa), (b1, s1), (b2, s2) = (
            [t.numpy() for t in quantize_nvfp4(torch.randn(r, k, generator=g))]
            for r in (rows, cols, cols))
        return (lambda: O.ref_dual(a, b1, b2, sa, s1, s2)), 4.0 * rows * cols * k, \
            f"oracle ref_dual on a {rows}x{cols} output block x K={k}"
    spec = I.GROUP_CONFIGS[cfg]
    ms = I.config3_m_sizes(spec["seed"], spec["groups"]) if cfg == 3 else \
        I.config4_m_sizes(spec["seed"], spec["experts"], spec["tokens"], spec["zipf_s"])
    k = spec["k"]
    rows, cols = min(rows, max(ms)), min(cols, spec["n"])
    (a, sa), (b, sb) = ([t.numpy() for t in quantize_nvfp4(torch.randn(r, k, generator=g))]
                        for r in (rows, cols))
    return (lambda: O.ref_group(a, b, sa, sb)), 2.0 * rows * cols * k, \
        f"oracle ref_group on a {rows}x{cols} output block x K={k}"


def cpu_oracle_protocol(cfg: int, steps: int, warmup: int) -> dict:
    """The CPU baseline of both bench arms: `warmup` untimed then `steps` timed
    oracle steps of configuration `cfg` (each a 2048 x 2048 block, all of K),
    plus configuration 0 in full (256 x 512 x 1024, repeated for >= 2 s), with
    the BLAS pool at every host thread.  Runs in a spawned child process
    (cpu_oracle_in_child) so neither arm's CUDA context, pinned buffers or
    clock sampler shares the host with it."""
    from threadpoolctl import threadpool_limits
    cores = cpu_cores()
    torch.set_num_threads(cores)
    with threadpool_limits(limits=cores):
        step, flop, sample = _cpu_step(cfg)
        for _ in range(warmup):
            step()
        secs = 0.0
        for _ in range(steps):
            t0 = time.perf_counter()
            step()
            secs += time.perf_counter() - t0
        step0, flop0, _ = _cpu_step(0, 256, 512)
        step0()
        reps0, secs0 = 0, 0.0
        while reps0 < 3 or secs0 < 2.0:
            t0 = time.perf_counter()
            step0()
            secs0 += time.perf_counter() - t0
            reps0 += 1
    return {"value": round(flop * steps / secs / 1e12, 5), "unit": "TFLOP/s", "cores": cores,
            "kind": "port", "steps": steps, "warmup": warmup,
            "ms_per_step": round(secs * 1e3 / steps, 2),
            "sample": f"{sample} per step (bounded sample, not extrapolated to the full "
                      f"configuration: TFLOP/s of the block itself), numpy + BLAS on {cores} "
                      f"threads, spawned process without a CUDA context",
            "full_config0": {"value": round(flop0 * reps0 / secs0 / 1e12, 5), "unit": "TFLOP/s",
                             "reps": reps0, "ms_per_call": round(secs0 * 1e3 / reps0, 3),
                             "sample": "configuration 0 in full (256x512x1024 dual GEMM), "
                                       "no extrapolation"}}


def cpu_oracle_in_child(cfg: int, steps: int, warmup: int) -> dict:
    import multiprocessing as mp
    with mp.get_context("spawn").Pool(1) as pool:
        return pool.apply(cpu_oracle_protocol, (cfg, steps, warmup))


def time_cpu_quant(x_dev, budget_s: float):
    """Oracle quantiser (numpy) on a 1024-row sample of one operand, bytes
    counted as on the device: fp32 in, e2m1 + plain and permuted scales out."""
    from oracle import nvfp4_oracle as O
    x = x_dev[:1024].detach().cpu().numpy()
    rows, k = x.shape
    nb = rows * k * 4 + rows * k // 2 + rows * k // 16 * 2
    O.quantize_nvfp4(x[:16])
    secs, reps = 0.0, 0
    while reps < 1 or secs < budget_s:
        t0 = time.perf_counter()
        O.quantize_nvfp4(x)
        secs += time.perf_counter() - t0
        reps += 1
    return {"value": round(nb * reps / secs / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"numpy oracle quantiser on {rows}x{k} fp32 rows, {reps} reps "
                      f"(~{budget_s:.0f} s, single-threaded numpy)"}


def time_cpu_moe(x_dev, ids_dev, experts, budget_s: float):
    """Oracle dispatch (numpy) on the first 1024 tokens, bytes counted as on
    the device: fp32 tokens + ids in, e2m1 rows + scale atoms + src/dst out."""
    from oracle import nvfp4_oracle as O
    x = x_dev[:1024].detach().cpu().numpy()
    ids = ids_dev[:1024].detach().cpu().numpy().reshape(-1, 1)
    t, k = x.shape
    (_, _, atom_off, _, _), _, _ = O.moe_dispatch(x[:16], ids[:16], experts)
    (_, _, atom_off, _, _), _, _ = O.moe_dispatch(x, ids, experts)
    nb = t * k * 4 + t * 4 + t * k // 2 + int(atom_off[-1]) * (k // 64) * 512 + 2 * t * 4
    secs, reps = 0.0, 0
    while reps < 1 or secs < budget_s:
        t0 = time.perf_counter()
        O.moe_dispatch(x, ids, experts)
        secs += time.perf_counter() - t0
        reps += 1
    return {"value": round(nb * reps / secs / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"numpy oracle dispatch (route + quantise + swizzle) of {t} tokens x K={k}, "
                      f"{reps} reps (~{budget_s:.0f} s, single-threaded numpy)"}


def time_cpu_moe_layer(data, budget_s: float, tokens: int = 256):
    """Oracle MoE layer (numpy: route + quantise + per-expert dequantised fp32
    GEMM + combine) on the first `tokens` tokens, TFLOP/s of the GEMM part."""
    from oracle import nvfp4_oracle as O
    x_dev, ids_dev, rw_dev, w = data[0], data[1], data[2], data[3]
    x = x_dev[:tokens].detach().cpu().numpy()
    ids = ids_dev[:tokens].detach().cpu().numpy().reshape(-1, 1)
    rw = rw_dev[:tokens].detach().cpu().numpy()
    used = sorted(set(int(v) for v in ids.reshape(-1)))
    wts = {}
    for e in used:
        b, sfp = w.w[e]
        n, kh = b.shape[0], b.shape[1]
        wts[e] = (b.detach().cpu().view(torch.uint8).numpy().reshape(n, kh),
                  O.unpermute_sf(sfp.detach().cpu().view(torch.uint8).permute(5, 2, 4, 0, 1, 3)
                                 .contiguous().numpy(), n, kh * 2 // 16)[:, :, 0])
    n = next(iter(wts.values()))[0].shape[0]
    k = x.shape[1]

    def step():
        (counts, row_off, _, src, dst), packed, _ = O.moe_dispatch(x, ids, len(w.w))
        _, sf = O.quantize_nvfp4(x[src])
        c = np.zeros((len(src), n), np.float16)
        for e in used:
            r0, r1 = int(row_off[e]), int(row_off[e + 1])
            if r1 > r0:
                c[r0:r1] = O.ref_group(packed[r0:r1], wts[e][0], sf[r0:r1], wts[e][1])
        O.moe_combine(c, dst, rw, x.shape[0], 1)

    torch.set_num_threads(cpu_cores())
    step()
    secs, reps = 0.0, 0
    while reps < 1 or secs < budget_s:
        t0 = time.perf_counter()
        step()
        secs += time.perf_counter() - t0
        reps += 1
    return {"value": round(2.0 * tokens * n * k * reps / secs / 1e12, 5), "unit": "TFLOP/s",
            "cores": cpu_cores(), "kind": "port",
            "sample": f"numpy oracle MoE layer (route, quantise, dequantised fp32 GEMM per expert, "
                      f"combine) on {tokens} tokens x K={k} x N={n}, {reps} reps (~{budget_s:.0f} s)"}


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count()


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------
def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_PEAKS["hbm_gbs"], FALLBACK_PEAKS["bf16_tflops"], "fallback"


def load_traffic(workload: str):
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        v = d.get(workload)
        if v is not None:
            return float(v["dram_bytes_per_call"])
    return None


# ---------------------------------------------------------------------------
# the reference's own benchmark shapes (task.yml) through custom_kernel
# ---------------------------------------------------------------------------
# nvfp4_dual_gemm/task.yml:58-62 and nvfp4_group_gemm/task.yml:59-63 (seed 1111);
# published geomeans: nvfp4_dual_gemm/README.md:19 (submission_v4) and
# nvfp4_group_gemm/README.md:33 (submission_v7), both on one B200.
TASK_DUAL = [(256, 4096, 7168), (512, 4096, 7168), (256, 3072, 4096), (512, 3072, 7168)]
TASK_GROUP = [([80, 176, 128, 72, 64, 248, 96, 160], 4096, 7168),
              ([40, 76, 168, 72, 164, 148, 196, 160], 7168, 2048),
              ([192, 320], 3072, 4096),
              ([128, 384], 4096, 1536)]
TASK_PUBLISHED_US = {"dual": 20.692, "group": 25.407}
TASK_SEED = 1111
TASK_INPUTS = 15        # distinct inputs per shape, as the reference's eval.py times them


def task_inputs(kind, shape, device):
    """The 15 inputs eval.py builds per benchmark (seed += 42 before each),
    made on the device by the restated reference generators: the reference
    harness's own tensors for these seeds."""
    from nvfp4_b200 import inputs as I
    out = []
    for i in range(TASK_INPUTS):
        seed = TASK_SEED + 42 * (i + 1)
        if kind == "dual":
            m, n, k = shape
            out.append(I.reference_dual_input(m, n, k, 1, seed, device=device))
        else:
            ms, n, k = shape
            out.append(I.reference_group_input(ms, [n] * len(ms), [k] * len(ms), len(ms), seed,
                                               device=device))
    return out


def task_flop(kind, shape):
    if kind == "dual":
        m, n, k = shape
        return 4.0 * m * n * k
    ms, n, k = shape
    return sum(2.0 * m * n * k for m in ms)


def task_suite_lines(args, device):
    """Per reference benchmark shape: L2 flushed, then the 15 distinct inputs
    run back to back between two CUDA events; the per-call mean of `steps`
    such batches.  One result per task: geomean us against the published
    geomean of the reference's best submission."""
    from nvfp4_b200 import _lib
    from nvfp4_b200.dual_gemm import custom_kernel as dual_kernel
    from nvfp4_b200.group_gemm import custom_kernel as group_kernel
    flush = L2Flush(device)
    lines = []
    for kind, shapes, fn in (("dual", TASK_DUAL, dual_kernel), ("group", TASK_GROUP, group_kernel)):
        per_shape, per_shape_std, tflops = [], [], []
        with ClockSampler(device.index, period_s=0.02) as clk:
            for shape in shapes:
                datas = task_inputs(kind, shape, device)
                for _ in range(args.warmup):
                    for d in datas:
                        fn(d)
                torch.cuda.synchronize()
                times = []
                with gc_paused():
                    for _ in range(args.steps):
                        flush()
                        e0 = torch.cuda.Event(enable_timing=True)
                        e1 = torch.cuda.Event(enable_timing=True)
                        e0.record()
                        for d in datas:
                            fn(d)
                        e1.record()
                        torch.cuda.synchronize()
                        times.append(e0.elapsed_time(e1) * 1e3 / len(datas))
                us = statistics.mean(times)
                per_shape.append(round(us, 3))
                per_shape_std.append(round(statistics.stdev(times), 3) if len(times) > 1 else 0.0)
                tflops.append(round(task_flop(kind, shape) / us / 1e6, 1))
                del datas
        assert _lib.device_status() == 0
        geo = float(np.exp(np.mean(np.log(per_shape))))
        pub = TASK_PUBLISHED_US[kind]
        lines.append({
            "metric": f"runtime geomean over the reference's task.yml benchmark shapes "
                      f"({'dual' if kind == 'dual' else 'grouped'} GEMM)",
            "value": round(geo, 3), "unit": "us", "higher_is_better": False,
            "vs_baseline": round(geo / pub, 4), "reference_published_us": pub,
            "per_shape_us": per_shape, "per_shape_std_us": per_shape_std, "per_shape_tflops": tflops,
            "shapes": [list(s) if kind == "dual" else [s[0], s[1], s[2]] for s in shapes],
            "method": f"{TASK_INPUTS} distinct inputs per shape (the reference generator's own "
                      f"tensors, seeds {TASK_SEED}+42i), L2 flushed before each batch, mean per "
                      f"call over {args.steps} batches, custom_kernel API",
            "n_gpus": 1, "clocks": clk.summary()})
    return lines


def run_task_suite(args):
    torch.cuda.set_device(0)
    for line in task_suite_lines(args, torch.device("cuda", 0)):
        print(json.dumps(line), flush=True)


def metric_name(cfg):
    if cfg == 5:
        return "NVFP4 quantisation bandwidth (fp32 -> e2m1 + e4m3 scales)"
    if cfg == 6:
        return "MoE dispatch bandwidth (route + fp32 -> NVFP4 per-expert operands)"
    if cfg == 7:
        return "NVFP4 effective TFLOPS (MoE expert layer: dispatch + grouped GEMM + combine)"
    return "NVFP4 effective TFLOPS (dual GEMM)" if cfg in (0, 1, 2) else \
        "NVFP4 effective TFLOPS (grouped GEMM)"


def scaling_of(cfg: int, dual_scaling: str) -> str:
    if cfg in (0, 1, 2):
        return dual_scaling
    return "weak" if cfg in (6, 7) else "strong"


def timed_calls(cfg, data, calls, flush, stream):
    """Per-call device ms of `calls` calls, L2 flushed before each (outside
    the events), CUDA events on the launching stream."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(calls)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(calls)]
    for i in range(calls):
        flush()
        starts[i].record(stream)
        call(cfg, data)
        ends[i].record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def all_max(pg, device, v: float) -> float:
    t = torch.tensor([v], dtype=torch.float64, device=device)
    if pg:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return t.item()


def all_sum(pg, device, v: float) -> float:
    t = torch.tensor([v], dtype=torch.float64, device=device)
    if pg:
        pg.all_reduce(t, op=pg.ReduceOp.SUM)
    return t.item()


def run_config(cfg, args, rank, world, device, pg, flush, *, dual_scaling="strong", e2e=True,
               sustained=False, cpu_baseline=False):
    """One configuration: warm-up, K timed calls, optionally the sustained
    loop, the end-to-end leg and the CPU baseline.  Returns rank 0's JSON
    line as a dict (every rank takes the same collective steps)."""
    from nvfp4_b200 import _lib
    data, flop, nbytes, desc = make_workload(cfg, rank, world, device, args.tokens, dual_scaling)
    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        call(cfg, data)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0

    with ClockSampler(device.index) as clk, gc_paused():
        if pg:                                  # ranks start the timed loop together
            pg.barrier()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed")
        launches0 = _lib.load().nvfp4_launch_count()
        per_call_ms = timed_calls(cfg, data, args.steps, flush, stream)
        launches = _lib.load().nvfp4_launch_count() - launches0
        torch.cuda.nvtx.range_pop()
    if pg:
        pg.barrier()
    status = _lib.device_status()
    assert status == 0, f"device status {status:#x}"
    t_max_s = all_max(pg, device, sum(per_call_ms)) / 1e3
    flop_all = all_sum(pg, device, flop)
    bytes_all = all_sum(pg, device, float(nbytes))
    ms_per_step = t_max_s * 1e3 / args.steps
    quant = cfg in (5, 6)        # bytes-moved metric for the quantiser and the dispatch
    unit = "GB/s" if quant else "TFLOP/s"
    value = bytes_all * args.steps / t_max_s / 1e9 if quant else flop_all * args.steps / t_max_s / 1e12
    clocks = clk.summary()
    scaling = scaling_of(cfg, dual_scaling)
    par = ("n-shard" if cfg in (0, 1, 2) and dual_scaling == "strong" else
           "n-replica" if cfg in (0, 1, 2) else "token-shard" if cfg in (6, 7) else
           "expert-lpt") + str(world)
    result = {
        "metric": metric_name(cfg), "value": round(value, 2), "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5), "us_per_call": round(ms_per_step * 1e3, 2),
        "us_per_call_std": round(statistics.stdev(per_call_ms) * 1e3, 2) if len(per_call_ms) > 1 else 0.0,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
        "dtype": ("int32 routing + fp32 -> e2m1 + e4m3 block16" if cfg == 6 else
                  "fp32 -> e2m1 + e4m3 block16") if quant
        else "fp32 tokens -> nvfp4 x nvfp4 -> fp32 acc -> fp16 -> fp32 combine" if cfg == 7
        else "nvfp4(e2m1+e4m3 block16) x nvfp4 -> fp32 acc -> fp16",
        "data": "synthetic: seeded N(0,1) fp32 quantised to NVFP4",
        "config": {**desc, "parallelism": par, "l2": L2Flush.describe},
    }
    if clocks.get("sm_mhz"):
        result["cycles_per_call"] = round(ms_per_step * 1e3 * clocks["sm_mhz"])

    if sustained:
        # back to back for >= args.sustain_s of kernel time (same calls on every rank)
        calls = max(args.steps, int(args.sustain_s * 1e3 / ms_per_step) + 1)
        with ClockSampler(device.index, period_s=0.02) as sclk, gc_paused():
            if pg:
                pg.barrier()
            torch.cuda.synchronize()
            sus_ms = timed_calls(cfg, data, calls, flush, stream)
        assert _lib.device_status() == 0
        ts = all_max(pg, device, sum(sus_ms)) / 1e3
        sc = sclk.summary()
        sus = {"value": round(flop_all * calls / ts / 1e12, 2), "unit": unit, "calls": calls,
               "kernel_seconds": round(ts, 3), "us_per_call": round(ts * 1e6 / calls, 2),
               "clocks": sc}
        if sc.get("sm_mhz"):
            sus["cycles_per_call"] = round(ts * 1e6 / calls * sc["sm_mhz"])
        result["sustained"] = sus

    if e2e:
        result["e2e"] = e2e_leg(cfg, data, args, device, stream, pg, flop_all, bytes_all)

    # ---- roofline of the dominant kernel (the GEMM kernel is the only launch)
    hbm_peak, bf16_peak, peak_kind = load_peaks()
    nvfp4_peak = 4.0 * bf16_peak
    avg_launch_s = statistics.mean(per_call_ms) / 1e3
    hbm_bound = cfg in (2, 5, 6)
    if hbm_bound:
        ach = nbytes / avg_launch_s / 1e9
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(ach / hbm_peak, 4)}
    else:
        ach = flop / avg_launch_s / 1e12
        roof = {"bound": "tensor", "achieved": round(ach, 1), "peak": nvfp4_peak,
                "unit": "TFLOP/s", "frac": round(ach / nvfp4_peak, 4)}
    roof["traffic"] = load_traffic(desc["workload"]) if world == 1 else None
    roof["algorithmic_bytes"] = nbytes
    roof["peak_source"] = (f"{peak_kind}: NVFP4 dense = 4 x bf16 {bf16_peak} TFLOP/s"
                           if not hbm_bound else f"{peak_kind}: HBM copy {hbm_peak} GB/s")
    if world > 1:
        roof["note"] = "per rank (rank 0's launches)"
    result["roofline"] = roof
    result["gpu_launches"] = launches   # this library's launches in the timed region (its counter)
    result["clocks"] = clocks

    if cpu_baseline and rank == 0 and world == 1 and not args.no_cpu_baseline:
        if cfg == 6:
            result["cpu_baseline"] = time_cpu_moe(data[0], data[1], data[2], args.cpu_budget)
        elif cfg == 7:
            result["cpu_baseline"] = time_cpu_moe_layer(data, args.cpu_budget)
        elif quant:
            result["cpu_baseline"] = time_cpu_quant(data[0][0], args.cpu_budget)
        else:
            result["cpu_baseline"] = cpu_oracle_in_child(cfg, args.steps, args.warmup)
    del data
    torch.cuda.empty_cache()
    return result


def _clone_data(x):
    """A second set of a GEMM configuration's device tensors (same shapes and
    strides; one-byte types copied as bytes)."""
    if isinstance(x, torch.Tensor):
        if x.element_size() == 1 and x.dtype != torch.uint8:
            return x.view(torch.uint8).clone().view(x.dtype)
        return x.clone()
    if isinstance(x, tuple):
        return tuple(_clone_data(v) for v in x)
    if isinstance(x, list):
        return [_clone_data(v) for v in x]
    return x


def e2e_leg(cfg, data, args, device, stream, pg, flop_all, bytes_all):
    """The metric through the public API with pinned host buffers.  Every step
    uploads its inputs and reads its result back.  The GEMM configurations
    alternate two sets of device buffers, as a serving loop would: step i+1's
    upload (its own stream) and step i-1's read-back (another stream; PCIe is
    full duplex) overlap step i's compute, and a step waits only for its own
    inputs and for the read-back that last used its buffers.  The quantiser and
    MoE configurations keep one set (step i+1's upload waits for step i)."""
    sets = [data, _clone_data(data)] if cfg in (0, 1, 2, 3, 4) else [data]
    bufs = [device_tensors(cfg, d) for d in sets]
    ins, outs = bufs[0]
    h_ins = [t.detach().cpu().pin_memory() for t in ins]
    h_outs = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in outs]
    h2d, d2h = nbytes_of(ins), nbytes_of(outs)
    for d in sets:
        call(cfg, d)
    torch.cuda.synchronize()
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    nb = len(sets)
    with gc_paused():
        es.record(stream)
        s_in.wait_event(es)
        s_out.wait_event(es)
        done_c = [None] * nb     # compute that last read buffer set b
        done_out = [None] * nb   # read-back that last read buffer set b
        last_out = None
        for i in range(args.e2e_steps):
            b = i % nb
            d_ins, d_outs = bufs[b]
            with torch.cuda.stream(s_in):              # the set's inputs are free once its last compute ended
                if done_c[b] is not None:
                    s_in.wait_event(done_c[b])
                for d, h in zip(d_ins, h_ins):
                    d.copy_(h, non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
            stream.wait_event(ev_in)
            if done_out[b] is not None:
                stream.wait_event(done_out[b])
            call(cfg, sets[b])
            ev_c = torch.cuda.Event()
            ev_c.record(stream)
            done_c[b] = ev_c
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_c)
                for h, d in zip(h_outs, d_outs):
                    h.copy_(d, non_blocking=True)
                last_out = torch.cuda.Event()
                last_out.record(s_out)
                done_out[b] = last_out
        stream.wait_event(last_out)
        ee.record(stream)
        torch.cuda.synchronize()
    t = all_max(pg, device, es.elapsed_time(ee) / 1e3)
    quant = cfg in (5, 6)
    v = (bytes_all * args.e2e_steps / t / 1e9) if quant else (flop_all * args.e2e_steps / t / 1e12)
    del h_ins, h_outs
    return {"value": round(v, 3), "unit": "GB/s" if quant else "TFLOP/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": args.e2e_steps,
            "api": "nvfp4_b200 public API (ctypes -> libnvfp4_b200.so)",
            "copies": "pinned host; two device buffer sets (GEMM configurations): step i+1's upload and "
                      "step i-1's read-back overlap step i's compute"}


def shape_run(args, device):
    """--shape / --group-shape: device-timed calls of one ad-hoc size (profiling runs)."""
    cfg, data, flop, nbytes, desc = shape_workload(args, device)
    flush = L2Flush(device)
    for _ in range(args.warmup):
        call(cfg, data)
    torch.cuda.synchronize()
    with ClockSampler(device.index) as clk, gc_paused():
        ms = timed_calls(cfg, data, args.steps, flush, torch.cuda.current_stream(device))
    us = statistics.mean(ms) * 1e3
    print(json.dumps({"metric": metric_name(cfg), "value": round(flop / us / 1e6, 2),
                      "unit": "TFLOP/s", "us_per_call": round(us, 2),
                      "hbm_gbs": round(nbytes / us / 1e3, 1), "config": desc,
                      "kernel_only": True, "clocks": clk.summary()}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=None, choices=[0, 1, 2, 3, 4, 5, 6, 7],
                    help="one configuration only (default: the suite, headline configuration 1). "
                         "0-4: BASELINE configurations; 5: device quantisation of config 1's "
                         "operands; 6: MoE dispatch of config 4's routing; 7: the MoE expert "
                         "layer around config 4")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="dual configurations with --config: N split over the ranks (strong) or "
                         "a full-N problem per rank (weak)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--sustain-s", type=float, default=2.0,
                    help="seconds of back-to-back kernel time in the headline's sustained figure")
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of CPU work for the configuration 5-7 baselines")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel-only", action="store_true",
                    help="device-timed calls only (no e2e, no CPU baseline): the profiling run")
    ap.add_argument("--suite", default=None, choices=["task"],
                    help="task: the reference's own task.yml benchmark shapes, one line per task")
    ap.add_argument("--shape", default=None,
                    help="M,N,K: kernel-only dual GEMM at this size (profiling runs)")
    ap.add_argument("--tokens", type=int, default=32768,
                    help="configuration 6: tokens to dispatch (32768 = configuration 4's routing)")
    ap.add_argument("--group-shape", default=None,
                    help="M1:M2:...,N,K: kernel-only grouped GEMM at these sizes (profiling runs)")
    args = ap.parse_args()
    assert args.warmup >= 3 or args.impl == "reference", "need >= 3 warm-up steps"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference_arm(args, 1 if args.config is None else args.config, rank, world)
    if args.suite == "task":
        return run_task_suite(args)

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if args.shape or args.group_shape:
        return shape_run(args, device)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
        pg = dist
    flush = L2Flush(device)
    full = not args.kernel_only

    def emit(line):
        if rank == 0:
            print(json.dumps(line), flush=True)

    ok = False
    try:
        if args.config is not None:
            emit(run_config(args.config, args, rank, world, device, pg, flush,
                            dual_scaling=args.scaling, e2e=full, sustained=full and args.config == 1,
                            cpu_baseline=full))
            ok = True
            return
        # the default suite: supporting lines first, the headline last.  On one
        # GPU a supporting line that fails prints its error and the suite goes
        # on to the headline (with several ranks every rank must take the same
        # collective steps, so a failure there ends the run)
        def extra(fn, what):
            if world > 1:
                return fn()
            try:
                return fn()
            except Exception as e:   # reported on the line, not swallowed
                emit({"metric": what, "error": f"{type(e).__name__}: {e}"[:400]})
                torch.cuda.synchronize()
        for c in ((2, 3, 4) if world == 1 else (2, 4)):
            line = extra(lambda: run_config(c, args, rank, world, device, pg, flush, e2e=full),
                         f"configuration {c}")
            if line is not None:
                emit(line)
        if world == 1:
            lines = extra(lambda: list(task_suite_lines(args, device)), "task-suite geomeans")
            for line in lines or []:
                emit(line)
        else:
            line = run_config(1, args, rank, world, device, pg, flush, dual_scaling="weak", e2e=False)
            line["note"] = "extra line: weak scaling (every rank a full-N problem); not the headline"
            emit(line)
        emit(run_config(1, args, rank, world, device, pg, flush, dual_scaling="strong", e2e=full,
                        sustained=full, cpu_baseline=full))
        ok = True
    finally:
        if pg:
            if ok:
                pg.barrier()
            pg.destroy_process_group()


def run_reference_arm(args, cfg, rank, world):
    """The reference's CPU path (its ref_kernel restated as the numpy oracle)
    on the host cores: rank 0 only; other ranks exit without work.  The
    dual / grouped configurations use cpu_oracle_protocol, the same protocol
    as the GPU arm's cpu_baseline."""
    if rank != 0:
        return
    if cfg in (5, 6):
        return run_reference_bytes_arm(args, cfg, world)
    if cfg == 7:
        return run_reference_layer_arm(args, world)
    r = cpu_oracle_in_child(cfg, args.steps, args.warmup)
    wl = f"dual_gemm_cfg{cfg}" if cfg in (0, 1, 2) else f"grouped_gemm_cfg{cfg}"
    print(json.dumps({
        "impl": "reference", "metric": metric_name(cfg), "value": r["value"], "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["ms_per_step"], "higher_is_better": True,
        "scaling": scaling_of(cfg, "strong"), "vs_baseline": None,
        "dtype": "fp32 (dequantised nvfp4)", "data": "synthetic: seeded N(0,1) quantised to NVFP4",
        "config": {"workload": wl, "sample": r["sample"]},
        "cpu_baseline": r,
        "e2e": {"value": r["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference_layer_arm(args, world, tokens: int = 128):
    """Configuration 7 on the host: the numpy oracle MoE layer on the first
    `tokens` tokens of configuration 4's routing (weights quantised on the
    host for the experts the sample touches)."""
    import types
    from nvfp4_b200 import inputs as I
    from nvfp4_b200.formats import quantize_nvfp4, swizzle_sf
    spec = I.GROUP_CONFIGS[4]
    k, n, experts = spec["k"], spec["n"], spec["experts"]
    g = torch.Generator().manual_seed(7000)
    ids = I.config4_expert_ids(tokens=32768)[:tokens]
    used = set(int(v) for v in ids)
    ws = []
    for e in range(experts):
        wf = torch.randn(n, k, generator=g)
        if e in used:
            p8, sf = quantize_nvfp4(wf)
            ws.append((p8.view(torch.float4_e2m1fn_x2).unsqueeze(-1), swizzle_sf(sf.unsqueeze(-1))))
        else:
            ws.append(None)
    w = types.SimpleNamespace(w=ws, n=n)
    x = torch.randn(tokens, k, generator=g)
    rw = torch.rand(tokens, generator=g)
    budget = max(1.0, 150.0 / max(1, args.steps))
    runs = [time_cpu_moe_layer((x, ids, rw, w), budget, tokens=tokens) for _ in range(args.steps)]
    v = statistics.mean(r["value"] for r in runs)
    print(json.dumps({
        "impl": "reference", "metric": metric_name(7), "value": round(v, 6), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(budget * 1e3, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32 (dequantised nvfp4)",
        "data": "synthetic: seeded N(0,1) fp32, configuration 4 routing",
        "config": {"workload": "moe_layer_cfg4", "sample_tokens": tokens, "budget_s": budget},
        "cpu_baseline": {**runs[0], "value": round(v, 6)},
        "e2e": {"value": round(v, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference_bytes_arm(args, cfg, world):
    """Configurations 5 and 6 on the host: the numpy oracle quantiser / dispatch
    (the reference has no such step; its inputs are built on the host) on a
    1024-row sample per step, GB/s counted as on the device."""
    from nvfp4_b200 import inputs as I
    g = torch.Generator().manual_seed(5)
    budget = max(0.5, 150.0 / max(1, args.steps))
    if cfg == 5:
        x = torch.randn(1024, I.DUAL_CONFIGS[1]["k"], generator=g)
        runs = [time_cpu_quant(x, budget) for _ in range(args.steps)]
        wl = "quantize_cfg1_operands"
    else:
        x = torch.randn(1024, I.GROUP_CONFIGS[4]["k"], generator=g)
        ids = I.config4_expert_ids()[:1024]
        runs = [time_cpu_moe(x, ids, 64, budget) for _ in range(args.steps)]
        wl = "moe_dispatch_cfg4"
    v = statistics.mean(r["value"] for r in runs)
    print(json.dumps({
        "impl": "reference", "metric": metric_name(cfg), "value": round(v, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(budget * 1e3, 1), "higher_is_better": True,
        "scaling": "weak" if cfg == 6 else "strong", "vs_baseline": None,
        "dtype": "fp32 -> e2m1 + e4m3 block16", "data": "synthetic: seeded N(0,1) fp32",
        "config": {"workload": wl, "sample_rows": 1024, "budget_s": budget},
        "cpu_baseline": {**runs[0], "value": round(v, 4)},
        "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    main()

"""Benchmark of the NVFP4 hot paths on B200; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]
    python bench.py --suite task     # the reference's task.yml shapes vs its published geomeans

Default workload: configuration 1 (dual GEMM M=8192 N=14336 K=4096, the
compute-bound SiLU-gated FFN shape).  A step is one dual-GEMM call over one
batch of synthetic inputs (seeded N(0,1) operands quantised to NVFP4).

* value: device time of the K timed calls (CUDA events on the launching
  stream, L2 flushed between calls outside the events), max over ranks;
  whole-job effective TFLOP/s = all ranks' FLOP / that time.
* e2e: the same metric through the public drop-in ``custom_kernel`` with the
  step's inputs copied from pinned host memory and the output copied back,
  inside the timed region.
* roofline: dominant kernel's achieved FLOP/s (or GB/s) against the NVFP4
  dense peak (4x the measured bf16 peak) or the measured HBM copy bandwidth.
* cpu_baseline / --impl reference: the CPU oracle (dequantise + fp32 matmul,
  the reference's ref_kernel restated) on a bounded sample of the workload.

Multi-GPU (torchrun, one rank per GPU): dual GEMM is sharded along N with the
per-rank shard fixed at the configuration's N (weak scaling, no collective on
the data path); grouped configurations assign experts by LPT (strong scaling).
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


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def dual_workload(cfg: int, rank: int, world: int, device):
    """Rank's dual GEMM: A replicated (same seed everywhere), B1/B2 = this
    rank's N-shard of a global N = N_cfg * world (weak scaling)."""
    from nvfp4_b200 import inputs as I
    spec = I.DUAL_CONFIGS[cfg]
    m, n, k = spec["m"], spec["n"], spec["k"]
    ga = torch.Generator().manual_seed(spec["seed"])
    a = torch.randn(m, k, generator=ga)
    gb = torch.Generator().manual_seed(spec["seed"] * 1000 + rank)
    if rank == 0:   # rank 0's shard is exactly the single-GPU configuration
        gb = torch.Generator().manual_seed(spec["seed"])
        torch.randn(m, k, generator=gb)
    b1 = torch.randn(n, k, generator=gb)
    b2 = torch.randn(n, k, generator=gb)
    data = I.dual_from_fp32(a, b1, b2, device=device)
    flop = 4.0 * m * n * k
    nbytes = m * k // 2 + 2 * n * k // 2 + (m + 2 * n) * k // 16 + 2 * m * n
    desc = dict(workload=f"dual_gemm_cfg{cfg}", m=m, n_per_rank=n, n_global=n * world, k=k, l=1)
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


def make_workload(cfg, rank, world, device, tokens=32768):
    if cfg == 5:
        return quant_workload(rank, world, device)
    if cfg == 6:
        return moe_workload(rank, world, device, tokens)
    if cfg == 7:
        return moe_layer_workload(rank, world, device, tokens)
    return dual_workload(cfg, rank, world, device) if cfg in (0, 1, 2) else \
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
def cpu_sample_step(cfg, data_cpu, rows, cols):
    """One bounded sample of the workload through the oracle: `rows` output
    rows x `cols` output columns (dual) or the same block of one group."""
    from oracle import nvfp4_oracle as O
    if cfg in (0, 1, 2):
        a, b1, b2, sfa, sfb1, sfb2 = data_cpu
        O.ref_dual(a[:rows], b1[:cols], b2[:cols], sfa[:rows], sfb1[:cols], sfb2[:cols])
        return 4.0 * rows * cols * a.shape[1] * 2
    a, b, sfa, sfb = data_cpu
    O.ref_group(a[:rows], b[:cols], sfa[:rows], sfb[:cols])
    return 2.0 * rows * cols * a.shape[1] * 2


def cpu_inputs(cfg, data):
    u8 = lambda t: t.detach().cpu().view(torch.uint8).numpy()[:, :, 0]
    if cfg in (0, 1, 2):
        return [u8(t) for t in data[:6]]
    abc, sfab, _, sizes = data
    i = max(range(len(sizes)), key=lambda j: sizes[j][0])   # largest group
    return [u8(abc[i][0]), u8(abc[i][1]), u8(sfab[i][0]), u8(sfab[i][1])]


def cpu_sample_shape(cfg, data_cpu):
    rows = min(data_cpu[0].shape[0], 2048)
    cols = min(data_cpu[1].shape[0], 2048)
    return rows, cols


def time_cpu(cfg, data_cpu, budget_s: float, min_reps: int = 1):
    rows, cols = cpu_sample_shape(cfg, data_cpu)
    cpu_sample_step(cfg, data_cpu, min(rows, 64), min(cols, 64))     # warm caches / threads
    flops, secs, reps = 0.0, 0.0, 0
    while reps < min_reps or secs < budget_s:
        t0 = time.perf_counter()
        flops += cpu_sample_step(cfg, data_cpu, rows, cols)
        secs += time.perf_counter() - t0
        reps += 1
    return flops / secs / 1e12, reps, rows, cols


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
            return float(v["dram_bytes_per_launch"])
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
    """The 15 inputs eval.py builds per benchmark (seed += 42 before each)."""
    from nvfp4_b200 import inputs as I
    out = []
    for i in range(TASK_INPUTS):
        seed = TASK_SEED + 42 * (i + 1)
        if kind == "dual":
            m, n, k = shape
            out.append(I.generate_dual_input(m, n, k, 1, seed, device=device))
        else:
            ms, n, k = shape
            out.append(I.generate_group_input(ms, [n] * len(ms), [k] * len(ms), len(ms), seed,
                                              device=device))
    return out


def task_flop(kind, shape):
    if kind == "dual":
        m, n, k = shape
        return 4.0 * m * n * k
    ms, n, k = shape
    return sum(2.0 * m * n * k for m in ms)


def run_task_suite(args):
    """Per reference benchmark shape: L2 flushed, then the 15 distinct inputs
    run back to back between two CUDA events; the per-call mean of `steps`
    such batches.  One JSON line per task: geomean us against the published
    geomean of the reference's best submission."""
    from nvfp4_b200 import _lib
    from nvfp4_b200.dual_gemm import custom_kernel as dual_kernel
    from nvfp4_b200.group_gemm import custom_kernel as group_kernel
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    for kind, shapes, fn in (("dual", TASK_DUAL, dual_kernel), ("group", TASK_GROUP, group_kernel)):
        per_shape, per_shape_std, tflops = [], [], []
        with ClockSampler(0, period_s=0.02) as clk:
            for shape in shapes:
                datas = task_inputs(kind, shape, device)
                for _ in range(args.warmup):
                    for d in datas:
                        fn(d)
                torch.cuda.synchronize()
                times = []
                with gc_paused():
                    for _ in range(args.steps):
                        flush.zero_()
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
        print(json.dumps({
            "metric": f"runtime geomean over the reference's task.yml benchmark shapes "
                      f"({'dual' if kind == 'dual' else 'grouped'} GEMM)",
            "value": round(geo, 3), "unit": "us", "higher_is_better": False,
            "vs_baseline": round(geo / pub, 4), "reference_published_us": pub,
            "per_shape_us": per_shape, "per_shape_std_us": per_shape_std, "per_shape_tflops": tflops,
            "shapes": [list(s) if kind == "dual" else [s[0], s[1], s[2]] for s in shapes],
            "method": f"{TASK_INPUTS} distinct seeded inputs per shape (reference generator "
                      f"distributions), L2 flushed before each batch, mean per call over "
                      f"{args.steps} batches, custom_kernel API",
            "n_gpus": 1, "clocks": clk.summary()}), flush=True)


def metric_name(cfg):
    if cfg == 5:
        return "NVFP4 quantisation bandwidth (fp32 -> e2m1 + e4m3 scales)"
    if cfg == 6:
        return "MoE dispatch bandwidth (route + fp32 -> NVFP4 per-expert operands)"
    if cfg == 7:
        return "NVFP4 effective TFLOPS (MoE expert layer: dispatch + grouped GEMM + combine)"
    return "NVFP4 effective TFLOPS (dual GEMM)" if cfg in (0, 1, 2) else \
        "NVFP4 effective TFLOPS (grouped GEMM)"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=1, choices=[0, 1, 2, 3, 4, 5, 6, 7],
                    help="0-4: BASELINE configurations; 5: device quantisation of config 1's "
                         "operands; 6: MoE dispatch of config 4's routing; 7: the MoE expert "
                         "layer around config 4")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-budget", type=float, default=12.0)
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
    if args.shape or args.group_shape:
        args.kernel_only = True
    assert args.warmup >= 3 or args.impl == "reference", "need >= 3 warm-up steps"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = args.config

    if args.impl == "reference":
        return run_reference_arm(args, cfg, rank, world)
    if args.suite == "task":
        return run_task_suite(args)

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
        pg = dist

    from nvfp4_b200 import _lib
    if args.shape or args.group_shape:
        cfg, data, flop, nbytes, desc = shape_workload(args, device)
    else:
        data, flop, nbytes, desc = make_workload(cfg, rank, world, device, args.tokens)
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)

    for _ in range(args.warmup):
        call(cfg, data)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clk, gc_paused():
        if pg:                                  # ranks start the timed loop together
            pg.barrier()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed")
        for i in range(args.steps):
            flush.zero_()                       # evict L2 between calls (outside the events)
            starts[i].record(stream)
            call(cfg, data)
            ends[i].record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    if pg:
        pg.barrier()
    status = _lib.device_status()
    assert status == 0, f"device status {status:#x}"
    per_call_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    t_total = torch.tensor([sum(per_call_ms)], dtype=torch.float64, device=device)
    flop_t = torch.tensor([flop], dtype=torch.float64, device=device)
    if pg:
        pg.all_reduce(t_total, op=pg.ReduceOp.MAX)
        pg.all_reduce(flop_t, op=pg.ReduceOp.SUM)
    t_max_s = t_total.item() / 1e3
    total_flop = flop_t.item() * args.steps
    ms_per_step = t_max_s * 1e3 / args.steps
    if cfg in (5, 6):   # bytes-moved metric for the quantiser and the dispatch
        bytes_t = torch.tensor([float(nbytes)], dtype=torch.float64, device=device)
        if pg:
            pg.all_reduce(bytes_t, op=pg.ReduceOp.SUM)
        value = bytes_t.item() * args.steps / t_max_s / 1e9
    else:
        value = total_flop / t_max_s / 1e12

    if args.kernel_only:
        if rank == 0:
            print(json.dumps({"metric": metric_name(cfg), "value": round(value, 2),
                              "unit": "GB/s" if cfg in (5, 6) else "TFLOP/s",
                              "us_per_call": round(ms_per_step * 1e3, 2),
                              "config": desc, "kernel_only": True, "clocks": clk.summary()}),
                  flush=True)
        if pg:
            pg.destroy_process_group()
        return

    # ---- e2e through the public API with pinned host buffers.  Every step
    # uploads its inputs and reads its result back; the upload of step i+1
    # runs on its own stream while step i's result is read back on another
    # (PCIe is full duplex), and a step's compute waits for its inputs and
    # for the previous read-back (the outputs are reused).
    ins, outs = device_tensors(cfg, data)
    h_ins = [t.detach().cpu().pin_memory() for t in ins]
    h_outs = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in outs]
    h2d, d2h = nbytes_of(ins), nbytes_of(outs)
    call(cfg, data)
    torch.cuda.synchronize()
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    with gc_paused():
        es.record(stream)
        s_in.wait_event(es)
        s_out.wait_event(es)
        done_out = None
        for _ in range(args.e2e_steps):
            with torch.cuda.stream(s_in):              # inputs are free once the last compute ended
                s_in.wait_stream(stream)
                for d, h in zip(ins, h_ins):
                    d.copy_(h, non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
            stream.wait_event(ev_in)
            if done_out is not None:
                stream.wait_event(done_out)
            call(cfg, data)
            ev_c = torch.cuda.Event()
            ev_c.record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_c)
                for h, d in zip(h_outs, outs):
                    h.copy_(d, non_blocking=True)
                done_out = torch.cuda.Event()
                done_out.record(s_out)
        stream.wait_event(done_out)
        ee.record(stream)
        torch.cuda.synchronize()
    e2e_t = torch.tensor([es.elapsed_time(ee) / 1e3], dtype=torch.float64, device=device)
    if pg:
        pg.all_reduce(e2e_t, op=pg.ReduceOp.MAX)
    quant = cfg in (5, 6)
    if quant:   # bytes-moved metric for the quantiser and the dispatch
        e2e_value = bytes_t.item() * args.e2e_steps / e2e_t.item() / 1e9
    else:
        e2e_value = flop_t.item() * args.e2e_steps / e2e_t.item() / 1e12
    unit = "GB/s" if quant else "TFLOP/s"

    # ---- roofline of the dominant kernel (the GEMM kernel is the only launch)
    hbm_peak, bf16_peak, peak_kind = load_peaks()
    nvfp4_peak = 4.0 * bf16_peak
    avg_launch_s = statistics.mean(per_call_ms) / 1e3
    hbm_bound = cfg in (2, 5, 6)
    traffic = load_traffic(desc["workload"])
    if hbm_bound:
        ach = nbytes / avg_launch_s / 1e9
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(ach / hbm_peak, 4)}
    else:
        ach = flop / avg_launch_s / 1e12
        roof = {"bound": "tensor", "achieved": round(ach, 1), "peak": nvfp4_peak,
                "unit": "TFLOP/s", "frac": round(ach / nvfp4_peak, 4)}
    roof["traffic"] = traffic
    roof["algorithmic_bytes"] = nbytes
    roof["peak_source"] = (f"{peak_kind}: NVFP4 dense = 4 x bf16 {bf16_peak} TFLOP/s"
                           if not hbm_bound else f"{peak_kind}: HBM copy {hbm_peak} GB/s")

    result = {
        "metric": metric_name(cfg), "value": round(value, 2), "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5), "us_per_call": round(ms_per_step * 1e3, 2),
        "us_per_call_std": round(statistics.stdev(per_call_ms) * 1e3, 2) if len(per_call_ms) > 1 else 0.0,
        "higher_is_better": True, "scaling": "weak" if cfg in (0, 1, 2, 6, 7) else "strong",
        "vs_baseline": None,
        "dtype": ("int32 routing + fp32 -> e2m1 + e4m3 block16" if cfg == 6 else
                  "fp32 -> e2m1 + e4m3 block16") if quant
        else "fp32 tokens -> nvfp4 x nvfp4 -> fp32 acc -> fp16 -> fp32 combine" if cfg == 7
        else "nvfp4(e2m1+e4m3 block16) x nvfp4 -> fp32 acc -> fp16",
        "data": "synthetic: seeded N(0,1) fp32 quantised to NVFP4",
        "config": {**desc, "parallelism": f"{'n-shard' if cfg in (0, 1, 2) else 'token-shard' if cfg in (6, 7) else 'expert-lpt'}{world}",
                   "l2": f"flushed ({L2_FLUSH_BYTES >> 20} MiB write) between timed calls"},
        "e2e": {"value": round(e2e_value, 3), "unit": unit, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": args.e2e_steps,
                "api": "nvfp4_b200 public API (ctypes -> libnvfp4_b200.so)",
                "copies": "pinned host; step i+1's upload overlaps step i's read-back"},
        "roofline": roof,
        "gpu_launches": args.steps * (4 if cfg == 6 else 6 if cfg == 7 else len(data) if quant else 1),
        "clocks": clk.summary(),
    }

    if rank == 0 and world == 1 and not args.no_cpu_baseline and cfg == 6:
        result["cpu_baseline"] = time_cpu_moe(data[0], data[1], data[2], args.cpu_budget)
    elif rank == 0 and world == 1 and not args.no_cpu_baseline and cfg == 7:
        result["cpu_baseline"] = time_cpu_moe_layer(data, args.cpu_budget)
    elif rank == 0 and world == 1 and not args.no_cpu_baseline and quant:
        result["cpu_baseline"] = time_cpu_quant(data[0][0], args.cpu_budget)
    elif rank == 0 and world == 1 and not args.no_cpu_baseline:
        dc = cpu_inputs(cfg, data)
        torch.set_num_threads(cpu_cores())
        v, reps, rows, cols = time_cpu(cfg, dc, args.cpu_budget)
        result["cpu_baseline"] = {
            "value": round(v, 5), "unit": "TFLOP/s", "cores": cpu_cores(), "kind": "port",
            "sample": f"oracle ref ({'dual' if cfg < 3 else 'group'}) on a {rows}x{cols} output "
                      f"block x K={dc[0].shape[1] * 2}, {reps} reps (~{args.cpu_budget:.0f} s)"}
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_reference_arm(args, cfg, rank, world):
    """The reference's CPU path (its ref_kernel restated as the numpy oracle)
    on the host cores: rank 0 only; other ranks exit without work."""
    if rank != 0:
        return
    from nvfp4_b200 import inputs as I
    if cfg in (5, 6):
        return run_reference_bytes_arm(args, cfg, world)
    if cfg == 7:
        return run_reference_layer_arm(args, world)
    if cfg in (0, 1, 2):
        spec = I.DUAL_CONFIGS[cfg]
        g = torch.Generator().manual_seed(spec["seed"])
        rows, cols = min(spec["m"], 2048), min(spec["n"], 2048)
        k = spec["k"]
        a = torch.randn(spec["m"], k, generator=g)[:rows]
        b1 = torch.randn(spec["n"], k, generator=g)[:cols]
        b2 = torch.randn(spec["n"], k, generator=g)[:cols]
        d = I.dual_from_fp32(a, b1, b2, device="cpu")
        dc = [t.view(torch.uint8).numpy()[:, :, 0] for t in d[:6]]
        wl = f"dual_gemm_cfg{cfg}"
    else:
        d = I.group_config_input(cfg, device="cpu") if cfg == 3 else None
        if d is None:   # config 4: largest expert only
            ms = I.config4_m_sizes()
            spec = I.GROUP_CONFIGS[4]
            gen = torch.Generator().manual_seed(7)
            mbig = min(max(ms), 2048)
            d = I.group_from_fp32([(torch.randn(mbig, spec["k"], generator=gen),
                                    torch.randn(spec["n"], spec["k"], generator=gen))], device="cpu")
        dc = cpu_inputs(cfg, d)
        wl = f"grouped_gemm_cfg{cfg}"
    torch.set_num_threads(cpu_cores())
    rows, cols = cpu_sample_shape(cfg, dc)
    for _ in range(args.warmup):
        cpu_sample_step(cfg, dc, rows, cols)
    budget = max(0.0, 150.0 / max(1, args.steps))
    flops, secs = 0.0, 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        flops += cpu_sample_step(cfg, dc, rows, cols)
        secs += time.perf_counter() - t0
    v = flops / secs / 1e12
    sample = (f"numpy oracle (dequantise + fp32 matmul) on a {rows}x{cols} output block "
              f"x K={dc[0].shape[1] * 2} per step")
    print(json.dumps({
        "impl": "reference", "metric": metric_name(cfg), "value": round(v, 5), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(secs * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "weak" if cfg in (0, 1, 2) else "strong", "vs_baseline": None,
        "dtype": "fp32 (dequantised nvfp4)", "data": "synthetic: seeded N(0,1) quantised to NVFP4",
        "config": {"workload": wl, "sample_rows": rows, "sample_cols": cols, "budget_s": budget},
        "cpu_baseline": {"value": round(v, 5), "unit": "TFLOP/s", "cores": cpu_cores(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(v, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
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

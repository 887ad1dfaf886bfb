"""CPU: host-side logic that needs no GPU: the grouped plan cache, the
multi-GPU partitioners, and the multi-rank timing reduction over gloo."""
import os
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nvfp4_b200 import inputs as I
from nvfp4_b200.group_gemm import _Plan
from nvfp4_b200.shard import imbalance, lpt_assign, n_shard


def _groups(ms, k=256, n=128, seed=0):
    g = torch.Generator().manual_seed(seed)
    return I.group_from_fp32([(torch.randn(m, k, generator=g), torch.randn(n, k, generator=g))
                              for m in ms], device="cpu")


def test_plan_matches_same_objects_only():
    abc, _, perm, sizes = _groups([64, 0, 130])
    plan = _Plan(abc, perm, sizes, table=None, device=None)
    assert plan.matches(abc, perm, sizes)
    assert plan.matches(list(abc), list(perm), list(sizes))           # new lists, same tensors
    swapped = list(abc)
    swapped[2] = (abc[2][0].clone(), abc[2][1], abc[2][2])
    assert not plan.matches(swapped, perm, sizes)                      # a replaced tensor
    assert not plan.matches(abc[:2], perm[:2], sizes[:2])              # a different count
    sizes2 = list(sizes)
    sizes2[0] = (64, 128, 256, 2)
    assert not plan.matches(abc, perm, sizes2)                         # a different size tuple


def test_plan_detects_storage_swap():
    abc, _, perm, sizes = _groups([64, 32])
    plan = _Plan(abc, perm, sizes, table=None, device=None)
    a = abc[0][0]
    a.set_(a.clone())                                                  # same object, new storage
    assert not plan.matches(abc, perm, sizes)


def test_plan_holds_no_strong_references():
    import gc
    import weakref
    abc, _, perm, sizes = _groups([64])
    plan = _Plan(abc, perm, sizes, table=None, device=None)
    probe = weakref.ref(abc[0][0])
    del abc, perm, sizes
    gc.collect()
    assert probe() is None
    assert plan.refs[0][0]() is None


def _dual_tensors(m=128, n=128, k=256):
    d = I.generate_dual_input(m, n, k, 1, seed=5, device="cpu")
    return (d[0], d[1], d[2], d[6], d[7], d[8], d[9])


def test_dual_plan_matches_same_objects_only():
    from nvfp4_b200.dual_gemm import _Plan as DualPlan
    ts = _dual_tensors()
    plan = DualPlan(ts, (128, 128, 256, 1), device=None)
    assert plan.matches(ts)
    assert plan.matches(list(ts))                                       # same tensors, new container
    assert not plan.matches(ts[:6] + (ts[6].clone(),))                  # a replaced output
    c = ts[6]
    c.set_(c.clone())                                                   # same object, new storage
    assert not plan.matches(ts)


def test_dual_plan_detects_restride_and_holds_no_references():
    import gc
    import weakref
    from nvfp4_b200.dual_gemm import _Plan as DualPlan
    ts = _dual_tensors()
    plan = DualPlan(ts, (128, 128, 256, 1), device=None)
    a = ts[0]
    a.as_strided_(a.shape, (a.stride(0), 1, a.stride(0) * a.shape[0] + 64))   # same storage, new strides
    assert not plan.matches(ts)
    probe = weakref.ref(ts[1])
    del ts, a
    gc.collect()
    assert probe() is None


@pytest.mark.parametrize("n,world", [(14336, 1), (14336, 2), (14336, 8), (7168, 8), (1000, 3)])
def test_n_shard_covers_and_aligns(n, world):
    spans = [n_shard(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a, b), (c, _) in zip(spans, spans[1:]):
        assert b == c
    for a, b in spans:
        assert a % 128 == 0
        assert b - a >= 0
    with pytest.raises(ValueError):
        n_shard(n, world, world)


def test_lpt_assignment_config4():
    ms = I.config4_m_sizes()
    costs = [float(m) for m in ms]
    for world in (1, 2, 4, 8):
        bins = lpt_assign(costs, world)
        assert sorted(i for b in bins for i in b) == list(range(len(ms)))
        # LPT guarantee: makespan <= 4/3 OPT; OPT >= max(mean, max item)
        opt_lb = max(sum(costs) / world, max(costs))
        assert max(sum(costs[i] for i in b) for b in bins) <= 4 / 3 * opt_lb + 1e-9
    assert imbalance(costs, lpt_assign(costs, 1)) == 1.0


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    # each rank's device time and FLOP, reduced the way bench.py reduces them
    t = torch.tensor([1.0 + rank], dtype=torch.float64)
    f = torch.tensor([10.0 * (rank + 1)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(f, op=dist.ReduceOp.SUM)
    if rank == 0:
        out.put((t.item(), f.item()))
    dist.barrier()
    dist.destroy_process_group()


def test_multi_rank_reduction_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    t, f = q.get(timeout=5)
    assert t == 2.0 and f == 30.0          # max time over ranks, summed work


def _failing_rank_main(rank, world, port, out):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    if rank == 1:
        # a step fails on this rank: it leaves between steps, before the barrier
        out.put((rank, "raised"))
        dist.destroy_process_group()
        return
    try:
        dist.monitored_barrier(timeout=datetime.timedelta(seconds=3))
        out.put((rank, "barrier passed"))
    except RuntimeError as e:
        out.put((rank, "error: " + str(e).splitlines()[0][:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_rank_failure_surfaces_as_error_not_hang():
    """A rank that fails between steps (and leaves) is reported to the others
    by the next barrier with a timeout, as an exception within seconds."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 31500 + os.getpid() % 1000
    procs = [ctx.Process(target=_failing_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    assert all(not p.is_alive() for p in procs), "a rank hung"
    got = dict(q.get(timeout=5) for _ in range(2))
    assert got[1] == "raised"
    assert got[0].startswith("error"), got[0]


def test_bench_timed_region_pauses_gc():
    import gc

    import bench
    assert gc.isenabled()
    with bench.gc_paused():
        assert not gc.isenabled()
    assert gc.isenabled()
    with pytest.raises(RuntimeError):
        with bench.gc_paused():
            raise RuntimeError("the collector comes back on errors too")
    assert gc.isenabled()


def test_bench_clock_sampler_reports_missing_nvml_instead_of_failing():
    # without a GPU driver the child sampler cannot start; the bench records
    # why and carries on with no clock samples
    import bench
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the sampler starts")
    with bench.ClockSampler(0, period_s=0.01) as clk:
        pass
    out = clk.summary()
    assert out["sm_mhz"] is None and out["error"]


def test_bench_strong_shards_concatenate_to_the_single_gpu_problem():
    """bench.py's strong-scaled dual workload: each rank's B1/B2 rows and
    permuted scale atoms are its contiguous 128-row slice of the single-GPU
    configuration's operands, and A is replicated."""
    import bench
    one, flop1, _, _ = bench.dual_workload(0, 0, 1, "cpu", "strong")
    u8 = lambda t: t.view(torch.uint8)
    for world in (2, 4):
        flops = 0.0
        for rank in range(world):
            d, flop, _, desc = bench.dual_workload(0, rank, world, "cpu", "strong")
            n0, n1 = desc["n_rows_this_rank"]
            assert desc["n_global"] == 512 and n1 - n0 == desc["n_this_rank"]
            assert torch.equal(u8(d[0]), u8(one[0]))
            for i in (1, 2):
                assert torch.equal(u8(d[i]), u8(one[i])[n0:n1])
                assert torch.equal(u8(d[i + 6]), u8(one[i + 6])[:, :, n0 // 128:n1 // 128])
            flops += flop
        assert flops == flop1


def test_bench_reference_arm_runs_on_the_host():
    """--impl reference: the oracle protocol in a spawned process, one JSON
    line with the reference-arm keys (no GPU needed)."""
    import json
    import subprocess
    import sys
    root = Path(__file__).resolve().parent.parent
    out = subprocess.run([sys.executable, str(root / "bench.py"), "--impl", "reference",
                          "--config", "0", "--steps", "2", "--warmup", "1"],
                         capture_output=True, text=True, timeout=600, cwd=root)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["steps"] == 2
    assert cb["full_config0"]["value"] > 0 and "no extrapolation" in cb["full_config0"]["sample"]

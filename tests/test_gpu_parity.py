"""GPU parity: the CUDA kernels (through the C ABI via the drop-in
``custom_kernel``s) against the CPU oracle on the same seeded inputs, at the
reference's task shapes (nvfp4_dual_gemm/task.yml:46-56,
nvfp4_group_gemm/task.yml:47-57), the benchmark configurations, and edge
cases.  Tolerance: rtol = atol = 1e-2 on fp16 outputs (fp32 accumulation),
NaN/inf-aware as in nvfp4_group_gemm/utils.py:31-86."""
import os

import numpy as np
import pytest
import torch

from nvfp4_b200 import _lib
from nvfp4_b200 import build as B
from nvfp4_b200 import dual_gemm as D
from nvfp4_b200 import group_gemm as G
from nvfp4_b200 import inputs as I
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2

DUAL_TASK_TESTS = [  # nvfp4_dual_gemm/task.yml:46-56 (m, n, k, l)
    (1536, 512, 7168, 1), (256, 512, 256, 1), (3072, 1024, 1536, 1), (7168, 1024, 256, 1),
    (7168, 2304, 2048, 1), (4608, 384, 7168, 1), (7168, 384, 2304, 1), (512, 768, 7168, 1),
    (4096, 768, 512, 1),
]
DUAL_TASK_BENCH = [(256, 4096, 7168, 1), (512, 4096, 7168, 1), (256, 3072, 4096, 1),
                   (512, 3072, 7168, 1)]  # nvfp4_dual_gemm/task.yml:58-62
GROUP_TASK_TESTS = [  # nvfp4_group_gemm/task.yml:47-57
    ([96, 128], [128, 256], [256, 512]), ([256, 72], [512, 384], [256, 256]),
    ([128, 128], [128, 256], [512, 256]), ([80, 128, 256], [384, 256, 128], [256, 512, 256]),
    ([64, 72, 96], [128, 384, 512], [512, 512, 256]), ([64, 256, 128], [768, 128, 256], [512, 256, 512]),
    ([128, 128, 64], [256, 512, 512], [768, 256, 768]),
    ([128] * 4, [128] * 4, [512, 256, 512, 256]), ([40, 56, 384, 512], [512, 384, 256, 128], [256] * 4),
    ([512, 384, 256, 128], [256] * 4, [512, 768, 512, 768]),
]


@pytest.fixture(scope="module", autouse=True)
def _lib_ready(cuda_device):
    B.build()
    _lib.load()
    assert _lib.device_status() == 0


def _np(t):
    return t.detach().cpu().view(torch.uint8).numpy() if t.dtype != torch.float16 \
        else t.detach().cpu().numpy()


def oracle_dual(data):
    a, b1, b2, sfa, sfb1, sfb2 = (_np(t) for t in data[:6])
    return O.ref_dual_batched(a, b1, b2, sfa, sfb1, sfb2)


def oracle_group(data):
    abc, sfab, _, _ = data
    return O.ref_grouped([(_np(a), _np(b), _np(sa), _np(sb)) for (a, b, _), (sa, sb) in zip(abc, sfab)])


def assert_close(got, want, what):
    bad, idx = O.allclose_report(got, want, RTOL, ATOL)
    if bad:
        i = tuple(idx[0])
        pytest.fail(f"{what}: {bad} mismatches of {want.size}; first {i}: got {got[i]} want {want[i]}")


def run_dual(data):
    out = D.custom_kernel(data)
    assert _lib.device_status() == 0
    return out.cpu().numpy()


@pytest.mark.parametrize("kernel", ["auto", "pair64", "pair128", "single"])
@pytest.mark.parametrize("m,n,k,l", DUAL_TASK_TESTS)
def test_dual_task_shapes(m, n, k, l, kernel, monkeypatch):
    if kernel == "single":
        monkeypatch.setenv("NVFP4_DUAL_KERNEL", "single")
    elif kernel != "auto":
        monkeypatch.setenv("NVFP4_DUAL_KERNEL", "pair")
        monkeypatch.setenv("NVFP4_DUAL_BN", kernel[4:])
    data = I.generate_dual_input(m, n, k, l, seed=1111, device="cuda")
    assert_close(run_dual(data), oracle_dual(data), f"dual {kernel} {m}x{n}x{k}")


@pytest.mark.parametrize("bn", ["64", "128"])
@pytest.mark.parametrize("m,n,k,l", DUAL_TASK_TESTS + DUAL_TASK_BENCH + [
    (256, 128, 256, 1), (384, 640, 1024, 2), (200, 264, 512, 1), (130, 72, 768, 1), (1, 8, 256, 1),
    (1000, 1000, 2048, 1), (100, 256, 1024, 3), (256, 4160, 2048, 1), (128, 1024, 2048, 1)])
def test_dual_pair_kernel_shapes(m, n, k, l, bn, monkeypatch):
    """CTA-pair kernel (each CTA loads half of the tile's B1 and B2 rows, the
    MMA thread copies the scale atoms into TMEM): task shapes, M and N ragged
    against the 256-row pair blocks and the tile width (the second CTA's B
    rows wholly past N at N = 8), batched L, and 64-wide tiles in the upper
    half of a 128-row scale block."""
    monkeypatch.setenv("NVFP4_DUAL_KERNEL", "pair")
    monkeypatch.setenv("NVFP4_DUAL_BN", bn)
    data = I.generate_dual_input(m, n, k, l, seed=5 + m + n + k, device="cuda")
    assert_close(run_dual(data), oracle_dual(data), f"dual pair{bn} {m}x{n}x{k}x{l}")


@pytest.mark.parametrize("bn", ["64", "128"])
@pytest.mark.parametrize("m,n,k,l", DUAL_TASK_BENCH + [(200, 264, 512, 1), (384, 640, 1024, 2)])
def test_dual_both_tile_widths(m, n, k, l, bn, monkeypatch):
    monkeypatch.setenv("NVFP4_DUAL_BN", bn)
    data = I.generate_dual_input(m, n, k, l, seed=42 + m, device="cuda")
    assert_close(run_dual(data), oracle_dual(data), f"dual bn={bn} {m}x{n}x{k}x{l}")


@pytest.mark.parametrize("m,n,k,l", DUAL_TASK_BENCH)
def test_dual_benchmark_shapes_automatic_choice(m, n, k, l):
    """The timed benchmark shapes with no knob set: the automatic kernel
    choice (the CTA pair: 64-wide tiles for the 256-row shapes, 128-wide for
    the 512-row ones)."""
    data = I.generate_dual_input(m, n, k, l, seed=2024 + m, device="cuda")
    assert_close(run_dual(data), oracle_dual(data), f"dual automatic {m}x{n}x{k}")


def test_dual_config2_full_output():
    """Configuration 2 (M=128, N=7168, K=16384; cluster split-K) in full:
    every one of the 128 x 7168 outputs against the oracle."""
    data = I.dual_config_input(2, device="cuda")
    assert_close(run_dual(data), oracle_dual(data), "dual cfg2 full output")


@pytest.mark.parametrize("splits", [2, 3, 5, 16])
@pytest.mark.parametrize("m,n,k,l", [(256, 512, 4096, 1), (200, 264, 2048, 1), (384, 640, 1024, 2),
                                     (128, 7168, 4096, 1)])
def test_dual_split_k(m, n, k, l, splits, monkeypatch):
    """Split-K reduction (partials in workspace, last split applies SiLU) at
    forced split counts, ragged M/N and batched L."""
    monkeypatch.setenv("NVFP4_DUAL_SPLITS", str(splits))
    data = I.generate_dual_input(m, n, k, l, seed=splits * 31 + m, device="cuda")
    assert_close(run_dual(data), oracle_dual(data), f"dual splitK={splits} {m}x{n}x{k}x{l}")


@pytest.mark.parametrize("cluster", ["2", "4"])
@pytest.mark.parametrize("m,n,k,l", [(256, 512, 4096, 1), (200, 264, 2048, 1), (384, 640, 1024, 2),
                                     (128, 7168, 4096, 1), (256, 3072, 4096, 1), (1, 8, 2048, 1)])
def test_dual_cluster_split_k(m, n, k, l, cluster, monkeypatch):
    """Cluster split-K (partials exchanged between the CTAs of a cluster, each
    CTA reducing and storing its own column slice) at 2 and 4 splits, ragged
    M/N, batched L; shapes where 4 splits do not fit fall back to 2."""
    monkeypatch.setenv("NVFP4_DUAL_CLUSTER", cluster)
    data = I.generate_dual_input(m, n, k, l, seed=int(cluster) * 17 + m, device="cuda")
    assert_close(run_dual(data), oracle_dual(data), f"dual cluster={cluster} {m}x{n}x{k}x{l}")


def test_dual_cluster_split_k_deterministic(monkeypatch):
    monkeypatch.setenv("NVFP4_DUAL_CLUSTER", "4")
    data = I.generate_dual_input(256, 1024, 4096, 1, seed=6, device="cuda")
    outs = [D.custom_kernel(data).clone() for _ in range(3)]
    assert all(torch.equal(outs[0], o) for o in outs[1:])


def test_dual_split_k_deterministic(monkeypatch):
    monkeypatch.setenv("NVFP4_DUAL_SPLITS", "4")
    data = I.generate_dual_input(256, 1024, 4096, 1, seed=5, device="cuda")
    outs = [D.custom_kernel(data).clone() for _ in range(3)]
    assert all(torch.equal(outs[0], o) for o in outs[1:])


def test_dual_config0_normal_inputs():
    data = I.dual_config_input(0, device="cuda")
    assert_close(run_dual(data), oracle_dual(data), "dual config 0")


def test_dual_small_m_and_ragged():
    for (m, n, k) in [(1, 8, 256), (7, 136, 256), (130, 72, 768), (128, 7168, 2048)]:
        data = I.generate_dual_input(m, n, k, 1, seed=m + n, device="cuda")
        assert_close(run_dual(data), oracle_dual(data), f"dual {m}x{n}x{k}")


def test_dual_deterministic():
    data = I.generate_dual_input(512, 1024, 2048, 1, seed=3, device="cuda")
    r1 = D.custom_kernel(data).clone()
    r2 = D.custom_kernel(data).clone()
    assert torch.equal(r1, r2)


def _rows(t, rows):
    """Row subset of a packed/scale tensor (index a uint8 view: CUDA indexing
    is not implemented for the fp4 dtype)."""
    return t.view(torch.uint8)[rows.to(t.device)]


def _sample_rows_check(data, rows):
    a, b1, b2, sfa, sfb1, sfb2 = data[:6]
    sub = lambda t: _np(_rows(t, rows))[:, :, 0]
    want = O.ref_dual(sub(a), _np(b1)[:, :, 0], _np(b2)[:, :, 0], sub(sfa),
                      _np(sfb1)[:, :, 0], _np(sfb2)[:, :, 0])
    return want


@pytest.mark.parametrize("cfg", [1, 2])
def test_dual_full_size_configs_sampled_rows(cfg):
    """Full BASELINE sizes: every row of a seeded sample of 96 rows (all
    columns) against the oracle, and no NaN anywhere in the output."""
    data = I.dual_config_input(cfg, device="cuda")
    out = D.custom_kernel(data)
    assert _lib.device_status() == 0
    m = out.shape[0]
    g = torch.Generator().manual_seed(cfg)
    rows = torch.randperm(m, generator=g)[:96].sort().values
    want = _sample_rows_check(data, rows)
    assert_close(out[rows.to(out.device), :, 0].cpu().numpy(), want, f"dual cfg{cfg} sampled rows")
    # fp16 overflow to +-inf is legitimate at large K (the oracle agrees on
    # the sampled rows); NaN never is
    assert not torch.isnan(out).any()


@pytest.mark.parametrize("bn", ["128", "256"])
@pytest.mark.parametrize("case", range(len(GROUP_TASK_TESTS)))
def test_group_task_shapes(case, bn, monkeypatch):
    monkeypatch.setenv("NVFP4_GROUPED_BN", bn)
    m, n, k = GROUP_TASK_TESTS[case]
    data = I.generate_group_input(m, n, k, len(m), seed=1111, device="cuda")
    outs = G.custom_kernel(data)
    assert _lib.device_status() == 0
    for i, (got, want) in enumerate(zip(outs, oracle_group(data))):
        assert_close(got.cpu().numpy(), want, f"group case {case} g{i}")


GROUP_TASK_BENCH = [  # nvfp4_group_gemm/task.yml:59-63 (m per group, n, k)
    ([80, 176, 128, 72, 64, 248, 96, 160], 4096, 7168), ([40, 76, 168, 72, 164, 148, 196, 160], 7168, 2048),
    ([192, 320], 3072, 4096), ([128, 384], 4096, 1536),
]


@pytest.mark.parametrize("bn", ["128", "auto"])
@pytest.mark.parametrize("case", range(len(GROUP_TASK_BENCH)))
def test_group_benchmark_shapes(case, bn, monkeypatch):
    if bn != "auto":
        monkeypatch.setenv("NVFP4_GROUPED_BN", bn)
    ms, n, k = GROUP_TASK_BENCH[case]
    data = I.generate_group_input(ms, [n] * len(ms), [k] * len(ms), len(ms), seed=1111, device="cuda")
    outs = G.custom_kernel(data)
    assert _lib.device_status() == 0
    # the widest group in full, sampled rows of the others
    abc, sfab, _, sizes = data
    wide = max(range(len(ms)), key=lambda i: ms[i])
    for i in range(len(ms)):
        (a, b, _), (sa, sb) = abc[i], sfab[i]
        rows = torch.arange(0, ms[i], 1 if i == wide else 13)
        want = O.ref_group(_np(_rows(a, rows))[:, :, 0], _np(b)[:, :, 0],
                           _np(_rows(sa, rows))[:, :, 0], _np(sb)[:, :, 0])
        assert_close(outs[i][rows.to(outs[i].device), :, 0].cpu().numpy(), want,
                     f"benchmark group case {case} g{i}")


@pytest.mark.parametrize("case", range(len(GROUP_TASK_TESTS)))
def test_group_pair_task_shapes(case, monkeypatch):
    """CTA-pair grouped kernel (256x256 tiles; a last block of at most 128
    rows runs as a transposed 128x256 half tile) on the task's test shapes:
    every group under 256 rows, so each is one full tile with its second CTA
    partly past M, or one half tile."""
    monkeypatch.setenv("NVFP4_GROUPED_KERNEL", "pair")
    m, n, k = GROUP_TASK_TESTS[case]
    data = I.generate_group_input(m, n, k, len(m), seed=1111, device="cuda")
    outs = G.custom_kernel(data)
    assert _lib.device_status() == 0
    for i, (got, want) in enumerate(zip(outs, oracle_group(data))):
        assert_close(got.cpu().numpy(), want, f"group pair case {case} g{i}")


def test_group_pair_ragged_and_chunked(monkeypatch):
    """CTA-pair grouped kernel: M around the 128/256-row block edges (half
    tiles of 1, 64, 127, 128 rows; full tiles whose second CTA holds 1 or 127
    rows), N below one tile and not a multiple of 256 (second 128-row B block
    past N, or a single block: a half tile's second CTA then stores nothing),
    K of 1..8 blocks per group, zero-M groups, and more groups than one launch
    holds (near-equal chunks of at most 48)."""
    monkeypatch.setenv("NVFP4_GROUPED_KERNEL", "pair")
    gen = torch.Generator().manual_seed(41)
    shapes = [(1, 8, 256), (0, 256, 512), (127, 136, 512), (128, 256, 256), (129, 264, 1024),
              (255, 384, 768), (256, 520, 256), (257, 256, 2048), (640, 1032, 512)]
    shapes += [(8 * (i % 40 + 1), 256 + 8 * (i % 5), 256 * (i % 3 + 1)) for i in range(50)]
    pairs = [(torch.randn(m, k, generator=gen), torch.randn(n, k, generator=gen)) for m, n, k in shapes]
    data = I.group_from_fp32(pairs, device="cuda")
    outs = G.custom_kernel(data)
    assert _lib.device_status() == 0
    for i, (got, want) in enumerate(zip(outs, oracle_group(data))):
        assert_close(got.cpu().numpy(), want, f"group pair g{i} {shapes[i]}")


def test_group_auto_pair_tails():
    """Automatic choice with long K (the CTA-pair kernel, no override): last
    blocks of at most 128 rows as half tiles — whole groups of <= 128 rows
    and the tails of larger groups (44 and 128 rows after 256, 128 after
    512, 232 after 768 as a full block) — and a 129-row group as one full
    pair block whose second CTA holds one row."""
    gen = torch.Generator().manual_seed(53)
    shapes = [(300, 256, 6144), (384, 384, 6144), (640, 264, 6144), (1000, 256, 6144),
              (129, 384, 6144), (100, 256, 6144), (64, 272, 6144)]
    pairs = [(torch.randn(m, k, generator=gen), torch.randn(n, k, generator=gen)) for m, n, k in shapes]
    data = I.group_from_fp32(pairs, device="cuda")
    outs = G.custom_kernel(data)
    assert _lib.device_status() == 0
    for i, (got, want) in enumerate(zip(outs, oracle_group(data))):
        assert_close(got.cpu().numpy(), want, f"group auto split g{i} {shapes[i]}")


@pytest.mark.parametrize("kernel", ["auto", "pair", "single"])
def test_group_batched_l(kernel, monkeypatch):
    """Groups with L = 2 and 3 batches (A, B, scales and C with L outermost
    in memory, as the reference lays them out): full and half pair tiles,
    ragged N, a zero-M group, under each grouped kernel."""
    if kernel != "auto":
        monkeypatch.setenv("NVFP4_GROUPED_KERNEL", kernel)
    gen = torch.Generator().manual_seed(67)
    shapes = [(200, 256, 6144, 2), (300, 384, 6144, 3), (64, 264, 6144, 2), (0, 256, 6144, 2),
              (384, 256, 6144, 2)]
    pairs = [(torch.randn(l, m, k, generator=gen), torch.randn(l, n, k, generator=gen))
             for m, n, k, l in shapes]
    data = I.group_from_fp32(pairs, device="cuda")
    outs = G.custom_kernel(data)
    assert _lib.device_status() == 0
    for i, (got, want) in enumerate(zip(outs, oracle_group(data))):
        assert got.shape == want.shape
        assert_close(got.cpu().numpy(), want, f"group L>1 {kernel} g{i} {shapes[i]}")


@pytest.mark.parametrize("kernel", ["pair", "single"])
def test_group_config3_both_kernels(kernel, monkeypatch):
    """Configuration 3 under each grouped kernel: sampled rows of every group."""
    monkeypatch.setenv("NVFP4_GROUPED_KERNEL", kernel)
    data = I.group_config_input(3, device="cuda")
    outs = G.custom_kernel(data)
    assert _lib.device_status() == 0
    abc, sfab, _, sizes = data
    for i in range(len(sizes)):
        (a, b, _), (sa, sb) = abc[i], sfab[i]
        rows = torch.arange(i % 5, sizes[i][0], 61)
        want = O.ref_group(_np(_rows(a, rows))[:, :, 0], _np(b)[:, :, 0],
                           _np(_rows(sa, rows))[:, :, 0], _np(sb)[:, :, 0])
        assert_close(outs[i][rows.to(outs[i].device), :, 0].cpu().numpy(), want,
                     f"cfg3 {kernel} group {i} sampled")


def test_group_ragged_k_and_chunks():
    # groups of different K (tiles of 2..12 K blocks), ragged M and N, zero-M
    # groups, and more groups than one launch holds
    gen = torch.Generator().manual_seed(31)
    shapes = [(0, 256, 512), (200, 264, 1536), (72, 512, 256), (0, 256, 768), (384, 256, 768)]
    shapes += [(8 * (i % 9 + 1), 256 + 8 * (i % 3), 256 * (i % 4 + 1)) for i in range(100)]
    pairs = [(torch.randn(m, k, generator=gen), torch.randn(n, k, generator=gen)) for m, n, k in shapes]
    data = I.group_from_fp32(pairs, device="cuda")
    outs = G.custom_kernel(data)
    assert _lib.device_status() == 0
    for i, (got, want) in enumerate(zip(outs, oracle_group(data))):
        assert_close(got.cpu().numpy(), want, f"group g{i} {shapes[i]}")


def test_group_deterministic():
    ms, n, k = GROUP_TASK_BENCH[0]
    data = I.generate_group_input(ms, [n] * len(ms), [k] * len(ms), len(ms), seed=9, device="cuda")
    runs = [[o.clone() for o in G.custom_kernel(data)] for _ in range(3)]
    assert _lib.device_status() == 0
    for r in runs[1:]:
        assert all(torch.equal(x, y) for x, y in zip(runs[0], r))


def test_group_zero_and_many_groups():
    # a zero-M group, ragged M, and more groups than one 16-entry launch holds
    ms = [0, 64, 40, 0, 200, 128] + [8 * (i + 1) for i in range(14)]
    g = len(ms)
    gen = torch.Generator().manual_seed(77)
    pairs = [(torch.randn(mi, 512, generator=gen), torch.randn(256, 512, generator=gen)) for mi in ms]
    data = I.group_from_fp32(pairs, device="cuda")
    outs = G.custom_kernel(data)
    assert _lib.device_status() == 0
    for i, (got, want) in enumerate(zip(outs, oracle_group(data))):
        assert_close(got.cpu().numpy(), want, f"group g{i} (m={ms[i]})")
    assert g > 16


def test_group_more_than_one_launch():
    ms = [16 * (i % 7 + 1) for i in range(100)]   # > 96 groups: two launches
    gen = torch.Generator().manual_seed(5)
    pairs = [(torch.randn(mi, 256, generator=gen), torch.randn(128, 256, generator=gen)) for mi in ms]
    data = I.group_from_fp32(pairs, device="cuda")
    outs = G.custom_kernel(data)
    assert _lib.device_status() == 0
    for i, (got, want) in enumerate(zip(outs, oracle_group(data))):
        assert_close(got.cpu().numpy(), want, f"group g{i}")


def test_group_config3_full_size():
    data = I.group_config_input(3, device="cuda")
    outs = G.custom_kernel(data)
    assert _lib.device_status() == 0
    # full check of the two smallest groups, sampled rows elsewhere
    abc, sfab, _, sizes = data
    order = sorted(range(len(sizes)), key=lambda i: sizes[i][0])
    for i in order[:2]:
        (a, b, _), (sa, sb) = abc[i], sfab[i]
        want = O.ref_group(_np(a)[:, :, 0], _np(b)[:, :, 0], _np(sa)[:, :, 0], _np(sb)[:, :, 0])
        assert_close(outs[i][:, :, 0].cpu().numpy(), want, f"cfg3 group {i}")
    for i in order[2:]:
        (a, b, _), (sa, sb) = abc[i], sfab[i]
        rows = torch.arange(0, sizes[i][0], 97)
        want = O.ref_group(_np(_rows(a, rows))[:, :, 0], _np(b)[:, :, 0],
                           _np(_rows(sa, rows))[:, :, 0], _np(sb)[:, :, 0])
        assert_close(outs[i][rows.to(outs[i].device), :, 0].cpu().numpy(), want,
                     f"cfg3 group {i} sampled")


def test_group_config4_sampled():
    data = I.group_config_input(4, device="cuda")
    outs = G.custom_kernel(data)
    assert _lib.device_status() == 0
    abc, sfab, _, sizes = data
    assert any(s[0] == 0 for s in sizes) or min(s[0] for s in sizes) < 128
    for i in range(0, len(sizes), 9):
        if sizes[i][0] == 0:
            continue
        (a, b, _), (sa, sb) = abc[i], sfab[i]
        rows = torch.arange(0, sizes[i][0], max(1, sizes[i][0] // 16))
        want = O.ref_group(_np(_rows(a, rows))[:, :, 0], _np(b)[:, :, 0],
                           _np(_rows(sa, rows))[:, :, 0], _np(sb)[:, :, 0])
        assert_close(outs[i][rows.to(outs[i].device), :, 0].cpu().numpy(), want, f"cfg4 expert {i}")


def test_oracle_matches_scaled_mm_live():
    """Pin the oracle (nibble order, scale layout, fp32 accumulation) against
    torch._scaled_mm called as nvfp4_dual_gemm/reference.py:56-73 does."""
    from nvfp4_b200.formats import to_blocked
    for (m, n, k) in [(128, 128, 256), (256, 384, 1024), (72, 144, 512)]:
        data = I.generate_dual_input(m, n, k, 1, seed=m * 7 + k, device="cuda")
        a, b1, _, sfa, sfb1 = data[0], data[1], data[2], data[3], data[4]
        r1 = torch._scaled_mm(a[:, :, 0], b1[:, :, 0].transpose(0, 1),
                              to_blocked(sfa[:, :, 0]).cuda(), to_blocked(sfb1[:, :, 0]).cuda(),
                              bias=None, out_dtype=torch.float32)
        ours = O.scaled_mm_f32(_np(a)[:, :, 0], _np(sfa)[:, :, 0], _np(b1)[:, :, 0], _np(sfb1)[:, :, 0])
        np.testing.assert_allclose(ours, r1.cpu().numpy(), rtol=1e-5, atol=1e-3)


def test_wait_timeout_reports_status():
    """A bounded wait on an mbarrier nothing completes ends with a status,
    not a hang; the context stays usable afterwards."""
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.nvfp4_wait_selftest(2_000_000, stream))
    bits = _lib.device_status(stream)
    assert bits != 0
    assert _lib.device_status(stream) == 0           # cleared
    data = I.generate_dual_input(256, 256, 256, 1, seed=9, device="cuda")
    assert_close(run_dual(data), oracle_dual(data), "dual after timeout self-test")


def test_device_quantisation_bit_exact():
    """formats.quantize_nvfp4 on the GPU == the oracle (bit-exact)."""
    from nvfp4_b200.formats import quantize_nvfp4
    g = torch.Generator().manual_seed(123)
    x = torch.randn(512, 1024, generator=g) * 3
    p, s = quantize_nvfp4(x.cuda())
    po, so = O.quantize_nvfp4(x.numpy())
    assert np.array_equal(s.cpu().numpy(), so) and np.array_equal(p.cpu().numpy(), po)


def _clone(x):
    if isinstance(x, torch.Tensor):
        if x.element_size() == 1 and x.dtype != torch.uint8:
            return x.view(torch.uint8).clone().view(x.dtype)
        return x.clone()
    if isinstance(x, (tuple, list)):
        return type(x)(_clone(v) for v in x)
    return x


def test_two_host_threads_on_their_own_streams(monkeypatch):
    """Two host threads, each on its own stream with its own buffers, run the
    dual GEMM (workspace split-K forced: each stream has its own workspace)
    and the grouped GEMM (CTA-pair kernel) interleaved; every output is
    bit-identical to a single-threaded run."""
    import threading
    monkeypatch.setenv("NVFP4_DUAL_SPLITS", "3")
    dual = I.generate_dual_input(256, 1024, 3072, 1, seed=21, device="cuda")
    gen = torch.Generator().manual_seed(22)
    group = I.group_from_fp32([(torch.randn(m, 6144, generator=gen), torch.randn(n, 6144, generator=gen))
                               for m, n in ((300, 256), (128, 384), (512, 264))], device="cuda")
    want_dual = D.custom_kernel(dual).clone()
    want_group = [c.clone() for c in G.custom_kernel(group)]
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    sets = [(_clone(dual), _clone(group)) for _ in range(2)]
    errors = []

    def work(d, g):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                for _ in range(10):
                    D.custom_kernel(d)
                    G.custom_kernel(g)
            s.synchronize()
        except Exception as e:   # surfaced below
            errors.append(e)

    threads = [threading.Thread(target=work, args=st) for st in sets]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    assert _lib.device_status() == 0
    for d, g in sets:
        assert torch.equal(d[9], want_dual)
        assert all(torch.equal(c, w) for (_, _, c), w in zip(g[0], want_group))


def _capture_and_replay(fn, outs):
    """Eager result, then the same call captured in a CUDA graph (warmed up on
    a side stream first, as torch documents) and replayed into zeroed outputs."""
    fn()
    torch.cuda.synchronize()
    want = [o.clone() for o in outs]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    for o in outs:
        o.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    for o, w in zip(outs, want):
        assert torch.equal(o, w)
    del graph


@pytest.mark.parametrize("m,n,k", [(256, 4096, 7168), (512, 3072, 7168), (128, 7168, 16384), (1536, 512, 7168)])
def test_dual_captured_in_a_cuda_graph(m, n, k):
    """The dual GEMM under its automatic choice (CTA pair 64/128-wide, cluster
    split-K) captured in a CUDA graph and replayed: bit-identical to eager."""
    data = I.generate_dual_input(m, n, k, 1, seed=m + n, device="cuda")
    _capture_and_replay(lambda: D.custom_kernel(data), [data[9]])


@pytest.mark.parametrize("k,groups", [(6144, 60), (1024, 5)])
def test_grouped_captured_in_a_cuda_graph(k, groups):
    """The grouped GEMM captured in a CUDA graph: long K with more groups than
    one launch holds (CTA-pair kernel, chained launches, half tiles) and short
    K (single-CTA kernel); bit-identical to eager."""
    gen = torch.Generator().manual_seed(k + groups)
    shapes = [(64 * (i % 5 + 1), 256 + 8 * (i % 3)) for i in range(groups)]
    data = I.group_from_fp32([(torch.randn(m, k, generator=gen), torch.randn(n, k, generator=gen))
                              for m, n in shapes], device="cuda")
    _capture_and_replay(lambda: G.custom_kernel(data), [c for _, _, c in data[0]])


def test_dual_workspace_split_captured_on_a_fresh_stream(monkeypatch):
    """Workspace split-K (forced) captured in a CUDA graph: the capture stream
    is new, so its workspace is created during the capture."""
    monkeypatch.setenv("NVFP4_DUAL_SPLITS", "3")
    data = I.generate_dual_input(256, 1024, 3072, 1, seed=77, device="cuda")
    _capture_and_replay(lambda: D.custom_kernel(data), [data[9]])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_calls_on_a_device_other_than_the_current_one():
    """Tensors on cuda:1 while cuda:0 is current (and the reverse): the
    drop-ins run on the tensors' device, per-device state (status word,
    kernel attributes, descriptors by address) stays apart, and the results
    match the same call made on cuda:0."""
    want = {}
    for dev in (0, 1):
        torch.cuda.set_device(0)
        dual = I.generate_dual_input(256, 1024, 7168, 1, seed=31, device=f"cuda:{dev}")
        gen = torch.Generator().manual_seed(32)
        group = I.group_from_fp32([(torch.randn(m, 6144, generator=gen), torch.randn(256, 6144, generator=gen))
                                   for m in (300, 100, 512)], device=f"cuda:{dev}")
        if dev == 1:
            torch.cuda.set_device(0)       # the current device is not the tensors'
        out_d = D.custom_kernel(dual)
        out_g = G.custom_kernel(group)
        assert out_d.device.index == dev and all(c.device.index == dev for c in out_g)
        torch.cuda.synchronize(dev)
        want[dev] = (out_d.cpu(), [c.cpu() for c in out_g])
    assert torch.equal(want[0][0], want[1][0])
    assert all(torch.equal(a, b) for a, b in zip(want[0][1], want[1][1]))
    assert torch.cuda.current_device() == 0
    for dev in (0, 1):
        with torch.cuda.device(dev):
            assert _lib.device_status() == 0

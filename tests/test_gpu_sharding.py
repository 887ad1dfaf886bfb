"""GPU: the dual GEMM's N-sharding (one process per GPU, no data-path
collective) computes exactly the unsharded output.

Rank r of P owns B1/B2 rows [n0, n1) = shard.n_shard(N, P, r) (128-row
multiples, so its scale atoms are a contiguous slice of the permuted scale
tensors), A is replicated, and it writes C[:, n0:n1].  Here all P shards run
one after another on one GPU, on views of the single-GPU operands, and each
rank's C is compared with the matching columns of the unsharded C.  Where a
shard makes the same kernel and split choice as the whole problem the two are
bit-identical (configuration 1: unsplit at every P; configuration 2 with the
K split pinned to the same 2-CTA cluster split); where the shard's smaller
tile count picks a different K split (configuration 2 at P = 8, automatic),
the summation order differs, so it is checked against the oracle instead.
"""
import pytest
import torch

from nvfp4_b200 import _lib
from nvfp4_b200 import build as B
from nvfp4_b200 import dual_gemm as D
from nvfp4_b200 import inputs as I
from nvfp4_b200.shard import n_shard
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib_ready(cuda_device):
    B.build()
    _lib.load()


def shard_of(data, n0, n1):
    """Rank tuple over rows [n0, n1) of B1/B2: views of the single-GPU tensors
    and a fresh C."""
    a, b1, b2, sfa, sfb1, sfb2, pa, pb1, pb2, c = data
    m, _, l = c.shape
    c_r = torch.full((l, m, n1 - n0), float("nan"), dtype=torch.float16,
                     device=c.device).permute(1, 2, 0)
    r0, r1 = n0 // 128, -(-n1 // 128)
    return (a, b1[n0:n1], b2[n0:n1], sfa, sfb1[n0:n1], sfb2[n0:n1], pa,
            pb1[:, :, r0:r1], pb2[:, :, r0:r1], c_r)


def run_shards(data, world):
    n = data[9].shape[1]
    outs = []
    for rank in range(world):
        n0, n1 = n_shard(n, world, rank)
        outs.append(((n0, n1), D.custom_kernel(shard_of(data, n0, n1)).clone()))
    assert _lib.device_status() == 0
    return outs


def test_config1_shards_bit_identical():
    data = I.dual_config_input(1, device="cuda")
    full = D.custom_kernel(data).clone()
    assert _lib.device_status() == 0
    for world in (2, 4, 8):
        for (n0, n1), c_r in run_shards(data, world):
            assert torch.equal(c_r, full[:, n0:n1]), f"P={world} rows [{n0}, {n1})"


def test_config2_shards_bit_identical_with_the_same_split(monkeypatch):
    monkeypatch.setenv("NVFP4_DUAL_CLUSTER", "2")
    data = I.dual_config_input(2, device="cuda")
    full = D.custom_kernel(data).clone()
    assert _lib.device_status() == 0
    for world in (2, 4, 8):
        for (n0, n1), c_r in run_shards(data, world):
            assert torch.equal(c_r, full[:, n0:n1]), f"P={world} rows [{n0}, {n1})"


def test_config2_eight_shards_automatic_choice():
    data = I.dual_config_input(2, device="cuda")
    u8 = lambda t: t.detach().cpu().view(torch.uint8).numpy()[:, :, 0]
    a, sfa = u8(data[0]), u8(data[3])
    for (n0, n1), c_r in run_shards(data, 8):
        want = O.ref_dual(a, u8(data[1])[n0:n1], u8(data[2])[n0:n1], sfa,
                          u8(data[4])[n0:n1], u8(data[5])[n0:n1])
        bad, idx = O.allclose_report(c_r[:, :, 0].cpu().numpy(), want, 1e-2, 1e-2)
        assert bad == 0, f"rows [{n0}, {n1}): {bad} mismatches, first {idx[:3]}"

"""GPU: the device quantiser (nvfp4_quantize) is bit-exact against the oracle
restatement of the quantisation and of the scale layouts, and its output
feeds the dual GEMM to the oracle's result."""
import numpy as np
import pytest
import torch

from nvfp4_b200 import _lib
from nvfp4_b200 import build as B
from nvfp4_b200 import dual_gemm as D
from nvfp4_b200.quantize import quantize
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _ready(cuda_device):
    B.build()
    _lib.load()


def _edge_rows(k):
    mags = np.array([0, 0.25, 0.5, 0.75, 1, 1.25, 1.5, 1.75, 2, 2.5, 3, 3.5, 4, 5, 6, 7, 1e4, 3e3],
                    np.float32)
    row = np.zeros(k, np.float32)
    vals = np.concatenate([mags, -mags])
    row[: len(vals)] = vals[:k]
    return row


@pytest.mark.parametrize("rows,k,l,scale", [(128, 64, 1, 1.0), (200, 1024, 1, 3.0),
                                            (1, 256, 2, 0.01), (385, 4096, 1, 1e3),
                                            (256, 7168, 1, 1.0), (1000, 2048, 3, 0.5)])
def test_quantize_bit_exact(rows, k, l, scale):
    g = torch.Generator().manual_seed(rows + k)
    x = torch.randn(l, rows, k, generator=g) * scale
    x[0, 0] = torch.from_numpy(_edge_rows(k))     # ties, saturation, large amax
    if rows > 1:
        x[0, 1, :16] = 0.0                        # zero block -> zero scale
        x[0, 1, 16:32] = 1e-12                    # scale underflows to zero
    packed, sf, sf_perm = quantize(x.cuda())
    assert _lib.device_status() == 0
    for b in range(l):
        po, so = O.quantize_nvfp4(x[b].numpy())
        assert np.array_equal(packed.view(torch.uint8)[:, :, b].cpu().numpy(), po)
        assert np.array_equal(sf.view(torch.uint8)[:, :, b].cpu().numpy(), so)
    mem = sf_perm.view(torch.uint8).permute(5, 2, 4, 0, 1, 3).contiguous().cpu().numpy()
    assert np.array_equal(mem, O.permuted_sf(sf.view(torch.uint8).cpu().numpy()))


def _special_rows(k, rng):
    """Blocks that stress the division-free quotient: values exactly at the
    e2m1 rounding thresholds times the block scale (ties) and their fp32
    neighbours, for scales of every e4m3 mantissa over a range of exponents;
    -0, subnormal and tiny values beside normal ones; +-inf (IEEE-division
    fallback); saturating scales."""
    thr = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    rows = []
    for mant in range(8):
        for exp in (-9, -4, 0, 3, 8):
            s = np.float32((1 + mant / 8) * 2.0 ** exp)
            amax = np.float32(s * 6)                 # e4m3(amax / 6) == s exactly
            blk = np.zeros(16, np.float32)
            blk[0] = amax
            t = thr * s
            pick = rng.choice(7, 5)
            blk[1:6] = t[pick]
            blk[6:11] = np.nextafter(t[pick], np.float32(np.inf))
            blk[11:15] = -np.nextafter(t[pick[:4]], np.float32(0))
            blk[15] = -0.0
            rows.append(blk)
    special = np.zeros(16, np.float32)
    special[:6] = [np.inf, -1.0, -0.0, 1e-40, -1e-40, 3.0e38]
    rows.append(special)
    rows.append(np.array([-0.0] * 8 + [1e-30] * 8, np.float32))
    rows.append(np.array([-np.inf] + [0.5] * 15, np.float32))
    rows.append(np.array([3.0e38, -2.9e38] + [1.0] * 14, np.float32))
    flat = np.concatenate(rows)
    n = -(-flat.size // k) * k
    flat = np.concatenate([flat, np.zeros(n - flat.size, np.float32)])
    return flat.reshape(-1, k)


@pytest.mark.parametrize("k", [64, 256])
def test_quantize_special_values_bit_exact(k):
    rng = np.random.default_rng(k)
    x = _special_rows(k, rng)
    wide = (rng.standard_normal((64, k)) * np.exp2(rng.integers(-30, 30, (64, 1)))).astype(np.float32)
    x = np.concatenate([x, wide])
    packed, sf, _ = quantize(torch.from_numpy(x).cuda())
    po, so = O.quantize_nvfp4(x)
    assert np.array_equal(sf.view(torch.uint8)[:, :, 0].cpu().numpy(), so)
    assert np.array_equal(packed.view(torch.uint8)[:, :, 0].cpu().numpy(), po)


def test_quantize_feeds_dual_gemm():
    m, n, k = 256, 384, 1024
    g = torch.Generator().manual_seed(11)
    qa = quantize(torch.randn(m, k, generator=g).cuda())
    q1 = quantize(torch.randn(n, k, generator=g).cuda())
    q2 = quantize(torch.randn(n, k, generator=g).cuda())
    c = torch.zeros((1, m, n), dtype=torch.float16, device="cuda").permute(1, 2, 0)
    data = (qa[0], q1[0], q2[0], qa[1], q1[1], q2[1], qa[2], q1[2], q2[2], c)
    out = D.custom_kernel(data).cpu().numpy()
    u8 = lambda t: t.cpu().view(torch.uint8).numpy()
    want = O.ref_dual_batched(u8(qa[0]), u8(q1[0]), u8(q2[0]), u8(qa[1]), u8(q1[1]), u8(q2[1]))
    assert O.allclose_report(out, want, 1e-2, 1e-2)[0] == 0


def test_quantize_reuses_out():
    g = torch.Generator().manual_seed(3)
    x1 = torch.randn(200, 512, generator=g).cuda()
    x2 = torch.randn(200, 512, generator=g).cuda()
    first = quantize(x1)
    ptrs = [t.data_ptr() for t in first]
    again = quantize(x2, out=first)
    assert [t.data_ptr() for t in again] == ptrs
    fresh = quantize(x2)
    assert all(torch.equal(a.view(torch.uint8), b.view(torch.uint8)) for a, b in zip(again, fresh))
    with pytest.raises(ValueError):
        quantize(torch.randn(128, 512).cuda(), out=first)


def test_quantize_rejects_bad_k():
    with pytest.raises(ValueError):
        quantize(torch.zeros(4, 100, device="cuda"))

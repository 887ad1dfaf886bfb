"""CPU: the product's host-side packing and swizzling (nvfp4_b200.formats,
nvfp4_b200.inputs) are bit-exact against the oracle restatement."""
from pathlib import Path

import numpy as np
import pytest
import torch

from nvfp4_b200 import formats as F
from nvfp4_b200 import inputs as I
from oracle import nvfp4_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def _edge_values():
    mags = np.array([0, 0.25, 0.5, 0.75, 1, 1.25, 1.5, 1.75, 2, 2.5, 3, 3.5, 4, 5, 6, 7, 100],
                    np.float32)
    return np.concatenate([mags, -mags])


@pytest.mark.parametrize("scale", [1.0, 1e-3, 37.0])
def test_quantize_bit_exact_vs_oracle(scale):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(64, 512, generator=g) * scale
    x[0, :34] = torch.from_numpy(_edge_values())   # ties and saturation in one block row
    x[1, :16] = 0.0                                 # all-zero block
    x[2, :16] = 1e-12                               # scale underflows to zero
    p, s = F.quantize_nvfp4(x)
    po, so = O.quantize_nvfp4(x.numpy())
    assert np.array_equal(s.numpy(), so)
    assert np.array_equal(p.numpy(), po)


def test_e2m1_codes_vs_oracle_dense_sweep():
    x = torch.linspace(-8, 8, 20001)
    assert np.array_equal(F.e2m1_codes(x).numpy(), O.f32_to_e2m1(x.numpy()))


def test_e4m3_codes_vs_oracle():
    g = torch.Generator().manual_seed(9)
    x = torch.rand(50000, generator=g) * 500 - 250
    assert np.array_equal(F.e4m3_codes(x).numpy(), O.f32_to_e4m3(x.numpy()))


@pytest.mark.parametrize("mn,sf_k,l", [(128, 16, 1), (200, 24, 1), (40, 4, 2), (384, 448, 1)])
def test_swizzle_bit_exact_vs_oracle(mn, sf_k, l):
    g = torch.Generator().manual_seed(mn + sf_k)
    sf = torch.randint(0, 256, (mn, sf_k, l), dtype=torch.uint8, generator=g)
    perm = F.swizzle_sf(sf)
    rm, rk = -(-mn // 128), -(-sf_k // 4)
    assert tuple(perm.shape) == (32, 4, rm, 4, rk, l)
    assert perm.dtype == torch.float8_e4m3fn
    mem = perm.view(torch.uint8).permute(5, 2, 4, 0, 1, 3)   # logical -> memory order
    assert mem.is_contiguous()
    assert np.array_equal(mem.numpy(), O.permuted_sf(sf.numpy()))


def test_to_blocked_matches_reference_fixture():
    z = np.load(GOLDEN / "swizzle_golden.npz")
    n = sum(1 for k in z.files if k.startswith("sf_"))
    for i in range(n):
        sf = torch.from_numpy(z[f"sf_{i}"])
        assert np.array_equal(F.to_blocked(sf).view(torch.uint8).numpy(), z[f"blocked_{i}"])
        perm = F.swizzle_sf(sf.unsqueeze(-1)).view(torch.uint8).permute(5, 2, 4, 0, 1, 3)
        assert np.array_equal(perm.contiguous().numpy(), z[f"perm_{i}"])


def test_generate_dual_input_layout():
    d = I.generate_dual_input(256, 384, 512, 2, seed=1111, device="cpu")
    a, b1, b2, sfa, sfb1, sfb2, pa, pb1, pb2, c = d
    assert a.dtype == torch.float4_e2m1fn_x2 and tuple(a.shape) == (256, 256, 2)
    assert a.stride() == (256, 1, 256 * 256)          # L outermost, K-major
    assert sfa.dtype == torch.float8_e4m3fn and tuple(sfa.shape) == (256, 32, 2)
    assert tuple(pa.shape) == (32, 4, 2, 4, 8, 2) and tuple(pb1.shape) == (32, 4, 3, 4, 8, 2)
    assert c.dtype == torch.float16 and tuple(c.shape) == (256, 384, 2)
    u = a.view(torch.uint8)
    assert int((u & 0x44).sum()) == 0                  # nibble bit 2 cleared (& 0b1011_1011)
    assert np.array_equal(pa.view(torch.uint8).permute(5, 2, 4, 0, 1, 3).contiguous().numpy(),
                          O.permuted_sf(sfa.view(torch.uint8).numpy()))


def test_generate_group_input_layout():
    abc, sfab, perm, sizes = I.generate_group_input([96, 128], [128, 256], [256, 512], 2,
                                                    seed=1111, device="cpu")
    assert sizes == [(96, 128, 256, 1), (128, 256, 512, 1)]
    a0 = abc[0][0].view(torch.uint8)
    assert set(torch.unique(a0).tolist()) <= {0, 1, 255}
    assert set(sfab[0][0].float().unique().tolist()) <= {1.0, 2.0}
    # scale padding rows (96..127) carry 1 or 2 like the reference's builder
    mem = perm[0][0].view(torch.uint8).permute(5, 2, 4, 0, 1, 3).contiguous().numpy()
    logical = O.unpermute_sf(mem, 96, 16)
    assert np.array_equal(logical, sfab[0][0].view(torch.uint8).numpy())


def test_group_from_fp32_batched_layout():
    """Batched (L = 2) grouped inputs from fp32: every tensor in the
    reference's layout ([rows, K/2, L], K-major, L outermost in memory), each
    batch slice bit-exact against the oracle quantiser, the permuted scales
    the swizzle of the logical ones per batch, and a zero-row group kept."""
    gen = torch.Generator().manual_seed(5)
    shapes = [(130, 264, 512, 2), (0, 256, 256, 2), (64, 128, 256, 1)]
    pairs = [(torch.randn(l, m, k, generator=gen), torch.randn(l, n, k, generator=gen))
             for m, n, k, l in shapes]
    abc, sfab, perm, sizes = I.group_from_fp32(pairs, device="cpu")
    assert sizes == [(m, n, k, l) for m, n, k, l in shapes]
    for (m, n, k, l), (a, b, c), (sa, sb), (pa, pb), (xa, xb) in zip(shapes, abc, sfab, perm, pairs):
        assert a.shape == (m, k // 2, l) and b.shape == (n, k // 2, l) and c.shape == (m, n, l)
        assert b.stride() == (k // 2, 1, n * k // 2)
        if m:   # an empty tensor's strides are never read
            assert a.stride() == (k // 2, 1, m * k // 2) and c.stride() == (n, 1, m * n)
        assert sa.shape == (m, k // 16, l) and sb.shape == (n, k // 16, l)
        for i in range(l):
            want_b, want_sb = O.quantize_nvfp4(xb[i].numpy())
            assert np.array_equal(b[:, :, i].view(torch.uint8).numpy(), want_b)
            assert np.array_equal(sb[:, :, i].view(torch.uint8).numpy(), want_sb)
            if m:
                want_a, want_sa = O.quantize_nvfp4(xa[i].numpy())
                assert np.array_equal(a[:, :, i].view(torch.uint8).numpy(), want_a)
                assert np.array_equal(sa[:, :, i].view(torch.uint8).numpy(), want_sa)
        for p_, s_, rows in ((pb, sb, n), (pa, sa, m)):
            if rows == 0:
                continue
            mem = p_.view(torch.uint8).permute(5, 2, 4, 0, 1, 3).contiguous().numpy()
            assert np.array_equal(O.unpermute_sf(mem, rows, k // 16), s_.view(torch.uint8).numpy())


def test_config_samplers_are_fixed():
    m3 = I.config3_m_sizes()
    assert len(m3) == 8 and all(v % 64 == 0 and 64 <= v <= 2048 for v in m3)
    assert m3 == I.config3_m_sizes()
    m4 = I.config4_m_sizes()
    assert len(m4) == 64 and sum(m4) == 32768 and m4 == I.config4_m_sizes()
    assert max(m4) > 10 * (32768 // 64) / 4            # skewed


def test_dual_config0_quantisation_matches_oracle():
    d = I.dual_config_input(0, device="cpu")
    g = torch.Generator().manual_seed(0)
    a = torch.randn(256, 1024, generator=g)
    pa, sa = O.quantize_nvfp4(a.numpy())
    assert np.array_equal(d[0].view(torch.uint8)[:, :, 0].numpy(), pa)
    assert np.array_equal(d[3].view(torch.uint8)[:, :, 0].numpy(), sa)


def test_reciprocal_fma_quotient_is_ieee_division():
    """The device quantiser forms x / s without a division: r = RN(1/s),
    q0 = RN(x*r), q1 = RN(q0 + RD(x - q0*s) * r) (two FMAs; the residual is
    exact whenever it is nonzero, asserted below, so its rounding direction
    only decides the sign of a zero residual, which leaves q0 unchanged).  Exhaustive
    check that q1 == RN(x/s) for every fp32 mantissa of x and every e4m3
    scale mantissa (1 + j/8); a power-of-two factor on x or s scales every
    step exactly, so this covers all normal operands.  FMAs are emulated in
    float64: the residual x - q0*s is exact there (checked), and the final
    sum is rounded to fp32 once unless it lands on an fp32 midpoint (checked
    to be absent)."""
    x = (np.arange(1 << 23, dtype=np.uint32) | np.uint32(0x3F800000)).view(np.float32)
    for j in range(8):
        s = np.float32(1 + j / 8)
        r = np.float32(1) / s
        q0 = x * r
        rho64 = x.astype(np.float64) - q0.astype(np.float64) * np.float64(s)
        rho = rho64.astype(np.float32)
        assert np.array_equal(rho.astype(np.float64), rho64)
        s64 = q0.astype(np.float64) + rho.astype(np.float64) * np.float64(r)
        q1 = s64.astype(np.float32)
        up = np.nextafter(q1, np.float32(np.inf)).astype(np.float64)
        dn = np.nextafter(q1, np.float32(-np.inf)).astype(np.float64)
        q1d = q1.astype(np.float64)
        assert not np.any((s64 == (q1d + up) / 2) | (s64 == (q1d + dn) / 2))
        assert np.array_equal(q1.view(np.uint32), (x / s).view(np.uint32)), f"scale mantissa {s}"

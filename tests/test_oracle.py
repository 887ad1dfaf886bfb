"""CPU: the oracle pinned against the reference's own golden vectors, and
known-answer tests of its element formats and GEMM restatement."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_to_blocked_matches_reference_fixture():
    z = np.load(GOLDEN / "swizzle_golden.npz")
    n = sum(1 for k in z.files if k.startswith("sf_"))
    assert n >= 8
    for i in range(n):
        sf = z[f"sf_{i}"]
        assert np.array_equal(O.to_blocked(sf), z[f"blocked_{i}"]), i
        if f"blocked_dual_{i}" in z.files:
            assert np.array_equal(O.to_blocked(sf), z[f"blocked_dual_{i}"]), i


def test_permuted_layout_matches_reference_fixture():
    z = np.load(GOLDEN / "swizzle_golden.npz")
    n = sum(1 for k in z.files if k.startswith("sf_"))
    for i in range(n):
        sf = z[f"sf_{i}"]
        perm = O.permuted_sf(sf[:, :, None])
        assert np.array_equal(perm, z[f"perm_{i}"]), i
        back = O.unpermute_sf(perm, sf.shape[0], sf.shape[1])
        assert np.array_equal(back[:, :, 0], sf)


def test_permuted_layout_is_blocked_per_batch():
    rng = np.random.default_rng(3)
    sf = rng.integers(0, 256, size=(256, 32, 3), dtype=np.uint8)
    perm = O.permuted_sf(sf)
    for b in range(3):
        assert np.array_equal(perm[b].ravel(), O.to_blocked(sf[:, :, b]))


def test_e4m3_decode_all_codes_match_torch():
    codes = np.arange(256, dtype=np.uint8)
    ours = O.e4m3_to_f32(codes)
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(ours), nan)
    assert np.array_equal(ours[~nan], ref[~nan])


def test_e4m3_encode_matches_torch_rne():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s
                        for s in (1e-3, 0.1, 1.0, 30.0, 200.0)])
    x = np.clip(x, -448, 448).astype(np.float32)
    # exact midpoints between neighbouring codes exercise ties-to-even
    vals = O.e4m3_to_f32(np.arange(0, 0x7E, dtype=np.uint8)).astype(np.float64)
    mids = ((vals[:-1] + vals[1:]) / 2).astype(np.float32)
    x = np.concatenate([x, mids, -mids])
    ours = O.f32_to_e4m3(x)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    ours_v, ref_v = O.e4m3_to_f32(ours), O.e4m3_to_f32(ref)
    assert np.array_equal(ours_v, ref_v)


def test_e2m1_known_answers():
    assert O.E2M1_TABLE.tolist()[:8] == [0, 0.5, 1, 1.5, 2, 3, 4, 6]
    x = np.array([0.0, 0.2, 0.25, 0.26, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.1, 7.0, -0.75, -9],
                 dtype=np.float32)
    want = [0.0, 0.0, 0.0, 0.5, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, 6.0, -1.0, -6.0]
    got = O.E2M1_TABLE[O.f32_to_e2m1(x)]
    assert got.tolist() == want
    packed = np.array([[0x21, 0xF9]], dtype=np.uint8)
    assert O.decode_e2m1_packed(packed).tolist() == [[0.5, 1.0, -0.5, -6.0]]


def test_quantize_known_answer():
    x = np.zeros((1, 32), dtype=np.float32)
    x[0, :16] = np.linspace(-3, 3, 16)
    x[0, 16] = 12.0
    packed, sf = O.quantize_nvfp4(x)
    assert sf.shape == (1, 2) and packed.shape == (1, 16)
    assert O.e4m3_to_f32(sf).tolist() == [[0.5, 2.0]]
    deq = O.dequantize(packed, sf)
    assert deq[0, 16] == 12.0 and np.all(deq[0, 17:] == 0)
    assert np.max(np.abs(deq[0, :16] - x[0, :16])) <= 0.5 + 1e-6
    # all-zero block -> zero scale and zero codes
    p0, s0 = O.quantize_nvfp4(np.zeros((2, 16), np.float32))
    assert not p0.any() and not s0.any()


def test_ref_dual_small_known_answer():
    # A = all +1 (code 2), B1 = all +0.5 (code 1), B2 = all +1, unit scales
    m, n, k = 4, 8, 64
    a = np.full((m, k // 2), 0x22, np.uint8)
    b1 = np.full((n, k // 2), 0x11, np.uint8)
    b2 = np.full((n, k // 2), 0x22, np.uint8)
    one = O.f32_to_e4m3(np.ones(1, np.float32))[0]
    sfa = np.full((m, k // 16), one, np.uint8)
    sfb = np.full((n, k // 16), one, np.uint8)
    r1 = 0.5 * k
    want = np.float16(r1 / (1 + np.exp(-r1)) * k)
    out = O.ref_dual(a, b1, b2, sfa, sfb, sfb)
    assert out.dtype == np.float16 and np.all(out == want)
    g = O.ref_group(a, b1, sfa, sfb)
    assert np.all(g == np.float16(r1))


def test_ref_dual_matches_float64_restatement():
    rng = np.random.default_rng(7)
    m, n, k = 16, 24, 256
    a = rng.integers(0, 256, (m, k // 2), dtype=np.uint8)
    b1 = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    b2 = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    sf = lambda r: O.f32_to_e4m3(rng.random((r, k // 16)).astype(np.float32))
    sfa, sfb1, sfb2 = sf(m), sf(n), sf(n)
    da = O.dequantize(a, sfa).astype(np.float64)
    r1 = da @ O.dequantize(b1, sfb1).astype(np.float64).T
    r2 = da @ O.dequantize(b2, sfb2).astype(np.float64).T
    want = (r1 / (1 + np.exp(-r1)) * r2).astype(np.float16)
    got = O.ref_dual(a, b1, b2, sfa, sfb1, sfb2)
    bad, _ = O.allclose_report(got, want, 1e-3, 1e-3)
    assert bad == 0


def test_allclose_report_inf_nan_rules():
    e = np.array([1.0, np.inf, -np.inf, np.nan, 2.0])
    assert O.allclose_report(e, e, 1e-3, 1e-3)[0] == 0
    r = np.array([1.0, np.inf, np.inf, np.nan, 2.1])
    assert O.allclose_report(r, e, 1e-3, 1e-3)[0] == 2


GOLDEN_MM = GOLDEN / "scaled_mm_golden.npz"


@pytest.mark.skipif(not GOLDEN_MM.exists(), reason="scaled_mm fixture not generated yet")
def test_oracle_matches_scaled_mm_fixture():
    """The oracle against torch._scaled_mm outputs recorded on a B200
    (tests/golden/make_golden.py --gpu)."""
    z = np.load(GOLDEN_MM)
    n = sum(1 for k in z.files if k.startswith("r1_"))
    assert n >= 3
    for i in range(n):
        r1 = O.scaled_mm_f32(z[f"a_{i}"], z[f"sfa_{i}"], z[f"b1_{i}"], z[f"sfb1_{i}"])
        np.testing.assert_allclose(r1, z[f"r1_{i}"], rtol=1e-5, atol=1e-3)
        h16 = O.ref_group(z[f"a_{i}"], z[f"b1_{i}"], z[f"sfa_{i}"], z[f"sfb1_{i}"])
        assert O.allclose_report(h16, z[f"h16_{i}"], 1e-3, 1e-3)[0] == 0
        d = O.ref_dual(z[f"a_{i}"], z[f"b1_{i}"], z[f"b2_{i}"], z[f"sfa_{i}"], z[f"sfb1_{i}"],
                       z[f"sfb2_{i}"])
        assert O.allclose_report(d, z[f"dual_{i}"], 1e-3, 1e-3)[0] == 0

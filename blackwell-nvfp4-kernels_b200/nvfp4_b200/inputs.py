"""Seeded input generators producing the reference task's tuples.

* ``generate_dual_input`` / ``generate_group_input``: the reference's own
  value distributions and tensor layouts (nvfp4_dual_gemm/reference.py:80-196,
  nvfp4_group_gemm/reference.py:126-196), drawn from a CPU generator so they
  are reproducible on any machine (the reference draws on the GPU, so the
  values differ, the distributions do not).
* ``dual_config_input`` / ``group_config_input``: the benchmark
  configurations: fp32 N(0,1) operands quantised with
  ``formats.quantize_nvfp4``.

Every tuple is built on CPU and moved to ``device``; quantisation can run on
the device (``quantize_on``) since it is bit-exact there too.
"""
from __future__ import annotations

import torch

from .formats import SF_VEC, ceil_div, quantize_nvfp4, swizzle_sf

# ---------------------------------------------------------------------------
# benchmark configurations
# ---------------------------------------------------------------------------
DUAL_CONFIGS = {
    0: dict(m=256, n=512, k=1024, l=1, seed=0),
    1: dict(m=8192, n=14336, k=4096, l=1, seed=1),
    2: dict(m=128, n=7168, k=16384, l=1, seed=2),
}
GROUP_CONFIGS = {
    3: dict(groups=8, n=4096, k=7168, seed=1),
    4: dict(experts=64, tokens=32768, zipf_s=1.1, n=2048, k=7168, seed=4),
}


def config3_m_sizes(seed: int = 1, groups: int = 8) -> list[int]:
    """M_g = 64 * U{1..32}: torch.randint(1, 33, (8,), generator=seed 1) * 64."""
    g = torch.Generator().manual_seed(seed)
    return [int(v) * 64 for v in torch.randint(1, 33, (groups,), generator=g)]


def config4_expert_ids(seed: int = 4, experts: int = 64, tokens: int = 32768,
                       s: float = 1.1) -> torch.Tensor:
    """Zipf(s) routing of `tokens` tokens over `experts` experts (int32 [tokens]):
    rank r in 1..experts has weight r**-s, ranks map to experts by a seeded
    permutation, tokens draw experts by seeded multinomial sampling with
    replacement."""
    g = torch.Generator().manual_seed(seed)
    w = torch.arange(1, experts + 1, dtype=torch.float64) ** (-s)
    perm = torch.randperm(experts, generator=g)
    ranks = torch.multinomial(w, tokens, replacement=True, generator=g)
    return perm[ranks].to(torch.int32)


def config4_m_sizes(seed: int = 4, experts: int = 64, tokens: int = 32768,
                    s: float = 1.1) -> list[int]:
    """Tokens per expert of :func:`config4_expert_ids` (configuration 4's M_g)."""
    expert = config4_expert_ids(seed, experts, tokens, s).long()
    return [int(v) for v in torch.bincount(expert, minlength=experts)]


def _pack_operand(x: torch.Tensor, quantize_on: str | torch.device):
    packed, sf = quantize_nvfp4(x.to(quantize_on))
    return packed, sf


def dual_from_fp32(a: torch.Tensor, b1: torch.Tensor, b2: torch.Tensor,
                   device="cuda", quantize_on=None):
    """Quantise fp32 A [M,K], B1/B2 [N,K] into the reference's 10-tuple (L=1)."""
    quantize_on = quantize_on or device
    m, k = a.shape
    n = b1.shape[0]
    pa, sa = _pack_operand(a, quantize_on)
    pb1, sb1 = _pack_operand(b1, quantize_on)
    pb2, sb2 = _pack_operand(b2, quantize_on)
    dev = torch.device(device)
    fp4 = lambda t: t.to(dev).unsqueeze(0).permute(1, 2, 0).view(torch.float4_e2m1fn_x2)
    sf3 = lambda t: t.to(dev).view(torch.float8_e4m3fn).unsqueeze(0).permute(1, 2, 0)
    sfa, sfb1, sfb2 = sf3(sa), sf3(sb1), sf3(sb2)
    c = torch.zeros((1, m, n), dtype=torch.float16, device=dev).permute(1, 2, 0)
    return (fp4(pa), fp4(pb1), fp4(pb2), sfa, sfb1, sfb2,
            swizzle_sf(sfa), swizzle_sf(sfb1), swizzle_sf(sfb2), c)


def dual_config_input(cfg: int, device="cuda", quantize_on=None):
    """BASELINE dual configuration 0, 1 or 2 as the reference 10-tuple."""
    spec = DUAL_CONFIGS[cfg]
    g = torch.Generator().manual_seed(spec["seed"])
    m, n, k = spec["m"], spec["n"], spec["k"]
    a = torch.randn(m, k, generator=g)
    b1 = torch.randn(n, k, generator=g)
    b2 = torch.randn(n, k, generator=g)
    return dual_from_fp32(a, b1, b2, device=device, quantize_on=quantize_on)


def group_from_fp32(pairs, device="cuda", quantize_on=None):
    """[(A_g, B_g)] fp32, A_g [M,K] and B_g [N,K] (L=1) or A_g [L,M,K] and
    B_g [L,N,K] (batched) -> the reference's grouped 4-tuple, every tensor in
    its layout: [rows, K/2, L] K-major with L outermost in memory."""
    quantize_on = quantize_on or device
    dev = torch.device(device)
    abc, sfab, sfab_perm, sizes = [], [], [], []
    for a, b in pairs:
        a3 = a if a.dim() == 3 else a.unsqueeze(0)
        b3 = b if b.dim() == 3 else b.unsqueeze(0)
        l, m, k = a3.shape
        n = b3.shape[1]
        if m > 0:
            pk = [_pack_operand(a3[i], quantize_on) for i in range(l)]
            pa = torch.stack([p_[0] for p_ in pk])
            sa = torch.stack([p_[1] for p_ in pk])
        else:
            pa = torch.zeros((l, 0, k // 2), dtype=torch.uint8)
            sa = torch.zeros((l, 0, k // SF_VEC), dtype=torch.uint8)
        pk = [_pack_operand(b3[i], quantize_on) for i in range(l)]
        pb = torch.stack([p_[0] for p_ in pk])
        sb = torch.stack([p_[1] for p_ in pk])
        fp4 = lambda t: t.to(dev).permute(1, 2, 0).view(torch.float4_e2m1fn_x2)
        sf3 = lambda t: t.to(dev).view(torch.float8_e4m3fn).permute(1, 2, 0)
        c = torch.zeros((l, m, n), dtype=torch.float16, device=dev).permute(1, 2, 0)
        sfa, sfb = sf3(sa), sf3(sb)
        abc.append((fp4(pa), fp4(pb), c))
        sfab.append((sfa, sfb))
        sfab_perm.append((swizzle_sf(sfa), swizzle_sf(sfb)))
        sizes.append((m, n, k, l))
    return abc, sfab, sfab_perm, sizes


def group_config_input(cfg: int, device="cuda", quantize_on=None, m_sizes=None):
    """BASELINE grouped configuration 3 or 4 as the reference 4-tuple."""
    spec = GROUP_CONFIGS[cfg]
    if m_sizes is None:
        m_sizes = config3_m_sizes(spec["seed"], spec["groups"]) if cfg == 3 else \
            config4_m_sizes(spec["seed"], spec["experts"], spec["tokens"], spec["zipf_s"])
    g = torch.Generator().manual_seed(1000 + spec["seed"])
    n, k = spec["n"], spec["k"]
    pairs = [(torch.randn(m, k, generator=g), torch.randn(n, k, generator=g)) for m in m_sizes]
    return group_from_fp32(pairs, device=device, quantize_on=quantize_on)


# ---------------------------------------------------------------------------
# the reference's own inputs
# ---------------------------------------------------------------------------
def _atom_image(fill: torch.Tensor, sf: torch.Tensor) -> torch.Tensor:
    """Permuted scale tensor whose padding holds `fill`: fill is the uint8
    atom image [l, ceil(mn/128), ceil(sf_k/4), 32, 4, 4] the reference starts
    from, sf the [mn, sf_k, l] scales written over it (row r = 128*mm + 32*mm4
    + mm32, block j = 4*kk + kk4 go to image index (l, mm, kk, mm32, mm4, kk4))."""
    mn, sf_k, l = sf.shape
    rm, rk = fill.shape[1], fill.shape[2]
    mat = fill.permute(0, 1, 4, 3, 2, 5).reshape(l, rm * 128, rk * 4).clone()
    mat[:, :mn, :sf_k] = sf.view(torch.uint8).permute(2, 0, 1)
    return swizzle_sf(mat.permute(1, 2, 0))


def reference_dual_input(m: int, n: int, k: int, l: int, seed: int, device="cuda"):
    """The dual-GEMM 10-tuple of nvfp4_dual_gemm/reference.py:80-196 for
    (m, n, k, l, seed), made by the same torch RNG calls in the same order
    (torch.manual_seed, then on `device`: randint of A, B1, B2 (:116, :125-127),
    randn of C (:134), rand of the three scale tensors (:145)), so on a GPU these
    are the reference's own inputs.  The padding of the permuted scale
    tensors, uninitialised memory in the reference (:165), is zero here; no
    kernel reads it for a stored output row."""
    torch.manual_seed(seed)
    dev = torch.device(device)
    sf_k = ceil_div(k, SF_VEC)

    def operand(mn):
        codes = torch.randint(255, size=(l, mn, k // 2), dtype=torch.uint8, device=dev)
        return (codes & 0b1011_1011).permute(1, 2, 0).view(torch.float4_e2m1fn_x2)

    a, b1, b2 = operand(m), operand(n), operand(n)
    c = torch.randn((l, m, n), dtype=torch.float16, device=dev).permute(1, 2, 0)

    def scales(mn):
        sf = torch.rand((l, mn, sf_k), dtype=torch.float32, device=dev) \
            .to(dtype=torch.float8_e4m3fn).permute(1, 2, 0)
        fill = torch.zeros((l, ceil_div(mn, 128), ceil_div(sf_k, 4), 32, 4, 4),
                           dtype=torch.uint8, device=dev)
        return sf, _atom_image(fill, sf)

    (sfa, pa), (sfb1, pb1), (sfb2, pb2) = scales(m), scales(n), scales(n)
    return (a, b1, b2, sfa, sfb1, sfb2, pa, pb1, pb2, c)


def reference_group_input(m, n, k, g: int, seed: int, device="cuda"):
    """The grouped-GEMM 4-tuple of nvfp4_group_gemm/reference.py:126-196 for
    (m, n, k, g, seed), made by the same torch RNG calls in the same order
    (torch.manual_seed, then per group: randint of A and B and randn of C on
    `device` (:168-179), randint of the plain scales on the CPU generator
    (:182-187), and for each permuted scale tensor a randint of its whole
    image on `device` that supplies the padding (:97)), so on a GPU these are
    the reference's own inputs.  The plain scales stay on the CPU, as there."""
    torch.manual_seed(seed)
    dev = torch.device(device)
    abc, sfab, sfab_perm, sizes = [], [], [], []
    for i in range(g):
        mi, ni, ki = m[i], n[i], k[i]
        sf_k = ceil_div(ki, SF_VEC)
        a = torch.randint(-1, 2, (1, mi, ki // 2), dtype=torch.int8, device=dev).permute(1, 2, 0)
        b = torch.randint(-1, 2, (1, ni, ki // 2), dtype=torch.int8, device=dev).permute(1, 2, 0)
        c = torch.randn((1, mi, ni), dtype=torch.float16, device=dev).permute(1, 2, 0)
        sfa = torch.randint(1, 3, (1, mi, sf_k), dtype=torch.int8) \
            .to(dtype=torch.float8_e4m3fn).permute(1, 2, 0)
        sfb = torch.randint(1, 3, (1, ni, sf_k), dtype=torch.int8) \
            .to(dtype=torch.float8_e4m3fn).permute(1, 2, 0)

        def permuted(mn, sf):
            fill = torch.randint(1, 3, (1, ceil_div(mn, 128), ceil_div(sf_k, 4), 32, 4, 4),
                                 dtype=torch.int8, device=dev).to(dtype=torch.float8_e4m3fn)
            return _atom_image(fill.view(torch.uint8), sf.to(dev))

        abc.append((a.view(torch.float4_e2m1fn_x2), b.view(torch.float4_e2m1fn_x2), c))
        sfab.append((sfa, sfb))
        sfab_perm.append((permuted(mi, sfa), permuted(ni, sfb)))
        sizes.append((mi, ni, ki, 1))
    return abc, sfab, sfab_perm, sizes


# ---------------------------------------------------------------------------
# reference-task distributions
# ---------------------------------------------------------------------------
def _ref_fp4_bytes(l, mn, k, g, mode):
    if mode == "dual":   # nvfp4_dual_gemm/reference.py:116-120
        return torch.randint(0, 255, (l, mn, k // 2), dtype=torch.uint8, generator=g) & 0xBB
    # nvfp4_group_gemm/reference.py:168-173: int8 in {-1, 0, 1}
    return torch.randint(-1, 2, (l, mn, k // 2), dtype=torch.int8, generator=g).view(torch.uint8)


def _ref_sf(l, mn, sf_k, g, mode):
    if mode == "dual":   # nvfp4_dual_gemm/reference.py:145-146: rand[0,1) -> e4m3
        return torch.rand((l, mn, sf_k), generator=g).to(torch.float8_e4m3fn)
    # nvfp4_group_gemm/reference.py:182-187: randint(1,3) -> e4m3 {1, 2}
    return torch.randint(1, 3, (l, mn, sf_k), dtype=torch.int8, generator=g).to(torch.float8_e4m3fn)


def generate_dual_input(m: int, n: int, k: int, l: int, seed: int, device="cuda"):
    """Reference-style dual input (10-tuple), layouts as
    nvfp4_dual_gemm/reference.py:80-196."""
    g = torch.Generator().manual_seed(seed)
    dev = torch.device(device)
    a = _ref_fp4_bytes(l, m, k, g, "dual")
    b1 = _ref_fp4_bytes(l, n, k, g, "dual")
    b2 = _ref_fp4_bytes(l, n, k, g, "dual")
    c = torch.randn((l, m, n), generator=g).to(torch.float16)
    sf_k = ceil_div(k, SF_VEC)
    sfa = _ref_sf(l, m, sf_k, g, "dual")
    sfb1 = _ref_sf(l, n, sf_k, g, "dual")
    sfb2 = _ref_sf(l, n, sf_k, g, "dual")
    to3 = lambda t: t.to(dev).permute(1, 2, 0)
    fp4 = lambda t: to3(t).view(torch.float4_e2m1fn_x2)
    sfa3, sfb13, sfb23 = to3(sfa), to3(sfb1), to3(sfb2)
    return (fp4(a), fp4(b1), fp4(b2), sfa3, sfb13, sfb23,
            swizzle_sf(sfa3), swizzle_sf(sfb13), swizzle_sf(sfb23), to3(c))


def generate_group_input(m, n, k, g: int, seed: int, device="cuda"):
    """Reference-style grouped input (4-tuple), layouts as
    nvfp4_group_gemm/reference.py:126-196 (scale padding filled with 1/2 like
    create_reordered_scale_factor_tensor, nvfp4_group_gemm/reference.py:95)."""
    gen = torch.Generator().manual_seed(seed)
    dev = torch.device(device)
    abc, sfab, sfab_perm, sizes = [], [], [], []
    for i in range(g):
        mi, ni, ki = m[i], n[i], k[i]
        a = _ref_fp4_bytes(1, mi, ki, gen, "group")
        b = _ref_fp4_bytes(1, ni, ki, gen, "group")
        c = torch.randn((1, mi, ni), generator=gen).to(torch.float16)
        sf_k = ceil_div(ki, SF_VEC)
        sfa = _ref_sf(1, mi, sf_k, gen, "group")
        sfb = _ref_sf(1, ni, sf_k, gen, "group")
        to3 = lambda t: t.to(dev).permute(1, 2, 0)
        fp4 = lambda t: to3(t).view(torch.float4_e2m1fn_x2)
        sfa3, sfb3 = to3(sfa), to3(sfb)
        pad = int(torch.randint(1, 3, (1,), generator=gen).to(torch.float8_e4m3fn)
                  .view(torch.uint8))
        abc.append((fp4(a), fp4(b), to3(c)))
        sfab.append((sfa3, sfb3))
        sfab_perm.append((swizzle_sf(sfa3, pad), swizzle_sf(sfb3, pad)))
        sizes.append((mi, ni, ki, 1))
    return abc, sfab, sfab_perm, sizes

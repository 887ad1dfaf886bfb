"""Host-side NVFP4 packing and scale-factor swizzling (torch; CPU or CUDA).

These produce exactly the byte images the reference task hands to a
``custom_kernel``:

* ``quantize_nvfp4``: fp32 [rows, K] -> e2m1 codes packed two per byte
  (element 2i in the low nibble) + one e4m3 scale per 16 K-elements.  The
  reference generators emit raw bit patterns instead
  (nvfp4_dual_gemm/reference.py:113-146); this quantiser is the one the
  benchmark configurations ask for: scale = e4m3_rne(amax/6),
  value = e2m1_rne(x / scale) saturating at +-6 (a value rounding to zero
  keeps its sign, as the sm_100 cvt.e2m1x2 conversion does), zero scale ->
  (+0) zero values.
* ``swizzle_sf``: [mn, sf_k, l] scales -> the permuted
  [32, 4, ceil(mn/128), 4, ceil(sf_k/4), l] tensor whose memory is the
  sequence of 512-byte atoms the kernels read
  (nvfp4_dual_gemm/reference.py:150-187, nvfp4_group_gemm/reference.py:80-123).
* ``to_blocked``: the flat cuBLAS layout of nvfp4_group_gemm/reference.py:14-36.

All bit-exact; the tests compare them with an independent restatement.
"""
from __future__ import annotations

import torch

SF_VEC = 16
E4M3_MAX = 448.0

# e2m1 rounding boundaries between consecutive magnitudes
# {0, .5, 1, 1.5, 2, 3, 4, 6}; a tie goes to the even code, so a boundary is
# crossed with ">" when the lower neighbour is even and ">=" when the upper is.
_E2M1_BOUNDS = ((0.25, False), (0.75, True), (1.25, False), (1.75, True),
                (2.5, False), (3.5, True), (5.0, False))


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


def e2m1_codes(q: torch.Tensor) -> torch.Tensor:
    """fp32 -> e2m1 nibble codes (uint8 0..15), nearest-even, saturating;
    the sign bit is the input's sign bit (also for zero)."""
    a = q.abs()
    code = torch.zeros(q.shape, dtype=torch.uint8, device=q.device)
    for bound, inclusive in _E2M1_BOUNDS:
        code += (a >= bound if inclusive else a > bound).to(torch.uint8)
    return code | (torch.signbit(q).to(torch.uint8) << 3)   # zero keeps its sign


def e4m3_codes(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> float8_e4m3fn bytes, nearest-even, saturating at 448."""
    return x.clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)


def quantize_nvfp4(x: torch.Tensor):
    """fp32 [rows, K] -> (packed uint8 [rows, K/2], scale bytes uint8 [rows, K/16])."""
    assert x.dim() == 2 and x.shape[1] % SF_VEC == 0, x.shape
    x = x.float()
    rows, k = x.shape
    blocks = x.view(rows, k // SF_VEC, SF_VEC)
    amax = blocks.abs().amax(dim=-1)
    sf = e4m3_codes(amax / 6.0)
    s = sf.view(torch.float8_e4m3fn).float().unsqueeze(-1)
    q = torch.where(s == 0, torch.zeros_like(blocks), blocks / torch.where(s == 0, 1.0, s))
    nib = e2m1_codes(q).view(rows, k)
    packed = nib[:, 0::2] | (nib[:, 1::2] << 4)
    return packed.contiguous(), sf.contiguous()


def swizzle_sf(sf: torch.Tensor, pad_value: int = 0) -> torch.Tensor:
    """[mn, sf_k, l] (uint8 or e4m3) -> float8_e4m3fn view of shape
    [32, 4, rest_mn, 4, rest_k, l] over contiguous [l, rest_mn, rest_k, 32, 4, 4]."""
    u = sf.view(torch.uint8) if sf.dtype != torch.uint8 else sf
    mn, sf_k, l = u.shape
    rest_mn, rest_k = ceil_div(mn, 128), ceil_div(sf_k, 4)
    padded = torch.full((l, rest_mn * 128, rest_k * 4), pad_value, dtype=torch.uint8,
                        device=u.device)
    padded[:, :mn, :sf_k] = u.permute(2, 0, 1)
    # rows r = mm*128 + mm4*32 + mm32, cols j = kk*4 + kk4
    t = padded.view(l, rest_mn, 4, 32, rest_k, 4)            # l, mm, mm4, mm32, kk, kk4
    atoms = t.permute(0, 1, 4, 3, 2, 5).contiguous()          # l, mm, kk, mm32, mm4, kk4
    return atoms.permute(3, 4, 1, 5, 2, 0).view(torch.float8_e4m3fn)


def to_blocked(sf2d: torch.Tensor) -> torch.Tensor:
    """[rows, cols] scales -> flat cuBLAS blocked layout, zero padded."""
    u = sf2d.view(torch.uint8) if sf2d.dtype != torch.uint8 else sf2d
    rows, cols = u.shape
    rb, cb = ceil_div(rows, 128), ceil_div(cols, 4)
    padded = torch.zeros((rb * 128, cb * 4), dtype=torch.uint8, device=u.device)
    padded[:rows, :cols] = u
    t = padded.view(rb, 4, 32, cb, 4)                         # rb, r4, r32, cb, c4
    return t.permute(0, 3, 2, 1, 4).reshape(-1).view(torch.float8_e4m3fn)

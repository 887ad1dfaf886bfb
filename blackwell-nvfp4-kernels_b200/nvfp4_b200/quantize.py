"""Device-side NVFP4 quantisation (kernel `nvfp4_quantize` in libnvfp4_b200.so).

``quantize(x)`` turns fp32 ``x`` ([rows, K] or [L, rows, K], on a CUDA device)
into the three tensors the reference task tuples carry for one operand
(nvfp4_dual_gemm/reference.py:196): packed values ``[rows, K/2, L]``
float4_e2m1fn_x2, plain scales ``[rows, K/16, L]`` float8_e4m3fn, and the
permuted scales ``[32, 4, ceil(rows/128), 4, K/64, L]`` float8_e4m3fn the
kernels read.  Bit-identical to ``formats.quantize_nvfp4`` + ``formats.swizzle_sf``.
"""
from __future__ import annotations

import torch

from . import _lib
from .dual_gemm import on_device


def quantize(x: torch.Tensor, out=None):
    """Returns (packed, sf, sf_perm).  ``out``: a tuple returned by an
    earlier call with the same shape, whose storage is reused (no allocation)."""
    if x.dim() == 2:
        x = x.unsqueeze(0)
    if x.dim() != 3 or x.dtype != torch.float32 or not x.is_cuda:
        raise ValueError("x must be a CUDA float32 tensor [rows, K] or [L, rows, K]")
    x = x.contiguous()
    l, rows, k = x.shape
    if k % 64:
        raise ValueError(f"K={k} must be a multiple of 64")
    rb, ka = -(-rows // 128), k // 64
    dev = x.device
    if out is not None:
        packed = out[0].view(torch.uint8).permute(2, 0, 1)
        sf = out[1].view(torch.uint8).permute(2, 0, 1)
        sf_perm = out[2].view(torch.uint8).permute(5, 2, 4, 0, 1, 3)
        if (tuple(packed.shape) != (l, rows, k // 2) or tuple(sf.shape) != (l, rows, k // 16)
                or tuple(sf_perm.shape) != (l, rb, ka, 32, 4, 4) or not packed.is_contiguous()
                or not sf.is_contiguous() or not sf_perm.is_contiguous()
                or any(t.device != dev for t in (packed, sf, sf_perm))):
            raise ValueError("out does not match x: pass the tuple an earlier call returned")
    else:
        packed = torch.empty((l, rows, k // 2), dtype=torch.uint8, device=dev)
        sf = torch.empty((l, rows, k // 16), dtype=torch.uint8, device=dev)
        sf_perm = torch.empty((l, rb, ka, 32, 4, 4), dtype=torch.uint8, device=dev)
    lib = _lib.load()
    _lib.check(on_device(dev, lambda st: lib.nvfp4_quantize(
        x.data_ptr(), rows, k, l, packed.data_ptr(), sf_perm.data_ptr(), sf.data_ptr(), st)))
    return (packed.permute(1, 2, 0).view(torch.float4_e2m1fn_x2),
            sf.permute(1, 2, 0).view(torch.float8_e4m3fn),
            sf_perm.permute(3, 4, 1, 5, 2, 0).view(torch.float8_e4m3fn))

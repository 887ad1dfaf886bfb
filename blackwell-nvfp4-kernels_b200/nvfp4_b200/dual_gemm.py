"""Drop-in ``custom_kernel`` for the NVFP4 dual GEMM task.

Same entry point, tuple and return value as the reference submissions
(nvfp4_dual_gemm/submission_v4.py:1256-1284): ``data`` is the 10-tuple of
nvfp4_dual_gemm/reference.py:196, the result is written into (and returned
as) its ``c``.  The kernels read a, b1, b2, the three permuted scale tensors
and c; the un-permuted scales are not needed.
"""
from __future__ import annotations

import torch

from . import _lib
from .formats import ceil_div


def _expect(cond: bool, msg: str):
    if not cond:
        raise ValueError(msg)


def _check_operand(name, t, rows, kh, l, device):
    _expect(t.dtype in (torch.float4_e2m1fn_x2, torch.uint8, torch.int8),
            f"{name}: expected float4_e2m1fn_x2, got {t.dtype}")
    _expect(tuple(t.shape) == (rows, kh, l), f"{name}: shape {tuple(t.shape)} != {(rows, kh, l)}")
    _expect(t.device == device, f"{name}: on {t.device}, expected {device}")
    ok = t.stride(0) == kh and t.stride(1) == 1 and (l == 1 or t.stride(2) == rows * kh)
    _expect(ok, f"{name}: strides {t.stride()} are not the K-major [L][{rows}][{kh}] layout")


def check_sf_perm(name, t, mn, k, l, device):
    """The permuted scale tensor must be the memory image
    [l][ceil(mn/128)][k/64][32][4][4] (its logical shape is [32,4,rm,4,rk,l])."""
    rm, rk = ceil_div(mn, 128), ceil_div(k // 16, 4)
    _expect(t.dtype in (torch.float8_e4m3fn, torch.uint8, torch.int8),
            f"{name}: expected float8_e4m3fn, got {t.dtype}")
    _expect(tuple(t.shape) == (32, 4, rm, 4, rk, l),
            f"{name}: shape {tuple(t.shape)} != {(32, 4, rm, 4, rk, l)}")
    _expect(t.device == device, f"{name}: on {t.device}, expected {device}")
    want = (16, 4, rk * 512, 1, 512, rm * rk * 512)
    got = t.stride()
    ok = all(g == w for g, w, s in zip(got, want, t.shape) if s > 1)
    _expect(ok, f"{name}: strides {got} are not the atom layout {want}")


def dual_gemm(a, b1, b2, sfa_perm, sfb1_perm, sfb2_perm, c) -> torch.Tensor:
    """c[:, :, l] = silu(A_l . B1_lᵀ) * (A_l . B2_lᵀ) in fp16, on c's stream."""
    _expect(c.dtype == torch.float16, f"c: expected float16, got {c.dtype}")
    _expect(c.is_cuda, "c must be a CUDA tensor")
    m, n, l = c.shape
    kh = a.shape[1]
    k = kh * 2
    dev = c.device
    _check_operand("a", a, m, kh, l, dev)
    _check_operand("b1", b1, n, kh, l, dev)
    _check_operand("b2", b2, n, kh, l, dev)
    check_sf_perm("sfa_permuted", sfa_perm, m, k, l, dev)
    check_sf_perm("sfb1_permuted", sfb1_perm, n, k, l, dev)
    check_sf_perm("sfb2_permuted", sfb2_perm, n, k, l, dev)
    _expect(c.stride(0) == n and c.stride(1) == 1 and (l == 1 or c.stride(2) == m * n),
            f"c: strides {c.stride()} are not the row-major [L][M][N] layout")
    lib = _lib.load()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(lib.nvfp4_dual_gemm(
            a.data_ptr(), b1.data_ptr(), b2.data_ptr(), sfa_perm.data_ptr(),
            sfb1_perm.data_ptr(), sfb2_perm.data_ptr(), c.data_ptr(), m, n, k, l, stream))
    return c


def custom_kernel(data):
    """Reference task entry point: data = (a, b1, b2, sfa, sfb1, sfb2,
    sfa_permuted, sfb1_permuted, sfb2_permuted, c); returns c."""
    a, b1, b2, _sfa, _sfb1, _sfb2, sfa_p, sfb1_p, sfb2_p, c = data
    return dual_gemm(a, b1, b2, sfa_p, sfb1_p, sfb2_p, c)

"""Drop-in ``custom_kernel`` for the NVFP4 grouped GEMM task.

Same entry point, tuple and return value as the reference submissions
(nvfp4_group_gemm/submission_v7.py:605-617): ``data`` is
``(abc_list, sfasfb_list, sfasfb_reordered_list, problem_sizes)``
(nvfp4_group_gemm/reference.py:196); every ``c_g`` is written in one
persistent launch and the list of ``c_g`` is returned.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .dual_gemm import _check_operand, _expect, check_sf_perm


def build_group_table(abc, sf_perm, sizes):
    """Validate every group and fill the C struct array nvfp4_group[G]."""
    _expect(len(abc) == len(sf_perm) == len(sizes), "group lists differ in length")
    table = (_lib.Group * max(len(abc), 1))()
    device = None
    for i, ((a, b, c), (sfa, sfb), size) in enumerate(zip(abc, sf_perm, sizes)):
        m, n, k, l = (int(v) for v in size)
        _expect(c.dtype == torch.float16 and c.is_cuda, f"group {i}: c must be CUDA float16")
        device = device or c.device
        _expect(c.device == device, f"group {i}: all groups must live on {device}")
        _expect(tuple(c.shape) == (m, n, l), f"group {i}: c shape {tuple(c.shape)} != {(m, n, l)}")
        if m > 0:
            _check_operand(f"group {i} a", a, m, k // 2, l, device)
            check_sf_perm(f"group {i} sfa", sfa, m, k, l, device)
            _expect(c.stride(0) == n and c.stride(1) == 1 and (l == 1 or c.stride(2) == m * n),
                    f"group {i}: c strides {c.stride()} are not row-major [L][M][N]")
        _check_operand(f"group {i} b", b, n, k // 2, l, device)
        check_sf_perm(f"group {i} sfb", sfb, n, k, l, device)
        table[i] = _lib.Group(a.data_ptr() if m > 0 else None, b.data_ptr(),
                              sfa.data_ptr() if m > 0 else None, sfb.data_ptr(),
                              c.data_ptr() if m > 0 else None, m, n, k, l)
    return table, device


def grouped_gemm(abc, sf_perm, sizes):
    """C_g = A_g . B_gᵀ (fp16) for all groups; returns [c_g]."""
    table, device = build_group_table(abc, sf_perm, sizes)
    if device is None:
        return []
    lib = _lib.load()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(lib.nvfp4_grouped_gemm(table, len(abc), stream))
    return [c for _, _, c in abc]


def custom_kernel(data):
    """Reference task entry point; returns the list of outputs c_g."""
    abc, _sfab, sfab_perm, sizes = data
    return grouped_gemm(abc, sfab_perm, sizes)

"""Drop-in ``custom_kernel`` for the NVFP4 grouped GEMM task.

Same entry point, tuple and return value as the reference submissions
(nvfp4_group_gemm/submission_v7.py:605-617): ``data`` is
``(abc_list, sfasfb_list, sfasfb_reordered_list, problem_sizes)``
(nvfp4_group_gemm/reference.py:196); every ``c_g`` is written in one
persistent launch and the list of ``c_g`` is returned.

Validating G groups touches ~20 tensor attributes per group, which for 64
groups costs more host time than the kernel.  A validated call is therefore
remembered as a plan: the next call with the same tensor objects (checked by
identity through weak references) at the same data pointers reuses the
C group table without re-validating; anything else is validated afresh.
"""
from __future__ import annotations

import threading
import weakref

import torch

from . import _lib
from .dual_gemm import _check_operand, _expect, check_sf_perm, on_device

_PLAN_SLOTS = 64        # >= the 15 rotating inputs of the reference's timing loop


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


class _Plan:
    """A validated group table plus weak references to the tensors it was
    built from (the plan never keeps user tensors alive)."""

    def __init__(self, abc, sf_perm, sizes, table, device):
        self.refs = [tuple(weakref.ref(t) for t in (a, b, c, sa, sb))
                     for (a, b, c), (sa, sb) in zip(abc, sf_perm)]
        self.ptrs = [tuple(t.data_ptr() for t in (a, b, c, sa, sb))
                     for (a, b, c), (sa, sb) in zip(abc, sf_perm)]
        self.sizes = [tuple(int(v) for v in s) for s in sizes]
        self.table, self.device = table, device

    def matches(self, abc, sf_perm, sizes) -> bool:
        if len(abc) != len(self.refs) or len(sf_perm) != len(self.refs):
            return False
        for (a, b, c), (sa, sb), refs, ptrs, size, want in zip(
                abc, sf_perm, self.refs, self.ptrs, sizes, self.sizes):
            if (a is not refs[0]() or b is not refs[1]() or c is not refs[2]()
                    or sa is not refs[3]() or sb is not refs[4]()):
                return False
            if (a.data_ptr(), b.data_ptr(), c.data_ptr(), sa.data_ptr(), sb.data_ptr()) != ptrs:
                return False
            if tuple(size) != want:
                return False
        return True


_plans: dict = {}
_plans_lock = threading.Lock()   # host threads may insert concurrently; lookups need no lock


def _plan_for(abc, sf_perm, sizes):
    key = (id(abc), id(sf_perm), id(sizes))
    plan = _plans.get(key)
    if plan is not None and plan.matches(abc, sf_perm, sizes):
        return plan
    table, device = build_group_table(abc, sf_perm, sizes)
    plan = _Plan(abc, sf_perm, sizes, table, device)
    with _plans_lock:
        if len(_plans) >= _PLAN_SLOTS:
            _plans.pop(next(iter(_plans)))
        _plans[key] = plan
    return plan


def clear_plan_cache() -> None:
    with _plans_lock:
        _plans.clear()


def grouped_gemm(abc, sf_perm, sizes):
    """C_g = A_g . B_gᵀ (fp16) for all groups; returns [c_g]."""
    plan = _plan_for(abc, sf_perm, sizes)
    if plan.device is None:
        return []
    lib = _lib.load()
    _lib.check(on_device(plan.device, lambda st: lib.nvfp4_grouped_gemm(plan.table, len(abc), st)))
    return [c for _, _, c in abc]


def custom_kernel(data):
    """Reference task entry point; returns the list of outputs c_g."""
    abc, _sfab, sfab_perm, sizes = data
    return grouped_gemm(abc, sfab_perm, sizes)

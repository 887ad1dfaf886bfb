"""Drop-in ``custom_kernel`` for the NVFP4 dual GEMM task.

Same entry point, tuple and return value as the reference submissions
(nvfp4_dual_gemm/submission_v4.py:1256-1284): ``data`` is the 10-tuple of
nvfp4_dual_gemm/reference.py:196, the result is written into (and returned
as) its ``c``.  The kernels read a, b1, b2, the three permuted scale tensors
and c; the un-permuted scales are not needed.
"""
from __future__ import annotations

import threading
import weakref

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


def _validate(a, b1, b2, sfa_perm, sfb1_perm, sfb2_perm, c):
    """Check every tensor against the task layout; returns (m, n, k, l, device)."""
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
    return m, n, k, l, dev


# torch's raw current-device / current-stream queries cost ~0.1 us; the public
# torch.cuda.current_stream() builds a Stream object (~3 us per call, as much
# as a small kernel).  The public calls remain the fallback.
_get_device = getattr(torch._C, "_cuda_getDevice", None)
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _current_stream_handle(index: int) -> int:
    if _raw_stream is not None:
        return _raw_stream(index)
    return torch.cuda.current_stream(index).cuda_stream


def on_device(device: torch.device, launch):
    """Run launch(stream_handle) with `device` current (the library launches
    on the current device) and its current stream; the device switch is
    skipped when `device` is current already (the common case)."""
    cur = _get_device() if _get_device is not None else torch.cuda.current_device()
    if cur == device.index:
        return launch(_current_stream_handle(cur))
    with torch.cuda.device(device):
        return launch(_current_stream_handle(device.index))


class _Plan:
    """A validated call: weak references to the seven tensors the kernel
    reads or writes, their data pointers, shapes and strides, and the size
    arguments.  A later call with the same tensor objects, still at the same
    addresses with the same shapes and strides, skips re-validation."""

    def __init__(self, ts, sizes, device):
        self.refs = tuple(weakref.ref(t) for t in ts)
        self.sig = tuple((t.data_ptr(), t.shape, t.stride()) for t in ts)
        self.ptrs = tuple(s[0] for s in self.sig)
        self.sizes, self.device = sizes, device

    def matches(self, ts) -> bool:
        for t, r in zip(ts, self.refs):
            if t is not r():
                return False
        return tuple((t.data_ptr(), t.shape, t.stride()) for t in ts) == self.sig


_PLAN_SLOTS = 64        # >= the 15 rotating inputs of the reference's timing loop
_plans: dict = {}
_plans_lock = threading.Lock()   # host threads may insert concurrently; lookups need no lock


def clear_plan_cache() -> None:
    with _plans_lock:
        _plans.clear()


def dual_gemm(a, b1, b2, sfa_perm, sfb1_perm, sfb2_perm, c) -> torch.Tensor:
    """c[:, :, l] = silu(A_l . B1_lᵀ) * (A_l . B2_lᵀ) in fp16, on c's stream."""
    ts = (a, b1, b2, sfa_perm, sfb1_perm, sfb2_perm, c)
    key = tuple(id(t) for t in ts)
    plan = _plans.get(key)
    if plan is None or not plan.matches(ts):
        m, n, k, l, dev = _validate(*ts)
        plan = _Plan(ts, (m, n, k, l), dev)
        with _plans_lock:
            if len(_plans) >= _PLAN_SLOTS:
                _plans.pop(next(iter(_plans)))
            _plans[key] = plan
    m, n, k, l = plan.sizes
    lib = _lib.load()
    _lib.check(on_device(plan.device,
                         lambda st: lib.nvfp4_dual_gemm(*plan.ptrs, m, n, k, l, st)))
    return c


def custom_kernel(data):
    """Reference task entry point: data = (a, b1, b2, sfa, sfb1, sfb2,
    sfa_permuted, sfb1_permuted, sfb2_permuted, c); returns c."""
    a, b1, b2, _sfa, _sfb1, _sfb2, sfa_p, sfb1_p, sfb2_p, c = data
    return dual_gemm(a, b1, b2, sfa_p, sfb1_p, sfb2_p, c)

"""GPU: the allocation-free dual GEMM entry point, nvfp4_dual_gemm_noalloc.

Some callers cannot let a library allocate device memory while they run:
serving engines that hand the entire HBM budget to weights and KV caches
before the first request, and hosts whose own memory manager must own every
device byte.  For them the C ABI offers nvfp4_dual_gemm_noalloc, which keeps
its split-K partial sums in a fixed array inside the library instead of a
workspace grown with cudaMalloc.  These tests call it through the C ABI and
check it against the ordinary entry point, nvfp4_dual_gemm, on two calls in a
row (the array is shared by every call and keeps the previous call's
contents), within the tolerance the parity tests use.  This file is named to
be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from nvfp4_b200 import _lib
from nvfp4_b200 import build as B
from nvfp4_b200 import inputs as I
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2


def _call(fn, d, m, n, k, l):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), d[6].data_ptr(),
              d[7].data_ptr(), d[8].data_ptr(), d[9].data_ptr(), m, n, k, l, stream)


@pytest.fixture(scope="module")
def lib(cuda_device):
    B.build()
    return _lib.load()


def test_noalloc_matches_allocating_entry_point_two_calls(lib):
    # shapes with under a quarter as many 128x128 tiles as SMs (16 each), so
    # both calls split K (4 and 8 splits) and keep their partials in the
    # fixed array, the second call finding the first call's contents there
    shapes = [(256, 1024, 2048, 1), (128, 2048, 4096, 1)]
    for i, (m, n, k, l) in enumerate(shapes):
        d = I.generate_dual_input(m, n, k, l, seed=900 + i, device="cuda")
        _lib.check(_call(lib.nvfp4_dual_gemm, d, m, n, k, l))
        assert _lib.device_status() == 0
        want = d[9].clone()
        d[9].zero_()
        _lib.check(_call(lib.nvfp4_dual_gemm_noalloc, d, m, n, k, l))
        assert _lib.device_status() == 0
        bad, idx = O.allclose_report(d[9].cpu().numpy(), want.cpu().numpy(), RTOL, ATOL)
        assert bad == 0, f"call {i} ({m}x{n}x{k}): {bad} mismatches, first {idx[:3]}"


def test_noalloc_rejects_shapes_beyond_its_scratch(lib, monkeypatch):
    # 48 tiles forced into 16 splits need 96 MiB of partials: beyond the 20 MiB array
    monkeypatch.setenv("NVFP4_DUAL_SPLITS", "16")
    m, n, k, l = 256, 3072, 8192, 1
    d = I.generate_dual_input(m, n, k, l, seed=7, device="cuda")
    st = _call(lib.nvfp4_dual_gemm_noalloc, d, m, n, k, l)
    assert st == _lib.NVFP4_ERR_SHAPE
    assert b"no-alloc scratch" in lib.nvfp4_last_error()
    assert _lib.device_status() == 0

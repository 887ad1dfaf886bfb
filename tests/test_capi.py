"""CPU: the C-ABI library loads, exports every symbol include/nvfp4_b200.h
declares, and rejects bad arguments before touching a GPU; the Python
drop-ins validate the reference tuples."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from nvfp4_b200 import _lib
from nvfp4_b200 import build as B
from nvfp4_b200 import dual_gemm as D
from nvfp4_b200 import group_gemm as G
from nvfp4_b200 import inputs as I

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "nvfp4_b200.h"


@pytest.fixture(scope="module")
def lib():
    B.build()
    return _lib.load()


def header_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(
        r"^\s*(?:const\s+)?(?:(?:unsigned|signed|long|short)\s+)*\w+\**\s+\**(nvfp4_\w+)\s*\(", text, re.M)))


def test_header_declares_what_python_binds():
    assert header_functions() == sorted(_lib.EXPORTED)


def test_library_exports_every_header_symbol(lib):
    for name in header_functions():
        assert hasattr(lib, name), name


def test_version_and_status_strings(lib):
    assert lib.nvfp4_version() >= 100
    assert isinstance(lib.nvfp4_launch_count(), int)
    assert lib.nvfp4_status_string(0) == b"ok"
    assert lib.nvfp4_status_string(_lib.NVFP4_ERR_TIMEOUT) == b"device wait timed out"
    assert lib.nvfp4_status_string(-99) == b"unknown status"


def test_no_load_multicast_in_sources():
    """No TMA or bulk load with cluster multicast anywhere (the kernels run in
    multi-GPU jobs); the only multicast is tcgen05.commit's arrive."""
    for p in (ROOT / "blackwell-nvfp4-kernels_b200" / "csrc").glob("*"):
        for i, line in enumerate(p.read_text().splitlines(), 1):
            if "multicast::cluster" in line:
                assert "tcgen05.commit" in line, f"{p.name}:{i}: {line.strip()}"
            assert not ("cp.async.bulk" in line and "multicast" in line), f"{p.name}:{i}"


def test_dual_rejects_bad_arguments_without_gpu(lib):
    p = ctypes.c_void_p(4096)   # never dereferenced: validation fails first
    f = lib.nvfp4_dual_gemm
    assert f(None, p, p, p, p, p, p, 128, 128, 256, 1, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert f(p, p, p, p, p, p, p, 0, 128, 256, 1, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert f(p, p, p, p, p, p, p, 128, 128, 320, 1, None) == _lib.NVFP4_ERR_SHAPE
    assert b"256" in lib.nvfp4_last_error()
    assert f(p, p, p, p, p, p, p, 128, 100, 256, 1, None) == _lib.NVFP4_ERR_SHAPE
    q = ctypes.c_void_p(4096 + 8)
    assert f(p, q, p, p, p, p, p, 128, 128, 256, 1, None) == _lib.NVFP4_ERR_ALIGNMENT


def test_grouped_rejects_bad_arguments_without_gpu(lib):
    t = (_lib.Group * 2)()
    t[0] = _lib.Group(4096, 4096, 4096, 4096, 4096, 128, 128, 256, 1)
    t[1] = _lib.Group(4096, 4096, 4096, 4096, 4096, 128, 128, 300, 1)
    assert lib.nvfp4_grouped_gemm(t, 2, None) == _lib.NVFP4_ERR_SHAPE
    t[1] = _lib.Group(None, 4096, 4096, 4096, 4096, 64, 128, 256, 1)
    assert lib.nvfp4_grouped_gemm(t, 2, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert lib.nvfp4_grouped_gemm(None, 1, None) == _lib.NVFP4_ERR_INVALID_ARG
    # only empty groups: nothing to launch
    t[0] = _lib.Group(None, None, None, None, None, 0, 128, 256, 1)
    assert lib.nvfp4_grouped_gemm(t, 1, None) == _lib.NVFP4_OK


def test_grouped_rejects_operands_beyond_the_descriptor_range_without_gpu(lib):
    # M*N*L is small, but max(M, N)*K*L = 2^41 bytes-worth of K elements: the
    # same bound the dual entry point applies before encoding tensor maps
    t = (_lib.Group * 1)()
    t[0] = _lib.Group(4096, 4096, 4096, 4096, 4096, 1 << 20, 8, 1 << 21, 1)
    assert lib.nvfp4_grouped_gemm(t, 1, None) == _lib.NVFP4_ERR_SHAPE
    assert b"too large" in lib.nvfp4_last_error()
    t[0] = _lib.Group(4096, 4096, 4096, 4096, 4096, 8, 1 << 19, 1 << 20, 4)
    assert lib.nvfp4_grouped_gemm(t, 1, None) == _lib.NVFP4_ERR_SHAPE
    # same for the allocation-free dual entry point, which shares the dual validation
    p = ctypes.c_void_p(4096)
    assert lib.nvfp4_dual_gemm_noalloc(p, p, p, p, p, p, p, 1 << 20, 8, 1 << 21, 1, None) == \
        _lib.NVFP4_ERR_SHAPE


def test_quantize_rejects_bad_arguments_without_gpu(lib):
    p = ctypes.c_void_p(4096)
    f = lib.nvfp4_quantize
    assert f(None, 128, 64, 1, p, p, None, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert f(p, 128, 96, 1, p, p, None, None) == _lib.NVFP4_ERR_SHAPE
    assert f(p, 128, 64, 1, ctypes.c_void_p(4096 + 4), p, None, None) == _lib.NVFP4_ERR_ALIGNMENT
    assert f(p, 128, 64, 1, p, p, ctypes.c_void_p(4097), None) == _lib.NVFP4_ERR_ALIGNMENT


def test_check_raises_with_detail(lib):
    p = ctypes.c_void_p(4096)
    st = lib.nvfp4_dual_gemm(p, p, p, p, p, p, p, 128, 128, 320, 1, None)
    with pytest.raises(_lib.Nvfp4Error, match="multiple of 256"):
        _lib.check(st)


def test_python_dropin_validates_tuples():
    d = I.generate_dual_input(256, 128, 256, 1, seed=1, device="cpu")
    with pytest.raises(ValueError, match="CUDA"):
        D.custom_kernel(d)
    g = I.generate_group_input([64], [128], [256], 1, seed=1, device="cpu")
    with pytest.raises(ValueError, match="CUDA"):
        G.custom_kernel(g)


def test_sf_layout_validation():
    d = I.generate_dual_input(256, 128, 256, 1, seed=1, device="cpu")
    pa = d[6]
    D.check_sf_perm("sfa", pa, 256, 256, 1, pa.device)
    bad = pa.contiguous()   # logical-order contiguous: not the atom memory image
    with pytest.raises(ValueError, match="strides"):
        D.check_sf_perm("sfa", bad, 256, 256, 1, bad.device)


def test_moe_sizes_and_rejections_without_gpu(lib):
    # workspace: one int per (chunk of 1024 pairs, expert); scales: upper bound of 128-row blocks
    assert lib.nvfp4_moe_workspace_bytes(32768, 1, 64) == 32 * 64 * 4
    assert lib.nvfp4_moe_workspace_bytes(0, 1, 8) == 8 * 4
    assert lib.nvfp4_moe_sf_bytes(32768, 1, 7168, 64) == (256 + 64) * 112 * 512
    assert lib.nvfp4_moe_sf_bytes(3, 2, 64, 64) == (1 + 6) * 1 * 512
    p = ctypes.c_void_p(4096)
    ws = lib.nvfp4_moe_workspace_bytes(100, 2, 8)
    f = lib.nvfp4_moe_dispatch
    assert f(p, p, 100, 2, 100, 8, p, p, p, p, p, p, p, p, ws, None) == _lib.NVFP4_ERR_SHAPE
    assert f(p, p, 100, 2, 128, 2000, p, p, p, p, p, p, p, p, ws, None) == _lib.NVFP4_ERR_SHAPE
    assert f(p, p, 100, 0, 128, 8, p, p, p, p, p, p, p, p, ws, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert f(None, p, 100, 2, 128, 8, p, p, p, p, p, p, p, p, ws, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert f(p, p, 100, 2, 128, 8, p, p, p, p, p, p, p, p, ws - 4, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert b"workspace" in lib.nvfp4_last_error()
    q = ctypes.c_void_p(4096 + 4)
    assert f(q, p, 100, 2, 128, 8, p, p, p, p, p, p, p, p, ws, None) == _lib.NVFP4_ERR_ALIGNMENT
    g = lib.nvfp4_moe_combine
    assert g(p, 10, p, None, 10, 0, 64, p, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert g(p, -1, p, None, 10, 1, 64, p, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert g(None, 10, p, None, 10, 1, 64, p, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert g(p, 10, p, None, 0, 1, 64, p, None) == _lib.NVFP4_OK      # nothing to combine
    assert g(ctypes.c_void_p(4097), 10, p, None, 10, 1, 64, p, None) == _lib.NVFP4_ERR_ALIGNMENT


def test_moe_grouped_gemm_rejects_without_gpu(lib):
    p = ctypes.c_void_p(4096)
    arr = (ctypes.c_void_p * 2)(4096, 4096)
    f = lib.nvfp4_moe_grouped_gemm
    assert f(p, 100, p, p, p, p, arr, arr, 2, 256, 300, p, None) == _lib.NVFP4_ERR_SHAPE   # K % 256
    assert f(p, 100, p, p, p, p, arr, arr, 2, 250, 256, p, None) == _lib.NVFP4_ERR_SHAPE   # N % 8
    assert f(p, 100, p, p, p, p, arr, arr, 0, 256, 256, p, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert f(p, 0, p, p, p, p, arr, arr, 2, 256, 256, p, None) == _lib.NVFP4_OK       # no rows
    bad = (ctypes.c_void_p * 2)(4096, None)
    assert f(p, 100, p, p, p, p, arr, bad, 2, 256, 256, p, None) == _lib.NVFP4_ERR_INVALID_ARG
    assert f(ctypes.c_void_p(4100), 100, p, p, p, p, arr, arr, 2, 256, 256, p, None) == \
        _lib.NVFP4_ERR_ALIGNMENT

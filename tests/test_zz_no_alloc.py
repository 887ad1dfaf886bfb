"""GPU: the allocation-free dual GEMM entry point, nvfp4_dual_gemm_noalloc.

Some callers cannot let a library allocate device memory while they run:
serving engines that hand the entire HBM budget to weights and KV caches
before the first request, and hosts whose own memory manager must own every
device byte.  For them the C ABI offers nvfp4_dual_gemm_noalloc.  It makes
the same kernel and split choices as nvfp4_dual_gemm, but a K split that
exchanges partial sums through global memory keeps them in a fixed array
inside the library instead of a workspace grown with cudaMalloc.

These tests call it through the C ABI, twice in a row per shape (the array is
shared by every call and keeps the previous call's contents), and check each
result against the CPU oracle within the tolerance the parity tests use, and
bit for bit against the ordinary entry point.  The cases cover each branch of
the kernel choice: the CTA-pair kernel and the single-CTA kernel's cluster K
split (partials exchanged between CTAs, no array) under the automatic choice,
and, with the single-CTA kernel forced, its K split through the fixed array
and its unsplit path.  This file is named to be collected last.
"""
import numpy as np
import pytest
import torch

from nvfp4_b200 import _lib
from nvfp4_b200 import build as B
from nvfp4_b200 import inputs as I
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2

# (m, n, k, l, kernel knob, branch) -- the branch nvfp4_dual_gemm takes on a
# 148-SM B200 (knob None: the automatic choice)
SHAPES = [
    (128, 2048, 4096, 1, "single", "K split into 8 through the fixed array"),
    (128, 1024, 4608, 1, "single", "K split into 9 through the fixed array"),
    (512, 4096, 1024, 1, "single", "unsplit"),
    (256, 1024, 8192, 1, "single", "cluster K split (4 CTAs)"),
    (128, 5120, 12288, 1, None, "cluster K split (2 CTAs), automatic"),
    (256, 3072, 4096, 1, None, "CTA pair, 64-wide tiles"),
    (512, 3072, 2048, 1, None, "CTA pair, 128-wide tiles"),
]


def _call(fn, d, m, n, k, l):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), d[6].data_ptr(),
              d[7].data_ptr(), d[8].data_ptr(), d[9].data_ptr(), m, n, k, l, stream)


def _oracle(d):
    u8 = lambda t: t.detach().cpu().view(torch.uint8).numpy()
    return O.ref_dual_batched(*(u8(t) for t in d[:6]))


@pytest.fixture(scope="module")
def lib(cuda_device):
    B.build()
    return _lib.load()


@pytest.mark.parametrize("m,n,k,l,knob,branch", SHAPES, ids=[s[5] for s in SHAPES])
def test_noalloc_matches_oracle_two_calls(lib, m, n, k, l, knob, branch, monkeypatch):
    if knob:
        monkeypatch.setenv("NVFP4_DUAL_KERNEL", knob)
    d = I.generate_dual_input(m, n, k, l, seed=900 + m + n, device="cuda")
    want = _oracle(d)
    outs = []
    for call in range(2):
        d[9].fill_(float("nan"))
        _lib.check(_call(lib.nvfp4_dual_gemm_noalloc, d, m, n, k, l))
        assert _lib.device_status() == 0
        got = d[9].cpu().numpy()
        bad, idx = O.allclose_report(got, want, RTOL, ATOL)
        assert bad == 0, f"{branch}, call {call}: {bad} mismatches, first {idx[:3]}"
        outs.append(d[9].clone())
    # the same kernels in the same order as the allocating entry point
    d[9].zero_()
    _lib.check(_call(lib.nvfp4_dual_gemm, d, m, n, k, l))
    assert _lib.device_status() == 0
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], d[9])


def test_noalloc_rejects_shapes_beyond_its_scratch(lib, monkeypatch):
    # 48 tiles forced into 16 splits need 96 MiB of partials: beyond the 20 MiB array
    monkeypatch.setenv("NVFP4_DUAL_SPLITS", "16")
    m, n, k, l = 256, 3072, 8192, 1
    d = I.generate_dual_input(m, n, k, l, seed=7, device="cuda")
    st = _call(lib.nvfp4_dual_gemm_noalloc, d, m, n, k, l)
    assert st == _lib.NVFP4_ERR_SHAPE
    assert b"no-alloc scratch" in lib.nvfp4_last_error()
    assert _lib.device_status() == 0


_FIRST_CALL_CAPTURED = r"""
import sys, torch
sys.path[:0] = ["blackwell-nvfp4-kernels_b200", "."]
import os
os.environ["NVFP4_DUAL_KERNEL"] = "single"
from nvfp4_b200 import _lib, inputs as I
lib = _lib.load()
m, n, k = 128, 2048, 4096                     # K split through the fixed array
d = I.generate_dual_input(m, n, k, 1, seed=12, device="cuda")
args = lambda c: (d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), d[6].data_ptr(),
                  d[7].data_ptr(), d[8].data_ptr(), c.data_ptr(), m, n, k, 1,
                  torch.cuda.current_stream().cuda_stream)
graph = torch.cuda.CUDAGraph()
with torch.cuda.graph(graph):                 # this process's first no-alloc call
    _lib.check(lib.nvfp4_dual_gemm_noalloc(*args(d[9])))
d[9].zero_()
graph.replay()
torch.cuda.synchronize()
want = torch.zeros_like(d[9])
_lib.check(lib.nvfp4_dual_gemm(*args(want)))
torch.cuda.synchronize()
assert _lib.device_status() == 0
assert torch.equal(d[9], want), "captured no-alloc call differs"
del graph
print("ok")
"""


def test_first_noalloc_call_inside_a_graph_capture():
    """A fresh process whose first no-alloc call is captured into a CUDA graph
    (the library looks up its fixed array during the capture): the replay
    matches the ordinary entry point bit for bit."""
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    r = subprocess.run([sys.executable, "-c", _FIRST_CALL_CAPTURED], cwd=root, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), (r.stdout[-2000:], r.stderr[-2000:])

"""nvfp4_b200: B200-native (sm_100a) NVFP4 dual GEMM (SiLU-gated) and
grouped GEMM behind the kazim05/Blackwell-nvfp4-kernels ``custom_kernel``
task API.  The compute lives in libnvfp4_b200.so (C ABI in
include/nvfp4_b200.h); this package validates the reference tuples and calls
it through ctypes.

    from nvfp4_b200.dual_gemm import custom_kernel    # dual GEMM task
    from nvfp4_b200.group_gemm import custom_kernel   # grouped GEMM task
"""
from . import dual_gemm, formats, group_gemm, inputs, quantize  # noqa: F401
from ._lib import Nvfp4Error, device_status, load  # noqa: F401

__all__ = ["dual_gemm", "group_gemm", "formats", "inputs", "quantize", "load", "device_status",
           "Nvfp4Error"]

"""ctypes binding of libnvfp4_b200.so (declarations in include/nvfp4_b200.h).

There is no fallback: if the library is missing or fails to load, importing
the ops raises, and every call that the library rejects raises
``Nvfp4Error`` with the library's own message.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libnvfp4_b200.so"

NVFP4_OK = 0
NVFP4_ERR_INVALID_ARG = -1
NVFP4_ERR_SHAPE = -2
NVFP4_ERR_ALIGNMENT = -3
NVFP4_ERR_CUDA = -4
NVFP4_ERR_DEVICE = -5
NVFP4_ERR_TIMEOUT = -6

# every symbol include/nvfp4_b200.h declares
EXPORTED = (
    "nvfp4_dual_gemm",
    "nvfp4_dual_gemm_noalloc",
    "nvfp4_grouped_gemm",
    "nvfp4_quantize",
    "nvfp4_moe_dispatch",
    "nvfp4_moe_workspace_bytes",
    "nvfp4_moe_sf_bytes",
    "nvfp4_moe_combine",
    "nvfp4_moe_grouped_gemm",
    "nvfp4_device_status",
    "nvfp4_wait_selftest",
    "nvfp4_status_string",
    "nvfp4_last_error",
    "nvfp4_version",
    "nvfp4_launch_count",
)


class Nvfp4Error(RuntimeError):
    def __init__(self, status: int, detail: str):
        super().__init__(f"nvfp4 status {status}: {detail}")
        self.status = status


class Group(ctypes.Structure):
    """struct nvfp4_group."""
    _fields_ = [
        ("a", ctypes.c_void_p),
        ("b", ctypes.c_void_p),
        ("sfa_perm", ctypes.c_void_p),
        ("sfb_perm", ctypes.c_void_p),
        ("c", ctypes.c_void_p),
        ("m", ctypes.c_int32),
        ("n", ctypes.c_int32),
        ("k", ctypes.c_int32),
        ("l", ctypes.c_int32),
    ]


_lib = None


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with argument types declared."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"{p} is missing: build it with `python -m nvfp4_b200.build` "
            "(the CUDA kernels have no CPU fallback)")
    lib = ctypes.CDLL(str(p))
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    lib.nvfp4_dual_gemm.argtypes = [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]
    lib.nvfp4_dual_gemm.restype = i32
    lib.nvfp4_dual_gemm_noalloc.argtypes = [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]
    lib.nvfp4_dual_gemm_noalloc.restype = i32
    lib.nvfp4_grouped_gemm.argtypes = [ctypes.POINTER(Group), i32, vp]
    lib.nvfp4_grouped_gemm.restype = i32
    lib.nvfp4_quantize.argtypes = [vp, i32, i32, i32, vp, vp, vp, vp]
    lib.nvfp4_quantize.restype = i32
    sz = ctypes.c_size_t
    lib.nvfp4_moe_dispatch.argtypes = [vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp,
                                       vp, sz, vp]
    lib.nvfp4_moe_dispatch.restype = i32
    lib.nvfp4_moe_workspace_bytes.argtypes = [i32, i32, i32]
    lib.nvfp4_moe_workspace_bytes.restype = sz
    lib.nvfp4_moe_sf_bytes.argtypes = [i32, i32, i32, i32]
    lib.nvfp4_moe_sf_bytes.restype = sz
    lib.nvfp4_moe_combine.argtypes = [vp, i32, vp, vp, i32, i32, i32, vp, vp]
    lib.nvfp4_moe_combine.restype = i32
    pp = ctypes.POINTER(ctypes.c_void_p)
    lib.nvfp4_moe_grouped_gemm.argtypes = [vp, i32, vp, vp, vp, vp, pp, pp, i32, i32, i32, vp, vp]
    lib.nvfp4_moe_grouped_gemm.restype = i32
    lib.nvfp4_device_status.argtypes = [vp, ctypes.POINTER(ctypes.c_uint)]
    lib.nvfp4_device_status.restype = i32
    lib.nvfp4_wait_selftest.argtypes = [ctypes.c_longlong, vp]
    lib.nvfp4_wait_selftest.restype = i32
    lib.nvfp4_status_string.argtypes = [i32]
    lib.nvfp4_status_string.restype = ctypes.c_char_p
    lib.nvfp4_last_error.argtypes = []
    lib.nvfp4_last_error.restype = ctypes.c_char_p
    lib.nvfp4_version.argtypes = []
    lib.nvfp4_version.restype = i32
    lib.nvfp4_launch_count.argtypes = []
    lib.nvfp4_launch_count.restype = ctypes.c_ulonglong
    if path is None:
        _lib = lib
    return lib


def check(status: int) -> None:
    """Raise Nvfp4Error for a non-zero status, with the library's detail."""
    if status != NVFP4_OK:
        lib = load()
        detail = lib.nvfp4_last_error().decode() or lib.nvfp4_status_string(status).decode()
        raise Nvfp4Error(status, detail)


def device_status(stream: int | None = None) -> int:
    """Synchronise `stream` and return (and clear) the device status bits."""
    bits = ctypes.c_uint(0)
    st = load().nvfp4_device_status(stream, ctypes.byref(bits))
    if st not in (NVFP4_OK, NVFP4_ERR_TIMEOUT):
        check(st)
    return int(bits.value)

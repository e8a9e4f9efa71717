"""ctypes binding of ``libpiper_merge.so`` (the sm_100a C ABI in ``include/piper_merge.h``).

The library is loaded from this package directory. There is no fallback: if
the shared object is missing or fails to load, every merge raises
``RuntimeError`` so that a GPU run can never silently take another path.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_NAME = "libpiper_merge.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

# Status codes (include/piper_merge.h).
OK = 0
EINVAL = 1
ECUDA = 2
EWORKSPACE = 3
ETIMEOUT = 4

# Formats.
FMT_MXFP8_E4M3 = 0
FMT_MXFP8_E5M2 = 1
FMT_MXFP4 = 2
FMT_NVFP4 = 3
FMT_FP8_E4M3 = 4
FMT_FP8_E5M2 = 5
FMT_INT8 = 6
FMT_GGUF_Q8_0 = 7
FMT_GGUF_Q4_0 = 8
FMT_BNB8 = 9
FMT_QUANTO_INT8 = 10
FMT_QUANTO_FP8_E4M3 = 11
FMT_QUANTO_FP8_E5M2 = 12
FMT_BNB4_NF4 = 13
FMT_BNB4_FP4 = 14

DT_BF16 = 0
DT_F16 = 1
DT_F32 = 2

FLAG_SWIZZLED = 1
FLAG_ASYMMETRIC = 2
FLAG_REDUCE_RANGE = 4
FLAG_STOCHASTIC = 8

# Weights packed into one kernel launch at most (their descriptors fill the
# kernel's parameter space); larger batches take several launches.
MAX_WEIGHTS_PER_LAUNCH = 48

EXPORTED_SYMBOLS = (
    "piper_merge_workspace_size",
    "piper_merge_batch",
    "piper_merge_mx",
    "piper_merge_nvfp4",
    "piper_merge_float8",
    "piper_merge_float8_noalloc",
    "piper_merge_int8",
    "piper_merge_gguf",
    "piper_merge_static_float8",
    "piper_merge_bnb8",
    "piper_merge_quanto",
    "piper_merge_bnb4",
    "piper_merge_last_error",
    "piper_merge_device_status",
    "piper_merge_version",
    "piper_merge_launches",
    "piper_merge_selftest_timeout",
)


class MergeDesc(ctypes.Structure):
    """Mirror of ``piper_merge_desc``."""

    _fields_ = [
        ("qdata", ctypes.c_void_p),
        ("scale", ctypes.c_void_p),
        ("zero_point", ctypes.c_void_p),
        ("global_scale", ctypes.c_void_p),
        ("b", ctypes.c_void_p),
        ("a", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("rank", ctypes.c_int64),
        ("block_rows", ctypes.c_int64),
        ("block_cols", ctypes.c_int64),
        ("format", ctypes.c_int32),
        ("compute_dtype", ctypes.c_int32),
        ("scale_dtype", ctypes.c_int32),
        ("scale_mode", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("strength", ctypes.c_float),
        ("seed", ctypes.c_uint64),
        ("offset_base", ctypes.c_uint64),
        ("codebook", ctypes.c_void_p),
        ("nested_absmax", ctypes.c_void_p),
        ("nested_code", ctypes.c_void_p),
        ("nested_offset", ctypes.c_void_p),
    ]


_lib = None
_lock = threading.Lock()


def library_path() -> Path:
    return Path(os.environ.get("PIPER_MERGE_LIB", LIB_PATH))


def load() -> ctypes.CDLL:
    """Load the native library (once) and declare its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"native merge library {path} is missing; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` (there is no CPU fallback)."
            )
        lib = ctypes.CDLL(str(path))
        vp, i32, i64, u64, f32, sz = (
            ctypes.c_void_p,
            ctypes.c_int32,
            ctypes.c_int64,
            ctypes.c_uint64,
            ctypes.c_float,
            ctypes.c_size_t,
        )
        lib.piper_merge_workspace_size.argtypes = [ctypes.POINTER(MergeDesc), i32, ctypes.POINTER(sz)]
        lib.piper_merge_batch.argtypes = [ctypes.POINTER(MergeDesc), i32, vp, sz, vp]
        lib.piper_merge_mx.argtypes = [vp, vp, vp, vp, i64, i64, i64, i32, i32, i32, i32, f32, i32, u64, u64, vp]
        lib.piper_merge_nvfp4.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i32, i32, f32, i32, u64, u64, vp, sz, vp]
        lib.piper_merge_float8.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64, i32, i32, f32, i32, u64, u64, vp, sz, vp]
        lib.piper_merge_int8.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i32, i32, i32, i32, f32, i32, u64, u64, vp, sz, vp]
        lib.piper_merge_gguf.argtypes = [vp, vp, vp, i64, i64, i64, i32, i32, f32, i32, u64, u64, vp]
        lib.piper_merge_static_float8.argtypes = [vp, vp, vp, vp, i64, i64, i64, i32, i32, f32, i32, u64, u64, vp, sz, vp]
        lib.piper_merge_bnb8.argtypes = [vp, vp, vp, vp, i64, i64, i64, f32, i32, u64, u64, vp]
        lib.piper_merge_quanto.argtypes = [vp, vp, vp, vp, i64, i64, i64, i32, i32, i32, f32, i32, u64, u64, vp, sz, vp]
        lib.piper_merge_bnb4.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i32, i32, f32, i32, u64, u64,
                                         vp, sz, vp]
        lib.piper_merge_last_error.restype = ctypes.c_char_p
        lib.piper_merge_last_error.argtypes = []
        lib.piper_merge_device_status.argtypes = [vp, ctypes.POINTER(ctypes.c_uint32)]
        lib.piper_merge_version.restype = ctypes.c_char_p
        lib.piper_merge_launches.restype = ctypes.c_uint64
        lib.piper_merge_launches.argtypes = []
        for name in (
            "piper_merge_workspace_size",
            "piper_merge_batch",
            "piper_merge_mx",
            "piper_merge_nvfp4",
            "piper_merge_float8",
            "piper_merge_float8_noalloc",
            "piper_merge_int8",
            "piper_merge_gguf",
            "piper_merge_static_float8",
            "piper_merge_bnb8",
            "piper_merge_quanto",
            "piper_merge_bnb4",
            "piper_merge_device_status",
            "piper_merge_selftest_timeout",
        ):
            getattr(lib, name).restype = ctypes.c_int
        _lib = lib
        return lib


def check(rc: int) -> None:
    """Raise the reference's exception type for a nonzero status."""
    if rc == OK:
        return
    msg = load().piper_merge_last_error().decode("utf-8", "replace")
    if rc == EINVAL:
        raise ValueError(msg)
    raise RuntimeError(f"piper merge failed (status {rc}): {msg}")


def current_stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def workspace_bytes(descs: list[MergeDesc]) -> int:
    arr = (MergeDesc * len(descs))(*descs)
    out = ctypes.c_size_t(0)
    check(load().piper_merge_workspace_size(arr, len(descs), ctypes.byref(out)))
    return int(out.value)


def merge_batch(descs: list[MergeDesc], device: torch.device, workspace: torch.Tensor | None = None) -> None:
    """Run ``piper_merge_batch`` on the current stream of ``device``.

    The workspace is taken from PyTorch's caching allocator on that stream when
    not supplied, so it is recycled safely in stream order.
    """
    if not descs:
        return
    lib = load()
    arr = (MergeDesc * len(descs))(*descs)
    need = ctypes.c_size_t(0)
    check(lib.piper_merge_workspace_size(arr, len(descs), ctypes.byref(need)))
    ws_ptr = None
    ws_len = 0
    if need.value > 0:
        if workspace is None or workspace.numel() < need.value:
            workspace = torch.empty(int(need.value) + 256, dtype=torch.uint8, device=device)
        ptr = workspace.data_ptr()
        aligned = (ptr + 255) // 256 * 256
        ws_ptr = aligned
        ws_len = workspace.numel() - (aligned - ptr)
    with torch.cuda.device(device):
        rc = lib.piper_merge_batch(arr, len(descs), ws_ptr, ws_len, current_stream_handle(device))
    check(rc)


def device_status(device: torch.device) -> int:
    """Read and clear the device-side status word (synchronises the current stream)."""
    lib = load()
    out = ctypes.c_uint32(0)
    with torch.cuda.device(device):
        rc = lib.piper_merge_device_status(current_stream_handle(device), ctypes.byref(out))
    if rc not in (OK, ETIMEOUT):
        check(rc)
    return int(out.value)


def version() -> str:
    return load().piper_merge_version().decode()


def launches() -> int:
    """Merge kernels launched by this process so far."""
    return int(load().piper_merge_launches())

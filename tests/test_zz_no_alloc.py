"""GPU: ``piper_merge_float8_noalloc`` (the workspace-free FP8 entry point,
called through the C ABI) gives the same codes and scales as
``piper_merge_float8`` with a caller's workspace, over two merges in a row,
and rejects a layout larger than its static scratch before launching
anything. It is for callers that cannot allocate device memory when they
merge (a C/C++ host without PyTorch's caching allocator, or a process whose
device memory is already reserved by a model cache).

Every case here goes through the static scratch array: per-tensor scales and
512-column groups always do, and the per-row weights (300 and 70 rows) are too
small to fill the GPU with whole 128-row strips, so they split their columns
over the reduce / encode launches, whose row maxima live in the scratch. (A
per-row weight with at least two strips per SM runs the one-launch fused pass
and needs none.) Collected last so it also runs after every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from piper_offload_b200 import _native as nat
from piper_offload_b200 import synthetic as S

pytestmark = pytest.mark.gpu

_c_p, _c_i64, _c_i32, _c_u64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_uint64


def _bind():
    lib = nat.load()
    fn = lib.piper_merge_float8_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [_c_p, _c_p, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_i32,
                   ctypes.c_float, _c_i32, _c_u64, _c_u64, _c_p]
    ref = lib.piper_merge_float8
    ref.restype = ctypes.c_int
    ref.argtypes = [_c_p, _c_p, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_i32,
                    ctypes.c_float, _c_i32, _c_u64, _c_u64, _c_p, ctypes.c_size_t, _c_p]
    return fn, ref


@pytest.mark.parametrize("seed", [None, 0x9C3EA68DBAC91AAD])
@pytest.mark.parametrize("rows,cols,layout", [(300, 512, "row"), (70, 130, "row"), (256, 1024, "tensor"),
                                             (200, 1024, "group512")])
def test_noalloc_matches_workspace_entry(cuda_device, seed, rows, cols, layout):
    fn, ref = _bind()
    w = S.normal((rows, cols), 0.02, seed=rows + cols, device=cuda_device)
    if layout == "group512":
        q = S.quantize_fp8(w, group=512)
        block = (1, 512)
    else:
        q = S.quantize_fp8(w, per_tensor=layout == "tensor")
        block = (1, cols) if layout == "row" else (rows, cols)
    b, a = S.lora_factors(rows, cols, 16, 0.01, seed=rows * 3 + 1, device=cuda_device)
    ref_q, ref_s = q.qdata.clone(), q.scale.clone()
    new_q, new_s = q.qdata.clone(), q.scale.clone()
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device=cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    has_seed = 0 if seed is None else 1
    for step in range(2):
        sd = 0 if seed is None else (seed + step) % (1 << 64)
        rc = ref(ref_q.data_ptr(), ref_s.data_ptr(), b.data_ptr(), a.data_ptr(), rows, cols, 16, block[0], block[1],
                 0, nat.DT_BF16, 1.0, has_seed, sd, 0, ws.data_ptr(), ws.numel(), stream)
        assert rc == 0, nat.load().piper_merge_last_error()
        rc = fn(new_q.data_ptr(), new_s.data_ptr(), b.data_ptr(), a.data_ptr(), rows, cols, 16, block[0], block[1],
                0, nat.DT_BF16, 1.0, has_seed, sd, 0, stream)
        assert rc == 0, nat.load().piper_merge_last_error()
    torch.cuda.synchronize(cuda_device)
    assert nat.device_status(cuda_device) == 0
    # Same kernels on the same inputs: identical results (tolerance: exact).
    assert torch.equal(ref_q.view(torch.uint8), new_q.view(torch.uint8))
    assert torch.equal(ref_s, new_s)


def test_noalloc_rejects_layout_beyond_static_scratch(cuda_device):
    fn, _ = _bind()
    # Groups of 512 columns are wider than a tile, so their maxima go through
    # the scratch: 70,000 rows x 2 groups = 140,000 quantization blocks > 65,536.
    rows, cols, group = 70000, 1024, 512
    q = torch.zeros((rows, cols), dtype=torch.uint8, device=cuda_device)
    s = torch.ones((rows, cols // group), dtype=torch.float32, device=cuda_device)
    b = torch.zeros((rows, 16), dtype=torch.bfloat16, device=cuda_device)
    a = torch.zeros((16, cols), dtype=torch.bfloat16, device=cuda_device)
    before = q.clone()
    rc = fn(q.data_ptr(), s.data_ptr(), b.data_ptr(), a.data_ptr(), rows, cols, 16, 1, group, 0, nat.DT_BF16, 1.0,
            0, 0, 0, torch.cuda.current_stream(cuda_device).cuda_stream)
    assert rc == nat.EWORKSPACE
    assert b"static scratch" in nat.load().piper_merge_last_error()
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(q, before)


# Child process for the context test below. It drives CUDA through the driver
# API only (no torch CUDA state), so it can create and destroy contexts freely:
# in each of two non-primary contexts, created one after the other, it merges
# the same inputs twice with the workspace entry point and twice with the
# workspace-free one, and requires identical codes and scales. A second
# context holds its own copy of the static scratch array, so the entry point
# has to find that copy's address again; a stale address from the first
# context would not be this context's memory.
_CONTEXT_CHILD = r'''
import ctypes, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
from piper_offload_b200 import synthetic as S
lib = ctypes.CDLL(sys.argv[2])
cu = ctypes.CDLL("libcuda.so.1")
P, I64, I32, U64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_uint64
lib.piper_merge_float8.argtypes = [P, P, P, P, I64, I64, I64, I64, I64, I32, I32, ctypes.c_float, I32, U64, U64,
                                   P, ctypes.c_size_t, P]
lib.piper_merge_float8_noalloc.argtypes = [P, P, P, P, I64, I64, I64, I64, I64, I32, I32, ctypes.c_float, I32,
                                           U64, U64, P]
lib.piper_merge_last_error.restype = ctypes.c_char_p
DPTR = ctypes.c_ulonglong
cu.cuMemAlloc_v2.argtypes = [ctypes.POINTER(DPTR), ctypes.c_size_t]
cu.cuMemFree_v2.argtypes = [DPTR]
cu.cuMemcpyHtoD_v2.argtypes = [DPTR, P, ctypes.c_size_t]
cu.cuMemcpyDtoH_v2.argtypes = [P, DPTR, ctypes.c_size_t]
cu.cuCtxCreate_v2.argtypes = [ctypes.POINTER(P), ctypes.c_uint, ctypes.c_int]
cu.cuCtxDestroy_v2.argtypes = [P]

def ck(r, what):
    if r != 0:
        raise SystemExit(f"{what} failed: CUresult {r}")

ck(cu.cuInit(0), "cuInit")
dev = ctypes.c_int(0)
ck(cu.cuDeviceGet(ctypes.byref(dev), 0), "cuDeviceGet")
rows, cols, rank = 256, 1024, 16
w = S.normal((rows, cols), 0.02, seed=5, device="cpu")
q = S.quantize_fp8(w, per_tensor=True)
b, a = S.lora_factors(rows, cols, rank, 0.01, seed=6, device="cpu")
host = {"q": q.qdata.view(torch.uint8).numpy().copy(), "s": q.scale.numpy().copy(),
        "b": b.view(torch.int16).numpy().copy(), "a": a.view(torch.int16).numpy().copy()}

def upload(arr):
    p = DPTR()
    ck(cu.cuMemAlloc_v2(ctypes.byref(p), arr.nbytes), "cuMemAlloc")
    ck(cu.cuMemcpyHtoD_v2(p, arr.ctypes.data, arr.nbytes), "cuMemcpyHtoD")
    return p

def download(p, like):
    out = np.empty_like(like)
    ck(cu.cuMemcpyDtoH_v2(out.ctypes.data, p, out.nbytes), "cuMemcpyDtoH")
    return out

for ctx_no in range(2):
    ctx = P()
    ck(cu.cuCtxCreate_v2(ctypes.byref(ctx), 0, dev), "cuCtxCreate")
    bufs = {k: upload(v) for k, v in host.items()}
    ref_q, ref_s = upload(host["q"]), upload(host["s"])
    ws = DPTR()
    ck(cu.cuMemAlloc_v2(ctypes.byref(ws), 1 << 20), "cuMemAlloc")
    for step in range(2):
        seed = 0x9C3EA68DBAC91AAD + step
        rc = lib.piper_merge_float8(ref_q.value, ref_s.value, bufs["b"].value, bufs["a"].value, rows, cols, rank,
                                    rows, cols, 0, 0, 1.0, 1, seed, 0, ws.value, 1 << 20, None)
        assert rc == 0, lib.piper_merge_last_error()
        rc = lib.piper_merge_float8_noalloc(bufs["q"].value, bufs["s"].value, bufs["b"].value, bufs["a"].value,
                                            rows, cols, rank, rows, cols, 0, 0, 1.0, 1, seed, 0, None)
        assert rc == 0, lib.piper_merge_last_error()
    ck(cu.cuCtxSynchronize(), "cuCtxSynchronize")
    got_q, got_s = download(bufs["q"], host["q"]), download(bufs["s"], host["s"])
    want_q, want_s = download(ref_q, host["q"]), download(ref_s, host["s"])
    assert np.array_equal(got_q, want_q), f"context {ctx_no}: codes differ"
    assert np.array_equal(got_s.view(np.uint32), want_s.view(np.uint32)), f"context {ctx_no}: scales differ"
    assert not np.array_equal(got_q, host["q"]), f"context {ctx_no}: nothing merged"
    for p in list(bufs.values()) + [ref_q, ref_s, ws]:
        ck(cu.cuMemFree_v2(p), "cuMemFree")
    ck(cu.cuCtxDestroy_v2(ctx), "cuCtxDestroy")
print("contexts ok")
'''


def test_noalloc_in_successive_contexts(cuda_device, tmp_path):
    """The workspace-free entry point in two non-primary CUDA contexts, one
    created after the other was destroyed, matches the workspace entry point
    in each (run in a child process that owns its contexts)."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = tmp_path / "contexts.py"
    script.write_text(_CONTEXT_CHILD)
    env = dict(os.environ)
    env.setdefault("CUDA_VISIBLE_DEVICES", str(cuda_device.index or 0))
    proc = subprocess.run([sys.executable, str(script), root, str(nat.library_path())], capture_output=True,
                          text=True, timeout=300, env=env)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "contexts ok" in proc.stdout

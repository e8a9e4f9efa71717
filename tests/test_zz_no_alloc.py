"""GPU: ``piper_merge_float8_noalloc`` (the workspace-free FP8 entry point,
called through the C ABI) gives the same codes and scales as
``piper_merge_float8`` with a caller's workspace, over two merges in a row,
and rejects a layout larger than its static scratch before launching
anything. Collected last so it also runs after every other test.
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

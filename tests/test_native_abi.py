"""CPU: the C-ABI library loads, exports every declared symbol, and rejects bad
arguments before touching the device."""

from __future__ import annotations

import contextlib
import ctypes
import re
from pathlib import Path

import pytest
import torch

from piper_offload_b200 import _native as nat

HEADER = Path(__file__).resolve().parents[1] / "include" / "piper_merge.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(piper_merge_\w+)\s*\(", text)))


def test_library_loads_and_exports_all_declared_symbols():
    lib = nat.load()
    names = declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name
    assert set(nat.EXPORTED_SYMBOLS) == set(names)


def test_version_string():
    assert "sm_100a" in nat.version()


def _desc(**kw) -> nat.MergeDesc:
    d = nat.MergeDesc()
    d.qdata = 0x1000
    d.b = 0x2000
    d.a = 0x3000
    d.scale = 0x4000
    d.rows, d.cols, d.rank = 64, 256, 16
    d.compute_dtype = nat.DT_BF16
    d.format = nat.FMT_FP8_E4M3
    d.block_rows, d.block_cols = 1, 256
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize(
    "kw,match",
    [
        ({"rows": 0}, "non-empty"),
        ({"rank": 300}, "rank above 256"),
        ({"format": 99}, "unknown format"),
        ({"compute_dtype": 7}, "float16, bfloat16, and float32"),
        ({"block_rows": 3, "block_cols": 7}, "per-group"),
        ({"format": nat.FMT_MXFP8_E4M3, "cols": 100}, "divisible by 32"),
        ({"format": nat.FMT_MXFP8_E4M3, "scale_mode": 9}, "scaling mode"),
        ({"format": nat.FMT_NVFP4, "cols": 40}, "divisible by 16"),
        ({"format": nat.FMT_GGUF_Q8_0, "cols": 48}, "divisible by 32"),
        ({"format": nat.FMT_INT8, "scale_dtype": 7}, "scales"),
        ({"qdata": None}, "null"),
    ],
)
def test_invalid_descriptors_are_rejected_on_host(kw, match):
    d = _desc(**kw)
    with pytest.raises(ValueError, match=match):
        nat.workspace_bytes([d])
    arr = (nat.MergeDesc * 1)(d)
    rc = nat.load().piper_merge_batch(arr, 1, None, 0, None)
    assert rc == nat.EINVAL


@pytest.mark.parametrize("fmt,extra", [
    (nat.FMT_FP8_E4M3, {}), (nat.FMT_INT8, {"scale_dtype": nat.DT_BF16}), (nat.FMT_MXFP8_E4M3, {}),
    (nat.FMT_MXFP4, {}), (nat.FMT_NVFP4, {}), (nat.FMT_GGUF_Q8_0, {}),
])
def test_fp32_factors_are_accepted_on_host(fmt, extra):
    """fp32 LoRA factors pass the host checks as the reference launchers accept
    them (_triton_float8_lora.py:311-318, _triton_mx_lora.py:311-316,
    _triton_nvfp4_lora.py:370-375)."""
    assert nat.workspace_bytes([_desc(format=fmt, compute_dtype=nat.DT_F32, **extra)]) >= 0


def test_workspace_sizes():
    assert nat.workspace_bytes([_desc(format=nat.FMT_MXFP8_E4M3)]) == 0
    # A per-row weight too small to fill the GPU with whole 128-row strips asks
    # for 16 bytes per row (column-split reduce / encode launches) ...
    assert nat.workspace_bytes([_desc()]) == 64 * 16
    # ... which is optional: with no workspace the fused launch runs (checked
    # on the GPU); enough strips for two per SM keep their maxima on chip.
    assert nat.workspace_bytes([_desc(rows=128 * 2 * 148)]) == 0
    # groups wider than a tile: 64 rows x 2 blocks x 16 bytes
    assert nat.workspace_bytes([_desc(cols=1024, block_cols=512)]) == 2048
    per_tensor = nat.workspace_bytes([_desc(block_rows=64, block_cols=256)])
    assert per_tensor == 256
    grouped_local = nat.workspace_bytes([_desc(block_cols=64)])
    assert grouped_local == 0
    two = nat.workspace_bytes([_desc(cols=1024, block_cols=512), _desc(block_rows=64, block_cols=256)])
    assert two == 2048 + 256
    # several small per-row weights together still fill fewer than two strips per SM
    assert nat.workspace_bytes([_desc(), _desc(rows=300)]) == 64 * 16 + (300 * 16 + 255) // 256 * 256  # 256-byte aligned


def test_workspace_too_small_is_reported():
    # A per-tensor layout needs workspace; the call is rejected before any launch.
    d = _desc(block_rows=64, block_cols=256)
    arr = (nat.MergeDesc * 1)(d)
    rc = nat.load().piper_merge_batch(arr, 1, ctypes.c_void_p(0x100000), 16, None)
    assert rc == nat.EWORKSPACE
    assert b"workspace" in nat.load().piper_merge_last_error()


def test_convenience_entry_points_validate():
    lib = nat.load()
    assert lib.piper_merge_mx(1, 1, 1, 1, 32, 64, 16, 5, 0, 0, 0, 1.0, 0, 0, 0, None) == nat.EINVAL
    assert lib.piper_merge_gguf(1, 1, 1, 32, 64, 16, 3, 0, 1.0, 0, 0, 0, None) == nat.EINVAL
    assert lib.piper_merge_float8(1, 1, 1, 1, 0, 64, 16, 1, 64, 0, 0, 1.0, 0, 0, 0, None, 0, None) == nat.EINVAL
    # new formats: argument errors are reported before anything is enqueued
    assert lib.piper_merge_static_float8(1, 1, 1, 1, 0, 64, 16, 0, 0, 1.0, 0, 0, 0, None, 0, None) == nat.EINVAL
    assert lib.piper_merge_quanto(1, 1, 1, 1, 32, 64, 16, 3, 1, 0, 1.0, 0, 0, 0, None, 0, None) == nat.EINVAL
    assert b"storage" in lib.piper_merge_last_error()
    assert lib.piper_merge_bnb8(1, 1, 1, 1, 32, 64, 0, 1.0, 0, 0, 0, None) == nat.EINVAL


def test_bnb4_validation_messages():
    lib = nat.load()
    size = ctypes.c_size_t()
    d = _desc(format=nat.FMT_BNB4_NF4, cols=96, codebook=0x5000)
    assert lib.piper_merge_workspace_size((nat.MergeDesc * 1)(d), 1, ctypes.byref(size)) == nat.EINVAL
    assert b"64-value blocks" in lib.piper_merge_last_error()
    d = _desc(format=nat.FMT_BNB4_FP4, codebook=0x5000, nested_absmax=0x6000, nested_code=0x7000,
              nested_offset=0x8000, flags=nat.FLAG_STOCHASTIC)
    assert lib.piper_merge_workspace_size((nat.MergeDesc * 1)(d), 1, ctypes.byref(size)) == nat.EINVAL
    assert b"nested" in lib.piper_merge_last_error()
    d = _desc(format=nat.FMT_BNB4_NF4, codebook=0x5000, nested_absmax=0x6000, nested_code=0x7000,
              nested_offset=0x8000)
    # raw block maxima for the nested pass, then 64 fp64 partial sums of their mean (256-byte aligned)
    assert nat.workspace_bytes([d]) == (64 * 256 // 64 * 4 + 130 * 4 + 255) // 256 * 256
    assert nat.workspace_bytes([_desc(format=nat.FMT_BNB4_NF4, codebook=0x5000)]) == 0


def test_new_format_validation_messages():
    # bitsandbytes: fp16 factors only; Quanto: per-row or per-tensor only.
    d = _desc(format=nat.FMT_BNB8, compute_dtype=nat.DT_BF16, block_rows=1, block_cols=256)
    assert nat.load().piper_merge_workspace_size((nat.MergeDesc * 1)(d), 1, ctypes.byref(ctypes.c_size_t())) == nat.EINVAL
    assert b"float16" in nat.load().piper_merge_last_error()
    d = _desc(format=nat.FMT_QUANTO_INT8, block_rows=1, block_cols=64)
    assert nat.load().piper_merge_workspace_size((nat.MergeDesc * 1)(d), 1, ctypes.byref(ctypes.c_size_t())) == nat.EINVAL
    assert b"last axis" in nat.load().piper_merge_last_error()
    # last-axis scales: one workspace slot (16 B) per column
    assert nat.workspace_bytes([_desc(format=nat.FMT_QUANTO_INT8, block_rows=64, block_cols=1)]) == 256 * 16
    # per-tensor Quanto and static FP8 take the two-pass workspace; a per-row
    # weight needs none once it has two 128-row strips per SM (a small one asks
    # for the optional 16 bytes per row); bitsandbytes 8-bit has the fused pass only
    assert nat.workspace_bytes([_desc(format=nat.FMT_QUANTO_FP8_E4M3, block_rows=64, block_cols=256)]) == 256
    assert nat.workspace_bytes([_desc(format=nat.FMT_QUANTO_INT8, block_rows=1, block_cols=256)]) == 64 * 16
    assert nat.workspace_bytes([_desc(format=nat.FMT_QUANTO_INT8, rows=128 * 2 * 148, block_rows=1,
                                      block_cols=256)]) == 0
    assert nat.workspace_bytes([_desc(format=nat.FMT_BNB8, compute_dtype=nat.DT_F16, block_rows=1,
                                      block_cols=256)]) == 0


class _FailingLib:
    """Stands in for the C-ABI library: validation succeeds, the launch reports a CUDA error."""

    def piper_merge_workspace_size(self, arr, count, out):
        return nat.OK

    def piper_merge_batch(self, arr, count, ws, ws_bytes, stream):
        return nat.ECUDA

    def piper_merge_last_error(self):
        return b"injected launch failure"


def test_injected_launch_error_raises_and_mutates_nothing(monkeypatch):
    # merge_batch surfaces a failing C-ABI return as RuntimeError with the
    # library's message; the (CPU) storages handed in are untouched.
    monkeypatch.setattr(nat, "load", lambda: _FailingLib())
    monkeypatch.setattr(nat, "current_stream_handle", lambda dev: None)
    monkeypatch.setattr(torch.cuda, "device", lambda dev: contextlib.nullcontext())
    q = torch.arange(64, dtype=torch.uint8)
    before = q.clone()
    d = _desc()
    d.qdata = q.data_ptr()
    with pytest.raises(RuntimeError, match="injected launch failure"):
        nat.merge_batch([d], torch.device("cpu"))
    assert torch.equal(q, before)

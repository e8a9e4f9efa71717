"""Raw-buffer merge launchers, drop-in for Piper Offload's Triton launchers.

Each function keeps the name, arguments, validation and exception types of the
reference launcher it replaces and runs the sm_100a kernels of
``libpiper_merge.so`` on ``torch.cuda.current_stream()``:

* :func:`merge_mx_lora_`     <- ``src/piper_offload/_triton_mx_lora.py:333-425``
* :func:`merge_nvfp4_lora`   <- ``src/piper_offload/_triton_nvfp4_lora.py:515-595``
* :func:`merge_float8_lora`  <- ``src/piper_offload/_triton_float8_lora.py:486-588``
* :func:`merge_int8_lora`    <- ``src/piper_offload/_triton_int8_lora.py:267-407``
* :func:`merge_gguf_lora_`   (new: the reference has no GGUF merge)

Unlike the reference, every update is applied in place: the returned tensors
are the input storage objects themselves, so the reference adapters'
``qt.qdata.copy_(qdata)`` copy-back becomes a no-op self copy.

``offset_base`` (keyword, default 0) is an extension for row-sharded merges:
it is added to every logical element offset before keying the stochastic
stream, so a shard can reproduce the unsharded merge's samples.
"""

from __future__ import annotations

import torch

from . import _native as nat

_MX_BLOCK_SIZE = 32
_NVFP4_BLOCK_SIZE = 16
MAX_GROUP_SIZE = 256  # _triton_float8_lora.py:23
_FP4_DTYPE = getattr(torch, "float4_e2m1fn_x2", None)
_E8M0_DTYPE = getattr(torch, "float8_e8m0fnu", None)

_MX_SCALING_MODES = {"floor": 0, "rceil": 1, "ceil": 2, "even": 3}


def _dt_id(dtype: torch.dtype, what: str) -> int:
    if dtype is torch.bfloat16:
        return nat.DT_BF16
    if dtype is torch.float16:
        return nat.DT_F16
    if dtype is torch.float32:
        return nat.DT_F32
    raise ValueError(f"merge supports float16, bfloat16, and float32 {what}, got {dtype}.")


def _factor_dt(b: torch.Tensor, a: torch.Tensor, *, allowed: tuple[torch.dtype, ...]) -> int:
    if b.dtype is not a.dtype:
        raise ValueError("merge requires matching LoRA factor dtypes.")
    if b.dtype not in allowed:
        names = ", ".join(str(d).replace("torch.", "") for d in allowed)
        raise ValueError(f"merge supports {names} LoRA factors, got {b.dtype}.")
    return _dt_id(b.dtype, "LoRA factors")


def _same_device(*ts: torch.Tensor | None) -> None:
    devs = {t.device for t in ts if t is not None}
    if len(devs) != 1:
        raise ValueError("merge requires all tensors on one CUDA device.")


def _seed_fields(rounding_seed: int | None) -> tuple[int, int]:
    if rounding_seed is None:
        return 0, 0
    seed = int(rounding_seed)
    if seed < 0:
        seed += 1 << 64  # the signed launch form of the same bits
    if not 0 <= seed < (1 << 64):
        raise ValueError("rounding_seed must be an unsigned 64-bit value.")
    return seed, nat.FLAG_STOCHASTIC


def _desc(**kw) -> nat.MergeDesc:
    d = nat.MergeDesc()
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------------- MX
def mx_format_parameters(elem_dtype: torch.dtype) -> int:
    """Format id for an MX element dtype (``_triton_mx_lora.py:298-308``)."""
    if elem_dtype is torch.float8_e4m3fn:
        return nat.FMT_MXFP8_E4M3
    if elem_dtype is torch.float8_e5m2:
        return nat.FMT_MXFP8_E5M2
    if _FP4_DTYPE is not None and elem_dtype is _FP4_DTYPE:
        return nat.FMT_MXFP4
    raise ValueError(f"MX merge does not support element dtype {elem_dtype}.")


def mx_expected_scale_shape(rows: int, cols: int, *, swizzled: bool) -> tuple[int, int]:
    if not swizzled:
        return rows, cols // _MX_BLOCK_SIZE
    return ((rows + 127) // 128) * 32, ((cols + 127) // 128) * 16


def merge_mx_lora_(
    qdata: torch.Tensor,
    scale: torch.Tensor,
    elem_dtype: torch.dtype,
    block_size: int,
    orig_dtype: torch.dtype,
    b: torch.Tensor,
    a: torch.Tensor,
    strength: float,
    *,
    scaling_mode: int,
    swizzled: bool,
    rounding_seed: int | None = None,
    offset_base: int = 0,
) -> None:
    """Merge one staged LoRA update directly into raw MX storage (in place)."""
    if qdata.device.type != "cuda":
        raise ValueError("MX merge requires CUDA tensors.")
    if qdata.ndim != 2 or scale.ndim != 2 or b.ndim != 2 or a.ndim != 2:
        raise ValueError("MX merge expects rank-two tensors.")
    if block_size != _MX_BLOCK_SIZE:
        raise ValueError("MX merge supports block size 32.")
    if b.dtype is not a.dtype or b.dtype is not orig_dtype:
        raise ValueError("MX merge requires factors in the weight's original dtype.")
    if orig_dtype not in (torch.bfloat16, torch.float32):  # _triton_mx_lora.py:311-316
        raise ValueError(f"MX merge supports bfloat16 and float32 weights and factors, got {orig_dtype}.")
    _same_device(qdata, scale, b, a)
    if not qdata.is_contiguous() or not scale.is_contiguous():
        raise ValueError("MX merge requires contiguous MX storage.")
    if scaling_mode not in (0, 1, 2, 3):
        raise ValueError(f"Unsupported MX scaling mode id {scaling_mode}.")
    rows, rank = b.shape
    if a.shape[0] != rank:
        raise ValueError("LoRA factor inner dimensions do not match.")
    cols = a.shape[1]
    if rows == 0 or cols == 0 or rank == 0:
        raise ValueError("MX merge requires non-empty weight and factors.")
    if cols % _MX_BLOCK_SIZE != 0:
        raise ValueError("MX merge requires columns divisible by 32.")
    fmt = mx_format_parameters(elem_dtype)
    expected_q = (rows, cols // 2) if fmt == nat.FMT_MXFP4 else (rows, cols)
    if tuple(qdata.shape) != expected_q:
        raise ValueError("MX qdata shape does not match its element format and LoRA factors.")
    if tuple(scale.shape) != mx_expected_scale_shape(rows, cols, swizzled=swizzled):
        raise ValueError("MX scale shape does not match its block layout.")
    if scale.dtype is not _E8M0_DTYPE and scale.dtype is not torch.uint8:
        raise ValueError(f"MX merge expects E8M0 scales, got {scale.dtype}.")
    if fmt == nat.FMT_MXFP4:
        if qdata.dtype is not torch.uint8:
            raise ValueError("MXFP4 merge expects packed uint8 qdata.")
    elif qdata.dtype is not elem_dtype:
        raise ValueError("MXFP8 qdata dtype does not match elem_dtype.")
    b = b.contiguous()
    a = a.contiguous()
    seed, sflag = _seed_fields(rounding_seed)
    d = _desc(
        qdata=qdata.data_ptr(), scale=scale.data_ptr(), b=b.data_ptr(), a=a.data_ptr(),
        rows=rows, cols=cols, rank=rank, format=fmt, compute_dtype=_dt_id(orig_dtype, "MX weights"),
        scale_mode=int(scaling_mode), flags=(nat.FLAG_SWIZZLED if swizzled else 0) | sflag,
        strength=float(strength), seed=seed, offset_base=int(offset_base),
    )
    nat.merge_batch([d], qdata.device)


# ------------------------------------------------------------------- NVFP4
def nvfp4_expected_scale_shape(rows: int, cols: int, *, swizzled: bool) -> tuple[int, int]:
    if swizzled:
        return (rows + 127) // 128 * 32, (cols + 63) // 64 * 16
    return rows, cols // _NVFP4_BLOCK_SIZE


def merge_nvfp4_lora(
    qdata: torch.Tensor,
    scale: torch.Tensor,
    per_tensor_scale: torch.Tensor | None,
    block_size: int,
    is_swizzled_scales: bool,
    b: torch.Tensor,
    a: torch.Tensor,
    strength: float,
    *,
    rounding_seed: int | None = None,
    offset_base: int = 0,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """Merge into packed NVFP4 storage in place and return its buffers."""
    if qdata.device.type != "cuda":
        raise ValueError("NVFP4 merge requires CUDA tensors.")
    if qdata.dtype is not torch.uint8:
        raise ValueError(f"NVFP4 merge expects packed uint8 data, got {qdata.dtype}.")
    if scale.dtype is not torch.float8_e4m3fn:
        raise ValueError("NVFP4 merge expects E4M3FN block scales.")
    if qdata.ndim != 2 or scale.ndim != 2 or b.ndim != 2 or a.ndim != 2:
        raise ValueError("NVFP4 merge expects rank-two tensors.")
    if not qdata.is_contiguous() or not scale.is_contiguous():
        raise ValueError("NVFP4 merge requires contiguous packed data and scales.")
    cdt = _factor_dt(b, a, allowed=(torch.bfloat16, torch.float32))
    _same_device(qdata, scale, b, a, per_tensor_scale)
    if block_size != _NVFP4_BLOCK_SIZE:
        raise ValueError("NVFP4 merge requires block_size=16.")
    rows, packed_cols = qdata.shape
    cols = packed_cols * 2
    rank = a.shape[0]
    if rows == 0 or cols == 0 or rank == 0:
        raise ValueError("NVFP4 merge requires non-empty tensors.")
    if packed_cols % 8 != 0:
        raise ValueError("NVFP4 merge requires columns divisible by 16.")
    if tuple(b.shape) != (rows, rank) or a.shape[1] != cols:
        raise ValueError("LoRA factors do not match the NVFP4 weight shape.")
    if tuple(scale.shape) != nvfp4_expected_scale_shape(rows, cols, swizzled=is_swizzled_scales):
        raise ValueError("NVFP4 scale shape does not match its swizzle metadata.")
    if per_tensor_scale is not None and (
        per_tensor_scale.dtype is not torch.float32 or per_tensor_scale.numel() != 1
    ):
        raise ValueError("NVFP4 merge expects one float32 per-tensor scale.")
    b = b.contiguous()
    a = a.contiguous()
    seed, sflag = _seed_fields(rounding_seed)
    d = _desc(
        qdata=qdata.data_ptr(), scale=scale.data_ptr(), global_scale=_ptr(per_tensor_scale),
        b=b.data_ptr(), a=a.data_ptr(), rows=rows, cols=cols, rank=rank, format=nat.FMT_NVFP4,
        compute_dtype=cdt, flags=(nat.FLAG_SWIZZLED if is_swizzled_scales else 0) | sflag,
        strength=float(strength), seed=seed, offset_base=int(offset_base),
    )
    nat.merge_batch([d], qdata.device)
    return qdata, scale, per_tensor_scale


# --------------------------------------------------------------------- FP8
def float8_layout(qdata: torch.Tensor, scale: torch.Tensor, block_size: tuple[int, ...]):
    """Normalized (rows, cols, per_row, per_tensor, group) of a scaled-FP8 layout.

    Mirrors ``_validate_inputs`` (``_triton_float8_lora.py:321-380``).
    """
    rows, cols = qdata.shape
    per_row = tuple(block_size) == (1, cols)
    per_tensor = tuple(block_size) == (rows, cols)
    group = (
        block_size[1]
        if (len(block_size) == 2 and block_size[0] == 1 and 0 < block_size[1] < cols and cols % block_size[1] == 0)
        else None
    )
    if per_row:
        if tuple(scale.shape) != (rows, 1):
            raise ValueError(
                f"per-row scaled-FP8 merge expects scale shape {(rows, 1)}, got {tuple(scale.shape)}."
            )
    elif per_tensor:
        if scale.numel() != 1:
            raise ValueError("per-tensor scaled-FP8 merge expects one scale.")
    elif group is not None:
        if group > MAX_GROUP_SIZE:
            raise ValueError(
                f"per-group scaled-FP8 merge supports group sizes up to {MAX_GROUP_SIZE}, got {group}."
            )
        if tuple(scale.shape) != (rows, cols // group):
            raise ValueError(
                "per-group scaled-FP8 merge expects scale shape "
                f"{(rows, cols // group)}, got {tuple(scale.shape)}."
            )
    else:
        raise ValueError(
            "scaled-FP8 merge supports per-row, per-tensor, and standard per-group layouts, "
            f"got block_size={block_size!r}."
        )
    return rows, cols, per_row, per_tensor, group


def merge_float8_lora(
    qdata: torch.Tensor,
    scale: torch.Tensor,
    block_size: tuple[int, ...],
    b: torch.Tensor,
    a: torch.Tensor,
    strength: float,
    *,
    rounding_seed: int | None = None,
    offset_base: int = 0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Merge into scaled-FP8 storage in place and return ``(qdata, scale)``."""
    if qdata.device.type != "cuda":
        raise ValueError("scaled-FP8 merge requires CUDA tensors.")
    if qdata.dtype not in (torch.float8_e4m3fn, torch.float8_e5m2):
        raise ValueError(f"scaled-FP8 merge supports E4M3FN and E5M2 storage, got {qdata.dtype}.")
    cdt = _factor_dt(b, a, allowed=(torch.float16, torch.bfloat16, torch.float32))
    if qdata.ndim != 2 or b.ndim != 2 or a.ndim != 2:
        raise ValueError("scaled-FP8 merge expects rank-two tensors.")
    _same_device(qdata, scale, b, a)
    if scale.dtype is not torch.float32:
        raise ValueError("scaled-FP8 merge expects float32 scales.")
    rows, cols, per_row, per_tensor, group = float8_layout(qdata, scale, tuple(block_size))
    rank = a.shape[0]
    if rows == 0 or cols == 0 or rank == 0:
        raise ValueError("scaled-FP8 merge requires non-empty weight and factors.")
    if tuple(b.shape) != (rows, rank) or a.shape[1] != cols:
        raise ValueError("LoRA factors do not match the scaled-FP8 weight shape.")
    if not qdata.is_contiguous() or not scale.is_contiguous():
        raise ValueError("scaled-FP8 merge requires contiguous storage for an in-place update.")
    b = b.contiguous()
    a = a.contiguous()
    brows, bcols = (rows, cols) if per_tensor else (1, cols if per_row else group)
    seed, sflag = _seed_fields(rounding_seed)
    d = _desc(
        qdata=qdata.data_ptr(), scale=scale.data_ptr(), b=b.data_ptr(), a=a.data_ptr(),
        rows=rows, cols=cols, rank=rank, block_rows=brows, block_cols=bcols,
        format=nat.FMT_FP8_E5M2 if qdata.dtype is torch.float8_e5m2 else nat.FMT_FP8_E4M3,
        compute_dtype=cdt, flags=sflag, strength=float(strength), seed=seed,
        offset_base=int(offset_base),
    )
    nat.merge_batch([d], qdata.device)
    return qdata, scale


def merge_static_float8_lora(
    qdata: torch.Tensor,
    scale: torch.Tensor,
    b: torch.Tensor,
    a: torch.Tensor,
    strength: float,
    *,
    rounding_seed: int | None = None,
    offset_base: int = 0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Static per-tensor FP8 merge in place (``merge_static_float8_lora``,
    ``_triton_static_float8_lora.py:174-295``); returns ``(qdata, scale)``.

    The reference's arithmetic is the per-tensor layout of the scaled-FP8
    merge: ``base = compute(fp8 * scale)``, ``merged = compute(base + acc *
    strength)``, ``scale = compute(amax / limit)`` (0 becomes 2**-23), codes
    ``fp8(clamp(merged / scale))`` or the stochastic FP8 rounding
    (``:23-158``), so it runs as one per-tensor FP8 descriptor.
    """
    if qdata.device.type != "cuda":
        raise ValueError("static-FP8 merge requires CUDA tensors.")
    if qdata.dtype not in (torch.float8_e4m3fn, torch.float8_e5m2):
        raise ValueError(f"static-FP8 merge supports E4M3FN and E5M2 storage, got {qdata.dtype}.")
    cdt = _factor_dt(b, a, allowed=(torch.float16, torch.bfloat16, torch.float32))
    if qdata.ndim != 2 or b.ndim != 2 or a.ndim != 2:
        raise ValueError("static-FP8 merge expects rank-two tensors.")
    _same_device(qdata, scale, b, a)
    if scale.dtype is not torch.float32 or scale.numel() != 1:
        raise ValueError("static-FP8 merge expects one float32 per-tensor scale.")
    rows, cols = qdata.shape
    rank = a.shape[0]
    if rows == 0 or cols == 0 or rank == 0:
        raise ValueError("static-FP8 merge requires non-empty weight and factors.")
    if tuple(b.shape) != (rows, rank) or a.shape[1] != cols:
        raise ValueError("LoRA factors do not match the FP8 weight shape.")
    if not qdata.is_contiguous():
        raise ValueError("static-FP8 merge requires contiguous storage for an in-place update.")
    b = b.contiguous()
    a = a.contiguous()
    seed, sflag = _seed_fields(rounding_seed)
    d = _desc(
        qdata=qdata.data_ptr(), scale=scale.data_ptr(), b=b.data_ptr(), a=a.data_ptr(),
        rows=rows, cols=cols, rank=rank, block_rows=rows, block_cols=cols,
        format=nat.FMT_FP8_E5M2 if qdata.dtype is torch.float8_e5m2 else nat.FMT_FP8_E4M3,
        compute_dtype=cdt, flags=sflag, strength=float(strength), seed=seed, offset_base=int(offset_base),
    )
    nat.merge_batch([d], qdata.device)
    return qdata, scale


# -------------------------------------------------------------------- INT8
def int8_block_numel(shape: tuple[int, int], block_size: tuple[int, int]) -> int:
    """``_block_numel`` (``_triton_int8_lora.py:251-264``)."""
    rows, cols = shape
    block_rows, block_cols = block_size
    if tuple(block_size) == tuple(shape):
        return rows * cols
    if block_rows == 1 and 0 < block_cols <= cols and cols % block_cols == 0:
        return block_cols
    raise ValueError(
        "INT8 merge supports two-dimensional per-tensor, per-row, "
        f"and per-group layouts, got shape {shape} with block size {block_size}."
    )


def merge_int8_lora(
    qdata: torch.Tensor,
    scale: torch.Tensor,
    zero_point: torch.Tensor | None,
    block_size: tuple[int, int],
    b: torch.Tensor,
    a: torch.Tensor,
    strength: float,
    *,
    asymmetric: bool,
    reduce_range: bool,
    rounding_seed: int | None = None,
    offset_base: int = 0,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Merge into affine-INT8 storage in place; returns ``(qdata, scale, zero_point)``.

    When ``zero_point`` is None the returned zero point is a zeros tensor, as in
    the reference.
    """
    if qdata.device.type != "cuda":
        raise ValueError("INT8 merge requires CUDA tensors.")
    if qdata.dtype is not torch.int8:
        raise ValueError(f"INT8 merge requires int8 weight storage, got {qdata.dtype}.")
    if qdata.ndim != 2 or b.ndim != 2 or a.ndim != 2:
        raise ValueError("INT8 merge expects rank-two tensors.")
    cdt = _factor_dt(b, a, allowed=(torch.float16, torch.bfloat16, torch.float32))
    sdt = _dt_id(scale.dtype, "scales")
    _same_device(qdata, scale, b, a, zero_point)
    rows, cols = qdata.shape
    rank = a.shape[0]
    if rows == 0 or cols == 0 or rank == 0:
        raise ValueError("INT8 merge requires non-empty weight and factors.")
    if tuple(b.shape) != (rows, rank) or a.shape[1] != cols:
        raise ValueError("LoRA factors do not match the INT8 weight shape.")
    block_numel = int8_block_numel((rows, cols), tuple(block_size))
    num_qparams = qdata.numel() // block_numel
    if scale.numel() != num_qparams:
        raise ValueError("INT8 scale shape does not match the quantization block layout.")
    if zero_point is not None and (zero_point.dtype is not torch.int8 or zero_point.numel() != num_qparams):
        raise ValueError("INT8 zero-point storage does not match the quantization blocks.")
    if not qdata.is_contiguous() or not scale.is_contiguous() or (
        zero_point is not None and not zero_point.is_contiguous()
    ):
        raise ValueError("INT8 merge requires contiguous storage for an in-place update.")
    b = b.contiguous()
    a = a.contiguous()
    per_tensor = block_numel == rows * cols and tuple(block_size) == (rows, cols)
    brows, bcols = (rows, cols) if per_tensor else (1, block_numel)
    seed, sflag = _seed_fields(rounding_seed)
    flags = sflag | (nat.FLAG_ASYMMETRIC if asymmetric else 0) | (nat.FLAG_REDUCE_RANGE if reduce_range else 0)
    d = _desc(
        qdata=qdata.data_ptr(), scale=scale.data_ptr(), zero_point=_ptr(zero_point),
        b=b.data_ptr(), a=a.data_ptr(), rows=rows, cols=cols, rank=rank, block_rows=brows,
        block_cols=bcols, format=nat.FMT_INT8, compute_dtype=cdt, scale_dtype=sdt, flags=flags,
        strength=float(strength), seed=seed, offset_base=int(offset_base),
    )
    nat.merge_batch([d], qdata.device)
    zp_out = zero_point if zero_point is not None else torch.zeros_like(scale, dtype=torch.int8)
    return qdata, scale, zp_out


# ----------------------------------------------------- bitsandbytes LLM.int8
def merge_bnb8_lora(
    cb: torch.Tensor,
    scb: torch.Tensor,
    b: torch.Tensor,
    a: torch.Tensor,
    strength: float,
    *,
    rounding_seed: int | None = None,
    offset_base: int = 0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """bitsandbytes row-wise int8 merge in place (``merge_bnb8_lora``,
    ``_triton_bnb8_lora.py:145-242``); returns ``(CB, SCB)``.

    ``base = f16(f16(CB / 127) * f16(SCB))``, ``merged = f16(clamp(base + acc *
    strength, +-65504))``, ``SCB = row max |merged|``, codes ``rint((merged /
    SCB) * 127)`` (0 where SCB is 0) or stochastic, clamped to [-127, 127].
    """
    if cb.device.type != "cuda":
        raise ValueError("BNB8 merge requires CUDA tensors.")
    if cb.dtype is not torch.int8 or scb.dtype is not torch.float32:
        raise ValueError("BNB8 merge expects int8 CB and float32 SCB tensors.")
    if b.dtype is not torch.float16 or a.dtype is not torch.float16:
        raise ValueError("BNB8 merge expects float16 LoRA factors.")
    if cb.ndim != 2 or b.ndim != 2 or a.ndim != 2:
        raise ValueError("BNB8 merge expects rank-two tensors.")
    _same_device(cb, scb, b, a)
    rows, cols = cb.shape
    rank = a.shape[0]
    if rows == 0 or cols == 0 or rank == 0:
        raise ValueError("BNB8 merge requires non-empty tensors.")
    if scb.numel() != rows:
        raise ValueError("BNB8 merge expects one SCB value per row.")
    if tuple(b.shape) != (rows, rank) or a.shape[1] != cols:
        raise ValueError("LoRA factors do not match the BNB8 weight shape.")
    if not cb.is_contiguous() or not scb.is_contiguous():
        raise ValueError("BNB8 merge requires contiguous storage for an in-place update.")
    b = b.contiguous()
    a = a.contiguous()
    seed, sflag = _seed_fields(rounding_seed)
    d = _desc(qdata=cb.data_ptr(), scale=scb.data_ptr(), b=b.data_ptr(), a=a.data_ptr(), rows=rows, cols=cols,
              rank=rank, block_rows=1, block_cols=cols, format=nat.FMT_BNB8, compute_dtype=nat.DT_F16,
              scale_dtype=nat.DT_F32, flags=sflag, strength=float(strength), seed=seed,
              offset_base=int(offset_base))
    nat.merge_batch([d], cb.device)
    return cb, scb


# ---------------------------------------------------------------- Quanto
def quanto_scale_axis(axis: int | None, scale: torch.Tensor, rows: int, cols: int) -> str:
    """``_scale_axis_id`` (``_triton_quanto_lora.py:184-199``): "tensor", "row" or "column"."""
    if axis is None and scale.numel() == 1:
        return "tensor"
    if axis == 0 and scale.numel() == rows:
        return "row"
    if axis in (-1, 1) and scale.numel() == cols:
        return "column"
    raise ValueError("Quanto qbytes merge expects a scalar scale, one scale per row for axis 0, "
                     "or one scale per column for the last axis.")


# Quantization block (rows, cols) of each Quanto scale layout in the C ABI.
QUANTO_BLOCK = {"tensor": lambda r, c: (r, c), "row": lambda r, c: (1, c), "column": lambda r, c: (r, 1)}


def _merge_quanto(qdata, scale, axis, b, a, strength, *, fmt: int, rounding_seed, offset_base):
    if qdata.device.type != "cuda":
        raise ValueError("Quanto qbytes merge requires CUDA tensors.")
    if scale.dtype is not b.dtype or b.dtype is not a.dtype:
        raise ValueError("Quanto qbytes merge requires matching scale and factor dtypes.")
    cdt = _factor_dt(b, a, allowed=(torch.float16, torch.bfloat16, torch.float32))
    if qdata.ndim != 2 or b.ndim != 2 or a.ndim != 2:
        raise ValueError("Quanto qbytes merge expects rank-two tensors.")
    _same_device(qdata, scale, b, a)
    rows, cols = qdata.shape
    rank = a.shape[0]
    if rows == 0 or cols == 0 or rank == 0:
        raise ValueError("Quanto qbytes merge requires non-empty tensors.")
    if tuple(b.shape) != (rows, rank) or a.shape[1] != cols:
        raise ValueError("LoRA factors do not match the Quanto weight shape.")
    kind = quanto_scale_axis(axis, scale, rows, cols)
    if not qdata.is_contiguous() or not scale.is_contiguous():
        raise ValueError("Quanto qbytes merge requires contiguous storage for an in-place update.")
    b = b.contiguous()
    a = a.contiguous()
    brows, bcols = QUANTO_BLOCK[kind](rows, cols)
    seed, sflag = _seed_fields(rounding_seed)
    d = _desc(qdata=qdata.data_ptr(), scale=scale.data_ptr(), b=b.data_ptr(), a=a.data_ptr(), rows=rows,
              cols=cols, rank=rank, block_rows=brows, block_cols=bcols, format=fmt, compute_dtype=cdt,
              scale_dtype=cdt, flags=sflag, strength=float(strength), seed=seed, offset_base=int(offset_base))
    nat.merge_batch([d], qdata.device)
    return qdata, scale


def merge_quanto_qint8_lora(qdata, scale, axis, b, a, strength, *, rounding_seed=None, offset_base=0):
    """Quanto qint8 merge in place (``merge_quanto_qint8_lora``, ``_triton_quanto_lora.py:317-342``);
    returns ``(qdata, scale)``: ``base = dtype(q * scale)`` (0 under a zero scale), the absmax
    scale ``dtype(amax / 127)`` (0 -> fp32 eps), codes ``rint(dtype(x / scale))`` or stochastic."""
    if qdata.dtype is not torch.int8:
        raise ValueError("Quanto qint8 merge expects int8 storage.")
    return _merge_quanto(qdata, scale, axis, b, a, strength, fmt=nat.FMT_QUANTO_INT8,
                         rounding_seed=rounding_seed, offset_base=offset_base)


def merge_quanto_qfloat8_lora(qdata, scale, axis, b, a, strength, *, rounding_seed=None, offset_base=0):
    """Quanto qfloat8 merge in place (``merge_quanto_qfloat8_lora``, ``_triton_quanto_lora.py:345-377``)."""
    if qdata.dtype not in (torch.float8_e4m3fn, torch.float8_e5m2):
        raise ValueError(f"Quanto qfloat8 merge expects E4M3FN or E5M2 storage, got {qdata.dtype}.")
    fmt = nat.FMT_QUANTO_FP8_E5M2 if qdata.dtype is torch.float8_e5m2 else nat.FMT_QUANTO_FP8_E4M3
    return _merge_quanto(qdata, scale, axis, b, a, strength, fmt=fmt, rounding_seed=rounding_seed,
                         offset_base=offset_base)


# ------------------------------------------------------- bitsandbytes 4-bit
BNB4_BLOCK = 64
BNB4_NESTED_BLOCK = 256


def bnb4_desc(packed, absmax, code, nested_absmax, nested_code, offset, logical_shape, blocksize, quant_type, b, a,
              strength, *, rounding_seed=None, offset_base=0, keep: list | None = None) -> nat.MergeDesc:
    """Validate a bitsandbytes 4-bit merge (``_triton_bnb4_lora.py:449-540``) and build its descriptor."""
    if packed.device.type != "cuda":
        raise ValueError("BNB4 merge requires CUDA tensors.")
    if packed.dtype is not torch.uint8:
        raise ValueError("BNB4 merge expects a raw uint8 packed view.")
    if quant_type not in ("nf4", "fp4"):
        raise ValueError("BNB4 merge supports NF4 and FP4.")
    if code.dtype is not torch.float32 or code.numel() != 16:
        raise ValueError("BNB4 merge expects a 16-value float32 codebook.")
    if b.dtype is not a.dtype:
        raise ValueError("BNB4 merge requires matching factor dtypes.")
    cdt = _factor_dt(b, a, allowed=(torch.float16, torch.bfloat16, torch.float32))
    if b.ndim != 2 or a.ndim != 2:
        raise ValueError("BNB4 merge expects rank-two factors.")
    rows, cols = logical_shape
    rank = a.shape[0]
    numel = rows * cols
    num_blocks = (numel + blocksize - 1) // blocksize
    nested = nested_absmax is not None
    if rows == 0 or cols == 0 or rank == 0:
        raise ValueError("BNB4 merge requires non-empty tensors.")
    if numel % 2 != 0 or packed.numel() != numel // 2:
        raise ValueError("BNB4 merge requires exact two-values-per-byte storage.")
    if blocksize != BNB4_BLOCK:
        raise ValueError("BNB4 merge expects the standard 64-value blocks.")
    if cols % blocksize != 0:
        raise ValueError("BNB4 merge requires row-aligned 64-value blocks.")
    if tuple(b.shape) != (rows, rank) or a.shape[1] != cols:
        raise ValueError("LoRA factors do not match the BNB4 weight shape.")
    if absmax.numel() != num_blocks:
        raise ValueError("BNB4 absmax shape does not match the logical weight.")
    _same_device(packed, absmax, code, b, a)
    if nested:
        if nested_code is None or offset is None:
            raise ValueError("Nested BNB4 merge requires its codebook and offset.")
        if (absmax.dtype is not torch.uint8 or nested_absmax.dtype is not torch.float32
                or nested_absmax.numel() != (num_blocks + BNB4_NESTED_BLOCK - 1) // BNB4_NESTED_BLOCK
                or nested_code.dtype is not torch.float32 or nested_code.numel() != 256
                or offset.dtype is not torch.float32 or offset.numel() != 1):
            raise ValueError("Nested BNB4 scale metadata has an unsupported layout.")
        _same_device(packed, nested_absmax, nested_code, offset)
        if rounding_seed is not None:
            raise ValueError("BNB4 stochastic merge does not support nested scales because their final effective "
                             "values are unavailable during terminal-code selection.")
    elif absmax.dtype is not torch.float32:
        raise ValueError("Non-nested BNB4 merge expects float32 absmax values.")
    for t in (packed, absmax, nested_absmax, offset):
        if t is not None and not t.is_contiguous():
            raise ValueError("BNB4 merge requires contiguous storage for an in-place update.")
    b = b.contiguous()
    a = a.contiguous()
    code = code.contiguous()
    nested_code = nested_code.contiguous() if nested_code is not None else None
    if keep is not None:
        keep.extend([b, a, code, nested_code])
    seed, sflag = _seed_fields(rounding_seed)
    return _desc(qdata=packed.data_ptr(), scale=absmax.data_ptr(), b=b.data_ptr(), a=a.data_ptr(), rows=rows,
              cols=cols, rank=rank, format=nat.FMT_BNB4_NF4 if quant_type == "nf4" else nat.FMT_BNB4_FP4,
              compute_dtype=cdt, flags=sflag, strength=float(strength), seed=seed, offset_base=int(offset_base),
              codebook=code.data_ptr(), nested_absmax=_ptr(nested_absmax), nested_code=_ptr(nested_code),
              nested_offset=_ptr(offset))


def merge_bnb4_lora(
    packed: torch.Tensor,
    absmax: torch.Tensor,
    code: torch.Tensor,
    nested_absmax: torch.Tensor | None,
    nested_code: torch.Tensor | None,
    offset: torch.Tensor | None,
    logical_shape: tuple[int, int],
    blocksize: int,
    quant_type: str,
    b: torch.Tensor,
    a: torch.Tensor,
    strength: float,
    *,
    rounding_seed: int | None = None,
    offset_base: int = 0,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None, torch.Tensor | None]:
    """bitsandbytes blockwise 4-bit merge in place (``merge_bnb4_lora``,
    ``_triton_bnb4_lora.py:434-604``); returns ``(packed, absmax, nested_absmax, offset)``.

    64-value blocks along rows, the first value of a byte in its high nibble.
    Plain absmax is fp32 per block; nested absmax is uint8 codes of
    ``nested_code`` scaled by ``nested_absmax`` (fp32 per 256 blocks) plus
    ``offset``, re-quantized after the merge (round-to-nearest only).
    """
    keep: list = []
    d = bnb4_desc(packed, absmax, code, nested_absmax, nested_code, offset, logical_shape, blocksize, quant_type, b,
                  a, strength, rounding_seed=rounding_seed, offset_base=offset_base, keep=keep)
    nat.merge_batch([d], packed.device)
    return packed, absmax, nested_absmax, offset


# -------------------------------------------------------------------- GGUF
GGUF_Q8_0 = 8
GGUF_Q4_0 = 2
GGUF_TYPE_SIZE = {GGUF_Q8_0: 34, GGUF_Q4_0: 18}


def gguf_logical_cols(packed_cols: int, quant_type: int) -> int:
    if quant_type not in GGUF_TYPE_SIZE:
        raise ValueError(f"GGUF merge supports Q8_0 and Q4_0, got quant type {quant_type}.")
    ts = GGUF_TYPE_SIZE[quant_type]
    if packed_cols % ts != 0:
        raise ValueError("GGUF raw row length is not a whole number of blocks.")
    return packed_cols // ts * 32


def validate_gguf_merge(raw: torch.Tensor, quant_type: int, b: torch.Tensor,
                        a: torch.Tensor) -> tuple[int, int, int, int]:
    """The GGUF merge's checks, raising ``ValueError`` before anything is
    enqueued; returns (compute dtype id, rows, logical cols, rank)."""
    if raw.device.type != "cuda":
        raise ValueError("GGUF merge requires CUDA tensors.")
    if raw.dtype is not torch.uint8 or raw.ndim != 2:
        raise ValueError("GGUF merge expects a rank-two uint8 tensor of raw blocks.")
    if not raw.is_contiguous():
        raise ValueError("GGUF merge requires contiguous raw blocks.")
    cdt = _factor_dt(b, a, allowed=(torch.float16, torch.bfloat16, torch.float32))
    _same_device(raw, b, a)
    rows = raw.shape[0]
    cols = gguf_logical_cols(raw.shape[1], int(quant_type))
    rank = a.shape[0]
    if rows == 0 or cols == 0 or rank == 0:
        raise ValueError("GGUF merge requires non-empty weight and factors.")
    if tuple(b.shape) != (rows, rank) or a.shape[1] != cols:
        raise ValueError("LoRA factors do not match the GGUF weight shape.")
    return cdt, rows, cols, rank


def merge_gguf_lora_(
    raw: torch.Tensor,
    quant_type: int,
    b: torch.Tensor,
    a: torch.Tensor,
    strength: float,
    *,
    rounding_seed: int | None = None,
    offset_base: int = 0,
) -> None:
    """Merge into raw GGUF Q8_0 / Q4_0 block rows in place.

    Decoding follows ``gguf_dequant._dequantize_Q8_0`` / ``_dequantize_Q4_0``
    (compute dtype = factor dtype), the update is added in fp32 and rounded to
    the compute dtype, and re-encoding follows gguf 0.19.0's
    ``quants.Q8_0/Q4_0.quantize_blocks`` bit for bit (round-to-nearest) or
    rounds each code stochastically by logical element offset.
    """
    cdt, rows, cols, rank = validate_gguf_merge(raw, quant_type, b, a)
    b = b.contiguous()
    a = a.contiguous()
    seed, sflag = _seed_fields(rounding_seed)
    d = _desc(
        qdata=raw.data_ptr(), b=b.data_ptr(), a=a.data_ptr(), rows=rows, cols=cols, rank=rank,
        format=nat.FMT_GGUF_Q8_0 if int(quant_type) == GGUF_Q8_0 else nat.FMT_GGUF_Q4_0,
        compute_dtype=cdt, flags=sflag, strength=float(strength), seed=seed,
        offset_base=int(offset_base),
    )
    nat.merge_batch([d], raw.device)

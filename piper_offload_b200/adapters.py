"""Tensor adapters with the reference's LoRA-merge capability, backed by sm_100a kernels.

Mirrors the merge half of Piper Offload's adapter protocol
(``src/piper_offload/tensor_adapters.py:214-278``):

* ``logical_shape(t)`` / ``compute_dtype(t)``
  (``LogicalShapeTensorAdapter`` / ``TensorAdapter.compute_dtype``);
* ``validate_lora_merge(target, b, a, strength, *, rounding_seed=None)``
  (``LoRAMergeValidationTensorAdapter``), raising ``ValueError`` before any
  mutation;
* ``merge_lora_(target, b, a, strength, *, rounding_seed=None)``
  (``LoRAMergeTensorAdapter``), updating the target's storage in place.

Targets are duck-typed on TorchAO's attribute names, so a real TorchAO
``Int8Tensor`` / ``Float8Tensor`` / ``NVFP4Tensor`` / ``MXTensor`` dispatches
the same way as the light stand-ins in ``piper_offload_b200.weights``:

=================  ==========================================================
adapter            reference gate / merge it replaces
=================  ==========================================================
Int8Adapter        int8_adapter.py:144-188 gate, :350-410 merge (act_pre_scale
                   folding :59-141)
Float8Adapter      float8_adapter.py:63-98 gate, :242-272 merge
StaticFloat8Ada.   static_float8_adapter.py:113-248 (layout rules
                   _torchao_static_float8.py:213-258)
Bnb8Adapter        bnb8bit_adapter.py:92-121 gate, :285-315 merge
QuantoAdapter      quanto_adapter.py:136-187 gate, :370-440 merge
Bnb4Adapter        bnb4bit_adapter.py:100-160 gate (plain / nested absmax)
Nvfp4Adapter       nvfp4_adapter.py:57-117 gate, :255-290 merge
MxAdapter          mx_adapter.py:90-137 gate, :274-309 merge
GgufAdapter        new: gguf_adapter.py:160-284 has no merge capability
=================  ==========================================================

Where the reference falls back to a TorchAO dequantize/requantize path for a
layout its Triton gate rejects, these adapters raise ``ValueError`` naming
the unsupported layout: the sm_100a path has no CPU or eager fallback.
Every adapter can also emit a ``MergeDesc`` so that many weights merge in one
``piper_merge_batch`` call (:func:`merge_lora_batch`).
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Any

import torch

from . import _native as nat
from . import kernels as K

_FP8_DTYPES = (torch.float8_e4m3fn, torch.float8_e5m2)
_FP4_DTYPE = getattr(torch, "float4_e2m1fn_x2", None)
_E8M0_DTYPE = getattr(torch, "float8_e8m0fnu", None)
MX_SCALING_MODES = {"floor": 0, "rceil": 1, "ceil": 2, "even": 3}


def _has(t: Any, *names: str) -> bool:
    return all(hasattr(t, n) for n in names)


def _seed(rounding_seed: int | None) -> tuple[int, int]:
    return K._seed_fields(rounding_seed)


def _factors(b: torch.Tensor, a: torch.Tensor, rows: int, cols: int, label: str) -> tuple[int, int]:
    if b.ndim != 2 or a.ndim != 2 or b.shape[1] != a.shape[0]:
        raise ValueError(f"{label}: LoRA factors must be rank two with matching inner dimensions, "
                         f"got B={tuple(b.shape)}, A={tuple(a.shape)}.")
    if tuple(b.shape) != (rows, b.shape[1]) or a.shape[1] != cols:
        raise ValueError(f"{label}: LoRA factors produce {(b.shape[0], a.shape[1])}, target is {(rows, cols)}.")
    if b.shape[1] == 0:
        raise ValueError(f"{label}: LoRA rank must be positive.")
    return b.shape[1], K._factor_dt(b, a, allowed=(torch.float16, torch.bfloat16, torch.float32))


def _cuda_same_device(label: str, *ts: torch.Tensor | None) -> torch.device:
    devs = {t.device for t in ts if t is not None}
    if len(devs) != 1:
        raise ValueError(f"{label}: merge requires all tensors on one CUDA device.")
    dev = next(iter(devs))
    if dev.type != "cuda":
        raise ValueError(f"{label}: the sm_100a merge requires CUDA tensors, got {dev}.")
    return dev


# ==================================================================== INT8
class Int8Adapter:
    """TorchAO ``Int8Tensor`` (affine int8, optional zero point and act_pre_scale)."""

    NAME = "torchao-int8"

    @staticmethod
    def matches(t: Any) -> bool:
        return _has(t, "qdata", "scale", "block_size") and getattr(t.qdata, "dtype", None) is torch.int8

    @staticmethod
    def logical_shape(t: Any) -> tuple[int, ...]:
        return tuple(t.qdata.shape)

    @staticmethod
    def compute_dtype(t: Any) -> torch.dtype:
        return t.dtype

    @staticmethod
    def _normalized_act_pre_scale(t: Any) -> torch.Tensor | None:
        """``act_pre_scale`` as (1,1) or (1, in_features) (int8_adapter.py:59-100)."""
        pre = getattr(t, "act_pre_scale", None)
        if pre is None:
            return None
        if not pre.dtype.is_floating_point:
            raise ValueError(f"TorchAO INT8 act_pre_scale must be floating-point for LoRA merge, got {pre.dtype}.")
        if pre.device != t.qdata.device:
            raise ValueError("TorchAO INT8 act_pre_scale must be on the weight device for LoRA merge.")
        cols = t.qdata.shape[-1]
        if pre.numel() == 1:
            norm = pre.reshape(1, 1)
        elif pre.ndim >= 1 and pre.shape[-1] == cols and all(s == 1 for s in pre.shape[:-1]):
            norm = pre.reshape(1, cols)
        else:
            raise ValueError(
                "TorchAO INT8 act_pre_scale must be a scalar or one value per input feature with only "
                f"singleton leading dimensions for LoRA merge; got shape {tuple(pre.shape)}."
            )
        if not bool(torch.isfinite(norm).all()):
            raise ValueError("TorchAO INT8 act_pre_scale must contain only finite values for LoRA merge.")
        if bool((norm == 0).any()):
            raise ValueError("TorchAO INT8 act_pre_scale must contain only non-zero values for LoRA merge.")
        return norm

    @classmethod
    def stored_factors(cls, t: Any, a: torch.Tensor, strength: float) -> tuple[torch.Tensor, float]:
        """Map A through act_pre_scale: B @ ((s * A) / p) in float64 (int8_adapter.py:103-126)."""
        pre = cls._normalized_act_pre_scale(t)
        if pre is None:
            return a, strength
        stored = a.to(torch.float64).mul(strength).div(pre.to(device=a.device, dtype=torch.float64)).to(a.dtype)
        if not bool(torch.isfinite(stored).all()):
            raise ValueError("TorchAO INT8 act_pre_scale produces non-finite stored-coordinate LoRA factors.")
        return stored.contiguous(), 1.0

    @classmethod
    def _check(cls, t: Any, b: torch.Tensor, a: torch.Tensor) -> tuple:
        label = "TorchAO INT8"
        if t.qdata.ndim != 2:
            raise ValueError(f"{label} merge expects a rank-two weight.")
        rows, cols = t.qdata.shape
        rank, cdt = _factors(b, a, rows, cols, label)
        if b.dtype is not t.dtype:
            raise ValueError(f"{label} merge requires factors in the weight's dtype {t.dtype}, got {b.dtype}.")
        dev = _cuda_same_device(label, t.qdata, t.scale, b, a, getattr(t, "zero_point", None))
        block = tuple(t.block_size)
        K.int8_block_numel((rows, cols), block)
        expected = (1, 1) if block == (rows, cols) else (rows, cols // block[1])
        if tuple(t.scale.shape) != expected and t.scale.numel() != expected[0] * expected[1]:
            raise ValueError(f"{label} scale shape {tuple(t.scale.shape)} does not match block size {block}.")
        zp = getattr(t, "zero_point", None)
        if zp is not None and (zp.dtype is not torch.int8 or zp.numel() != expected[0] * expected[1]):
            raise ValueError(f"{label} zero-point storage does not match the quantization blocks.")
        return rows, cols, rank, cdt, dev

    @classmethod
    def validate_lora_merge(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                            rounding_seed: int | None = None) -> None:
        _seed(rounding_seed)
        stored_a, _ = cls.stored_factors(target, a, strength)
        cls._check(target, b, stored_a)

    @classmethod
    def merge_desc(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                   rounding_seed: int | None = None, offset_base: int = 0, keep: list | None = None) -> nat.MergeDesc:
        a, strength = cls.stored_factors(target, a, strength)
        rows, cols, rank, cdt, _ = cls._check(target, b, a)
        b = b.contiguous()
        a = a.contiguous()
        if keep is not None:
            keep.extend([b, a])
        zp = getattr(target, "zero_point", None)
        # The reference treats a stored all-zero zero point as symmetric (int8_adapter.py:384).
        asym = zp is not None and bool(zp.any())
        block = tuple(target.block_size)
        per_tensor = block == (rows, cols)
        seed, sflag = _seed(rounding_seed)
        flags = sflag | (nat.FLAG_ASYMMETRIC if asym else 0) | (
            nat.FLAG_REDUCE_RANGE if bool(getattr(target, "reduce_range", False)) else 0)
        return K._desc(
            qdata=target.qdata.data_ptr(), scale=target.scale.data_ptr(), zero_point=K._ptr(zp),
            b=b.data_ptr(), a=a.data_ptr(), rows=rows, cols=cols, rank=rank,
            block_rows=rows if per_tensor else 1, block_cols=cols if per_tensor else block[1],
            format=nat.FMT_INT8, compute_dtype=cdt, scale_dtype=K._dt_id(target.scale.dtype, "scales"),
            flags=flags, strength=float(strength), seed=seed, offset_base=int(offset_base))

    @classmethod
    def merge_lora_(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                    rounding_seed: int | None = None, offset_base: int = 0) -> None:
        keep: list = []
        d = cls.merge_desc(target, b, a, strength, rounding_seed=rounding_seed, offset_base=offset_base, keep=keep)
        nat.merge_batch([d], target.qdata.device)


# ===================================================================== FP8
class Float8Adapter:
    """TorchAO ``Float8Tensor`` (scaled FP8, fp32 per-row / per-tensor / per-group scales)."""

    NAME = "torchao-float8"

    @staticmethod
    def matches(t: Any) -> bool:
        return _has(t, "qdata", "scale", "block_size") and getattr(t.qdata, "dtype", None) in _FP8_DTYPES \
            and not _has(t, "elem_dtype")

    @staticmethod
    def logical_shape(t: Any) -> tuple[int, ...]:
        return tuple(t.qdata.shape)

    @staticmethod
    def compute_dtype(t: Any) -> torch.dtype:
        return t.dtype

    @classmethod
    def _check(cls, t: Any, b: torch.Tensor, a: torch.Tensor) -> tuple:
        label = "TorchAO scaled-FP8"
        if t.qdata.ndim != 2:
            raise ValueError(f"{label} merge expects a rank-two weight.")
        if t.scale.dtype is not torch.float32:
            raise ValueError(f"{label} merge expects float32 scales.")
        rows, cols = t.qdata.shape
        rank, cdt = _factors(b, a, rows, cols, label)
        if b.dtype is not t.dtype:
            raise ValueError(f"{label} merge requires factors in the weight's dtype {t.dtype}, got {b.dtype}.")
        dev = _cuda_same_device(label, t.qdata, t.scale, b, a)
        if not t.qdata.is_contiguous():
            raise ValueError(f"{label} merge requires contiguous qdata (requantization fills the standard layout).")
        _, _, per_row, per_tensor, group = K.float8_layout(t.qdata, t.scale, tuple(t.block_size))
        return rows, cols, rank, cdt, dev, per_row, per_tensor, group

    @classmethod
    def validate_lora_merge(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                            rounding_seed: int | None = None) -> None:
        _seed(rounding_seed)
        cls._check(target, b, a)

    @classmethod
    def merge_desc(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                   rounding_seed: int | None = None, offset_base: int = 0, keep: list | None = None) -> nat.MergeDesc:
        rows, cols, rank, cdt, _, per_row, per_tensor, group = cls._check(target, b, a)
        b = b.contiguous()
        a = a.contiguous()
        if keep is not None:
            keep.extend([b, a])
        seed, sflag = _seed(rounding_seed)
        brows, bcols = (rows, cols) if per_tensor else (1, cols if per_row else group)
        return K._desc(
            qdata=target.qdata.data_ptr(), scale=target.scale.data_ptr(), b=b.data_ptr(), a=a.data_ptr(),
            rows=rows, cols=cols, rank=rank, block_rows=brows, block_cols=bcols,
            format=nat.FMT_FP8_E5M2 if target.qdata.dtype is torch.float8_e5m2 else nat.FMT_FP8_E4M3,
            compute_dtype=cdt, flags=sflag, strength=float(strength), seed=seed, offset_base=int(offset_base))

    @classmethod
    def merge_lora_(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                    rounding_seed: int | None = None, offset_base: int = 0) -> None:
        keep: list = []
        d = cls.merge_desc(target, b, a, strength, rounding_seed=rounding_seed, offset_base=offset_base, keep=keep)
        nat.merge_batch([d], target.qdata.device)


# ============================================================ static FP8
class StaticFloat8Adapter:
    """TorchAO ``PrototypeFloat8Tensor`` with a static activation scale
    (``static_float8_adapter.py:113-248``): per-tensor FP8 weight, fp32 scale.
    The merge rewrites ``qdata`` and ``scale`` and leaves ``act_quant_scale``."""

    NAME = "torchao-static-float8"

    @staticmethod
    def matches(t: Any) -> bool:
        return _has(t, "qdata", "scale", "act_quant_scale") and t.act_quant_scale is not None \
            and getattr(t.qdata, "dtype", None) in _FP8_DTYPES

    @staticmethod
    def logical_shape(t: Any) -> tuple[int, ...]:
        return tuple(t.qdata.shape)

    @staticmethod
    def compute_dtype(t: Any) -> torch.dtype:
        return t.dtype

    @classmethod
    def _check(cls, t: Any, b: torch.Tensor, a: torch.Tensor) -> tuple:
        label = "static FP8"
        if not isinstance(t.act_quant_scale, torch.Tensor):
            raise TypeError("PrototypeFloat8Tensor.act_quant_scale must be a tensor")
        if t.act_quant_scale.numel() != 1:
            raise ValueError("StaticFloat8Adapter supports a per-tensor activation scale containing exactly one value.")
        if tuple(getattr(t, "block_size", t.qdata.shape)) != tuple(t.qdata.shape):
            raise ValueError("StaticFloat8Adapter supports only the per-tensor FP8 weight layout used by TorchAO's "
                             "static workflow; use Float8Tensor's dynamic activation path for other weight "
                             "granularities.")
        if t.qdata.ndim != 2:
            raise ValueError(f"{label} merge expects a rank-two weight.")
        if t.scale.dtype is not torch.float32 or t.scale.numel() != 1:
            raise ValueError(f"{label} merge expects one float32 per-tensor scale.")
        rows, cols = t.qdata.shape
        rank, cdt = _factors(b, a, rows, cols, label)
        dev = _cuda_same_device(label, t.qdata, t.scale, b, a)
        if not t.qdata.is_contiguous():
            raise ValueError(f"{label} merge requires contiguous qdata.")
        return rows, cols, rank, cdt, dev

    @classmethod
    def validate_lora_merge(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                            rounding_seed: int | None = None) -> None:
        _seed(rounding_seed)
        cls._check(target, b, a)

    @classmethod
    def merge_desc(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                   rounding_seed: int | None = None, offset_base: int = 0, keep: list | None = None) -> nat.MergeDesc:
        rows, cols, rank, cdt, _ = cls._check(target, b, a)
        b = b.contiguous()
        a = a.contiguous()
        if keep is not None:
            keep.extend([b, a])
        seed, sflag = _seed(rounding_seed)
        return K._desc(
            qdata=target.qdata.data_ptr(), scale=target.scale.data_ptr(), b=b.data_ptr(), a=a.data_ptr(),
            rows=rows, cols=cols, rank=rank, block_rows=rows, block_cols=cols,
            format=nat.FMT_FP8_E5M2 if target.qdata.dtype is torch.float8_e5m2 else nat.FMT_FP8_E4M3,
            compute_dtype=cdt, flags=sflag, strength=float(strength), seed=seed, offset_base=int(offset_base))

    @classmethod
    def merge_lora_(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                    rounding_seed: int | None = None, offset_base: int = 0) -> None:
        keep: list = []
        d = cls.merge_desc(target, b, a, strength, rounding_seed=rounding_seed, offset_base=offset_base, keep=keep)
        nat.merge_batch([d], target.qdata.device)


# ================================================= bitsandbytes LLM.int8
class Bnb8Adapter:
    """bitsandbytes ``Int8Params`` (``CB`` int8 rows, fp32 ``SCB`` per row);
    ``bnb8bit_adapter.py:92-121`` gate, ``:285-315`` merge. LLM.int8 computes in fp16."""

    NAME = "bitsandbytes-int8"

    @staticmethod
    def matches(t: Any) -> bool:
        return _has(t, "CB", "SCB") and isinstance(t.CB, torch.Tensor) and t.CB.dtype is torch.int8

    @staticmethod
    def logical_shape(t: Any) -> tuple[int, ...]:
        return tuple(t.CB.shape)

    @staticmethod
    def compute_dtype(t: Any) -> torch.dtype:
        return torch.float16

    @classmethod
    def _check(cls, t: Any, b: torch.Tensor, a: torch.Tensor) -> tuple:
        label = "bitsandbytes 8-bit"
        if t.CB.ndim != 2:
            raise ValueError(f"{label} merge expects a rank-two weight.")
        if not isinstance(t.SCB, torch.Tensor) or t.SCB.dtype is not torch.float32:
            raise ValueError(f"{label} merge expects float32 SCB.")
        rows, cols = t.CB.shape
        if t.SCB.numel() != rows:
            raise ValueError(f"{label} merge expects one SCB value per row.")
        rank, _ = _factors(b, a, rows, cols, label)
        if b.dtype is not torch.float16 or a.dtype is not torch.float16:
            raise ValueError(f"{label} merge expects float16 LoRA factors.")
        dev = _cuda_same_device(label, t.CB, t.SCB, b, a)
        if not t.CB.is_contiguous() or not t.SCB.is_contiguous():
            raise ValueError(f"{label} merge requires contiguous CB and SCB.")
        return rows, cols, rank, dev

    @classmethod
    def validate_lora_merge(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                            rounding_seed: int | None = None) -> None:
        _seed(rounding_seed)
        cls._check(target, b, a)

    @classmethod
    def merge_desc(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                   rounding_seed: int | None = None, offset_base: int = 0, keep: list | None = None) -> nat.MergeDesc:
        rows, cols, rank, _ = cls._check(target, b, a)
        b = b.contiguous()
        a = a.contiguous()
        if keep is not None:
            keep.extend([b, a])
        seed, sflag = _seed(rounding_seed)
        return K._desc(qdata=target.CB.data_ptr(), scale=target.SCB.data_ptr(), b=b.data_ptr(), a=a.data_ptr(),
                       rows=rows, cols=cols, rank=rank, block_rows=1, block_cols=cols, format=nat.FMT_BNB8,
                       compute_dtype=nat.DT_F16, scale_dtype=nat.DT_F32, flags=sflag, strength=float(strength),
                       seed=seed, offset_base=int(offset_base))

    @classmethod
    def merge_lora_(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                    rounding_seed: int | None = None, offset_base: int = 0) -> None:
        keep: list = []
        d = cls.merge_desc(target, b, a, strength, rounding_seed=rounding_seed, offset_base=offset_base, keep=keep)
        nat.merge_batch([d], target.CB.device)


# ================================================= bitsandbytes 4-bit
class Bnb4Adapter:
    """bitsandbytes ``Params4bit`` (NF4 / FP4, plain or nested absmax);
    ``bnb4bit_adapter.py:100-160`` gate. The merge runs in the quant state's dtype."""

    NAME = "bitsandbytes-4bit"

    @staticmethod
    def matches(t: Any) -> bool:
        qs = getattr(t, "quant_state", None)
        return qs is not None and hasattr(qs, "quant_type") and isinstance(getattr(t, "data", None), torch.Tensor)

    @staticmethod
    def logical_shape(t: Any) -> tuple[int, ...]:
        return tuple(t.quant_state.shape)

    @staticmethod
    def compute_dtype(t: Any) -> torch.dtype:
        return t.quant_state.dtype

    @classmethod
    def _desc(cls, t: Any, b, a, strength, rounding_seed, offset_base, keep) -> nat.MergeDesc:
        qs = t.quant_state
        st2 = qs.state2
        if st2 is not None and getattr(st2, "blocksize", 256) != 256:
            raise ValueError("Nested BNB4 scale metadata has an unsupported layout.")
        _cuda_same_device("bitsandbytes 4-bit", t.data, qs.absmax, b, a)
        return K.bnb4_desc(t.data, qs.absmax, qs.code, None if st2 is None else st2.absmax,
                           None if st2 is None else st2.code, qs.offset if st2 is not None else None,
                           tuple(qs.shape), qs.blocksize, qs.quant_type, b, a, strength, rounding_seed=rounding_seed,
                           offset_base=offset_base, keep=keep)

    @classmethod
    def validate_lora_merge(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                            rounding_seed: int | None = None) -> None:
        _seed(rounding_seed)
        cls._desc(target, b, a, strength, rounding_seed, 0, None)

    @classmethod
    def merge_desc(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                   rounding_seed: int | None = None, offset_base: int = 0, keep: list | None = None) -> nat.MergeDesc:
        return cls._desc(target, b, a, strength, rounding_seed, offset_base, keep)

    @classmethod
    def merge_lora_(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                    rounding_seed: int | None = None, offset_base: int = 0) -> None:
        keep: list = []
        d = cls.merge_desc(target, b, a, strength, rounding_seed=rounding_seed, offset_base=offset_base, keep=keep)
        nat.merge_batch([d], target.data.device)


# ================================================================ Quanto
class QuantoAdapter:
    """optimum-quanto ``WeightQBytesTensor`` (qint8 / qfloat8 ``_data``, ``_scale``
    in the weight dtype); ``quanto_adapter.py:136-187`` gate, ``:370-440`` merge."""

    NAME = "quanto-qbytes"

    @staticmethod
    def matches(t: Any) -> bool:
        return _has(t, "_data", "_scale", "axis", "qtype")

    @staticmethod
    def logical_shape(t: Any) -> tuple[int, ...]:
        return tuple(t.size())

    @staticmethod
    def compute_dtype(t: Any) -> torch.dtype:
        return t.dtype

    @classmethod
    def _check(cls, t: Any, b: torch.Tensor, a: torch.Tensor) -> tuple:
        label = "Quanto qbytes"
        data, scale = t._data, t._scale
        if data.ndim != 2 or tuple(data.shape) != tuple(t.size()):
            raise ValueError("Quanto LoRA merge requires a rank-two weight whose qbytes storage matches its "
                             "logical shape.")
        if getattr(t.qtype, "bits", None) != 8:
            raise ValueError("Quanto qbytes LoRA merge requires an 8-bit qtype.")
        if getattr(t.qtype, "dtype", None) is not data.dtype:
            raise ValueError("Quanto qbytes storage dtype does not match its qtype metadata.")
        if not scale.dtype.is_floating_point:
            raise ValueError("Quanto qbytes LoRA merge requires floating-point scales.")
        rows, cols = data.shape
        kind = K.quanto_scale_axis(t.axis, scale, rows, cols)
        rank, cdt = _factors(b, a, rows, cols, label)
        if scale.dtype is not b.dtype:
            raise ValueError(f"{label} merge requires matching scale and factor dtypes.")
        if data.dtype is torch.int8:
            fmt = nat.FMT_QUANTO_INT8
        elif data.dtype is torch.float8_e4m3fn:
            fmt = nat.FMT_QUANTO_FP8_E4M3
        elif data.dtype is torch.float8_e5m2:
            fmt = nat.FMT_QUANTO_FP8_E5M2
        else:
            raise ValueError(f"Quanto qbytes merge supports qint8 and qfloat8 storage, got {data.dtype}.")
        dev = _cuda_same_device(label, data, scale, b, a)
        if not data.is_contiguous() or not scale.is_contiguous():
            raise ValueError(f"{label} merge requires contiguous storage.")
        return rows, cols, rank, cdt, fmt, kind, dev

    @classmethod
    def validate_lora_merge(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                            rounding_seed: int | None = None) -> None:
        _seed(rounding_seed)
        cls._check(target, b, a)

    @classmethod
    def merge_desc(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                   rounding_seed: int | None = None, offset_base: int = 0, keep: list | None = None) -> nat.MergeDesc:
        rows, cols, rank, cdt, fmt, kind, _ = cls._check(target, b, a)
        b = b.contiguous()
        a = a.contiguous()
        if keep is not None:
            keep.extend([b, a])
        seed, sflag = _seed(rounding_seed)
        brows, bcols = K.QUANTO_BLOCK[kind](rows, cols)
        return K._desc(qdata=target._data.data_ptr(), scale=target._scale.data_ptr(), b=b.data_ptr(),
                       a=a.data_ptr(), rows=rows, cols=cols, rank=rank, block_rows=brows,
                       block_cols=bcols, format=fmt, compute_dtype=cdt, scale_dtype=cdt, flags=sflag,
                       strength=float(strength), seed=seed, offset_base=int(offset_base))

    @classmethod
    def merge_lora_(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                    rounding_seed: int | None = None, offset_base: int = 0) -> None:
        keep: list = []
        d = cls.merge_desc(target, b, a, strength, rounding_seed=rounding_seed, offset_base=offset_base, keep=keep)
        nat.merge_batch([d], target._data.device)


# =================================================================== NVFP4
class Nvfp4Adapter:
    """TorchAO ``NVFP4Tensor`` (packed e2m1, e4m3 block scales, optional fp32 global scale)."""

    NAME = "torchao-nvfp4"

    @staticmethod
    def matches(t: Any) -> bool:
        return _has(t, "qdata", "scale", "per_tensor_scale", "is_swizzled_scales") and \
            getattr(t.qdata, "dtype", None) is torch.uint8

    @staticmethod
    def logical_shape(t: Any) -> tuple[int, ...]:
        rows, packed = t.qdata.shape
        return rows, packed * 2

    @staticmethod
    def compute_dtype(t: Any) -> torch.dtype:
        return t.orig_dtype

    @classmethod
    def validate_lora_merge(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                            rounding_seed: int | None = None) -> None:
        """Reject layouts whose quantizers cannot be preserved (nvfp4_adapter.py:227-252)."""
        _seed(rounding_seed)
        if not target.qdata.is_contiguous():
            raise ValueError(
                "Cannot merge LoRA into a non-contiguous (e.g. transposed) NVFP4 weight: requantization "
                "produces the standard packed layout, which cannot fill a transposed target. Use routed "
                "LoRA for this weight.")
        pts = target.per_tensor_scale
        if pts is not None and pts.numel() != 1:
            raise ValueError(
                "Cannot merge LoRA into an NVFP4 weight with a non-scalar per_tensor_scale (e.g. "
                "per-expert grouped/MoE scales); the merge recomputes a single global scale and would drop "
                "per-group precision. Use routed LoRA for this weight.")
        cls._check(target, b, a)

    @classmethod
    def _check(cls, t: Any, b: torch.Tensor, a: torch.Tensor) -> tuple:
        label = "TorchAO NVFP4"
        rows, cols = cls.logical_shape(t)
        if getattr(t, "block_size", 16) != 16:
            raise ValueError(f"{label} merge requires block_size=16.")
        rank, _ = _factors(b, a, rows, cols, label)
        if b.dtype is not t.orig_dtype or b.dtype not in (torch.bfloat16, torch.float32):  # nvfp4_adapter.py:73
            raise ValueError(f"{label} merge requires bfloat16 or float32 factors in the weight's original dtype.")
        _cuda_same_device(label, t.qdata, t.scale, b, a, t.per_tensor_scale)
        if tuple(t.scale.shape) != K.nvfp4_expected_scale_shape(rows, cols, swizzled=bool(t.is_swizzled_scales)):
            raise ValueError("NVFP4 scale shape does not match its swizzle metadata.")
        if cols % 16:
            raise ValueError("NVFP4 merge requires columns divisible by 16.")
        return rows, cols, rank

    @classmethod
    def merge_desc(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                   rounding_seed: int | None = None, offset_base: int = 0, keep: list | None = None) -> nat.MergeDesc:
        rows, cols, rank = cls._check(target, b, a)
        b = b.contiguous()
        a = a.contiguous()
        if keep is not None:
            keep.extend([b, a])
        seed, sflag = _seed(rounding_seed)
        return K._desc(
            qdata=target.qdata.data_ptr(), scale=target.scale.data_ptr(),
            global_scale=K._ptr(target.per_tensor_scale), b=b.data_ptr(), a=a.data_ptr(), rows=rows, cols=cols,
            rank=rank, format=nat.FMT_NVFP4, compute_dtype=K._dt_id(b.dtype, "LoRA factors"),
            flags=(nat.FLAG_SWIZZLED if target.is_swizzled_scales else 0) | sflag, strength=float(strength),
            seed=seed, offset_base=int(offset_base))

    @classmethod
    def merge_lora_(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                    rounding_seed: int | None = None, offset_base: int = 0) -> None:
        keep: list = []
        d = cls.merge_desc(target, b, a, strength, rounding_seed=rounding_seed, offset_base=offset_base, keep=keep)
        nat.merge_batch([d], target.qdata.device)


# ====================================================================== MX
def mx_scaling_mode_id(t: Any) -> int | None:
    """Scale rounding from ``act_quant_kwargs.scaling_mode``, FLOOR by default (mx_adapter.py:66-73)."""
    mode = getattr(getattr(t, "act_quant_kwargs", None), "scaling_mode", None)
    if mode is None:
        return MX_SCALING_MODES["floor"]
    value = getattr(mode, "value", mode)
    return MX_SCALING_MODES.get(value) if isinstance(value, str) else None


class MxAdapter:
    """TorchAO ``MXTensor`` (MXFP8 e4m3/e5m2, MXFP4 e2m1; E8M0 block-32 scales)."""

    NAME = "torchao-mx"

    @staticmethod
    def matches(t: Any) -> bool:
        return _has(t, "qdata", "scale", "elem_dtype", "block_size")

    @staticmethod
    def logical_shape(t: Any) -> tuple[int, ...]:
        rows, cols = t.qdata.shape
        return (rows, cols * 2) if t.elem_dtype is _FP4_DTYPE and _FP4_DTYPE is not None else (rows, cols)

    @staticmethod
    def compute_dtype(t: Any) -> torch.dtype:
        return t.orig_dtype

    @classmethod
    def validate_lora_merge(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                            rounding_seed: int | None = None) -> None:
        _seed(rounding_seed)
        if not target.qdata.is_contiguous():
            raise ValueError(
                "Cannot merge LoRA into a non-contiguous (e.g. transposed) MX weight: requantization produces "
                "the standard packed layout, which cannot fill a transposed target. Use routed LoRA for this "
                "weight.")
        cls._check(target, b, a)

    @classmethod
    def _check(cls, t: Any, b: torch.Tensor, a: torch.Tensor) -> tuple:
        rows, cols = cls.logical_shape(t)
        rank, _ = _factors(b, a, rows, cols, "TorchAO MX")
        mode = mx_scaling_mode_id(t)
        if mode is None:
            raise ValueError("TorchAO MX merge supports FLOOR, RCEIL, CEIL and EVEN scale rounding.")
        if t.block_size != 32:
            raise ValueError("MX merge supports block size 32.")
        if b.dtype is not t.orig_dtype or t.orig_dtype not in (torch.bfloat16, torch.float32):  # mx_adapter.py:61
            raise ValueError("MX merge requires bfloat16 or float32 factors in the weight's original dtype.")
        fmt = K.mx_format_parameters(t.elem_dtype)
        _cuda_same_device("TorchAO MX", t.qdata, t.scale, b, a)
        if tuple(t.scale.shape) != K.mx_expected_scale_shape(rows, cols, swizzled=bool(t.is_swizzled_scales)):
            raise ValueError("MX scale shape does not match its block layout.")
        if cols % 32:
            raise ValueError("MX merge requires columns divisible by 32.")
        return rows, cols, rank, fmt, mode

    @classmethod
    def merge_desc(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                   rounding_seed: int | None = None, offset_base: int = 0, keep: list | None = None) -> nat.MergeDesc:
        rows, cols, rank, fmt, mode = cls._check(target, b, a)
        b = b.contiguous()
        a = a.contiguous()
        if keep is not None:
            keep.extend([b, a])
        seed, sflag = _seed(rounding_seed)
        return K._desc(
            qdata=target.qdata.data_ptr(), scale=target.scale.data_ptr(), b=b.data_ptr(), a=a.data_ptr(),
            rows=rows, cols=cols, rank=rank, format=fmt, compute_dtype=K._dt_id(b.dtype, "LoRA factors"),
            scale_mode=mode,
            flags=(nat.FLAG_SWIZZLED if target.is_swizzled_scales else 0) | sflag, strength=float(strength),
            seed=seed, offset_base=int(offset_base))

    @classmethod
    def merge_lora_(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                    rounding_seed: int | None = None, offset_base: int = 0) -> None:
        keep: list = []
        d = cls.merge_desc(target, b, a, strength, rounding_seed=rounding_seed, offset_base=offset_base, keep=keep)
        nat.merge_batch([d], target.qdata.device)


# ==================================================================== GGUF
class GgufAdapter:
    """GGUF Q8_0 / Q4_0 raw block rows (``GGUFWeight``: uint8 data + ``quant_type``).

    The reference moves GGUF weights but never merges them ("GGUF (k-quants) --
    routed only", README.md:1001); this adapter adds the merge capability.
    """

    NAME = "gguf"

    @staticmethod
    def matches(t: Any) -> bool:
        return hasattr(t, "quant_type") and int(getattr(t, "quant_type", -1)) in (K.GGUF_Q8_0, K.GGUF_Q4_0)

    @staticmethod
    def _raw(t: Any) -> torch.Tensor:
        return t.raw if hasattr(t, "raw") else t

    @classmethod
    def logical_shape(cls, t: Any) -> tuple[int, ...]:
        raw = cls._raw(t)
        return raw.shape[0], K.gguf_logical_cols(raw.shape[1], int(t.quant_type))

    @staticmethod
    def compute_dtype(t: Any) -> torch.dtype:
        return getattr(t, "compute_dtype", torch.bfloat16)

    @classmethod
    def validate_lora_merge(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                            rounding_seed: int | None = None) -> None:
        _seed(rounding_seed)
        cls._check(target, b, a)

    @classmethod
    def _check(cls, t: Any, b: torch.Tensor, a: torch.Tensor) -> tuple:
        raw = cls._raw(t)
        if raw.dtype is not torch.uint8 or raw.ndim != 2 or not raw.is_contiguous():
            raise ValueError("GGUF merge expects contiguous rank-two uint8 raw blocks.")
        rows, cols = cls.logical_shape(t)
        rank, cdt = _factors(b, a, rows, cols, "GGUF")
        _cuda_same_device("GGUF", raw, b, a)
        return rows, cols, rank, cdt

    @classmethod
    def merge_desc(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                   rounding_seed: int | None = None, offset_base: int = 0, keep: list | None = None) -> nat.MergeDesc:
        rows, cols, rank, cdt = cls._check(target, b, a)
        b = b.contiguous()
        a = a.contiguous()
        if keep is not None:
            keep.extend([b, a])
        seed, sflag = _seed(rounding_seed)
        return K._desc(
            qdata=cls._raw(target).data_ptr(), b=b.data_ptr(), a=a.data_ptr(), rows=rows, cols=cols, rank=rank,
            format=nat.FMT_GGUF_Q8_0 if int(target.quant_type) == K.GGUF_Q8_0 else nat.FMT_GGUF_Q4_0,
            compute_dtype=cdt, flags=sflag, strength=float(strength), seed=seed, offset_base=int(offset_base))

    @classmethod
    def merge_lora_(cls, target: Any, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                    rounding_seed: int | None = None, offset_base: int = 0) -> None:
        keep: list = []
        d = cls.merge_desc(target, b, a, strength, rounding_seed=rounding_seed, offset_base=offset_base, keep=keep)
        nat.merge_batch([d], cls._raw(target).device)


# ================================================================ registry
_ADAPTERS: list[type] = [MxAdapter, Nvfp4Adapter, StaticFloat8Adapter, Float8Adapter, Int8Adapter,
                         Bnb8Adapter, QuantoAdapter, Bnb4Adapter, GgufAdapter]


def register_adapter(adapter: type, *, first: bool = True) -> None:
    """Add an adapter (dispatch order mirrors ``tensor_adapter_registry.py:38-51``)."""
    if adapter in _ADAPTERS:
        _ADAPTERS.remove(adapter)
    _ADAPTERS.insert(0 if first else len(_ADAPTERS), adapter)


def select_adapter(t: Any) -> type:
    for ad in _ADAPTERS:
        if ad.matches(t):
            return ad
    raise NotImplementedError(f"no LoRA-merge adapter for {type(t).__name__}")


def target_device(t: Any) -> torch.device:
    for name in ("raw", "qdata", "CB", "_data", "data"):
        raw = getattr(t, name, None)
        if isinstance(raw, torch.Tensor):
            return raw.device
    return t.device


def merge_lora_batch(ops: Sequence[tuple], *, workspace: torch.Tensor | None = None) -> None:
    """Merge many weights with one C-ABI call per device.

    ``ops``: ``(target, b, a, strength, rounding_seed[, offset_base])`` tuples.
    Every op is validated before any launch, so a bad op mutates nothing
    (the preflight of ``merge.py:118-125``).
    """
    by_dev: dict[torch.device, list] = {}
    keep: list = []
    for op in ops:
        target, b, a, strength, seed = op[:5]
        offset_base = op[5] if len(op) > 5 else 0
        ad = select_adapter(target)
        d = ad.merge_desc(target, b, a, strength, rounding_seed=seed, offset_base=offset_base, keep=keep)
        by_dev.setdefault(target_device(target), []).append(d)
    for dev, descs in by_dev.items():
        nat.merge_batch(descs, dev, workspace)

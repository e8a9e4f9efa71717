"""Light stand-ins for the quantized weight wrappers the adapters merge into.

They carry TorchAO's attribute names (``Int8Tensor``, ``Float8Tensor``,
``NVFP4Tensor``, ``MXTensor``) and the reference's ``GGUFWeight``
(``gguf_adapter.py:61-105``) so that the adapters can be used and tested
without TorchAO, which is absent from this image. A real TorchAO tensor with
the same attributes dispatches to the same adapter.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch


@dataclass
class Int8Weight:
    qdata: torch.Tensor
    scale: torch.Tensor
    block_size: tuple[int, int]
    dtype: torch.dtype = torch.bfloat16
    zero_point: torch.Tensor | None = None
    act_pre_scale: torch.Tensor | None = None
    reduce_range: bool = False

    @property
    def shape(self) -> torch.Size:
        return self.qdata.shape


@dataclass
class Float8Weight:
    qdata: torch.Tensor
    scale: torch.Tensor
    block_size: tuple[int, int]
    dtype: torch.dtype = torch.bfloat16

    @property
    def shape(self) -> torch.Size:
        return self.qdata.shape


@dataclass
class StaticFloat8Weight:
    """TorchAO's calibrated ``PrototypeFloat8Tensor``: per-tensor FP8 weight plus
    a static activation scale that a merge leaves alone
    (``static_float8_adapter.py:241-248``)."""

    qdata: torch.Tensor
    scale: torch.Tensor
    act_quant_scale: torch.Tensor
    block_size: tuple[int, int] = ()
    dtype: torch.dtype = torch.bfloat16

    def __post_init__(self) -> None:
        if not self.block_size:
            self.block_size = tuple(self.qdata.shape)

    @property
    def shape(self) -> torch.Size:
        return self.qdata.shape


@dataclass
class Bnb8Weight:
    """bitsandbytes ``Int8Params`` before its first forward: row-major int8
    ``CB`` and one fp32 ``SCB`` per row (``bnb8bit_adapter.py:1-35``)."""

    CB: torch.Tensor
    SCB: torch.Tensor

    @property
    def shape(self) -> torch.Size:
        return self.CB.shape


@dataclass(frozen=True)
class QuantoQType:
    """The parts of an optimum-quanto ``qtype`` the merge reads."""

    name: str
    bits: int
    is_floating_point: bool
    dtype: torch.dtype
    qmax: float


QINT8 = QuantoQType("qint8", 8, False, torch.int8, 127.0)
QFLOAT8_E4M3 = QuantoQType("qfloat8_e4m3fn", 8, True, torch.float8_e4m3fn, 448.0)
QFLOAT8_E5M2 = QuantoQType("qfloat8_e5m2", 8, True, torch.float8_e5m2, 57344.0)


@dataclass
class QuantoWeight:
    """optimum-quanto ``WeightQBytesTensor``: ``_data`` codes, ``_scale`` in the
    compute dtype, ``axis`` (None, 0 or -1) and ``qtype`` (``quanto_adapter.py:1-30``)."""

    _data: torch.Tensor
    _scale: torch.Tensor
    axis: int | None
    qtype: QuantoQType
    dtype: torch.dtype | None = None

    def __post_init__(self) -> None:
        if self.dtype is None:
            self.dtype = self._scale.dtype

    @property
    def shape(self) -> torch.Size:
        return self._data.shape

    def size(self) -> torch.Size:
        return self._data.shape


@dataclass
class Bnb4State:
    """The parts of a bitsandbytes ``QuantState`` the merge reads
    (``bnb4bit_adapter.py:100-160``); ``state2`` / ``offset`` for nested absmax."""

    absmax: torch.Tensor
    code: torch.Tensor
    shape: tuple[int, int]
    quant_type: str = "nf4"
    blocksize: int = 64
    dtype: torch.dtype = torch.bfloat16
    state2: "Bnb4State | None" = None
    offset: torch.Tensor | None = None

    @property
    def nested(self) -> bool:
        return self.state2 is not None


@dataclass
class Bnb4Weight:
    """bitsandbytes ``Params4bit``: packed uint8 ``data`` (two values per byte,
    the first in the high nibble) and its ``quant_state``."""

    data: torch.Tensor
    quant_state: Bnb4State

    @property
    def shape(self) -> torch.Size:
        return torch.Size(self.quant_state.shape)


@dataclass
class NVFP4Weight:
    qdata: torch.Tensor
    scale: torch.Tensor
    per_tensor_scale: torch.Tensor | None = None
    block_size: int = 16
    orig_dtype: torch.dtype = torch.bfloat16
    is_swizzled_scales: bool = False

    @property
    def shape(self) -> tuple[int, int]:
        return self.qdata.shape[0], self.qdata.shape[1] * 2


@dataclass
class MXScalingMode:
    value: str = "floor"


@dataclass
class MXActQuantKwargs:
    scaling_mode: Any = None


@dataclass
class MXWeight:
    qdata: torch.Tensor
    scale: torch.Tensor
    elem_dtype: Any
    block_size: int = 32
    orig_dtype: torch.dtype = torch.bfloat16
    is_swizzled_scales: bool = False
    act_quant_kwargs: Any = field(default_factory=MXActQuantKwargs)

    @property
    def shape(self) -> tuple[int, int]:
        fp4 = getattr(torch, "float4_e2m1fn_x2", None)
        rows, cols = self.qdata.shape
        return (rows, cols * 2) if fp4 is not None and self.elem_dtype is fp4 else (rows, cols)


@dataclass
class GGUFWeight:
    raw: torch.Tensor
    quant_type: int
    compute_dtype: torch.dtype = torch.bfloat16

    @property
    def shape(self) -> tuple[int, int]:
        from .kernels import gguf_logical_cols

        return self.raw.shape[0], gguf_logical_cols(self.raw.shape[1], self.quant_type)

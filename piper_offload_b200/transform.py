"""LoRA transform and permanent merge, mirroring the reference's merge driver.

* :class:`LoRATransform` restates the merge half of ``src/piper_offload/lora.py``
  (``LoRATransform`` :314-724): per-merge seeds ``derive_seed(target_key,
  merge_index)`` (:356-359), validation before application (:361-428),
  single-factor staging ``B, A -> .to(device, compute_dtype).contiguous()``
  (:596-626) and multi-LoRA packing ``A = [s_i * A_i]``, ``B = [B_i]`` with unit
  strength (:685-724), then the adapter's ``merge_lora_`` (:535-567).
* :func:`merge_lora` restates ``src/piper_offload/merge.py:54-214``: reject a
  LoRA passed twice, drop zero strengths, check that every targeted weight
  exists, group factors per weight, validate every weight before mutating
  any, then apply. Unlike the reference's per-weight loop, application is one
  batched C-ABI call per device (``piper_merge_batch``).

Factors are staged once per application. The reference stages them in
validation and again in application (``lora.py:406-413`` and ``:543-549``), one
host-to-device copy per factor tensor each time. Here validation keeps what it
staged for the next application, and :func:`stage_factors` stages a whole
batch with one host-to-device copy per device: host-resident factors are
converted to the compute dtype on the host into one pinned buffer.

Weights are addressed by name in a mapping (the reference walks an
``nn.Module``); a LoRA is a mapping from weight name to ``(A, B)`` factors.
"""

from __future__ import annotations

import logging
from collections.abc import Mapping, Sequence
from dataclasses import dataclass
from typing import Any

import torch

from . import adapters as AD
from .seeding import derive_seed

log = logging.getLogger(__name__)


@dataclass(frozen=True)
class LoRAFactor:
    """One LoRA pair: ``a`` (rank x in_features), ``b`` (out_features x rank)."""

    a: torch.Tensor
    b: torch.Tensor
    strength: float = 1.0

    def __post_init__(self) -> None:
        if self.a.ndim != 2 or self.b.ndim != 2:
            raise ValueError("LoRA factors must be rank two.")
        if self.b.shape[1] != self.a.shape[0]:
            raise ValueError(
                f"LoRA factor inner dimensions do not match: B={tuple(self.b.shape)}, A={tuple(self.a.shape)}.")

    @property
    def produced_shape(self) -> tuple[int, int]:
        return self.b.shape[0], self.a.shape[1]

    def scaled(self, strength: float) -> "LoRAFactor":
        return LoRAFactor(self.a, self.b, self.strength * strength)


@dataclass
class _Plan:
    adapter: type
    compute_dtype: torch.dtype
    logical_shape: tuple[int, ...]


class LoRATransform:
    """LoRA factors applied to one quantized weight (merge path of ``lora.py:314``)."""

    __slots__ = ("_factors", "_merge_index", "_stochastic_rounding", "_target_key", "_plan", "_staged")

    def __init__(self, factors: Sequence[LoRAFactor], *, stochastic_rounding: bool = False,
                 target_key: str = "") -> None:
        if stochastic_rounding and not target_key:
            raise ValueError("Stochastic LoRATransform requires a non-empty target_key.")
        if not factors:
            raise ValueError("LoRATransform requires at least one factor.")
        self._factors = list(factors)
        self._stochastic_rounding = stochastic_rounding
        self._target_key = target_key
        self._merge_index = 0
        self._plan: _Plan | None = None
        self._staged: tuple[torch.Tensor, torch.Tensor, float] | None = None

    @property
    def merge_index(self) -> int:
        return self._merge_index

    def _rounding_seed(self) -> int | None:
        if not self._stochastic_rounding:
            return None
        return derive_seed(self._target_key, self._merge_index)

    # ------------------------------------------------------------ validation
    def _make_plan(self, target: Any) -> _Plan:
        try:
            adapter = AD.select_adapter(target)
        except NotImplementedError as exc:
            raise ValueError(
                f"Tensor type {type(target).__name__} has no registered tensor adapter. "
                "Merge requires a tensor adapter with LoRA merge support.") from exc
        shape = tuple(adapter.logical_shape(target))
        dtype = adapter.compute_dtype(target)
        if not dtype.is_floating_point:
            raise ValueError(f"LoRA merge requires a floating-point compute dtype, got {dtype}.")
        for f in self._factors:
            if tuple(f.produced_shape) != shape:
                raise ValueError(
                    f"LoRA factor shape mismatch: B@A produces {tuple(f.produced_shape)}, target shape is {shape}.")
        return _Plan(adapter, dtype, shape)

    def validate_target(self, target: Any, *,
                        staged: tuple[torch.Tensor, torch.Tensor, float] | None = None) -> None:
        """Preflight the weight update and remember the plan (``lora.py:361-428``).

        The staged factors (``staged``, else staged here) are kept for the next
        application, so a validated merge copies its factors to the device once.
        """
        self._plan = None
        self._staged = None
        plan = self._make_plan(target)
        b, a, s = staged if staged is not None else self._stage(target, plan)
        plan.adapter.validate_lora_merge(target, b, a, s, rounding_seed=self._rounding_seed())
        self._plan = plan
        self._staged = (b, a, s)

    def _take_staged(self, target: Any) -> tuple[torch.Tensor, torch.Tensor, float]:
        staged, self._staged = self._staged, None
        return staged if staged is not None else self._stage(target, self._plan)

    # --------------------------------------------------------------- staging
    def _stage(self, target: Any, plan: _Plan) -> tuple[torch.Tensor, torch.Tensor, float]:
        device = AD.target_device(target)
        dt = plan.compute_dtype
        if len(self._factors) == 1:
            f = self._factors[0]
            return (f.b.to(device=device, dtype=dt, non_blocking=True).contiguous(),
                    f.a.to(device=device, dtype=dt, non_blocking=True).contiguous(), f.strength)
        total = sum(f.a.shape[0] for f in self._factors)
        rows, cols = plan.logical_shape
        a_packed = torch.empty((total, cols), device=device, dtype=dt)
        b_packed = torch.empty((rows, total), device=device, dtype=dt)
        off = 0
        for f in self._factors:
            nxt = off + f.a.shape[0]
            a_slice = a_packed[off:nxt]
            a_slice.copy_(f.a, non_blocking=True)
            b_packed[:, off:nxt].copy_(f.b, non_blocking=True)
            if f.strength != 1.0:
                a_slice.mul_(f.strength)
            off = nxt
        return b_packed, a_packed, 1.0

    # ----------------------------------------------------------- application
    def merge_op(self, target: Any) -> tuple:
        """Stage this transform's next application as a ``merge_lora_batch`` op."""
        if self._plan is None:
            raise RuntimeError("LoRA weight target must be validated before application.")
        b, a, s = self._take_staged(target)
        op = (target, b, a, s, self._rounding_seed())
        self._merge_index += 1
        return op

    def apply_weight(self, target: Any) -> None:
        """Apply to a previously validated target (``lora.py:445-463``)."""
        if self._plan is None:
            raise RuntimeError("LoRA weight target must be validated before application.")
        b, a, s = self._take_staged(target)
        self._plan.adapter.merge_lora_(target, b, a, s, rounding_seed=self._rounding_seed())
        self._merge_index += 1


_STAGE_ALIGN = 256  # byte alignment of each staged factor inside the shared buffers


def stage_factors(pairs: Sequence[tuple[LoRATransform, Any]]) -> list[tuple[torch.Tensor, torch.Tensor, float]]:
    """Stage the factors of many ``(transform, target)`` pairs for their next application.

    Equal to each transform's own staging, value for value. Factors that live
    on the host and are bound for a CUDA device are converted to the compute
    dtype on the host, packed into one pinned buffer per device and moved with
    one copy; multi-LoRA ``A`` slices are then scaled on the device exactly as
    the per-weight packing does (``lora.py:685-724``). Pairs with any factor
    already on a device, or whose target is on the host, stage per weight.
    """
    out: list = [None] * len(pairs)
    plans = [t._make_plan(x) for t, x in pairs]
    groups: dict[torch.device, list[int]] = {}
    for i, ((t, x), plan) in enumerate(zip(pairs, plans)):
        dev = AD.target_device(x)
        host = all(f.a.device.type == "cpu" and f.b.device.type == "cpu" for f in t._factors)
        if dev.type == "cuda" and host:
            groups.setdefault(dev, []).append(i)
        else:
            out[i] = t._stage(x, plan)
    for dev, idx in groups.items():
        layout = []  # per pair: (b_off, b_shape, a_off, a_shape, dtype, scales)
        total = 0
        for i in idx:
            t, plan = pairs[i][0], plans[i]
            rows, cols = plan.logical_shape
            rank = sum(f.a.shape[0] for f in t._factors)
            esz = torch.empty((), dtype=plan.compute_dtype).element_size()
            b_off = total
            total += -(-rows * rank * esz // _STAGE_ALIGN) * _STAGE_ALIGN
            a_off = total
            total += -(-rank * cols * esz // _STAGE_ALIGN) * _STAGE_ALIGN
            layout.append((b_off, (rows, rank), a_off, (rank, cols), plan.compute_dtype))
        host_buf = torch.empty(total, dtype=torch.uint8, pin_memory=True)
        for i, (b_off, b_shape, a_off, a_shape, dt) in zip(idx, layout):
            fs = pairs[i][0]._factors
            hb = _view(host_buf, b_off, b_shape, dt)
            ha = _view(host_buf, a_off, a_shape, dt)
            r0 = 0
            for f in fs:
                r1 = r0 + f.a.shape[0]
                hb[:, r0:r1].copy_(f.b)
                ha[r0:r1].copy_(f.a)
                r0 = r1
        dev_buf = torch.empty(total, dtype=torch.uint8, device=dev)
        dev_buf.copy_(host_buf, non_blocking=True)
        for i, (b_off, b_shape, a_off, a_shape, dt) in zip(idx, layout):
            fs = pairs[i][0]._factors
            b = _view(dev_buf, b_off, b_shape, dt)
            a = _view(dev_buf, a_off, a_shape, dt)
            if len(fs) == 1:
                out[i] = (b, a, fs[0].strength)
                continue
            r0 = 0
            for f in fs:
                r1 = r0 + f.a.shape[0]
                if f.strength != 1.0:
                    a[r0:r1].mul_(f.strength)
                r0 = r1
            out[i] = (b, a, 1.0)
    return out


def _view(buf: torch.Tensor, off: int, shape: tuple[int, int], dtype: torch.dtype) -> torch.Tensor:
    n = shape[0] * shape[1] * torch.empty((), dtype=dtype).element_size()
    return buf[off:off + n].view(dtype).view(shape)


def _as_factor(value: Any) -> LoRAFactor:
    if isinstance(value, LoRAFactor):
        return value
    a, b = value
    return LoRAFactor(a, b)


def merge_lora(weights: Mapping[str, Any], loras: Sequence[tuple[Mapping[str, Any], float]], *,
               stochastic_rounding: bool = True) -> int:
    """Permanently merge LoRAs into quantized weights; returns the number of weights merged.

    ``loras`` is a sequence of ``(targets, strength)`` where ``targets`` maps
    weight names to ``LoRAFactor`` or ``(A, B)`` pairs.
    """
    seen: set[int] = set()
    grouped: dict[str, list[LoRAFactor]] = {}
    for targets, strength in loras:
        if id(targets) in seen:
            raise ValueError("merge_lora() received the same LoRA more than once.")
        seen.add(id(targets))
        if strength == 0:
            continue
        missing = sorted(set(targets) - set(weights))
        if missing:
            raise ValueError(f"LoRA targets weights missing from the model: {missing[:5]}")
        for name, value in targets.items():
            grouped.setdefault(name, []).append(_as_factor(value).scaled(strength))
    transforms = {name: LoRATransform(f, stochastic_rounding=stochastic_rounding, target_key=name)
                  for name, f in grouped.items()}
    pairs = [(t, weights[name]) for name, t in transforms.items()]
    for (t, target), staged in zip(pairs, stage_factors(pairs)):  # every weight validates before any mutates
        t.validate_target(target, staged=staged)
    AD.merge_lora_batch([t.merge_op(target) for t, target in pairs])
    if transforms:
        log.info("merged LoRA into %d weight(s)", len(transforms))
    return len(transforms)

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

    __slots__ = ("_factors", "_merge_index", "_stochastic_rounding", "_target_key", "_plan")

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

    @property
    def merge_index(self) -> int:
        return self._merge_index

    def _rounding_seed(self) -> int | None:
        if not self._stochastic_rounding:
            return None
        return derive_seed(self._target_key, self._merge_index)

    # ------------------------------------------------------------ validation
    def validate_target(self, target: Any) -> None:
        """Preflight the weight update and remember the plan (``lora.py:361-428``)."""
        self._plan = None
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
        plan = _Plan(adapter, dtype, shape)
        b, a, s = self._stage(target, plan)
        adapter.validate_lora_merge(target, b, a, s, rounding_seed=self._rounding_seed())
        self._plan = plan

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
        b, a, s = self._stage(target, self._plan)
        op = (target, b, a, s, self._rounding_seed())
        self._merge_index += 1
        return op

    def apply_weight(self, target: Any) -> None:
        """Apply to a previously validated target (``lora.py:445-463``)."""
        if self._plan is None:
            raise RuntimeError("LoRA weight target must be validated before application.")
        b, a, s = self._stage(target, self._plan)
        self._plan.adapter.merge_lora_(target, b, a, s, rounding_seed=self._rounding_seed())
        self._merge_index += 1


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
    for name, t in transforms.items():  # every weight validates before any mutates
        t.validate_target(weights[name])
    AD.merge_lora_batch([t.merge_op(weights[name]) for name, t in transforms.items()])
    if transforms:
        log.info("merged LoRA into %d weight(s)", len(transforms))
    return len(transforms)

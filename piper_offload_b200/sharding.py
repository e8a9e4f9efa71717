"""Shard-local merges and the multi-GPU partition of a merge workload.

DTensor shard-local merge (``src/piper_offload/dtensor_adapter.py:116-600``):
:func:`local_shape_and_offsets` applies Replicate / contiguous Shard
placements left to right (``:116-178``), :func:`local_lora_factors` narrows
B's rows and A's columns to the local shard (``:272-300``) and
:func:`localize_rounding_seed` keeps replicas aligned while giving shards
distinct samples, ``derive_seed(seed, *offsets)`` (``:200-207``). No
collective is needed: the LoRA rank dimension is never sharded.

:func:`shard_merge_desc_args` adds the second seed semantics the B200 build
needs for row shards: ``mode="global"`` keeps the unsharded seed and keys the
stochastic stream by GLOBAL element offsets, so any row partition reproduces
the single-GPU merge byte for byte.

:func:`partition` is the multi-GPU planner: weights are independent, so the
work is split with no data-path collective, by whole weights (bytes-balanced
longest-processing-time greedy) and, for layouts whose scales never span rows
(per-row / per-block formats), by contiguous 128-row output shards.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import torch

from .seeding import derive_seed


def _shard_size_and_offset(size: int, chunks: int, index: int) -> tuple[int, int]:
    try:
        from torch.distributed.tensor import Shard

        s, o = Shard.local_shard_size_and_offset(size, chunks, index)
        return int(s), int(o)
    except (ImportError, AttributeError):  # pragma: no cover - same rule, restated
        block = (size + chunks - 1) // chunks
        start = block * index
        if size < start:
            return 0, size
        return min(size, start + block) - start, start


def _placement_kind(p) -> tuple[str, int | None]:
    if isinstance(p, tuple):
        return p[0], (p[1] if len(p) > 1 else None)
    name = type(p).__name__
    if name == "Replicate":
        return "replicate", None
    if name == "Shard" and type(p).__module__.startswith("torch"):
        return "shard", p.dim
    return name.lower(), getattr(p, "dim", None)


def local_shape_and_offsets(global_shape: Sequence[int], mesh_shape: Sequence[int], coordinate: Sequence[int],
                            placements: Sequence) -> tuple[tuple[int, ...], tuple[int, ...]]:
    """This rank's contiguous shard shape and global offsets."""
    if not (len(mesh_shape) == len(coordinate) == len(placements)):
        raise ValueError(
            "DTensor LoRA merge requires one placement and coordinate per mesh dimension; mesh shape is "
            f"{tuple(mesh_shape)}, coordinate is {tuple(coordinate)}, and placements are {tuple(placements)}.")
    local = list(global_shape)
    offsets = [0] * len(global_shape)
    for mesh_dim, (size, coord, p) in enumerate(zip(mesh_shape, coordinate, placements, strict=True)):
        kind, dim = _placement_kind(p)
        if kind == "replicate":
            continue
        if kind != "shard":
            raise ValueError(
                "DTensor LoRA merge supports only Replicate and contiguous Shard placements; mesh dimension "
                f"{mesh_dim} uses {p!r}. Use routed LoRA for this layout.")
        if dim < 0:
            dim += len(global_shape)
        if not 0 <= dim < len(global_shape):
            raise ValueError(f"DTensor LoRA merge placement {p!r} refers to tensor dimension {dim}, but the "
                             f"target shape is {tuple(global_shape)}.")
        shard, rel = _shard_size_and_offset(local[dim], size, coord)
        local[dim] = shard
        offsets[dim] = global_shape[dim] if shard == 0 else offsets[dim] + rel
    return tuple(local), tuple(offsets)


def localize_rounding_seed(seed: int | None, offsets: Sequence[int]) -> int | None:
    return None if seed is None else derive_seed(seed, *offsets)


def local_lora_factors(b: torch.Tensor, a: torch.Tensor, *, global_shape: Sequence[int],
                       local_shape: Sequence[int], offsets: Sequence[int]) -> tuple[torch.Tensor, torch.Tensor]:
    """Accept global or already-local factors and return this shard's slices."""
    if b.ndim != 2 or a.ndim != 2 or b.shape[1] != a.shape[0]:
        raise ValueError("DTensor LoRA factors must be rank two with matching inner dimensions, "
                         f"got B={tuple(b.shape)}, A={tuple(a.shape)}.")
    produced = (b.shape[0], a.shape[1])
    if produced == tuple(local_shape):
        return b.contiguous(), a.contiguous()
    if produced == tuple(global_shape):
        return (b.narrow(0, offsets[0], local_shape[0]).contiguous(),
                a.narrow(1, offsets[1], local_shape[1]).contiguous())
    raise ValueError(f"DTensor LoRA factors must match either the global or local weight shape: global="
                     f"{tuple(global_shape)}, local={tuple(local_shape)}, B={tuple(b.shape)}, A={tuple(a.shape)}.")


def shard_merge_args(seed: int | None, *, global_shape: Sequence[int], offsets: Sequence[int],
                     mode: str = "dtensor") -> tuple[int | None, int]:
    """``(rounding_seed, offset_base)`` for a shard-local merge.

    ``mode="dtensor"`` is the reference rule (local offsets, per-shard seed);
    ``mode="global"`` reproduces the unsharded stream (row shards only).
    """
    if mode == "dtensor":
        return localize_rounding_seed(seed, offsets), 0
    if mode == "global":
        if offsets[1] != 0:
            raise ValueError("global-offset stochastic merges require full-width (row) shards.")
        return seed, int(offsets[0]) * int(global_shape[1])
    raise ValueError(f"unknown shard seed mode {mode!r}")


# ---------------------------------------------------------------- partition
@dataclass(frozen=True)
class WorkItem:
    key: str
    rows: int
    cols: int
    bytes_per_row: int
    row_splittable: bool = True


@dataclass(frozen=True)
class Shard:
    key: str
    row_begin: int
    row_end: int
    cols: int
    bytes: int

    @property
    def offset_base(self) -> int:
        """First element's global offset (stochastic stream of the unsharded merge)."""
        return self.row_begin * self.cols


def partition(items: Sequence[WorkItem], world: int, *, split_rows: bool = True,
              granularity: int = 128) -> list[list[Shard]]:
    """Bytes-balanced assignment of weights (and row shards) to ``world`` ranks."""
    if world < 1:
        raise ValueError("world size must be positive")
    total = sum(it.rows * it.bytes_per_row for it in items)
    target = total / world if world else total
    pieces: list[Shard] = []
    for it in items:
        nbytes = it.rows * it.bytes_per_row
        if split_rows and it.row_splittable and world > 1 and nbytes > target and it.rows > granularity:
            n = min(world, -(-nbytes // int(max(target, 1))), -(-it.rows // granularity))
            step = -(-it.rows // n)
            step = -(-step // granularity) * granularity
            for r0 in range(0, it.rows, step):
                r1 = min(it.rows, r0 + step)
                pieces.append(Shard(it.key, r0, r1, it.cols, (r1 - r0) * it.bytes_per_row))
        else:
            pieces.append(Shard(it.key, 0, it.rows, it.cols, nbytes))
    pieces.sort(key=lambda s: (-s.bytes, s.key, s.row_begin))
    loads = [0] * world
    out: list[list[Shard]] = [[] for _ in range(world)]
    for p in pieces:
        r = min(range(world), key=lambda i: (loads[i], i))
        out[r].append(p)
        loads[r] += p.bytes
    for lst in out:
        lst.sort(key=lambda s: (s.key, s.row_begin))
    return out

"""Streamed-block merge pipeline for host-resident quantized weights.

Piper Offload keeps models in pinned host memory and moves transformer blocks
onto the GPU through a prefetch stream, so that the copy of block i+1 overlaps
the work on block i (``streamed_component.py:1398-1419``, ``_load_block`` on a
``torch.cuda.Stream``). ``merge_streamed`` applies that pattern to LoRA
merging. Weights whose storages live in pinned host memory are merged in place
through a ring of ``depth`` device slots on three CUDA streams:

* host-to-device copies of block i+1 on an upload stream;
* the merge of block i on the caller's current stream (one C-ABI batch per block);
* device-to-host copies of block i-1 on a download stream.

Events order the three streams. A slot is refilled only after its previous
block has been downloaded. On return the caller's stream is ordered after every
download; call ``torch.cuda.synchronize`` (or wait on that stream) before
reading the host tensors. Results equal ``adapters.merge_lora_batch`` on the
same weights bit for bit (same kernels, same seeds).
"""

from __future__ import annotations

import copy
from dataclasses import dataclass
from typing import Sequence

import torch

from .adapters import merge_lora_batch

STORAGE_NAMES = ("qdata", "scale", "zero_point", "per_tensor_scale", "raw", "CB", "SCB", "_data", "_scale")


@dataclass
class StreamedOp:
    """One weight merge: ``target`` is a weight wrapper (``weights.py`` types)
    whose storage tensors are pinned host tensors; ``b``/``a`` are the factors
    (pinned host or device)."""

    target: object
    b: torch.Tensor
    a: torch.Tensor
    strength: float
    rounding_seed: int | None = None
    offset_base: int = 0


def storages(target) -> list[tuple[str, torch.Tensor]]:
    """The (name, tensor) storage fields of a weight wrapper."""
    out = []
    for name in STORAGE_NAMES:
        t = getattr(target, name, None)
        if isinstance(t, torch.Tensor):
            out.append((name, t))
    return out


def block_signature(block: Sequence[StreamedOp]) -> tuple:
    """Types, shapes and dtypes that decide whether a device slot can be reused."""
    sig = []
    for op in block:
        sig.append((type(op.target).__name__,
                    tuple((n, tuple(t.shape), t.dtype) for n, t in storages(op.target)),
                    tuple(op.b.shape), op.b.dtype, tuple(op.a.shape), op.a.dtype))
    return tuple(sig)


class _Slot:
    def __init__(self, block: Sequence[StreamedOp], device: torch.device, streams: Sequence[torch.cuda.Stream]):
        self.signature = block_signature(block)
        self.twins = []
        self.factors = []
        for op in block:
            twin = copy.copy(op.target)
            for name, t in storages(op.target):
                d = torch.empty_like(t, device=device)
                for s in streams:
                    d.record_stream(s)
                setattr(twin, name, d)
            bd = torch.empty_like(op.b, device=device)
            ad = torch.empty_like(op.a, device=device)
            for s in streams:
                bd.record_stream(s)
                ad.record_stream(s)
            self.twins.append(twin)
            self.factors.append((bd, ad))


def _check_host(block: Sequence[StreamedOp]) -> None:
    for op in block:
        for name, t in storages(op.target):
            if t.device.type != "cpu":
                raise ValueError(f"merge_streamed expects host storages; {name} is on {t.device}.")


def merge_streamed(blocks: Sequence[Sequence[StreamedOp]], device, *, depth: int = 3,
                   workspace: torch.Tensor | None = None) -> None:
    """Merge every op of every block in place in its host storages.

    ``depth`` device slots hold a block each (3 lets upload, merge and
    download run at once). Every block is validated, through the same
    preflight as ``merge_lora_batch``, before its merge is enqueued; an invalid
    op raises ``ValueError`` and leaves that block's host storages unchanged.
    """
    if depth < 1:
        raise ValueError("depth must be at least 1.")
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("merge_streamed needs a CUDA device.")
    compute = torch.cuda.current_stream(dev)
    up = torch.cuda.Stream(dev)
    down = torch.cuda.Stream(dev)
    try:
        slots: list[_Slot | None] = [None] * depth
        freed: list[torch.cuda.Event | None] = [None] * depth
        for i, block in enumerate(blocks):
            _check_host(block)
            k = i % depth
            slot = slots[k]
            if slot is None or slot.signature != block_signature(block):
                if freed[k] is not None:
                    compute.wait_event(freed[k])  # the old slot's tensors are released in stream order
                with torch.cuda.stream(compute):
                    slot = _Slot(block, dev, (up, down))
                slots[k] = slot
            with torch.cuda.stream(up):
                if freed[k] is None:
                    up.wait_stream(compute)  # a fresh slot: its memory may have had earlier users on `compute`
                else:
                    up.wait_event(freed[k])  # the slot's previous block has been downloaded
                for op, twin, (bd, ad) in zip(block, slot.twins, slot.factors):
                    for name, src in storages(op.target):
                        getattr(twin, name).copy_(src, non_blocking=True)
                    bd.copy_(op.b, non_blocking=True)
                    ad.copy_(op.a, non_blocking=True)
                uploaded = torch.cuda.Event()
                uploaded.record(up)
            compute.wait_event(uploaded)
            with torch.cuda.stream(compute):
                merge_lora_batch([(twin, bd, ad, op.strength, op.rounding_seed, op.offset_base)
                                  for op, twin, (bd, ad) in zip(block, slot.twins, slot.factors)],
                                 workspace=workspace)
                merged = torch.cuda.Event()
                merged.record(compute)
            down.wait_event(merged)
            with torch.cuda.stream(down):
                for op, twin in zip(block, slot.twins):
                    for name, dst in storages(op.target):
                        dst.copy_(getattr(twin, name), non_blocking=True)
                done = torch.cuda.Event()
                done.record(down)
            freed[k] = done
    finally:
        compute.wait_stream(down)  # the caller's stream follows every issued download


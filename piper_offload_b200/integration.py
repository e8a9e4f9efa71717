"""The B200 merge bound into an imported Piper Offload 0.2.5 package.

``install(po)`` is the drop-in at run time: the reference's adapters,
registry, ``LoRATransform`` and ``merge_lora()`` stay as they are, and

* every tensor adapter module that imported a raw-buffer Triton launcher at
  load time gets the matching launcher of :mod:`piper_offload_b200.kernels`
  (same arguments, return values and ``ValueError`` behaviour) in its place:
  ``float8_adapter.py:51-60``, ``int8_adapter.py:47-53``,
  ``nvfp4_adapter.py:47-54``, ``mx_adapter.py:47-52``,
  ``static_float8_adapter.py:40-47``, ``bnb8bit_adapter.py:59-66``,
  ``quanto_adapter.py:65-76`` and ``bnb4bit_adapter.py:65-72``; the adapters'
  layout gates, which test those names for ``None``, then route to the B200
  kernels;
* a GGUF adapter that adds the merge capability the reference's GgufAdapter
  lacks (GGUF weights are routed-only there, ``lora.py:752-753``) is
  registered with ``register_adapter`` (``tensor_adapter_registry.py:59``),
  which checks it before the built-in adapters.

The returned callable undoes both. The reference package is the caller's: it
is passed in (or imported as ``piper_offload``), never imported by the rest of
this package.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Any

import torch

from . import kernels as K

# adapter module -> (attribute, replacement) pairs
_BINDINGS = {
    "float8_adapter": (("_triton_merge_float8_lora", K.merge_float8_lora), ("_TRITON_MAX_GROUP_SIZE", K.MAX_GROUP_SIZE)),
    "int8_adapter": (("_triton_merge_int8_lora", K.merge_int8_lora),),
    "nvfp4_adapter": (("_triton_merge_nvfp4_lora", K.merge_nvfp4_lora),),
    "mx_adapter": (("_triton_merge_mx_lora_", K.merge_mx_lora_),),
    "static_float8_adapter": (("_triton_merge_static_float8_lora", K.merge_static_float8_lora),),
    "bnb8bit_adapter": (("_triton_merge_bnb8_lora", K.merge_bnb8_lora),),
    "quanto_adapter": (("_triton_merge_quanto_qint8_lora", K.merge_quanto_qint8_lora),
                       ("_triton_merge_quanto_qfloat8_lora", K.merge_quanto_qfloat8_lora)),
    "bnb4bit_adapter": (("_triton_merge_bnb4_lora", K.merge_bnb4_lora),),
}


def gguf_merge_adapter(po: Any) -> type:
    """The reference's GgufAdapter with the LoRA merge capability added: the
    raw Q8_0 / Q4_0 blocks are merged in place by ``piper_merge_gguf``."""
    gguf_adapter = __import__(f"{po.__name__}.gguf_adapter", fromlist=["GgufAdapter"])
    base = gguf_adapter.GgufAdapter

    class B200GgufAdapter(base):  # type: ignore[misc, valid-type]
        @staticmethod
        def logical_shape(t: torch.Tensor) -> tuple[int, ...]:
            raw = t.as_subclass(torch.Tensor)
            return (raw.shape[0], K.gguf_logical_cols(raw.shape[1], int(t.quant_type)))

        @staticmethod
        def validate_lora_merge(t: torch.Tensor, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                                rounding_seed: int | None = None) -> None:
            K.validate_gguf_merge(t.as_subclass(torch.Tensor), int(t.quant_type), b, a)

        @staticmethod
        def merge_lora_(t: torch.Tensor, b: torch.Tensor, a: torch.Tensor, strength: float, *,
                        rounding_seed: int | None = None) -> None:
            K.merge_gguf_lora_(t.as_subclass(torch.Tensor), int(t.quant_type), b, a, strength,
                               rounding_seed=rounding_seed)

    B200GgufAdapter.__name__ = "B200GgufAdapter"
    B200GgufAdapter.__qualname__ = "B200GgufAdapter"
    return B200GgufAdapter


def install(po: Any = None) -> Callable[[], None]:
    """Bind the B200 launchers into ``po`` (default: ``import piper_offload``)
    and register the GGUF merge adapter; returns the undo callable."""
    if po is None:
        import piper_offload as po  # noqa: PLC0415 - the caller's reference install
    saved: list[tuple[Any, str, Any]] = []
    for mod_name, pairs in _BINDINGS.items():
        mod = __import__(f"{po.__name__}.{mod_name}", fromlist=["_"])
        for attr, value in pairs:
            if hasattr(mod, attr):
                saved.append((mod, attr, getattr(mod, attr)))
                setattr(mod, attr, value)
    registry = __import__(f"{po.__name__}.tensor_adapter_registry", fromlist=["register_adapter"])
    unregister = registry.register_adapter(gguf_merge_adapter(po))

    def undo() -> None:
        unregister()
        for mod, attr, value in reversed(saved):
            setattr(mod, attr, value)

    return undo

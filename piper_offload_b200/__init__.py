"""B200-native fused quantized LoRA merge (drop-in for Piper Offload's merge path)."""

from .seeding import derive_seed  # noqa: F401

__all__ = ["derive_seed"]

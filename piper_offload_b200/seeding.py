"""Stable seed derivation, identical to ``piper_offload.seeding.derive_seed``.

Restates ``src/piper_offload/seeding.py:10-36``: BLAKE2s with an 8-byte digest
over ``b"piper-offload-seed-v1\\0"`` followed by each part, strings as
``b"s" + len(u64 LE) + utf-8`` and integers as ``b"i" + u64 LE``; the digest is
read as a little-endian unsigned 64-bit integer. The format is a published
contract (seeds must agree across implementations), so the encoding is kept
byte for byte.
"""

from __future__ import annotations

from hashlib import blake2s

__all__ = ["derive_seed"]

_UINT64_LIMIT = 1 << 64
_DOMAIN = b"piper-offload-seed-v1\0"


def derive_seed(*parts: str | int) -> int:
    """Return a stable unsigned 64-bit seed derived from typed identity parts."""
    h = blake2s(digest_size=8)
    h.update(_DOMAIN)
    for part in parts:
        if isinstance(part, str):
            data = part.encode("utf-8")
            h.update(b"s" + len(data).to_bytes(8, "little") + data)
        elif isinstance(part, int) and not isinstance(part, bool):
            if not 0 <= part < _UINT64_LIMIT:
                raise ValueError("derive_seed() integer parts must be unsigned 64-bit values")
            h.update(b"i" + part.to_bytes(8, "little"))
        else:
            raise TypeError("derive_seed() parts must be strings or unsigned 64-bit integers")
    return int.from_bytes(h.digest(), "little")

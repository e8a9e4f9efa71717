"""Counter-based uniform stream of the reference (TEST INFRASTRUCTURE ONLY).

Restates ``_random(seed, offsets) = tl.rand(seed, offsets.to(tl.uint64))``
(reference ``src/piper_offload/_triton_stochastic_quantization.py:18-21``),
i.e. Triton's open-source Philox4x32-10 (``triton/language/random.py:13-156``
in triton 3.6.0):

* key ``(k0, k1) = (seed & 0xffffffff, seed >> 32)`` of the uint64 seed
  (``_seed_argument`` at ``_triton_stochastic_quantization.py:11-15`` only
  reinterprets the bits as int64 for the launch);
* counter ``(off & 0xffffffff, off >> 32, 0, 0)`` of the logical element
  offset;
* ten rounds of ``c0' = hi(B*c2) ^ c1 ^ k0``, ``c2' = hi(A*c0) ^ c3 ^ k1``,
  ``c1' = lo(B*c2)``, ``c3' = lo(A*c0)`` with A=0xD2511F53, B=0xCD9E8D57 and
  key increments 0x9E3779B9 / 0xBB67AE85;
* output word c0 bit-cast to int32, folded with ``x < 0 ? -x - 1 : x`` and
  multiplied in fp32 by the fp32 constant 4.6566127342e-10.
"""

from __future__ import annotations

import numpy as np

_MASK = np.uint64(0xFFFFFFFF)
ROUND_A = np.uint64(0xD2511F53)
ROUND_B = np.uint64(0xCD9E8D57)
KEY_A = 0x9E3779B9
KEY_B = 0xBB67AE85
UNIFORM_SCALE = np.float32(4.6566127342e-10)


def philox_c0(seed: int, offsets: np.ndarray, rounds: int = 10) -> np.ndarray:
    """First Philox4x32 output word (uint32) for each 64-bit offset."""
    seed &= (1 << 64) - 1
    off = np.asarray(offsets, dtype=np.uint64)
    c0 = off & _MASK
    c1 = off >> np.uint64(32)
    c2 = np.zeros_like(c0)
    c3 = np.zeros_like(c0)
    k0 = seed & 0xFFFFFFFF
    k1 = seed >> 32
    for _ in range(rounds):
        p0 = ROUND_A * c0  # < 2**64, exact in uint64
        p1 = ROUND_B * c2
        n0 = (p1 >> np.uint64(32)) ^ c1 ^ np.uint64(k0)
        n2 = (p0 >> np.uint64(32)) ^ c3 ^ np.uint64(k1)
        c1 = p1 & _MASK
        c3 = p0 & _MASK
        c0, c2 = n0, n2
        k0 = (k0 + KEY_A) & 0xFFFFFFFF
        k1 = (k1 + KEY_B) & 0xFFFFFFFF
    return c0.astype(np.uint32)


def philox_uniform(seed: int, offsets: np.ndarray) -> np.ndarray:
    """``tl.rand(seed, offsets)`` as fp32 in [0, 1)."""
    x = philox_c0(seed, offsets).view(np.int32).astype(np.int64)
    x = np.where(x < 0, -x - 1, x)
    return (x.astype(np.float32) * UNIFORM_SCALE).astype(np.float32)

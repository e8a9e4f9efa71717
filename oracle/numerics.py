"""Bit-exact scalar numerics used by the oracle (TEST INFRASTRUCTURE ONLY).

Every helper works element-wise on numpy arrays and reproduces the rounding
of the GPU instruction that the reference Triton kernels lower to:

* ``x.to(tl.bfloat16)`` / ``x.to(tl.float16)``: round-to-nearest-even casts.
* ``x.to(tl.float8e4nv)`` and stores into ``float8_e4m3fn`` / ``float8_e5m2``
  pointers: round-to-nearest-even with saturation to the largest finite value
  (``cvt.rn.satfinite``); NaN stays NaN.
* ``tl.minimum`` / ``tl.maximum``: IEEE minNum/maxNum (a NaN operand yields
  the other operand).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
U32 = np.uint32


def f32(x: np.ndarray | float) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def bits_f32(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)


def from_bits_f32(b: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(b, dtype=np.uint32).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit pattern (uint16), round to nearest even, NaN kept quiet."""
    b = bits_f32(x).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    rounded = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    quiet = (b >> 16) | 0x40
    return np.where(nan, quiet, rounded).astype(np.uint16)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return from_bits_f32(np.asarray(h, dtype=np.uint32) << 16)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 value (returned as fp32)."""
    return bf16_to_f32(bf16_bits(x))


def f16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest fp16 value (returned as fp32)."""
    with np.errstate(over="ignore"):
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to_compute(x: np.ndarray, compute: str) -> np.ndarray:
    """``value.to(compute_dtype).to(float32)`` for compute in {bf16, f16, f32}."""
    if compute == "bf16":
        return bf16_round(x)
    if compute == "f16":
        return f16_round(x)
    return np.asarray(x, dtype=np.float32)


def maxnum(a, b) -> np.ndarray:
    return np.fmax(np.asarray(a, dtype=np.float32), np.asarray(b, dtype=np.float32))


def minnum(a, b) -> np.ndarray:
    return np.fmin(np.asarray(a, dtype=np.float32), np.asarray(b, dtype=np.float32))


def clamp(x, lo, hi) -> np.ndarray:
    """``tl.minimum(tl.maximum(x, lo), hi)``."""
    return minnum(maxnum(x, np.float32(lo)), np.float32(hi))


# ---------------------------------------------------------------------------
# 8-bit floating point formats (OCP FP8 E4M3FN / E5M2)
# ---------------------------------------------------------------------------


def _fp8_table(exp_bits: int, man_bits: int, bias: int) -> np.ndarray:
    """Values of all 256 codes (NaN/inf where the format defines them)."""
    codes = np.arange(256, dtype=np.int64)
    sign = np.where(codes & 0x80, -1.0, 1.0)
    exp = (codes >> man_bits) & ((1 << exp_bits) - 1)
    man = codes & ((1 << man_bits) - 1)
    sub = exp == 0
    val = np.where(
        sub,
        man * 2.0 ** (1 - bias - man_bits),
        (1.0 + man / (1 << man_bits)) * np.exp2(exp.astype(np.float64) - bias),
    )
    return (sign * val).astype(np.float64)


_E4M3 = _fp8_table(4, 3, 7)
_E4M3[0x7F] = np.nan
_E4M3[0xFF] = np.nan
_E5M2 = _fp8_table(5, 2, 15)
for _c in range(0x7C, 0x80):
    _E5M2[_c] = np.inf if _c == 0x7C else np.nan
    _E5M2[_c | 0x80] = -np.inf if _c == 0x7C else np.nan

E4M3_MAX = 448.0
E5M2_MAX = 57344.0
_E4M3_POS = _E4M3[:0x7F].copy()  # codes 0x00..0x7E, ascending
_E5M2_POS = _E5M2[:0x7C].copy()  # codes 0x00..0x7B, ascending


def decode_e4m3(code: np.ndarray) -> np.ndarray:
    return _E4M3[np.asarray(code, dtype=np.uint8)].astype(np.float32)


def decode_e5m2(code: np.ndarray) -> np.ndarray:
    return _E5M2[np.asarray(code, dtype=np.uint8)].astype(np.float32)


def _encode_fp8(x: np.ndarray, table: np.ndarray, max_code: int) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    mag = np.abs(x).astype(np.float64)
    sign = (bits_f32(x) >> 24).astype(np.uint8) & np.uint8(0x80)
    finite = np.isfinite(mag)
    m = np.where(finite, mag, 0.0)
    hi = np.searchsorted(table, m, side="left")  # first code with value >= m
    hi = np.minimum(hi, max_code)
    lo = np.maximum(hi - 1, 0)
    vhi = table[hi]
    vlo = table[lo]
    exact = vhi == m
    dlo = m - vlo
    dhi = vhi - m
    pick_hi = (dhi < dlo) | ((dhi == dlo) & ((hi & 1) == 0))
    code = np.where(exact, hi, np.where(pick_hi, hi, lo))
    # satfinite: anything at or beyond the largest finite value saturates.
    code = np.where(m >= table[max_code], max_code, code).astype(np.uint8)
    code = np.where(np.isinf(mag), np.uint8(max_code), code)
    out = code | sign
    nan_code = np.uint8(0x7F)
    return np.where(np.isnan(x), nan_code | sign, out).astype(np.uint8)


def encode_e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 -> E4M3FN code, RTNE, saturating (``cvt.rn.satfinite.e4m3x2.f32``)."""
    return _encode_fp8(x, _E4M3_POS, 0x7E)


def encode_e5m2(x: np.ndarray) -> np.ndarray:
    """fp32 -> E5M2 code, RTNE, saturating (``cvt.rn.satfinite.e5m2x2.f32``)."""
    return _encode_fp8(x, _E5M2_POS, 0x7B)


def fp8_codec(e4m3: bool):
    return (encode_e4m3, decode_e4m3, E4M3_MAX) if e4m3 else (encode_e5m2, decode_e5m2, E5M2_MAX)


# ---------------------------------------------------------------------------
# E2M1 (FP4) helpers: reference _triton_mx_lora.py:40-94 and
# _triton_nvfp4_lora.py:24-85 / _triton_stochastic_quantization.py:82-106.
# ---------------------------------------------------------------------------

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def e2m1_value(code: np.ndarray) -> np.ndarray:
    """Magnitude of the low three bits (``_e2m1_value``)."""
    return E2M1_VALUES[np.asarray(code, dtype=np.int64) & 7]


def decode_e2m1(code: np.ndarray) -> np.ndarray:
    """Signed value of a 4-bit code (``_decode_fp4``, ``_triton_nvfp4_lora.py:24-52``,
    ``_triton_mx_lora.py:40-64``).

    The sign is applied as ``-magnitude``, which Triton lowers to ``0.0 - x``
    (``triton/language/semantic.py`` ``minus``), so code 8 decodes to +0.0.
    """
    code = np.asarray(code, dtype=np.int64)
    mag = E2M1_VALUES[code & 7]
    return np.where((code & 8) != 0, np.float32(0.0) - mag, mag).astype(np.float32)


def encode_e2m1(x: np.ndarray) -> np.ndarray:
    """RTNE threshold ladder of ``_encode_fp4``; sign from the fp32 sign bit."""
    x = np.asarray(x, dtype=np.float32)
    m = np.abs(x)
    code = np.where(
        m <= 0.25, 0,
        np.where(m < 0.75, 1,
        np.where(m <= 1.25, 2,
        np.where(m < 1.75, 3,
        np.where(m <= 2.5, 4,
        np.where(m < 3.5, 5,
        np.where(m <= 5.0, 6, 7)))))))
    sign = np.where((bits_f32(x) >> 31) != 0, 8, 0)
    return (code | sign).astype(np.int64)


# ---------------------------------------------------------------------------
# E8M0 (MX shared exponent): reference _triton_mx_lora.py:30-37.
# ---------------------------------------------------------------------------


def decode_e8m0(code: np.ndarray) -> np.ndarray:
    code = np.asarray(code, dtype=np.uint32)
    bits = np.where(code == 0, np.uint32(1 << 22), code << 23)
    val = from_bits_f32(bits.astype(np.uint32))
    return np.where(code != 255, val, np.float32(np.nan)).astype(np.float32)


def rint_half_even(x: np.ndarray) -> np.ndarray:
    """``libdevice.llrint``: round half to even to an integer (as int64)."""
    return np.rint(np.asarray(x, dtype=np.float32)).astype(np.int64)


def ieee_div(a, b) -> np.ndarray:
    """fp32 IEEE quotient (correctly rounded)."""
    with np.errstate(divide="ignore", invalid="ignore", over="ignore", under="ignore"):
        return (np.asarray(a, dtype=np.float32) / np.asarray(b, dtype=np.float32)).astype(np.float32)


# The reference's ``x / CONST`` (constexpr or literal divisor, e.g. ``/ 2688.0``,
# ``/ FP8_LIMIT``, ``/ MAX_POS``): on sm_100 with triton 3.6 it evaluates as
# ``x * fp32(1 / CONST)`` (measured on a B200: identical to that product for all
# of 1M random x with CONST = 2688, 6, 448 and 127.5, and to IEEE division for
# only 26-78 % of them). The Triton CPU interpreter that recorded the golden
# fixtures divides in IEEE fp32 instead, so those fixtures are checked with
# ``set_constant_division("ieee")``.
_constant_division = "reciprocal"


def set_constant_division(mode: str) -> None:
    """``"reciprocal"`` (the GPU's evaluation, default) or ``"ieee"`` (the interpreter's)."""
    global _constant_division
    if mode not in ("reciprocal", "ieee"):
        raise ValueError(mode)
    _constant_division = mode


def constant_division() -> str:
    return _constant_division


# The reference's fp32-compute ``base = values * scale; merged = base + acc * strength``
# is compiled for the GPU with floating-point contraction, which fuses the first
# product into the add (``"gpu"``, default). The Triton CPU interpreter that
# recorded the golden fixtures evaluates each operation on its own with one
# rounding each (``"separate"``), so those fixtures are checked in that mode.
_fp32_contraction = "gpu"


def set_fp32_contraction(mode: str) -> None:
    """``"gpu"`` (the compiled kernels) or ``"separate"`` (the interpreter)."""
    global _fp32_contraction
    if mode not in ("gpu", "separate"):
        raise ValueError(mode)
    _fp32_contraction = mode


def fp32_contraction() -> str:
    return _fp32_contraction


def fdiv(a, b) -> np.ndarray:
    """fp32 quotient of the reference's ``x / CONST`` (see ``set_constant_division``)."""
    if _constant_division == "ieee":
        return ieee_div(a, b)
    rcp = np.float32(1.0) / np.asarray(b, dtype=np.float32)
    with np.errstate(over="ignore", invalid="ignore", under="ignore"):
        return (np.asarray(a, dtype=np.float32) * rcp).astype(np.float32)


# The reference's ``tensor / tensor`` quotients are Triton's default fp32
# division, which on sm_100 is the approximate ``div.full.f32`` (measured: it
# differs from IEEE in up to ~30% of random operand pairs, by <= 2 ulp). The
# oracle cannot restate that instruction; by default it uses IEEE division
# (a documented tie class), and GPU parity tests may install a device hook
# that evaluates exactly those quotients with Triton's own ``/``.
_tensor_division = None


def set_tensor_division(fn) -> None:
    """Install ``fn(a, b) -> fp32 quotient`` for tensor/tensor divisions (None = IEEE)."""
    global _tensor_division
    _tensor_division = fn


def fdiv_t(a, b) -> np.ndarray:
    """fp32 quotient of a ``tensor / tensor`` division in the reference kernels."""
    if _tensor_division is None:
        return ieee_div(a, b)
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    shape = np.broadcast_shapes(a.shape, b.shape)
    out = _tensor_division(np.broadcast_to(a, shape).reshape(-1), np.broadcast_to(b, shape).reshape(-1))
    return np.asarray(out, dtype=np.float32).reshape(shape)


def fma_f32_exact(a, b, c) -> np.ndarray:
    """Single-rounding ``a * b + c`` in fp32, exact in every case (``fma.rn.f32``).

    The product of two fp32 values is exact in fp64. Their fp64 sum ``s``
    with the TwoSum error ``e`` (Knuth) is the exact result ``s + e``. fp32
    rounding points are fp64 values, so rounding ``s`` to fp32 gives the
    fused result unless ``s`` lies exactly on an fp32 midpoint with ``e``
    nonzero; then the exact result lies on the side of ``e``.
    """
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    c = np.asarray(c, dtype=np.float64)
    with np.errstate(over="ignore", invalid="ignore"):
        p = a * b
        s = p + c
        bb = s - p
        e = (p - (s - bb)) + (c - bb)
        r = s.astype(np.float32)
        r64 = r.astype(np.float64)
        d = s - r64
        toward = np.where(d > 0, np.float32(np.inf), np.float32(-np.inf)).astype(np.float32)
        other = np.nextafter(r, toward).astype(np.float32)
        mid = (d != 0) & np.isfinite(s) & (np.abs(other.astype(np.float64) - r64) == 2.0 * np.abs(d))
        # On a midpoint the exact value lies past it (toward `other`) when e has d's sign.
        past = mid & (e != 0) & (np.sign(e) == np.sign(d))
        return np.where(past, other, r).astype(np.float32)


def fma_f32(a, b, c) -> np.ndarray:
    """Single-rounding ``a * b + c`` in fp32 (Triton contracts mul+add into FMA).

    The exact product of two fp32 values fits in fp64; adding ``c`` in fp64
    and rounding once to fp32 equals the fused result except when the fp64
    sum is itself inexact and lands on an fp32 midpoint, which needs operands
    more than 29 binades apart and cannot change the bf16 value downstream.
    """
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    c = np.asarray(c, dtype=np.float64)
    with np.errstate(over="ignore", invalid="ignore"):
        return (a * b + c).astype(np.float32)

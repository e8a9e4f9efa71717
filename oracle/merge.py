"""numpy restatement of the reference LoRA-merge kernels (TEST INFRASTRUCTURE ONLY).

Arrays in, arrays out. Factors ``b`` (M x r) and ``a`` (r x N) are fp32 numpy
arrays holding the exact compute-dtype values (bf16 / fp16 values upcast).
``compute`` is the LoRA factor dtype: ``"bf16"``, ``"f16"`` or ``"f32"``.
``seed`` is ``None`` for round-to-nearest, else the uint64 rounding seed.

Every function cites the reference lines whose arithmetic it restates.
"""

from __future__ import annotations

import numpy as np

from .numerics import (
    bf16_round,
    bits_f32,
    clamp,
    decode_e2m1,
    decode_e8m0,
    e2m1_value,
    encode_e2m1,
    f16_round,
    fdiv,
    fdiv_t,
    fma_f32,
    fma_f32_exact,
    fp32_contraction,
    fp8_codec,
    from_bits_f32,
    maxnum,
    minnum,
    rint_half_even,
    round_to_compute,
)
from .philox import philox_uniform

EPS_2_23 = np.float32(1.1920928955078125e-07)
FLT_MIN = np.float32(1.1754943508222875e-38)


# ---------------------------------------------------------------------------
# The rank-r update.
# ---------------------------------------------------------------------------


def lora_delta(b: np.ndarray, a: np.ndarray, compute: str = "bf16") -> np.ndarray:
    """fp32 ``B @ A`` as the reference's ``tl.dot`` forms it.

    bf16 / fp16 factors (tensor-core dot): correctly rounded (tie class: GPU
    summation order). The reference accumulates into ``tl.zeros``
    (``accumulator += tl.dot(b, a)``), so an all-zero sum is +0.0 whatever the
    signs of its products.

    fp32 factors (``input_precision="ieee"``, e.g. ``_triton_float8_lora.py:53-66``):
    one fused multiply-add per rank step in rank order from +0, across the rank
    blocks (16 for rank <= 16, else 32); the zero-padded steps of the last
    block add +0, which turns a -0 sum into +0.
    """
    if compute == "f32":
        b = np.asarray(b, np.float32)
        a = np.asarray(a, np.float32)
        rank = b.shape[1]
        acc = np.zeros((b.shape[0], a.shape[1]), np.float32)
        for k in range(rank):
            acc = fma_f32_exact(b[:, k:k + 1], a[k:k + 1, :], acc)
        block = 16 if rank <= 16 else 32
        if rank % block:
            acc = (acc + np.float32(0.0)).astype(np.float32)
        return acc
    acc = (np.asarray(b, np.float64) @ np.asarray(a, np.float64)).astype(np.float32)
    return (np.float32(0.0) + acc).astype(np.float32)


def merged_values(base: np.ndarray, acc: np.ndarray, strength: float, compute: str) -> np.ndarray:
    """``(base.to(f32) + acc * strength).to(compute)``; Triton contracts it to an FMA."""
    return round_to_compute(fma_f32(acc, np.float32(strength), base), compute)


def merged_values_f32_product(values: np.ndarray, scale: np.ndarray, acc: np.ndarray, strength: float) -> np.ndarray:
    """fp32 compute of ``base = values * scale; merged = base + acc * strength``.

    With no cast between them (``COMPUTE_DTYPE == 2``, e.g. ``_triton_float8_lora.py:80-92``,
    ``_triton_int8_lora.py:78-94``), the sum of two products is contracted on the
    first one (LLVM's ``(fadd (fmul x, y), z) -> (fma x, y, z)``): the update is
    rounded on its own and the element product enters the fused add exactly.
    """
    update = (np.asarray(acc, np.float32) * np.float32(strength)).astype(np.float32)
    if fp32_contraction() == "separate":
        prod = (np.asarray(values, np.float32) * np.asarray(scale, np.float32)).astype(np.float32)
        return (prod + update).astype(np.float32)
    return fma_f32_exact(np.asarray(values, np.float32), np.asarray(scale, np.float32), update)


def nanmax_reduce(x: np.ndarray, axis: int) -> np.ndarray:
    """``tl.max`` reduction: maxNum combine, NaN only if every element is NaN."""
    return np.fmax.reduce(np.asarray(x, np.float32), axis=axis)


def nanmin_reduce(x: np.ndarray, axis: int) -> np.ndarray:
    return np.fmin.reduce(np.asarray(x, np.float32), axis=axis)


# ---------------------------------------------------------------------------
# Stochastic rounding helpers: _triton_stochastic_quantization.py:24-175.
# ---------------------------------------------------------------------------


def sr_round_to_int(values, deterministic, seed, offsets, qmin, qmax):
    """``_stochastic_round_to_int`` (``_triton_stochastic_quantization.py:24-39``)."""
    values = np.asarray(values, np.float32)
    interior = (values > qmin) & (values < qmax)
    safe = np.where(interior, values, np.float32(0.0)).astype(np.float32)
    lower = np.floor(safe).astype(np.float32)
    prob = (safe - lower).astype(np.float32)
    u = philox_uniform(seed, offsets)
    rounded = lower + (u < prob).astype(np.float32)
    return np.where(interior & (prob > 0), rounded, np.asarray(deterministic, np.float32)).astype(np.float32)


def sr_float8(values, seed, offsets, e4m3: bool, limit: float) -> np.ndarray:
    """``_stochastic_float8`` (``_triton_stochastic_quantization.py:132-175``); returns codes."""
    encode, decode, _ = fp8_codec(e4m3)
    v = np.asarray(values, np.float32)
    mag = np.abs(v)
    det_bits = encode(mag).astype(np.int64)
    det_val = decode(det_bits)
    rounded_down = det_val > mag
    lower_bits = np.where(rounded_down, det_bits - 1, det_bits) & 0xFF
    upper_bits = np.where(rounded_down, det_bits, det_bits + 1) & 0xFF
    lower = decode(lower_bits)
    upper = decode(upper_bits)
    with np.errstate(invalid="ignore"):
        ok = upper > lower
    prob = np.where(ok, fdiv_t(mag - lower, upper - lower), np.float32(0.0))
    u = philox_uniform(seed, offsets)
    mag_bits = np.where(u < prob, upper_bits, lower_bits)
    sign = (bits_f32(v) >> 24).astype(np.int64) & 0x80
    chosen = mag_bits | sign
    det_signed = det_bits | sign
    interior = (mag < limit) & (prob > 0)
    return np.where(interior, chosen, det_signed).astype(np.uint8)


def sr_e2m1(values, deterministic, seed, offsets) -> np.ndarray:
    """``_stochastic_e2m1_code`` (``_triton_stochastic_quantization.py:109-129``)."""
    v = np.asarray(values, np.float32)
    mag = np.abs(v)
    det = np.asarray(deterministic, np.int64)
    nearest_code = det & 7
    nearest = e2m1_value(nearest_code)
    rounded_down = nearest > mag
    lower_code = np.where(rounded_down, nearest_code - 1, nearest_code)
    upper_code = np.where(rounded_down, nearest_code, nearest_code + 1)
    lower = e2m1_value(lower_code)
    upper = e2m1_value(upper_code)
    prob = np.where(upper > lower, fdiv_t(mag - lower, upper - lower), np.float32(0.0))
    u = philox_uniform(seed, offsets)
    mag_code = np.where(u < prob, upper_code, lower_code)
    sign = (bits_f32(v) >> 28).astype(np.int64) & 8
    chosen = mag_code | sign
    interior = (mag > 0) & (mag < 6.0) & (prob > 0)
    return np.where(interior, chosen, det).astype(np.int64)


def logical_offsets(rows: int, cols: int, base: int = 0) -> np.ndarray:
    r = np.arange(rows, dtype=np.uint64)[:, None]
    c = np.arange(cols, dtype=np.uint64)[None, :]
    return (np.uint64(base) + r * np.uint64(cols) + c).astype(np.uint64)


# ---------------------------------------------------------------------------
# Swizzled (blocked 128x4) scale layout shared by MX and NVFP4:
# _triton_mx_lora.py:97-112, _triton_nvfp4_lora.py:88-104.
# ---------------------------------------------------------------------------


def scale_index(rows: int, scale_cols: int, swizzled: bool) -> np.ndarray:
    r = np.arange(rows, dtype=np.int64)[:, None]
    c = np.arange(scale_cols, dtype=np.int64)[None, :]
    if not swizzled:
        return r * scale_cols + c
    col_blocks = (scale_cols + 3) // 4
    tile = ((r // 128) * col_blocks + c // 4) * 512
    rin = r % 128
    return tile + (rin % 32) * 16 + (rin // 32) * 4 + (c % 4)


def unpack_fp4(packed: np.ndarray) -> np.ndarray:
    """Byte j holds element 2j in its low nibble and 2j+1 in its high nibble."""
    p = np.asarray(packed, np.uint8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.int64)
    out[..., 0::2] = p & 0xF
    out[..., 1::2] = p >> 4
    return out


def pack_fp4(codes: np.ndarray) -> np.ndarray:
    c = np.asarray(codes, np.int64) & 0xF
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


# ---------------------------------------------------------------------------
# MX: _triton_mx_lora.py:115-295.
# ---------------------------------------------------------------------------

MX_FORMATS = {
    # elem: (target_max_pow2, max_pos, mbits)  -- _triton_mx_lora.py:298-308
    "e4m3": (8, 448.0, 3),
    "e5m2": (15, 57344.0, 2),
    "e2m1": (2, 6.0, 1),
}
MX_SCALE_MODES = {"floor": 0, "rceil": 1, "ceil": 2, "even": 3}


def exact_ceil_log2(x: np.ndarray) -> np.ndarray:
    """``ceil(log2(x))`` for positive finite fp32 x, computed exactly."""
    x = np.asarray(x, np.float32)
    mant, exp = np.frexp(x.astype(np.float64))  # x = mant * 2**exp, mant in [0.5, 1)
    return np.where(mant == 0.5, exp - 1, exp).astype(np.float64)


def mx_calculate_scale(max_abs, target_pow2, max_pos, mbits, mode):
    """``_calculate_scale`` (``_triton_mx_lora.py:115-159``) -> (E8M0 code, inverse scale)."""
    max_abs = np.asarray(max_abs, np.float32)
    if mode == 1:  # RCEIL
        descale = fdiv(max_abs, np.float32(max_pos))
        with np.errstate(divide="ignore", invalid="ignore"):
            pos = np.isfinite(descale) & (descale > 0)
            lg = np.where(pos, exact_ceil_log2(np.where(pos, descale, 1.0)),
                          np.where(descale == 0, -np.inf, np.where(np.isnan(descale), np.nan, np.inf)))
        unbiased = np.fmin(np.fmax(lg, -127.0), 127.0)
        encoded = (unbiased + 127.0).astype(np.int64)
        encoded = np.where(np.isnan(descale), 255, encoded)
        inv = np.where(encoded == 0, np.float32(1.0), np.exp2(-unbiased).astype(np.float32))
        return encoded.astype(np.uint8), inv.astype(np.float32)
    bits = bits_f32(max_abs).astype(np.int64)
    if mode == 3:  # EVEN
        bias = {3: 524288, 2: 1048576}.get(mbits, 2097152)
        bits = ((bits + bias) & 0xFFFFFFFF) & (-8388608 & 0xFFFFFFFF)
    extracted = ((bits >> 23) & 255) - 127
    if mode == 2:  # CEIL
        extracted = extracted + ((bits & 8388607) > 0).astype(np.int64)
    unbiased = np.clip(extracted - target_pow2, -127, 128)
    encoded = (unbiased + 127).astype(np.int64) & 0xFF
    encoded = np.where(np.isnan(max_abs), 255, encoded)
    scale = from_bits_f32((encoded.astype(np.uint32) << 23).astype(np.uint32))
    scale = maxnum(scale, FLT_MIN)
    return encoded.astype(np.uint8), fdiv_t(np.float32(1.0), scale)


def merge_mx(qdata, scale, elem, b, a, strength, *, scaling_mode=0, swizzled=False, seed=None,
             compute="bf16", offset_base=0):
    """In-place MX merge (``_merge_mx_kernel``, ``_triton_mx_lora.py:162-295``).

    ``qdata``: uint8 codes (M x N for e4m3/e5m2, M x N/2 packed for e2m1).
    ``scale``: uint8 E8M0 codes in plain (M x N/32) or swizzled layout.
    Returns new ``(qdata, scale)`` arrays.
    """
    target, max_pos, mbits = MX_FORMATS[elem]
    M = b.shape[0]
    N = a.shape[1]
    nb = N // 32
    acc = lora_delta(b, a, compute)
    if elem == "e2m1":
        codes = unpack_fp4(qdata)
        base_lp = decode_e2m1(codes)
    else:
        _, decode, _ = fp8_codec(elem == "e4m3")
        base_lp = decode(qdata)
    sidx = scale_index(M, nb, swizzled)
    flat_scale = np.asarray(scale, np.uint8).reshape(-1).copy()
    enc_in = flat_scale[sidx]
    bscale = np.repeat(decode_e8m0(enc_in), 32, axis=1)
    if compute == "bf16":
        base = bf16_round(bf16_round(base_lp) * bf16_round(bscale))
    else:
        base = (base_lp * bscale).astype(np.float32)
    merged = merged_values(base, acc, strength, compute)
    max_abs = nanmax_reduce(np.abs(merged).reshape(M, nb, 32), axis=2)
    enc_out, inv = mx_calculate_scale(max_abs, target, max_pos, mbits, scaling_mode)
    normalized = (merged * np.repeat(inv, 32, axis=1)).astype(np.float32)
    normalized = clamp(normalized, -max_pos, max_pos)
    flat_scale[sidx] = enc_out
    offs = logical_offsets(M, N, offset_base)
    if elem == "e2m1":
        out = encode_e2m1(normalized)
        if seed is not None:
            out = sr_e2m1(normalized, out, seed, offs)
        new_q = pack_fp4(out)
    else:
        encode, _, _ = fp8_codec(elem == "e4m3")
        if seed is not None:
            new_q = sr_float8(normalized, seed, offs, elem == "e4m3", max_pos)
        else:
            new_q = encode(normalized)
    return new_q.astype(np.uint8), flat_scale.reshape(np.shape(scale))


# ---------------------------------------------------------------------------
# NVFP4: _triton_nvfp4_lora.py:107-367 and the global-scale pass 190-266.
# ---------------------------------------------------------------------------


def _nvfp4_merged(qdata, scale, global_scale, swizzled, b, a, strength, compute):
    """``_merged_tile`` over the whole tensor (``_triton_nvfp4_lora.py:107-187``)."""
    from .numerics import decode_e4m3

    M = b.shape[0]
    N = a.shape[1]
    sc = N // 16
    codes = unpack_fp4(qdata)
    base = decode_e2m1(codes)
    sidx = scale_index(M, sc, swizzled)
    flat_scale = np.asarray(scale, np.uint8).reshape(-1)
    bs = decode_e4m3(flat_scale[sidx])
    if compute == "bf16":
        bs = bf16_round(bs)
    if global_scale is not None:
        bs = (bs * np.float32(global_scale)).astype(np.float32)
        if compute == "bf16":
            bs = bf16_round(bs)
    base = (base * np.repeat(bs, 16, axis=1)).astype(np.float32)
    if compute == "bf16":
        base = bf16_round(base)
    acc = lora_delta(b, a, compute)
    update = (acc * np.float32(strength)).astype(np.float32)
    summed = fma_f32(acc, np.float32(strength), base)
    merged = np.where(update == 0.0, base, summed).astype(np.float32)
    if compute == "bf16":
        merged = bf16_round(merged)
    return merged, sidx


def merge_nvfp4(qdata, scale, per_tensor_scale, b, a, strength, *, swizzled=False, seed=None,
                compute="bf16", offset_base=0, global_amax=None):
    """NVFP4 merge (``merge_nvfp4_lora``, ``_triton_nvfp4_lora.py:515-595``).

    ``qdata`` uint8 (M x N/2), ``scale`` uint8 E4M3 codes (plain or swizzled),
    ``per_tensor_scale`` fp32 scalar or None. Returns ``(qdata, scale, global)``;
    the returned scale has zeros in swizzle padding like the reference's
    ``torch.zeros_like`` output buffer. ``global_amax`` (two-level only)
    replaces the maximum |merged| of these rows with the whole tensor's, so a
    row strip of a larger weight is encoded as the whole-tensor merge encodes
    it (``_recompute_global_scale``, ``_triton_nvfp4_lora.py:437-512``).
    """
    from .numerics import encode_e4m3, decode_e4m3

    M = b.shape[0]
    N = a.shape[1]
    sc = N // 16
    g_in = None if per_tensor_scale is None else np.float32(per_tensor_scale)
    merged, sidx = _nvfp4_merged(qdata, scale, g_in, swizzled, b, a, strength, compute)
    g_out = None
    if g_in is not None:
        amax = nanmax_reduce(np.abs(merged).reshape(-1), axis=0) if global_amax is None else np.float32(global_amax)
        g_out = maxnum(fdiv(amax, np.float32(2688.0)), EPS_2_23)
    blocks = merged.reshape(M, sc, 16)
    max_abs = nanmax_reduce(np.abs(blocks), axis=2)
    block_scale = fdiv(max_abs, np.float32(6.0))
    fp8_scale = fdiv_t(block_scale, g_out) if g_out is not None else block_scale
    fp8_scale = clamp(fp8_scale, 0.015625, 448.0)
    fp8_codes = encode_e4m3(fp8_scale)
    fp8_scale = decode_e4m3(fp8_codes)
    new_scale = np.zeros(np.asarray(scale).size, dtype=np.uint8)
    new_scale[sidx] = fp8_codes
    if g_out is not None:
        recip = fdiv_t(fdiv_t(np.float32(1.0), g_out), fp8_scale)
        normalized = (merged * np.repeat(recip, 16, axis=1)).astype(np.float32)
    else:
        normalized = fdiv_t(merged, np.repeat(fp8_scale, 16, axis=1))
    normalized = clamp(normalized, -6.0, 6.0)
    codes = encode_e2m1(normalized)
    if seed is not None:
        codes = sr_e2m1(normalized, codes, seed, logical_offsets(M, N, offset_base))
    new_q = pack_fp4(codes)
    return new_q, new_scale.reshape(np.shape(scale)), g_out


# ---------------------------------------------------------------------------
# Scaled FP8: _triton_float8_lora.py:26-308.
# ---------------------------------------------------------------------------


def merge_float8(qdata, scale, block_size, b, a, strength, *, e4m3=True, seed=None, compute="bf16",
                 offset_base=0):
    """Scaled-FP8 merge (``merge_float8_lora``, ``_triton_float8_lora.py:486-588``).

    ``qdata`` uint8 codes (M x N); ``scale`` fp32 of shape (M,1) per-row,
    (1,1)/() per-tensor or (M, N/g) per-group. Returns ``(qdata, scale)``.
    """
    encode, decode, limit = fp8_codec(e4m3)
    M = b.shape[0]
    N = a.shape[1]
    acc = lora_delta(b, a, compute)
    scale = np.asarray(scale, np.float32)
    per_row = tuple(block_size) == (1, N)
    per_tensor = tuple(block_size) == (M, N)
    lp = decode(qdata)
    if per_row:
        s_in = scale.reshape(M, 1)
    elif per_tensor:
        s_in = scale.reshape(1, 1)
    else:
        g = block_size[1]
        s_in = np.repeat(scale.reshape(M, N // g), g, axis=1)
    if compute == "f32":
        merged = merged_values_f32_product(lp, np.broadcast_to(s_in, lp.shape), acc, strength)
    else:
        base = round_to_compute((lp * s_in).astype(np.float32), compute)
        merged = merged_values(base, acc, strength, compute)
    absv = np.abs(merged)
    if per_row or per_tensor:
        amax = nanmax_reduce(absv, axis=1) if per_row else nanmax_reduce(absv.reshape(-1), axis=0)
        new_scale = round_to_compute(fdiv(amax, np.float32(limit)), compute)
        new_scale = np.where(new_scale == 0.0, EPS_2_23, new_scale).astype(np.float32)
        s_out = new_scale.reshape(M, 1) if per_row else new_scale.reshape(1, 1)
    else:
        g = block_size[1]
        amax = nanmax_reduce(absv.reshape(M, N // g, g), axis=2)
        new_scale = round_to_compute(fdiv(amax, np.float32(limit)), compute)
        new_scale = np.where(new_scale == 0.0, EPS_2_23, new_scale).astype(np.float32)
        s_out = np.repeat(new_scale, g, axis=1)
    scaled = clamp(fdiv_t(merged, s_out), -limit, limit)
    if seed is not None:
        new_q = sr_float8(scaled, seed, logical_offsets(M, N, offset_base), e4m3, limit)
    else:
        new_q = encode(scaled)
    return new_q, new_scale.reshape(scale.shape).astype(np.float32)


def merge_static_float8(qdata, scale, b, a, strength, *, e4m3=True, seed=None, compute="bf16", offset_base=0):
    """Static per-tensor FP8 merge (``merge_static_float8_lora``,
    ``_triton_static_float8_lora.py:23-158``): the per-tensor layout of
    :func:`merge_float8` (dense ``compute(fp8 * scale)``, tile maxima of
    ``|merged|``, ``compute(amax / limit)`` with 0 -> 2**-23, ``merged / scale``
    clamped, RTNE or stochastic FP8)."""
    M = np.asarray(b).shape[0]
    N = np.asarray(a).shape[1]
    return merge_float8(qdata, np.asarray(scale, np.float32).reshape(1, 1), (M, N), b, a, strength, e4m3=e4m3,
                        seed=seed, compute=compute, offset_base=offset_base)


# ---------------------------------------------------------------------------
# bitsandbytes LLM.int8: _triton_bnb8_lora.py:20-142.
# ---------------------------------------------------------------------------


def merge_bnb8(cb, scb, b, a, strength, *, seed=None, offset_base=0):
    """bitsandbytes row-wise int8 merge (``merge_bnb8_lora``, ``_triton_bnb8_lora.py:145-242``).

    ``cb`` int8 (M x N), ``scb`` fp32 (M,). fp16 arithmetic: ``normalized =
    f16(cb / 127.0)`` (IEEE constant division), ``base = f16(normalized *
    f16(scb))``, ``merged = f16(clamp(base + acc * strength, +-65504))``; the new
    SCB is the row max of ``|merged|``; codes ``rint(merged / SCB * 127)`` (0
    where SCB is 0) or stochastic, clamped to [-127, 127]. Returns ``(cb, scb)``.
    """
    from .numerics import f16_round

    M = b.shape[0]
    N = a.shape[1]
    cbf = np.asarray(cb, np.int8).astype(np.float32)
    normalized = f16_round((cbf / np.float32(127.0)).astype(np.float32))
    s16 = f16_round(np.asarray(scb, np.float32).reshape(M, 1))
    base = f16_round((normalized * s16).astype(np.float32))
    acc = lora_delta(b, a, "f16")
    merged = f16_round(clamp(fma_f32(acc, np.float32(strength), base), -65504.0, 65504.0))
    new_scb = nanmax_reduce(np.abs(merged), axis=1).astype(np.float32)
    safe = np.where(new_scb == 0.0, np.float32(1.0), new_scb).reshape(M, 1)
    scaled = (fdiv_t(merged, safe) * np.float32(127.0)).astype(np.float32)
    scaled = np.where(new_scb.reshape(M, 1) == 0.0, np.float32(0.0), scaled).astype(np.float32)
    quant = rint_half_even(scaled).astype(np.float32)
    if seed is not None:
        quant = sr_round_to_int(scaled, quant, seed, logical_offsets(M, N, offset_base), -127, 127)
    quant = np.clip(quant, -127, 127).astype(np.int8)
    return quant, new_scb.reshape(np.shape(scb))


# ---------------------------------------------------------------------------
# bitsandbytes 4-bit (NF4 / FP4): _triton_bnb4_lora.py:28-375.
# ---------------------------------------------------------------------------

BNB4_BLOCK = 64
BNB4_NESTED_BLOCK = 256
# Ordered FP4 magnitude levels and thresholds (_triton_bnb4_lora.py:53-105).
_FP4_LEVELS = np.array([0.0, 0.0052083334885537624, 0.1666666716337204, 0.25, 0.3333333432674408, 0.5,
                        0.6666666865348816, 1.0], dtype=np.float32)
_FP4_THRESHOLDS = np.array([0.0026041667442768812, 0.08593750256113708, 0.2083333358168602, 0.2916666716337204,
                            0.4166666716337204, 0.5833333432674408, 0.8333333432674408], dtype=np.float32)
_FP4_STORE_TO_LEVEL = np.array([0, 1, 6, 7, 4, 5, 2, 3], dtype=np.int64)  # _fp4_storage_to_level


def _fp4_level_to_store(level):
    level = np.asarray(level, np.int64)
    return np.where(level < 2, level, np.where(level < 4, level + 4, np.where(level < 6, level, level - 4)))


def sorted_code_lower_bound(values, code, max_index: int):
    """Index reached by the reference's binary search (``:29-50``): the number of
    entries among ``code[0:max_index]`` that are ``< value``."""
    values = np.asarray(values, np.float32)
    code = np.asarray(code, np.float32)
    low = np.zeros(values.shape, np.int64)
    high = np.full(values.shape, max_index, np.int64)
    steps = int(max_index).bit_length()
    for _ in range(steps):
        middle = (low + high) // 2
        right = code[middle] < values
        low = np.where(right, middle + 1, low)
        high = np.where(right, high, middle)
    return low


def nearest_sorted_code(values, code, max_index: int):
    """``_nearest_sorted_code`` (``_triton_bnb4_lora.py:29-50``)."""
    values = np.asarray(values, np.float32)
    code = np.asarray(code, np.float32)
    upper_index = sorted_code_lower_bound(values, code, max_index)
    lower_index = np.maximum(upper_index - 1, 0)
    lower = code[lower_index]
    upper = code[upper_index]
    choose_lower = np.abs((values - lower).astype(np.float32)) <= np.abs((values - upper).astype(np.float32))
    return np.where(choose_lower, lower_index, upper_index)


def stochastic_sorted_code(values, deterministic, code, seed, offsets, max_index: int):
    """``_stochastic_sorted_code`` (``_triton_stochastic_quantization.py:43-79``)."""
    values = np.asarray(values, np.float32)
    code = np.asarray(code, np.float32)
    upper_index = sorted_code_lower_bound(values, code, max_index)
    upper = code[upper_index]
    exact = upper == values
    lower_index = np.where(exact, upper_index, np.maximum(upper_index - 1, 0))
    lower = code[lower_index]
    width = (upper - lower).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        prob = np.where(width > 0.0, fdiv_t((values - lower).astype(np.float32), np.where(width > 0, width, 1.0)),
                        np.float32(0.0)).astype(np.float32)
    u = philox_uniform(seed, offsets)
    chosen = np.where(u < prob, upper_index, lower_index)
    interior = (values > code[0]) & (values < code[max_index]) & ~exact
    return np.where(interior, chosen, np.asarray(deterministic, np.int64))


def nearest_fp4_code(values):
    """``_nearest_fp4_code`` (``_triton_bnb4_lora.py:53-75``)."""
    values = np.asarray(values, np.float32)
    mag = np.abs(values)
    level = (mag[..., None] > _FP4_THRESHOLDS).sum(axis=-1).astype(np.int64)
    code = _fp4_level_to_store(level)
    return np.where((values < 0.0) & (level != 0), code + 8, code)


def stochastic_fp4_code(values, deterministic, seed, offsets):
    """``_stochastic_fp4_code`` (``_triton_bnb4_lora.py:135-160``)."""
    values = np.asarray(values, np.float32)
    deterministic = np.asarray(deterministic, np.int64)
    mag = np.abs(values)
    nearest_level = _FP4_STORE_TO_LEVEL[deterministic & 7]
    nearest = _FP4_LEVELS[nearest_level]
    down = nearest > mag
    lower_level = np.where(down, nearest_level - 1, nearest_level)
    upper_level = np.where(down, nearest_level, nearest_level + 1)
    lower = _FP4_LEVELS[np.clip(lower_level, 0, 7)]
    upper = _FP4_LEVELS[np.clip(upper_level, 0, 7)]
    width = (upper - lower).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        prob = np.where(upper > lower, fdiv_t((mag - lower).astype(np.float32), np.where(width > 0, width, 1.0)),
                        np.float32(0.0)).astype(np.float32)
    level = np.where(philox_uniform(seed, offsets) < prob, upper_level, lower_level)
    sign = np.where((values < 0.0) & (level != 0), 8, 0)
    chosen = _fp4_level_to_store(level) + sign
    interior = (mag > 0.0) & (mag < 1.0) & (prob > 0.0)
    return np.where(interior, chosen, deterministic)


def unpack_bnb4(packed, rows: int, cols: int) -> np.ndarray:
    """Code index of every element: element 2j is the high nibble of byte j (``:217-226``)."""
    p = np.asarray(packed, np.uint8).reshape(rows, cols // 2).astype(np.int64)
    out = np.empty((rows, cols), np.int64)
    out[:, 0::2] = p >> 4
    out[:, 1::2] = p & 15
    return out


def pack_bnb4(codes) -> np.ndarray:
    codes = np.asarray(codes, np.int64)
    return ((codes[:, 0::2] << 4) | codes[:, 1::2]).astype(np.uint8)


def bnb4_nested_quantize(raw_absmax, nested_code):
    """Nested (double) quantization of the new block maxima (``:316-375``, ``:399-431``).

    ``offset = sum(raw) / n``; per 256-block: ``nested = max |raw - offset|``,
    code ``nearest(clamp((raw - offset) / nested, -1, 1))`` over the 256-entry
    table. The reference sums in Triton's reduction order; here the sum is
    exact and rounded once (tie class: fp32 summation order of the mean).
    """
    raw = np.asarray(raw_absmax, np.float32).reshape(-1)
    n = raw.size
    # ``tl.sum(values) / TOTAL_VALUES`` with a runtime divisor: Triton's fp32 division (``fdiv_t``).
    offset = np.float32(fdiv_t(np.float32(np.sum(raw.astype(np.float64))), np.float32(n)))
    centered = (raw - offset).astype(np.float32)
    nblk = (n + BNB4_NESTED_BLOCK - 1) // BNB4_NESTED_BLOCK
    pad = np.zeros(nblk * BNB4_NESTED_BLOCK, np.float32)
    pad[:n] = np.abs(centered)
    nested_absmax = nanmax_reduce(pad.reshape(nblk, BNB4_NESTED_BLOCK), axis=1).astype(np.float32)
    safe = np.where(nested_absmax == 0.0, np.float32(1.0), nested_absmax)
    scaled = clamp(fdiv_t(centered, np.repeat(safe, BNB4_NESTED_BLOCK)[:n]), -1.0, 1.0)
    q = nearest_sorted_code(scaled, nested_code, 255).astype(np.uint8)
    return q, nested_absmax, offset


def merge_bnb4(packed, absmax, code, b, a, strength, *, quant_type="nf4", nested_absmax=None, nested_code=None,
               offset=None, seed=None, compute="bf16", offset_base=0):
    """bitsandbytes blockwise 4-bit merge (``merge_bnb4_lora``, ``_triton_bnb4_lora.py:434-604``).

    Blocks of 64 values along each row. ``absmax`` fp32 per block, or uint8
    codes of the nested quantization (``nested_absmax`` fp32 per 256 blocks,
    ``nested_code`` 256 fp32, ``offset`` fp32). ``base = compute(code[q] *
    scale)`` with ``scale = nested_code[c] * nested_absmax + offset`` (one fused
    multiply-add) when nested; ``merged = compute(base + acc * strength)``;
    new block scale ``max |merged|``; ``clamp(merged / scale, -1, 1)`` encoded
    to the nearest NF4 table entry (ties to the lower) or the FP4 thresholds,
    or stochastically. Returns ``(packed, absmax[, nested_absmax, offset])``.
    """
    M = b.shape[0]
    N = a.shape[1]
    nb = N // BNB4_BLOCK
    code = np.asarray(code, np.float32)
    idx = unpack_bnb4(packed, M, N)
    base = code[idx]
    if nested_absmax is not None:
        q = np.asarray(absmax, np.uint8).reshape(M, nb).astype(np.int64)
        flat = np.arange(M * nb).reshape(M, nb) // BNB4_NESTED_BLOCK
        ns = np.asarray(nested_absmax, np.float32).reshape(-1)[flat]
        scales = fma_f32(np.asarray(nested_code, np.float32)[q], ns, np.float32(offset))
    else:
        scales = np.asarray(absmax, np.float32).reshape(M, nb)
    acc = lora_delta(b, a, compute)
    if compute == "f32":
        merged = merged_values_f32_product(base, np.repeat(scales, BNB4_BLOCK, axis=1), acc, strength)
    else:
        base = round_to_compute((base * np.repeat(scales, BNB4_BLOCK, axis=1)).astype(np.float32), compute)
        merged = merged_values(base, acc, strength, compute)
    out_scale = nanmax_reduce(np.abs(merged).reshape(M, nb, BNB4_BLOCK), axis=2).astype(np.float32)
    safe = np.where(out_scale == 0.0, np.float32(1.0), out_scale)
    normalized = clamp(fdiv_t(merged, np.repeat(safe, BNB4_BLOCK, axis=1)), -1.0, 1.0)
    offs = logical_offsets(M, N, offset_base)
    if quant_type == "nf4":
        codes = nearest_sorted_code(normalized, code, 15)
        if seed is not None:
            codes = stochastic_sorted_code(normalized, codes, code, seed, offs, 15)
    else:
        codes = nearest_fp4_code(normalized)
        if seed is not None:
            codes = stochastic_fp4_code(normalized, codes, seed, offs)
    new_packed = pack_bnb4(codes).reshape(np.shape(packed))
    if nested_absmax is None:
        return new_packed, out_scale.reshape(np.shape(absmax))
    q, nabs, off = bnb4_nested_quantize(out_scale, nested_code)
    return new_packed, q.reshape(np.shape(absmax)), nabs.reshape(np.shape(nested_absmax)), off


# ---------------------------------------------------------------------------
# Quanto qbytes: _triton_quanto_lora.py:28-168, 202-217.
# ---------------------------------------------------------------------------


def merge_quanto(qdata, scale, axis_kind, b, a, strength, *, storage="int8", seed=None, compute="bf16",
                 offset_base=0):
    """Quanto qint8 / qfloat8 merge (``_merge_quanto_qbytes_lora``, ``_triton_quanto_lora.py:220-314``).

    ``storage`` is ``"int8"``, ``"e4m3"`` or ``"e5m2"``; ``qdata`` int8 or uint8
    FP8 codes; ``scale`` holds compute-dtype values, one per tensor / row /
    column (``axis_kind`` "tensor" / "row" / "column"). ``base = compute(q *
    scale)`` (0 where the scale is 0), ``merged = compute(base + acc *
    strength)``; the new scale is ``compute(amax * fp32(1 / qmax))`` (torch on
    CUDA divides by a host scalar through its reciprocal), 0 -> fp32 eps;
    ``s = merged / scale``; int8: ``rint(compute(s))`` or stochastic on ``s``,
    clamp [-128, 127]; FP8: RTNE of ``clamp(compute(s))`` or stochastic FP8 of
    ``clamp(s)``. Returns ``(qdata, scale)``.
    """
    M = b.shape[0]
    N = a.shape[1]
    if storage == "int8":
        lp = np.asarray(qdata, np.int8).astype(np.float32)
        qmax = np.float32(127.0)
    else:
        encode, decode, limit = fp8_codec(storage == "e4m3")
        lp = decode(np.asarray(qdata, np.uint8))
        qmax = np.float32(limit)
    s_in = np.asarray(scale, np.float32)
    shape_b = {"tensor": (1, 1), "row": (M, 1), "column": (1, N)}[axis_kind]
    s_b = s_in.reshape(shape_b)
    with np.errstate(invalid="ignore"):
        prod = (lp * s_b).astype(np.float32)
    base = round_to_compute(np.where(s_b == 0.0, np.float32(0.0), prod).astype(np.float32), compute)
    acc = lora_delta(b, a, compute)
    merged = merged_values(base, acc, strength, compute)
    absm = np.abs(merged)
    if axis_kind == "tensor":
        amax = nanmax_reduce(absm.reshape(-1), axis=0).reshape(1, 1)
    elif axis_kind == "row":
        amax = nanmax_reduce(absm, axis=1).reshape(M, 1)
    else:
        amax = nanmax_reduce(absm, axis=0).reshape(1, N)
    inv = np.float32(np.float32(1.0) / qmax)
    new_s = round_to_compute((amax * inv).astype(np.float32), compute)
    new_s = np.where(new_s == 0.0, EPS_2_23, new_s).astype(np.float32)
    ss = fdiv_t(merged, new_s)
    offs = logical_offsets(M, N, offset_base)
    if storage == "int8":
        det = rint_half_even(round_to_compute(ss, compute)).astype(np.float32)
        quant = det if seed is None else sr_round_to_int(ss, det, seed, offs, -128, 127)
        new_q = np.clip(quant, -128, 127).astype(np.int8)
    else:
        if seed is None:
            new_q = encode(clamp(round_to_compute(ss, compute), -qmax, qmax))
        else:
            new_q = sr_float8(clamp(ss, -qmax, qmax), seed, offs, storage == "e4m3", float(qmax))
    return new_q, new_s.reshape(np.shape(scale)).astype(np.float32)


# ---------------------------------------------------------------------------
# Affine INT8: _triton_int8_lora.py:24-236.
# ---------------------------------------------------------------------------


def merge_int8(qdata, scale, zero_point, block_size, b, a, strength, *, asymmetric=False,
               reduce_range=False, seed=None, compute="bf16", qparam="bf16", offset_base=0):
    """Affine-INT8 merge (``merge_int8_lora``, ``_triton_int8_lora.py:267-407``).

    ``qdata`` int8 (M x N); ``scale`` float values (already in ``qparam``
    precision) with one entry per quantization block; ``zero_point`` int8 or
    None. Returns ``(qdata, scale, zero_point)`` (scale rounded to ``qparam``).
    """
    qmin, qmax = (-64, 63) if reduce_range else (-128, 127)
    M = b.shape[0]
    N = a.shape[1]
    if tuple(block_size) == (M, N):
        block_numel = M * N
    else:
        block_numel = block_size[1]
    nq = (M * N) // block_numel
    flat_q = np.asarray(qdata, np.int8).reshape(-1).astype(np.float32)
    s_flat = np.asarray(scale, np.float32).reshape(-1)
    zp_flat = (np.zeros(nq, np.int64) if zero_point is None
               else np.asarray(zero_point, np.int8).reshape(-1).astype(np.int64))
    qidx = np.arange(M * N, dtype=np.int64) // block_numel
    base = round_to_compute(flat_q - zp_flat[qidx].astype(np.float32), compute)
    sv_in = s_flat[qidx]
    if {compute, qparam} == {"bf16", "f16"}:
        # ``base * scale`` (:80) with one bf16 and one fp16 operand: Triton
        # converts both to fp16 and rounds the product to fp16
        # (triton/language/semantic.py, computation_type_impl).
        prod = f16_round((f16_round(base) * f16_round(sv_in)).astype(np.float32))
    else:
        prod = (base * sv_in).astype(np.float32)
    acc = lora_delta(b, a, compute).reshape(-1)
    if compute == "f32":
        dense = merged_values_f32_product(base, sv_in, acc, strength)
    else:
        base = round_to_compute(prod, compute)
        dense = merged_values(base, acc, strength, compute)
    blocks = dense.reshape(nq, block_numel)
    min_v = nanmin_reduce(minnum(blocks, np.float32(0.0)), axis=1)
    max_v = nanmax_reduce(maxnum(blocks, np.float32(0.0)), axis=1)
    min_v = round_to_compute(min_v, compute)
    max_v = round_to_compute(max_v, compute)
    if asymmetric:
        rng = round_to_compute((max_v - min_v).astype(np.float32), compute)
        s = fdiv(rng, np.float32(qmax - qmin))
    else:
        s = fdiv(maxnum(-min_v, max_v), np.float32((qmax - qmin) / 2.0))
    s = round_to_compute(s, compute)
    s = maxnum(s, EPS_2_23)
    s = round_to_compute(s, compute)
    if asymmetric:
        ratio = round_to_compute(fdiv_t(min_v, s), compute)
        zp = np.clip(qmin - rint_half_even(ratio), qmin, qmax)
    else:
        zp = np.zeros(nq, np.int64)
    # The output scale buffer has the scale tensor's dtype.
    s_store = round_to_compute(s, qparam)
    values = dense
    sv = s_store[qidx]
    stochastic_scaled = fdiv_t(values, sv)
    inv = round_to_compute(fdiv_t(np.float32(1.0), sv), qparam)
    scaled = round_to_compute((values * inv).astype(np.float32), qparam)
    quant = rint_half_even(scaled) + zp[qidx]
    quant = quant.astype(np.float32)
    if seed is not None:
        offs = (np.uint64(offset_base) + np.arange(M * N, dtype=np.uint64)).astype(np.uint64)
        quant = sr_round_to_int((stochastic_scaled + zp[qidx].astype(np.float32)).astype(np.float32),
                                quant, seed, offs, qmin, qmax)
    quant = np.clip(quant, qmin, qmax).astype(np.int8).reshape(M, N)
    return quant, s_store.reshape(np.shape(scale)), zp.astype(np.int8).reshape(np.shape(scale))


# ---------------------------------------------------------------------------
# GGUF Q8_0 / Q4_0. Decoding follows gguf_dequant.py:57-61 and :107-115 (the
# reference's bf16 dequantization on H2D). The reference has no GGUF merge;
# re-encoding follows the gguf package (0.19.0) quantizers
# gguf/quants.py Q8_0.quantize_blocks and Q4_0.quantize_blocks.
# ---------------------------------------------------------------------------

Q8_0 = 8
Q4_0 = 2
GGUF_BLOCK = {Q8_0: (32, 34), Q4_0: (32, 18)}


def gguf_dequant(raw: np.ndarray, quant_type: int, rows: int, cols: int, compute="bf16") -> np.ndarray:
    """``gguf_dequant.dequantize(data, qtype, dtype=bf16)`` for Q8_0/Q4_0 as fp32 values."""
    bs, ts = GGUF_BLOCK[quant_type]
    blocks = np.asarray(raw, np.uint8).reshape(-1, ts)
    d = blocks[:, :2].copy().view(np.float16).astype(np.float32)
    d = round_to_compute(d, compute)
    if quant_type == Q8_0:
        q = blocks[:, 2:].view(np.int8).astype(np.float32)
    else:
        qs = blocks[:, 2:]
        q = np.concatenate([qs & 0xF, qs >> 4], axis=1).astype(np.int64) - 8
        q = q.astype(np.float32)
    out = round_to_compute((d * q).astype(np.float32), compute)
    return out.reshape(rows, cols)


def roundf_away(x: np.ndarray) -> np.ndarray:
    """``gguf.quants.np_roundf``: round half away from zero."""
    a = np.abs(x)
    fl = np.floor(a)
    return (np.sign(x) * (fl + np.floor(2 * (a - fl)))).astype(np.float32)


def gguf_quantize(values: np.ndarray, quant_type: int, seed=None, offset_base=0) -> np.ndarray:
    """Re-encode fp32 values (M x N) into raw GGUF blocks.

    RTN reproduces ``gguf.quants.Q8_0/Q4_0.quantize_blocks`` bit for bit.
    SR (no reference stream exists) draws ``_random`` by logical element
    offset and rounds the pre-rounding quotient to an adjacent integer code,
    the same rule as ``_stochastic_round_to_int``.
    """
    M, N = values.shape
    v = np.asarray(values, np.float32).reshape(-1, 32)
    nblk = v.shape[0]
    offs = (np.uint64(offset_base) + np.arange(M * N, dtype=np.uint64)).reshape(-1, 32)
    if quant_type == Q8_0:
        d = (np.max(np.abs(v), axis=1, keepdims=True) / np.float32(127)).astype(np.float32)
        with np.errstate(divide="ignore"):
            inv = np.where(d == 0, np.float32(0), (np.float32(1) / d)).astype(np.float32)
        x = (v * inv).astype(np.float32)
        q = roundf_away(x)
        if seed is not None:
            q = sr_round_to_int(x, q, seed, offs, -127, 127)
        q = np.clip(q, -128, 127).astype(np.int8).view(np.uint8)
        dh = d.astype(np.float16).view(np.uint8).reshape(nblk, 2)
        return np.concatenate([dh, q], axis=1).reshape(M, N // 32 * 34)
    imax = np.abs(v).argmax(axis=1)[:, None]
    mx = np.take_along_axis(v, imax, axis=1)
    d = (mx / np.float32(-8)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), (np.float32(1) / d)).astype(np.float32)
    x = (v * inv).astype(np.float32)
    q = np.trunc((x + np.float32(8.5)).astype(np.float32))
    if seed is not None:
        q = sr_round_to_int((x + np.float32(8.0)).astype(np.float32), q, seed, offs, 0, 15)
    q = np.clip(q, 0, 15).astype(np.uint8)
    packed = (q[:, :16] | (q[:, 16:] << 4)).astype(np.uint8)
    dh = d.astype(np.float16).view(np.uint8).reshape(nblk, 2)
    return np.concatenate([dh, packed], axis=1).reshape(M, N // 32 * 18)


def merge_gguf(raw, quant_type, b, a, strength, *, seed=None, compute="bf16", offset_base=0):
    """GGUF merge: dequant (bf16) + fp32 FMA update rounded to bf16 + gguf re-encode."""
    M = b.shape[0]
    N = a.shape[1]
    base = gguf_dequant(raw, quant_type, M, N, compute)
    merged = merged_values(base, lora_delta(b, a, compute), strength, compute)
    return gguf_quantize(merged, quant_type, seed=seed, offset_base=offset_base)

"""Seeded synthetic quantized weights and LoRA factors (torch, any device).

The reference benchmarks its merge on no public dataset; these builders make
model-shaped stand-ins: a bf16 base drawn from N(0, std) (optionally with a
fraction of outliers), quantized into each raw layout with simple
torch-op quantizers whose scale conventions follow the layouts the reference
reads (per-row symmetric INT8, per-row FP8, NVFP4 two-level, MX E8M0 FLOOR,
GGUF Q8_0/Q4_0). The quantizers only produce valid inputs; the merge itself
re-derives every scale.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

E2M1_GRID = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def generator(seed: int, device: torch.device | str) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def normal(shape, std: float, *, seed: int, device, dtype=torch.bfloat16, outlier_frac: float = 0.0,
           outlier_scale: float = 8.0) -> torch.Tensor:
    g = generator(seed, device)
    x = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std
    if outlier_frac > 0:
        mask = torch.rand(shape, generator=g, device=device) < outlier_frac
        x = torch.where(mask, x * outlier_scale, x)
    return x.to(dtype)


def lora_factors(rows: int, cols: int, rank: int, std: float, *, seed: int, device,
                 dtype=torch.bfloat16) -> tuple[torch.Tensor, torch.Tensor]:
    """(B, A) with B: rows x rank and A: rank x cols, both N(0, std)."""
    b = normal((rows, rank), std, seed=seed, device=device, dtype=dtype)
    a = normal((rank, cols), std, seed=seed + 1, device=device, dtype=dtype)
    return b, a


def encode_e2m1(x: torch.Tensor) -> torch.Tensor:
    """Round-to-nearest-even E2M1 code (4 bits, sign in bit 3) of fp32 values."""
    m = x.abs()
    code = torch.zeros_like(x, dtype=torch.int32)
    for i, t in enumerate((0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)):
        above = (m > t) if i % 2 == 0 else (m >= t)
        code = code + above.to(torch.int32)
    sign = (x.view(torch.int32) >> 31) & 1
    return (code | (sign << 3)).to(torch.uint8)


def pack_fp4(codes: torch.Tensor) -> torch.Tensor:
    c = codes.to(torch.uint8) & 0xF
    return (c[..., 0::2] | (c[..., 1::2] << 4)).contiguous()


def to_blocked(scale2d: torch.Tensor) -> torch.Tensor:
    """Blocked layout with a flat index of (row_blk*colblks + col_blk)*512 + lane*16 + grp*4 + col."""
    rows, sc = scale2d.shape
    rp = (rows + 127) // 128 * 128
    cp = (sc + 3) // 4 * 4
    padded = torch.zeros((rp, cp), dtype=scale2d.dtype, device=scale2d.device)
    padded[:rows, :sc] = scale2d
    t = padded.view(rp // 128, 4, 32, cp // 4, 4).permute(0, 3, 2, 1, 4).contiguous()
    return t.view(-1)


@dataclass
class QuantizedWeight:
    """Raw buffers of one quantized weight (attribute names follow TorchAO)."""

    qdata: torch.Tensor
    scale: torch.Tensor | None = None
    zero_point: torch.Tensor | None = None
    per_tensor_scale: torch.Tensor | None = None
    rows: int = 0
    cols: int = 0


def quantize_int8_per_row(w: torch.Tensor) -> QuantizedWeight:
    wf = w.float()
    amax = wf.abs().amax(dim=1, keepdim=True).clamp_min(1e-12)
    scale = (amax / 127.0).to(torch.bfloat16)
    q = torch.round(wf / scale.float()).clamp(-128, 127).to(torch.int8)
    return QuantizedWeight(q, scale, None, None, w.shape[0], w.shape[1])


def quantize_int8_codes(rows: int, cols: int, *, seed: int, device, std: float = 0.02) -> QuantizedWeight:
    """Codes uniform in [-127, 127] and bf16 row scales |N(0, std)| row-absmax / 127."""
    g = generator(seed, device)
    q = torch.randint(-127, 128, (rows, cols), generator=g, device=device, dtype=torch.int16).to(torch.int8)
    base = torch.randn((rows, cols), generator=g, device=device) * std
    scale = (base.abs().amax(dim=1, keepdim=True) / 127.0).to(torch.bfloat16)
    return QuantizedWeight(q, scale, None, None, rows, cols)


def quantize_fp8(w: torch.Tensor, *, group: int | None = None, per_tensor: bool = False,
                 dtype=torch.float8_e4m3fn) -> QuantizedWeight:
    wf = w.float()
    rows, cols = wf.shape
    limit = torch.finfo(dtype).max
    if per_tensor:
        scale = (wf.abs().amax().clamp_min(1e-12) / limit).reshape(1, 1)
        s_full = scale
    elif group is None:
        scale = wf.abs().amax(dim=1, keepdim=True).clamp_min(1e-12) / limit
        s_full = scale
    else:
        scale = wf.view(rows, cols // group, group).abs().amax(dim=2).clamp_min(1e-12) / limit
        s_full = scale.repeat_interleave(group, dim=1)
    q = (wf / s_full).clamp(-limit, limit).to(dtype)
    return QuantizedWeight(q, scale.float().contiguous(), None, None, rows, cols)


def quantize_nvfp4(w: torch.Tensor, *, two_level: bool = True, swizzled: bool = False) -> QuantizedWeight:
    wf = w.float()
    rows, cols = wf.shape
    blocks = wf.view(rows, cols // 16, 16)
    amax16 = blocks.abs().amax(dim=2)
    if two_level:
        g = (wf.abs().amax() / 2688.0).clamp_min(2 ** -23)
        bs = (amax16 / 6.0 / g).clamp(0.015625, 448.0).to(torch.float8_e4m3fn)
        denom = bs.float() * g
        pts = g.reshape(1).float()
    else:
        bs = (amax16 / 6.0).clamp(0.015625, 448.0).to(torch.float8_e4m3fn)
        denom = bs.float()
        pts = None
    codes = encode_e2m1((blocks / denom.unsqueeze(2)).clamp(-6, 6)).view(rows, cols)
    scale = bs.view(torch.uint8)
    if swizzled:
        scale = to_blocked(scale).view((rows + 127) // 128 * 32, (cols + 63) // 64 * 16)
    return QuantizedWeight(pack_fp4(codes), scale.contiguous().view(torch.float8_e4m3fn), None, pts, rows, cols)


_MX = {"e4m3": (8, torch.float8_e4m3fn), "e5m2": (15, torch.float8_e5m2), "e2m1": (2, None)}


def quantize_mx(w: torch.Tensor, elem: str, *, swizzled: bool = False) -> QuantizedWeight:
    wf = w.float()
    rows, cols = wf.shape
    target, dt = _MX[elem]
    blocks = wf.view(rows, cols // 32, 32)
    amax = blocks.abs().amax(dim=2).clamp_min(2 ** -126)
    exp = torch.floor(torch.log2(amax)).to(torch.int32) - target
    exp = exp.clamp(-127, 127)
    code = (exp + 127).to(torch.uint8)
    scale_val = torch.pow(2.0, exp.float())
    norm = blocks / scale_val.unsqueeze(2)
    if elem == "e2m1":
        q = pack_fp4(encode_e2m1(norm.clamp(-6, 6)).view(rows, cols))
    else:
        lim = torch.finfo(dt).max
        q = norm.clamp(-lim, lim).view(rows, cols).to(dt)
    scale = code
    if swizzled:
        scale = to_blocked(code).view((rows + 127) // 128 * 32, (cols + 127) // 128 * 16)
    return QuantizedWeight(q.contiguous(), scale.contiguous(), None, None, rows, cols)


def quantize_gguf(w: torch.Tensor, quant_type: int) -> QuantizedWeight:
    """Q8_0 (8) / Q4_0 (2) raw blocks following gguf's quantize_blocks formulas."""
    wf = w.float()
    rows, cols = wf.shape
    blocks = wf.reshape(-1, 32)
    if quant_type == 8:
        d = blocks.abs().amax(dim=1, keepdim=True) / 127.0
        inv = torch.where(d == 0, torch.zeros_like(d), 1.0 / d)
        x = blocks * inv
        a = x.abs()
        fl = torch.floor(a)
        q = (torch.sign(x) * (fl + torch.floor(2 * (a - fl)))).clamp(-128, 127).to(torch.int8)
        dh = d.to(torch.float16).view(torch.uint8).view(-1, 2)
        raw = torch.cat([dh, q.view(torch.uint8)], dim=1)
        return QuantizedWeight(raw.reshape(rows, cols // 32 * 34).contiguous(), None, None, None, rows, cols)
    idx = blocks.abs().argmax(dim=1, keepdim=True)
    mx = torch.gather(blocks, 1, idx)
    d = mx / -8.0
    inv = torch.where(d == 0, torch.zeros_like(d), 1.0 / d)
    q = torch.trunc(blocks * inv + 8.5).clamp(0, 15).to(torch.uint8)
    packed = q[:, :16] | (q[:, 16:] << 4)
    dh = d.to(torch.float16).view(torch.uint8).view(-1, 2)
    raw = torch.cat([dh, packed], dim=1)
    return QuantizedWeight(raw.reshape(rows, cols // 32 * 18).contiguous(), None, None, None, rows, cols)


# ------------------------------------------------ bitsandbytes and Quanto layouts
def quantize_bnb8(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """bitsandbytes LLM.int8 row-wise storage: ``CB = round(w * 127 / SCB)``, ``SCB = row max |w|`` (fp32)."""
    wf = w.float()
    scb = wf.abs().amax(dim=1).clamp_min(1e-12)
    cb = torch.round(wf * 127.0 / scb[:, None]).clamp(-127, 127).to(torch.int8)
    return cb.contiguous(), scb.contiguous()


def quantize_quanto(w: torch.Tensor, storage: str, axis: int | None = 0,
                    dtype: torch.dtype = torch.bfloat16) -> tuple[torch.Tensor, torch.Tensor]:
    """Quanto qbytes: absmax scale (``dtype``) per row (axis 0), per column (axis -1) or per tensor."""
    wf = w.float()
    qmax = 127.0 if storage == "int8" else torch.finfo(torch.float8_e4m3fn if storage == "e4m3"
                                                       else torch.float8_e5m2).max
    if axis == 0:
        amax = wf.abs().amax(dim=1, keepdim=True)
    elif axis == -1:
        amax = wf.abs().amax(dim=0, keepdim=True)
    else:
        amax = wf.abs().amax()
    scale = (amax.clamp_min(1e-12) / qmax).to(dtype)
    x = wf / scale.float()
    if storage == "int8":
        data = torch.round(x).clamp(-128, 127).to(torch.int8)
    else:
        data = x.clamp(-qmax, qmax).to(torch.float8_e4m3fn if storage == "e4m3" else torch.float8_e5m2)
    return data.contiguous(), scale.contiguous()


def nf4_style_table(device) -> torch.Tensor:
    """A 16-entry NF4-style table: normal quantiles scaled to [-1, 1] with an exact zero
    (the construction of the QLoRA paper; synthetic, for benchmarking)."""
    pos = torch.erfinv(torch.linspace(0.0, 0.9677, 9)[1:] * 1.0).double()  # 8 positive quantiles
    neg = -torch.erfinv(torch.linspace(0.0, 0.9677, 8)[1:] * 1.0).double()  # 7 negative quantiles
    vals = torch.cat([neg / neg.abs().max(), torch.zeros(1, dtype=torch.float64), pos / pos.max()])
    return vals.sort().values.float().to(device).contiguous()


def _nearest_index(x: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    return (x[..., None] - table).abs().argmin(dim=-1)


def quantize_bnb4(w: torch.Tensor, *, nested: bool = False):
    """bitsandbytes 4-bit blockwise storage (64-value blocks along rows, first value of a
    byte in its high nibble) with an NF4-style table; nested absmax quantized with a
    256-entry table. Returns ``(packed (numel/2, 1) uint8, absmax, code, nested_absmax,
    nested_code, offset)``."""
    rows, cols = w.shape
    dev = w.device
    code = nf4_style_table(dev)
    blocks = w.float().reshape(rows, cols // 64, 64)
    absmax = blocks.abs().amax(dim=2).clamp_min(1e-12)
    idx = torch.empty(rows, cols // 64, 64, dtype=torch.int64, device=dev)
    for r0 in range(0, rows, 1024):  # bounded temporary
        idx[r0:r0 + 1024] = _nearest_index(blocks[r0:r0 + 1024] / absmax[r0:r0 + 1024, :, None], code)
    idx = idx.reshape(rows, cols)
    packed = ((idx[:, 0::2] << 4) | idx[:, 1::2]).to(torch.uint8).reshape(-1, 1).contiguous()
    if not nested:
        return packed, absmax.reshape(-1).contiguous(), code, None, None, None
    flat = absmax.reshape(-1)
    offset = flat.mean().reshape(())
    centered = flat - offset
    nblk = (flat.numel() + 255) // 256
    pad = torch.zeros(nblk * 256, device=dev)
    pad[:flat.numel()] = centered.abs()
    nested_absmax = pad.reshape(nblk, 256).amax(dim=1).clamp_min(1e-12)
    nested_code = torch.linspace(-1.0, 1.0, 256, device=dev)
    scaled = centered / nested_absmax.repeat_interleave(256)[:flat.numel()]
    q = torch.empty(flat.numel(), dtype=torch.uint8, device=dev)
    for i0 in range(0, flat.numel(), 1 << 16):
        q[i0:i0 + (1 << 16)] = _nearest_index(scaled[i0:i0 + (1 << 16)], nested_code).to(torch.uint8)
    return packed, q.contiguous(), code, nested_absmax.contiguous(), nested_code.contiguous(), \
        offset.float().contiguous()

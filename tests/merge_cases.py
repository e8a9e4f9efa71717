"""Shared builders for the merge parity tests: one seeded case per format.

A case holds CPU copies of the input buffers (for the oracle) and runs the
sm_100a path through ``piper_offload_b200.kernels`` on a CUDA device. The
oracle (``oracle.merge``) is the checker; results are compared code for code.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from oracle import merge as om
from piper_offload_b200 import kernels as K
from piper_offload_b200 import synthetic as S

FORMATS = ("mxfp8", "mxfp8_e5m2", "mxfp4", "nvfp4", "nvfp4_1l", "fp8_row", "fp8_tensor",
           "fp8_group", "int8_row", "int8_tensor", "int8_group", "int8_asym", "q8_0", "q4_0")


def f32np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float32)


def u8np(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy().copy()


@dataclass
class Case:
    fmt: str
    rows: int
    cols: int
    rank: int
    seed: int | None = None
    strength: float = 1.0
    swizzled: bool = False
    scale_mode: int = 0
    group: int = 64
    factor_dtype: torch.dtype = torch.bfloat16
    base_std: float = 0.02
    lora_std: float = 0.01
    outliers: float = 0.0
    offset_base: int = 0
    tensors: dict = field(default_factory=dict)

    # ------------------------------------------------------------- build
    def build(self, device="cpu", data_seed: int = 0) -> "Case":
        w = S.normal((self.rows, self.cols), self.base_std, seed=data_seed, device="cpu",
                     outlier_frac=self.outliers)
        b, a = S.lora_factors(self.rows, self.cols, self.rank, self.lora_std, seed=data_seed + 10,
                              device="cpu", dtype=self.factor_dtype)
        f = self.fmt
        if f.startswith("mx"):
            elem = {"mxfp8": "e4m3", "mxfp8_e5m2": "e5m2", "mxfp4": "e2m1"}[f]
            q = S.quantize_mx(w, elem, swizzled=self.swizzled)
        elif f.startswith("nvfp4"):
            q = S.quantize_nvfp4(w, two_level=(f == "nvfp4"), swizzled=self.swizzled)
        elif f == "fp8_row":
            q = S.quantize_fp8(w)
        elif f == "fp8_tensor":
            q = S.quantize_fp8(w, per_tensor=True)
        elif f == "fp8_group":
            q = S.quantize_fp8(w, group=self.group)
        elif f.startswith("int8"):
            q = S.quantize_int8_per_row(w)
            if f == "int8_tensor":
                q.scale = (w.float().abs().amax() / 127.0).reshape(1, 1).to(torch.bfloat16)
            elif f == "int8_group":
                g = self.group
                sc = (w.float().view(self.rows, self.cols // g, g).abs().amax(2) / 127.0).to(torch.bfloat16)
                q.scale = sc
            elif f == "int8_asym":
                q.zero_point = torch.randint(-20, 21, (self.rows, 1), generator=S.generator(data_seed + 5, "cpu"),
                                             dtype=torch.int32).to(torch.int8)
        elif f == "q8_0":
            q = S.quantize_gguf(w, 8)
        elif f == "q4_0":
            q = S.quantize_gguf(w, 2)
        else:
            raise KeyError(f)
        self.tensors = {"q": q, "b": b, "a": a}
        return self

    # ------------------------------------------------------------ native
    def run_native(self, device) -> dict:
        q = self.tensors["q"]
        b = self.tensors["b"].to(device)
        a = self.tensors["a"].to(device)
        f = self.fmt
        out = {}
        qd = q.qdata.to(device)
        sc = q.scale.to(device) if q.scale is not None else None
        kw = dict(rounding_seed=self.seed, offset_base=self.offset_base)
        if f.startswith("mx"):
            elem = {"mxfp8": torch.float8_e4m3fn, "mxfp8_e5m2": torch.float8_e5m2,
                    "mxfp4": getattr(torch, "float4_e2m1fn_x2", None)}[f]
            if f == "mxfp4" and elem is None:
                raise RuntimeError("torch lacks float4_e2m1fn_x2")
            scale_e8 = sc.view(torch.float8_e8m0fnu)
            K.merge_mx_lora_(qd, scale_e8, elem, 32, self.factor_dtype, b, a, self.strength,
                             scaling_mode=self.scale_mode, swizzled=self.swizzled, **kw)
            out["q"] = u8np(qd)
            out["scale"] = u8np(scale_e8)
        elif f.startswith("nvfp4"):
            pts = q.per_tensor_scale.to(device) if q.per_tensor_scale is not None else None
            K.merge_nvfp4_lora(qd, sc, pts, 16, self.swizzled, b, a, self.strength, **kw)
            out["q"] = u8np(qd)
            out["scale"] = u8np(sc)
            out["global"] = None if pts is None else float(pts.cpu())
        elif f.startswith("fp8"):
            block = {"fp8_row": (1, self.cols), "fp8_tensor": (self.rows, self.cols),
                     "fp8_group": (1, self.group)}[f]
            K.merge_float8_lora(qd, sc, block, b, a, self.strength, **kw)
            out["q"] = u8np(qd)
            out["scale"] = f32np(sc)
        elif f.startswith("int8"):
            block = {"int8_row": (1, self.cols), "int8_tensor": (self.rows, self.cols),
                     "int8_group": (1, self.group), "int8_asym": (1, self.cols)}[f]
            zp = q.zero_point.to(device) if q.zero_point is not None else None
            asym = zp is not None
            K.merge_int8_lora(qd, sc, zp, block, b, a, self.strength, asymmetric=asym,
                              reduce_range=False, **kw)
            out["q"] = qd.cpu().numpy().copy()
            out["scale"] = f32np(sc)
            out["zp"] = None if zp is None else zp.cpu().numpy().copy()
        else:
            qt = 8 if f == "q8_0" else 2
            K.merge_gguf_lora_(qd, qt, b, a, self.strength, **kw)
            out["q"] = u8np(qd)
        return out

    # ------------------------------------------------------------ oracle
    def run_oracle(self) -> dict:
        q = self.tensors["q"]
        b = f32np(self.tensors["b"])
        a = f32np(self.tensors["a"])
        cdt = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[self.factor_dtype]
        f = self.fmt
        kw = dict(seed=self.seed, offset_base=self.offset_base)
        if f.startswith("mx"):
            elem = {"mxfp8": "e4m3", "mxfp8_e5m2": "e5m2", "mxfp4": "e2m1"}[f]
            nq, ns = om.merge_mx(u8np(q.qdata), u8np(q.scale), elem, b, a, self.strength,
                                 scaling_mode=self.scale_mode, swizzled=self.swizzled, compute=cdt, **kw)
            return {"q": nq, "scale": ns}
        if f.startswith("nvfp4"):
            pts = None if q.per_tensor_scale is None else float(q.per_tensor_scale)
            nq, ns, g = om.merge_nvfp4(u8np(q.qdata), u8np(q.scale), pts, b, a, self.strength,
                                       swizzled=self.swizzled, compute=cdt, **kw)
            return {"q": nq, "scale": ns, "global": None if g is None else float(g)}
        if f.startswith("fp8"):
            block = {"fp8_row": (1, self.cols), "fp8_tensor": (self.rows, self.cols),
                     "fp8_group": (1, self.group)}[f]
            nq, ns = om.merge_float8(u8np(q.qdata), f32np(q.scale), block, b, a, self.strength,
                                     e4m3=True, compute=cdt, **kw)
            return {"q": nq, "scale": ns}
        if f.startswith("int8"):
            block = {"int8_row": (1, self.cols), "int8_tensor": (self.rows, self.cols),
                     "int8_group": (1, self.group), "int8_asym": (1, self.cols)}[f]
            zp = None if q.zero_point is None else q.zero_point.numpy()
            nq, ns, nz = om.merge_int8(q.qdata.numpy(), f32np(q.scale), zp, block, b, a, self.strength,
                                       asymmetric=zp is not None, compute=cdt,
                                       qparam={torch.float16: "f16", torch.float32: "f32"}.get(q.scale.dtype, "bf16"),
                                       **kw)
            return {"q": nq, "scale": ns, "zp": None if zp is None else nz}
        qt = om.Q8_0 if f == "q8_0" else om.Q4_0
        return {"q": om.merge_gguf(u8np(q.qdata), qt, b, a, self.strength, compute=cdt, **kw)}


# ---------------------------------------------------------------- compare
def code_values(fmt: str, q: np.ndarray) -> np.ndarray:
    """Integer 'code position' of each element so one step = 1 apart."""
    from oracle.merge import unpack_fp4

    if fmt in ("mxfp4", "nvfp4", "nvfp4_1l"):
        c = unpack_fp4(q)
        mag = c & 7
        return np.where(c & 8, -mag, mag)
    if fmt.startswith("int8"):
        return q.astype(np.int64)
    if fmt in ("q8_0", "q4_0"):
        ts = 34 if fmt == "q8_0" else 18
        blocks = q.reshape(-1, ts)[:, 2:]
        if fmt == "q8_0":
            return blocks.view(np.int8).astype(np.int64)
        return np.concatenate([blocks & 0xF, blocks >> 4], axis=1).astype(np.int64)
    c = q.astype(np.int64)
    mag = c & 0x7F
    return np.where(c & 0x80, -mag, mag)


@dataclass
class Diff:
    n: int
    code_mismatch: int
    max_step: int
    scale_mismatch: int
    extra: str = ""

    @property
    def frac(self) -> float:
        return self.code_mismatch / max(self.n, 1)


def compare(case: Case, got: dict, want: dict) -> Diff:
    gv = code_values(case.fmt, got["q"])
    wv = code_values(case.fmt, want["q"])
    diff = np.abs(gv - wv)
    n = gv.size
    mism = int(np.count_nonzero(diff))
    max_step = int(diff.max()) if n else 0
    sm = 0
    if "scale" in want and want["scale"] is not None:
        gs = np.asarray(got["scale"]).reshape(-1)
        ws = np.asarray(want["scale"]).reshape(-1)
        sm = int(np.count_nonzero(gs.view(np.uint8) != ws.view(np.uint8))) if gs.dtype == np.uint8 else int(
            np.count_nonzero(gs != ws))
    if case.fmt in ("q8_0", "q4_0"):
        ts = 34 if case.fmt == "q8_0" else 18
        gd = got["q"].reshape(-1, ts)[:, :2]
        wd = want["q"].reshape(-1, ts)[:, :2]
        sm = int(np.count_nonzero(np.any(gd != wd, axis=1)))
    extra = ""
    if want.get("global") is not None:
        extra = f"global got={got['global']!r} want={want['global']!r}"
        if got["global"] != want["global"]:
            sm += 1
    if want.get("zp") is not None:
        sm += int(np.count_nonzero(got["zp"] != want["zp"]))
    return Diff(n, mism, max_step, sm, extra)


# Reference test shapes (the reference tests): 35x69 r7 INT8, 70x130 r7
# FP8, 19x80 r13 NVFP4, 19x96 r7 MX, 16x64 SR.
SMALL_SHAPES = {
    "mxfp8": (19, 96, 7), "mxfp8_e5m2": (19, 96, 7), "mxfp4": (19, 96, 7),
    "nvfp4": (19, 80, 13), "nvfp4_1l": (19, 80, 13),
    "fp8_row": (70, 130, 7), "fp8_tensor": (70, 130, 7), "fp8_group": (70, 128, 7),
    "int8_row": (35, 69, 7), "int8_tensor": (35, 69, 19), "int8_group": (35, 128, 7),
    "int8_asym": (35, 69, 7), "q8_0": (19, 96, 7), "q4_0": (19, 96, 7),
}

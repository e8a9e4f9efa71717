"""Reference-kernel fixtures: load them, and run the oracle or the sm_100a path on their inputs.

``tests/golden/merge_reference.{npz,json}`` hold the inputs and outputs of the
reference's Triton merge launchers, recorded by
``tests/golden/make_merge_golden.py``. Every case's factors are small-integer
multiples of a power of two, so the rank-r dot product is exact in any
summation order and the outputs are a bit-level target for any correct
implementation.
"""

from __future__ import annotations

import json
from functools import lru_cache
from pathlib import Path

import numpy as np
import torch

from oracle import merge as om

GOLDEN = Path(__file__).resolve().parent / "golden"
TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


@lru_cache(maxsize=1)
def _load():
    cases = json.loads((GOLDEN / "merge_reference.json").read_text())
    with np.load(GOLDEN / "merge_reference.npz") as z:
        arrays = {k: z[k] for k in z.files}
    return cases, arrays


def cases() -> list[dict]:
    return _load()[0]


def arr(case: dict, name: str) -> np.ndarray | None:
    return _load()[1].get(f"{case['id']}.{name}")


def case_label(case: dict) -> str:
    keys = [k for k in ("launcher", "rows", "cols", "rank", "e4m3", "elem", "storage", "axis", "quant_type", "nested",
                        "block",
                        "scaling_mode", "swizzled", "two_level", "asymmetric", "reduce_range", "dtype", "scale_dtype",
                        "strength") if k in case]
    sr = "sr" if case["seed"] is not None else "rtn"
    return "-".join(str(case[k]) for k in keys) + "-" + sr


def _float_values(a: np.ndarray, dt: str) -> np.ndarray:
    """fp32 values of a stored bf16/f16 (int16 bits) or f32 array."""
    if dt == "f32":
        return a.astype(np.float32)
    return torch.from_numpy(a.copy()).view(TORCH_DT[dt]).float().numpy()


def factors(case: dict) -> tuple[np.ndarray, np.ndarray]:
    return _float_values(arr(case, "b"), case["dtype"]), _float_values(arr(case, "a"), case["dtype"])


def expected(case: dict) -> dict:
    """The reference's outputs, as comparable numpy arrays."""
    out = {"q": arr(case, "out_qdata").reshape(-1).view(np.uint8)}
    sc = arr(case, "out_scale")
    if case["launcher"] == "int8":
        out["scale"] = _float_values(sc, case["scale_dtype"]).reshape(-1)
        out["zp"] = arr(case, "out_zero_point").reshape(-1)
    elif case["launcher"] in ("float8", "static_float8", "bnb8"):
        out["scale"] = sc.astype(np.float32).reshape(-1)
    elif case["launcher"] == "quanto":
        out["scale"] = _float_values(sc, case["dtype"]).reshape(-1)
    elif case["launcher"] == "bnb4":
        out["scale"] = sc.reshape(-1).view(np.uint8) if case["nested"] else sc.astype(np.float32).reshape(-1)
        if case["nested"]:
            out["nested_absmax"] = arr(case, "out_nested_absmax").astype(np.float32).reshape(-1)
            out["offset"] = arr(case, "out_offset").astype(np.float32).reshape(-1)
    else:
        out["scale"] = sc.reshape(-1).view(np.uint8)
    g = arr(case, "out_per_tensor_scale")
    if g is not None:
        out["global"] = g.astype(np.float32).reshape(-1)
    return out


def oracle(case: dict) -> dict:
    """The oracle on the case's inputs, in the layout of ``expected``."""
    b, a = factors(case)
    q = arr(case, "qdata")
    kw = dict(seed=case["seed"], compute=case["dtype"])
    s = case["strength"]
    L = case["launcher"]
    if L == "float8":
        nq, ns = om.merge_float8(q.view(np.uint8), arr(case, "scale"), tuple(case["block"]), b, a, s,
                                 e4m3=case["e4m3"], **kw)
        return {"q": nq.reshape(-1).view(np.uint8), "scale": np.asarray(ns, np.float32).reshape(-1)}
    if L == "static_float8":
        nq, ns = om.merge_static_float8(q.view(np.uint8), arr(case, "scale"), b, a, s, e4m3=case["e4m3"], **kw)
        return {"q": nq.reshape(-1).view(np.uint8), "scale": np.asarray(ns, np.float32).reshape(-1)}
    if L == "bnb4":
        nested = case["nested"]
        res = om.merge_bnb4(q, arr(case, "scale"), arr(case, "code"), b, a, s, quant_type=case["quant_type"],
                            nested_absmax=arr(case, "nested_absmax") if nested else None,
                            nested_code=arr(case, "nested_code") if nested else None,
                            offset=float(arr(case, "offset")) if nested else None, **kw)
        out = {"q": np.asarray(res[0], np.uint8).reshape(-1)}
        if nested:
            out["scale"] = np.asarray(res[1], np.uint8).reshape(-1)
            out["nested_absmax"] = np.asarray(res[2], np.float32).reshape(-1)
            out["offset"] = np.asarray([res[3]], np.float32)
        else:
            out["scale"] = np.asarray(res[1], np.float32).reshape(-1)
        return out
    if L == "bnb8":
        nq, ns = om.merge_bnb8(q, arr(case, "scale"), b, a, s, seed=case["seed"])
        return {"q": nq.reshape(-1).view(np.uint8), "scale": np.asarray(ns, np.float32).reshape(-1)}
    if L == "quanto":
        kind = {None: "tensor", 0: "row", -1: "column"}[case["axis"]]
        qa = q if case["storage"] == "int8" else q.view(np.uint8)
        nq, ns = om.merge_quanto(qa, _float_values(arr(case, "scale"), case["dtype"]), kind, b, a, s,
                                 storage=case["storage"], **kw)
        return {"q": nq.reshape(-1).view(np.uint8), "scale": np.asarray(ns, np.float32).reshape(-1)}
    if L == "int8":
        sdt = case["scale_dtype"]
        nq, ns, nz = om.merge_int8(q, _float_values(arr(case, "scale"), sdt), arr(case, "zero_point"),
                                   tuple(case["block"]), b, a, s, asymmetric=case["asymmetric"],
                                   reduce_range=case["reduce_range"], qparam=sdt, **kw)
        return {"q": nq.reshape(-1).view(np.uint8), "scale": np.asarray(ns, np.float32).reshape(-1),
                "zp": np.asarray(nz, np.int8).reshape(-1)}
    if L == "nvfp4":
        pts = arr(case, "per_tensor_scale")
        nq, ns, g = om.merge_nvfp4(q, arr(case, "scale"), None if pts is None else float(pts), b, a, s,
                                   swizzled=case["swizzled"], **kw)
        out = {"q": nq.reshape(-1), "scale": np.asarray(ns, np.uint8).reshape(-1)}
        if g is not None:
            out["global"] = np.asarray([g], np.float32)
        return out
    nq, ns = om.merge_mx(q.view(np.uint8), arr(case, "scale"), case["elem"], b, a, s,
                         scaling_mode=case["scaling_mode"], swizzled=case["swizzled"], **kw)
    return {"q": nq.reshape(-1), "scale": np.asarray(ns, np.uint8).reshape(-1)}


def native(case: dict, device) -> dict:
    """The sm_100a path (``piper_offload_b200.kernels``) on the case's inputs."""
    from piper_offload_b200 import kernels as K

    def dev(a: np.ndarray, dtype=None) -> torch.Tensor:
        t = torch.from_numpy(a.copy())
        if dtype is not None:
            t = t.view(dtype)
        return t.to(device)

    fdt = TORCH_DT[case["dtype"]]
    b = dev(arr(case, "b"), fdt)
    a = dev(arr(case, "a"), fdt)
    s = case["strength"]
    kw = dict(rounding_seed=case["seed"])
    L = case["launcher"]
    if L == "float8":
        q = dev(arr(case, "qdata"), torch.float8_e4m3fn if case["e4m3"] else torch.float8_e5m2)
        sc = dev(arr(case, "scale"))
        K.merge_float8_lora(q, sc, tuple(case["block"]), b, a, s, **kw)
        return {"q": q.view(torch.uint8).cpu().numpy().reshape(-1), "scale": sc.cpu().numpy().reshape(-1)}
    if L == "static_float8":
        q = dev(arr(case, "qdata"), torch.float8_e4m3fn if case["e4m3"] else torch.float8_e5m2)
        sc = dev(arr(case, "scale"))
        K.merge_static_float8_lora(q, sc, b, a, s, **kw)
        return {"q": q.view(torch.uint8).cpu().numpy().reshape(-1), "scale": sc.cpu().numpy().reshape(-1)}
    if L == "bnb4":
        nested = case["nested"]
        q = dev(arr(case, "qdata"))
        sc = dev(arr(case, "scale"))
        nabs = dev(arr(case, "nested_absmax")) if nested else None
        off = dev(arr(case, "offset")).reshape(()) if nested else None
        K.merge_bnb4_lora(q, sc, dev(arr(case, "code")), nabs, dev(arr(case, "nested_code")) if nested else None, off,
                          (case["rows"], case["cols"]), 64, case["quant_type"], b, a, s, **kw)
        out = {"q": q.cpu().numpy().reshape(-1)}
        out["scale"] = sc.cpu().numpy().reshape(-1).view(np.uint8) if nested else sc.cpu().numpy().reshape(-1)
        if nested:
            out["nested_absmax"] = nabs.cpu().numpy().reshape(-1)
            out["offset"] = off.cpu().numpy().reshape(-1)
        return out
    if L == "bnb8":
        q = dev(arr(case, "qdata"))
        sc = dev(arr(case, "scale"))
        K.merge_bnb8_lora(q, sc, b, a, s, **kw)
        return {"q": q.cpu().numpy().reshape(-1).view(np.uint8), "scale": sc.cpu().numpy().reshape(-1)}
    if L == "quanto":
        if case["storage"] == "int8":
            q = dev(arr(case, "qdata"))
            fn = K.merge_quanto_qint8_lora
        else:
            q = dev(arr(case, "qdata"), torch.float8_e4m3fn if case["storage"] == "e4m3" else torch.float8_e5m2)
            fn = K.merge_quanto_qfloat8_lora
        sc = dev(arr(case, "scale"), fdt)
        fn(q, sc, case["axis"], b, a, s, **kw)
        return {"q": q.view(torch.uint8).cpu().numpy().reshape(-1), "scale": sc.float().cpu().numpy().reshape(-1)}
    if L == "int8":
        q = dev(arr(case, "qdata"))
        sdt = TORCH_DT[case["scale_dtype"]]
        sc = dev(arr(case, "scale"), None if case["scale_dtype"] == "f32" else sdt)
        zp_in = arr(case, "zero_point")
        zp = None if zp_in is None else dev(zp_in)
        _, _, zo = K.merge_int8_lora(q, sc, zp, tuple(case["block"]), b, a, s, asymmetric=case["asymmetric"],
                                     reduce_range=case["reduce_range"], **kw)
        return {"q": q.cpu().numpy().reshape(-1).view(np.uint8), "scale": sc.float().cpu().numpy().reshape(-1),
                "zp": zo.cpu().numpy().reshape(-1)}
    if L == "nvfp4":
        q = dev(arr(case, "qdata"))
        sc = dev(arr(case, "scale"), torch.float8_e4m3fn)
        pts_in = arr(case, "per_tensor_scale")
        pts = None if pts_in is None else dev(pts_in)
        _, _, g = K.merge_nvfp4_lora(q, sc, pts, 16, case["swizzled"], b, a, s, **kw)
        out = {"q": q.cpu().numpy().reshape(-1), "scale": sc.view(torch.uint8).cpu().numpy().reshape(-1)}
        if g is not None:
            out["global"] = g.float().cpu().numpy().reshape(-1)
        return out
    elem = {"e4m3": torch.float8_e4m3fn, "e5m2": torch.float8_e5m2, "e2m1": torch.float4_e2m1fn_x2}[case["elem"]]
    q = dev(arr(case, "qdata"), None if case["elem"] == "e2m1" else elem)
    sc = dev(arr(case, "scale"), torch.float8_e8m0fnu)
    K.merge_mx_lora_(q, sc, elem, 32, fdt, b, a, s, scaling_mode=case["scaling_mode"],
                     swizzled=case["swizzled"], **kw)
    return {"q": q.view(torch.uint8).cpu().numpy().reshape(-1), "scale": sc.view(torch.uint8).cpu().numpy().reshape(-1)}


def mismatches(got: dict, want: dict) -> dict:
    """Per output field, the indices whose bits differ."""
    out = {}
    for k, w in want.items():
        g = np.asarray(got[k])
        w = np.asarray(w)
        if g.dtype != w.dtype:
            g = g.astype(w.dtype)
        if w.dtype == np.float32:
            g, w = g.view(np.uint32), w.view(np.uint32)
        out[k] = np.nonzero(g.reshape(-1) != w.reshape(-1))[0]
    return out

"""Record the reference's own Triton merge kernels as golden fixtures (run in the build container).

Usage: ``python tests/golden/make_merge_golden.py /path/to/piper-offload``

The raw-buffer launchers of Piper Offload 0.2.5 --
``merge_float8_lora`` (``_triton_float8_lora.py:486``), ``merge_int8_lora``
(``_triton_int8_lora.py:267``), ``merge_nvfp4_lora`` (``_triton_nvfp4_lora.py:515``),
``merge_mx_lora_`` (``_triton_mx_lora.py:333``), ``merge_static_float8_lora``
(``_triton_static_float8_lora.py:174``), ``merge_bnb8_lora``
(``_triton_bnb8_lora.py:145``) and ``merge_quanto_qint8_lora`` /
``merge_quanto_qfloat8_lora`` (``_triton_quanto_lora.py:317, 345``) -- run
unmodified under the
Triton CPU interpreter (``TRITON_INTERPRET=1``, triton 3.6). Their inputs and
outputs go to ``merge_reference.npz`` with one manifest entry per case in
``merge_reference.json``.

The interpreter emulates a few device operations loosely. This script replaces
exactly those, so that every operation the kernels use computes what the GPU
instruction computes:

* float narrowing (``x.to(tl.bfloat16)``, ``.to(tl.float8e4nv)`` ...): the
  interpreter truncates on ``fp_trunc`` and rounds ties and mantissa carries
  incorrectly; here every conversion is one round-to-nearest-even step through
  torch's exact casts, as ``cvt.rn`` does;
* ``tl.dot`` on bf16 operands: the interpreter multiplies the raw uint16 bit
  patterns; here operands are decoded, summed in float64 and rounded once to
  fp32 (the fixtures use factors whose dot products are exact in any order);
* binary arithmetic on two bf16 tensors (``base * scale`` in the INT8 kernel):
  computed on decoded values and rounded once to bf16, as ``mul.rn.bf16`` does;
* ``libdevice.llrint`` / ``libdevice.rint``: absent from the interpreter;
  ``numpy.rint`` (round half to even, the ``cvt.rni`` default mode);
* Quanto's torch-side scale recompute (``_absmax_scale``) runs on CPU tensors
  here, where torch divides ``amax / qmax``; on CUDA tensors torch multiplies
  by the fp32 reciprocal of the host scalar, which this script applies (a GPU
  test checks that torch behaviour on the device).

Unary and reduction operations on bf16/fp8 tensors, which none of these kernels
use, raise instead of running on bit patterns. The launchers' CUDA-device check
(``qdata.device.type != "cuda"``) is lifted so that CPU tensors reach the
kernels; nothing else in the reference is changed. Divisions run as IEEE
``numpy.divide``, which the oracle reproduces without its GPU-division hook.
"""

from __future__ import annotations

import __future__
import inspect
import json
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

SEED = 0x9C3EA68DBAC91AAD  # derive_seed("layer.0.weight", 0)


# ---------------------------------------------------------------- interpreter
def patch_interpreter() -> None:
    import triton.language as tl
    from triton.runtime import interpreter as ti

    torch_of = {tl.float32: torch.float32, tl.float16: torch.float16, tl.bfloat16: torch.bfloat16,
                tl.float8e4nv: torch.float8_e4m3fn, tl.float8e5: torch.float8_e5m2, tl.float64: torch.float64}
    bits_of = {8: torch.uint8, 16: torch.int16, 32: torch.int32, 64: torch.int64}
    narrow = (tl.bfloat16, tl.float8e4nv, tl.float8e5)

    def convert_float(data, src, dst, rounding_mode=None):  # noqa: ARG001
        t = torch.from_numpy(np.ascontiguousarray(data).copy())
        if t.dtype != torch_of[src]:
            t = t.view(torch_of[src])
        out = t.to(torch_of[dst])
        if dst in (tl.float32, tl.float16, tl.float64):
            return out.numpy()
        return out.view(bits_of[dst.primitive_bitwidth]).numpy().view(ti._get_np_dtype(dst))

    def to_f64(h):
        if h.dtype.scalar in narrow:
            return convert_float(h.data, h.dtype.scalar, tl.float32).astype(np.float64)
        return h.data.astype(np.float64)

    def f64_to_bf16_bits(x):
        x = np.asarray(x, np.float64)
        fin = np.isfinite(x) & (x != 0)
        ax = np.abs(x[fin])
        if ax.size and (ax.min() < 2.0**-126 or ax.max() >= 2.0**127):
            raise NotImplementedError("bf16 result outside the normal range")
        u = x.view(np.uint64).copy()
        lsb = (u >> np.uint64(45)) & np.uint64(1)
        r = (u + np.uint64((1 << 44) - 1) + lsb) & ~np.uint64((1 << 45) - 1)
        u = np.where(fin, r, u)
        f32 = u.view(np.float64).astype(np.float32)  # exact: at most 8 significant bits
        return (f32.view(np.uint32) >> np.uint32(16)).astype(np.uint16)

    ti._convert_float = convert_float
    orig_cast = ti.InterpreterBuilder.cast_impl

    def cast_impl(self, src, dst_type):
        s, d = src.dtype.scalar, dst_type.scalar
        if s in narrow or d in narrow:
            if not (s.is_floating() and d.is_floating()):
                raise NotImplementedError((s, d))
            return ti.TensorHandle(convert_float(src.data, s, d), d)
        return orig_cast(self, src, dst_type)

    ti.InterpreterBuilder.cast_impl = cast_impl
    ti.InterpreterBuilder.create_fp_ext = lambda self, src, dst_type: self.cast_impl(src, dst_type)
    ti.InterpreterBuilder.create_fp_trunc = lambda self, src, dst_type: self.cast_impl(src, dst_type)

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):  # noqa: ARG001
        prod = (to_f64(a) @ to_f64(b)).astype(np.float32)
        return ti.TensorHandle((prod + d.data).astype(np.float32), d.dtype.scalar)

    ti.InterpreterBuilder.create_dot = create_dot

    compare = {np.less, np.greater, np.less_equal, np.greater_equal, np.equal, np.not_equal}
    arith = {np.add, np.subtract, np.multiply, np.divide, np.maximum, np.minimum}
    orig_binary = ti.InterpreterBuilder.binary_op

    def binary_op(self, lhs, rhs, fn):
        s = lhs.dtype.scalar
        if s in (tl.float8e4nv, tl.float8e5):
            raise NotImplementedError(f"arithmetic on {s}")
        if s == tl.bfloat16:
            if rhs.dtype.scalar != tl.bfloat16:
                raise NotImplementedError("mixed bf16 operands")
            x, y = to_f64(lhs), to_f64(rhs)
            if fn in compare:
                return ti.TensorHandle(fn(x, y), tl.int1)
            if fn not in arith:
                raise NotImplementedError(fn)
            return ti.TensorHandle(f64_to_bf16_bits(fn(x, y)), s)
        return orig_binary(self, lhs, rhs, fn)

    ti.InterpreterBuilder.binary_op = binary_op
    orig_unary = ti.InterpreterBuilder.unary_op

    def unary_op(self, arg, fn):
        if arg.dtype.scalar in narrow:
            raise NotImplementedError(f"unary op on {arg.dtype.scalar}")
        return orig_unary(self, arg, fn)

    ti.InterpreterBuilder.unary_op = unary_op
    orig_min_max = ti.ReduceOps.min_max

    def min_max(self, input, val_reduce_op, idx_reduce_op=None):  # noqa: A002
        if input.dtype in narrow:
            raise NotImplementedError(f"reduction on {input.dtype}")
        return orig_min_max(self, input, val_reduce_op, idx_reduce_op)

    ti.ReduceOps.min_max = min_max


class _Libdevice:
    """``libdevice.llrint`` (to int64) and ``libdevice.rint``: round half to even."""

    @staticmethod
    def llrint(x):
        import triton.language as tl
        from triton.runtime import interpreter as ti

        data = np.rint(x.handle.data).astype(np.int64)
        ty = x.type.with_element_ty(tl.int64) if x.type.is_block() else tl.int64
        return tl.core.tensor(ti.TensorHandle(data, tl.int64), ty)

    @staticmethod
    def rint(x):
        import triton.language as tl
        from triton.runtime import interpreter as ti

        return tl.core.tensor(ti.TensorHandle(np.rint(x.handle.data), x.dtype), x.type)


def _cuda_absmax_scale(quanto):
    """Quanto's ``_absmax_scale`` (``_triton_quanto_lora.py:202-217``) as it runs on
    CUDA tensors: there ``amax / qmax`` (a tensor over a host scalar) is computed
    by torch as ``amax * fp32(1 / qmax)``; on the CPU tensors of this script torch
    would divide. Every other step is the reference's."""

    def absmax_scale(dense, scale, scale_axis, qmax):
        if scale_axis == quanto._AXIS_ROW:
            amax = dense.abs().amax(dim=1, keepdim=True)
        elif scale_axis == quanto._AXIS_COLUMN:
            amax = dense.abs().amax(dim=0, keepdim=True)
        else:
            amax = dense.abs().amax()
        inv = torch.tensor(float(np.float32(1.0) / np.float32(qmax)), dtype=torch.float32)
        output = (amax.float() * inv).to(dense.dtype).to(dtype=scale.dtype).reshape(scale.shape)
        eps = torch.finfo(torch.float32).eps
        return torch.where(output == 0, torch.full_like(output, eps), output)

    return absmax_scale


def lift_device_check(mod, fname: str, tensor: str = "qdata") -> None:
    src = inspect.getsource(getattr(mod, fname))
    needle = f'{tensor}.device.type != "cuda"'
    if src.count(needle) != 1:
        raise RuntimeError(f"{mod.__name__}.{fname}: device check not found")
    code = compile(src.replace(needle, "False"), mod.__file__, "exec",
                   flags=__future__.annotations.compiler_flag, dont_inherit=True)
    exec(code, mod.__dict__)  # noqa: S102


def load_reference(src: Path):
    import make_golden

    make_golden.install_reference(src)
    patch_interpreter()
    from piper_offload import _triton_float8_lora as f8
    from piper_offload import _triton_int8_lora as i8
    from piper_offload import _triton_mx_lora as mx
    from piper_offload import _triton_bnb4_lora as bnb4
    from piper_offload import _triton_bnb8_lora as bnb8
    from piper_offload import _triton_nvfp4_lora as n4
    from piper_offload import _triton_quanto_lora as qo
    from piper_offload import _triton_static_float8_lora as sf8

    for mod, fname in ((f8, "_validate_inputs"), (i8, "merge_int8_lora"), (n4, "_validate_inputs"),
                       (mx, "merge_mx_lora_"), (sf8, "merge_static_float8_lora"), (qo, "_merge_quanto_qbytes_lora")):
        lift_device_check(mod, fname)
    lift_device_check(bnb8, "merge_bnb8_lora", tensor="cb")
    lift_device_check(bnb4, "merge_bnb4_lora", tensor="packed")
    for mod in (i8, bnb8, qo):
        mod.libdevice = _Libdevice
    qo._absmax_scale = _cuda_absmax_scale(qo)
    return {"float8": f8, "int8": i8, "nvfp4": n4, "mx": mx, "static_float8": sf8, "bnb8": bnb8, "quanto": qo,
            "bnb4": bnb4}


# ---------------------------------------------------------------------- inputs
DTYPES = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def exact_factors(g, rows, cols, rank, dt, exp=8, zero_b=False):
    """Small-integer multiples of 2**-exp: every dot product and its scaling by
    the fixtures' strengths is exact in fp32, in any summation order."""
    b = torch.randint(-15, 16, (rows, rank), generator=g).float() * 2.0**-exp
    a = torch.randint(-15, 16, (rank, cols), generator=g).float() * 2.0**-exp
    if zero_b:
        b.zero_()
    return b.to(dt), a.to(dt)


class Writer:
    def __init__(self):
        self.arrays: dict[str, np.ndarray] = {}
        self.cases: list[dict] = []

    def add(self, meta: dict, **arrays) -> None:
        cid = f"c{len(self.cases):03d}"
        meta = {"id": cid, **meta}
        for k, v in arrays.items():
            if v is None:
                continue
            t = v.detach().contiguous().cpu()
            if t.dtype in (torch.bfloat16, torch.float16):
                t = t.view(torch.int16)
            elif t.dtype in (torch.float8_e4m3fn, torch.float8_e5m2, torch.float8_e8m0fnu):
                t = t.view(torch.uint8)
            self.arrays[f"{cid}.{k}"] = t.numpy().copy()
        self.cases.append(meta)

    def save(self) -> None:
        np.savez_compressed(HERE / "merge_reference.npz", **self.arrays)
        (HERE / "merge_reference.json").write_text(json.dumps(self.cases, indent=1))


def gen_float8(f8, w: Writer, g) -> None:
    def one(rows, cols, rank, e4m3, layout, seed, dt, strength=1.0, zero_b=False, group=10):
        fdt = torch.float8_e4m3fn if e4m3 else torch.float8_e5m2
        limit = torch.finfo(fdt).max
        base = torch.randn(rows, cols, generator=g) * 0.02
        if layout == "row":
            block = (1, cols)
            s = base.abs().amax(1, keepdim=True) / limit
            sx = s
        elif layout == "tensor":
            block = (rows, cols)
            s = (base.abs().amax() / limit).reshape(1, 1)
            sx = s
        else:
            block = (1, group)
            s = base.reshape(rows, cols // group, group).abs().amax(2) / limit
            sx = s.repeat_interleave(group, 1)
        s = s.float()
        q = (base / sx).clamp(-limit, limit).to(fdt)
        if zero_b:
            q.view(torch.uint8)[:, ::5] = 0x80  # negative-zero codes
        b, a = exact_factors(g, rows, cols, rank, DTYPES[dt], zero_b=zero_b)
        oq, os_ = f8.merge_float8_lora(q.clone(), s.clone(), block, b, a, strength, rounding_seed=seed)
        w.add({"launcher": "float8", "rows": rows, "cols": cols, "rank": rank, "e4m3": e4m3,
               "block": list(block), "seed": seed, "dtype": dt, "strength": strength},
              qdata=q, scale=s, b=b, a=a, out_qdata=oq, out_scale=os_)

    for e4m3 in (True, False):
        for layout in ("row", "tensor", "group"):
            for seed in (None, SEED):
                one(70, 130, 7, e4m3, layout, seed, "bf16")
            one(70, 130, 7, e4m3, layout, SEED if e4m3 else None, "f16")
    one(16, 64, 7, True, "row", SEED, "bf16")
    one(70, 130, 7, True, "row", SEED, "bf16", strength=-0.75)
    one(70, 130, 7, True, "row", None, "bf16", zero_b=True)
    one(70, 130, 7, True, "tensor", SEED, "bf16", zero_b=True)
    one(8, 512, 19, True, "group", SEED, "bf16", group=256)


def gen_int8(i8, w: Writer, g) -> None:
    def one(rows, cols, rank, layout, asym, rr, seed, dt, sdt="bf16", strength=1.0, group=23, zero_b=False):
        qmin, qmax = (-64, 63) if rr else (-128, 127)
        q = torch.randint(qmin, qmax + 1, (rows, cols), generator=g, dtype=torch.int8)
        if layout == "row":
            block, sshape = (1, cols), (rows, 1)
        elif layout == "tensor":
            block, sshape = (rows, cols), (1, 1)
        else:
            block, sshape = (1, group), (rows, cols // group)
        scale = (torch.rand(sshape, generator=g) * 2e-4 + 1e-4).to(DTYPES[sdt])
        zp = torch.randint(-10, 10, sshape, generator=g, dtype=torch.int8) if asym else None
        b, a = exact_factors(g, rows, cols, rank, DTYPES[dt], exp=9, zero_b=zero_b)
        oq, os_, oz = i8.merge_int8_lora(q.clone(), scale.clone(), None if zp is None else zp.clone(), block, b, a,
                                         strength, asymmetric=asym, reduce_range=rr, rounding_seed=seed)
        w.add({"launcher": "int8", "rows": rows, "cols": cols, "rank": rank, "block": list(block),
               "asymmetric": asym, "reduce_range": rr, "seed": seed, "dtype": dt, "scale_dtype": sdt,
               "strength": strength},
              qdata=q, scale=scale, zero_point=zp, b=b, a=a, out_qdata=oq, out_scale=os_, out_zero_point=oz)

    for layout in ("row", "tensor", "group"):
        for asym in (False, True):
            for rr in (False, True):
                for seed in (None, SEED):
                    one(35, 69, 7, layout, asym, rr, seed, "bf16")
            one(35, 69, 7, layout, asym, not asym, SEED if asym else None, "f16")
    for layout in ("row", "tensor"):
        for asym in (False, True):
            one(35, 69, 19, layout, asym, False, SEED, "bf16")
    one(35, 69, 7, "row", False, False, SEED, "bf16", sdt="f16")
    one(35, 69, 7, "row", True, False, None, "bf16", sdt="f32")
    one(35, 69, 7, "row", True, False, SEED, "bf16", strength=-1.25)
    one(35, 69, 7, "row", False, False, None, "bf16", zero_b=True)


def gen_nvfp4(n4, w: Writer, g) -> None:
    def one(rows, cols, rank, swizzled, two_level, seed, strength=1.0, zero_b=False):
        q = torch.randint(0, 256, (rows, cols // 2), generator=g, dtype=torch.uint8)
        if zero_b:
            q[:, ::3] = 0x88  # negative-zero codes in both nibbles
        sshape = ((rows + 127) // 128 * 32, (cols + 63) // 64 * 16) if swizzled else (rows, cols // 16)
        if two_level:
            scale = (torch.rand(sshape, generator=g) * 3 + 0.5).to(torch.float8_e4m3fn)
            pts = torch.tensor(0.003, dtype=torch.float32)
        else:
            scale = (torch.rand(sshape, generator=g) * 0.01 + 0.002).to(torch.float8_e4m3fn)
            pts = None
        b, a = exact_factors(g, rows, cols, rank, torch.bfloat16, zero_b=zero_b)
        oq, os_, og = n4.merge_nvfp4_lora(q.clone(), scale.clone(), None if pts is None else pts.clone(), 16,
                                          swizzled, b, a, strength, rounding_seed=seed)
        w.add({"launcher": "nvfp4", "rows": rows, "cols": cols, "rank": rank, "swizzled": swizzled,
               "two_level": two_level, "seed": seed, "dtype": "bf16", "strength": strength},
              qdata=q, scale=scale, per_tensor_scale=pts, b=b, a=a, out_qdata=oq, out_scale=os_,
              out_per_tensor_scale=og)

    for rank in (13, 40):
        for swizzled in (False, True):
            for two_level in (False, True):
                for seed in (None, SEED):
                    one(19, 80, rank, swizzled, two_level, seed)
    one(19, 80, 13, False, False, None, zero_b=True)
    one(19, 80, 13, True, True, SEED, zero_b=True)
    one(19, 80, 13, False, True, SEED, strength=-0.5)


def gen_mx(mx, w: Writer, g) -> None:
    elem_dtypes = {"e4m3": torch.float8_e4m3fn, "e5m2": torch.float8_e5m2, "e2m1": torch.float4_e2m1fn_x2}

    def one(rows, cols, rank, elem, mode, swizzled, seed, strength=1.0, zero_b=False):
        if elem == "e2m1":
            q = torch.randint(0, 256, (rows, cols // 2), generator=g, dtype=torch.uint8)
            if zero_b:
                q[:, ::3] = 0x88
        else:
            q = (torch.randn(rows, cols, generator=g) * 100).clamp(-400, 400).to(elem_dtypes[elem])
        sshape = ((rows + 127) // 128 * 32, (cols + 127) // 128 * 16) if swizzled else (rows, cols // 32)
        scale = torch.randint(110, 122, sshape, generator=g, dtype=torch.uint8).view(torch.float8_e8m0fnu)
        b, a = exact_factors(g, rows, cols, rank, torch.bfloat16, exp=9, zero_b=zero_b)
        oq, os_ = q.clone(), scale.clone()
        mx.merge_mx_lora_(oq, os_, elem_dtypes[elem], 32, torch.bfloat16, b, a, strength, scaling_mode=mode,
                          swizzled=swizzled, rounding_seed=seed)
        w.add({"launcher": "mx", "rows": rows, "cols": cols, "rank": rank, "elem": elem, "scaling_mode": mode,
               "swizzled": swizzled, "seed": seed, "dtype": "bf16", "strength": strength},
              qdata=q, scale=scale, b=b, a=a, out_qdata=oq, out_scale=os_)

    for elem in ("e4m3", "e5m2", "e2m1"):
        for mode in (0, 1, 2, 3):
            for swizzled in (False, True):
                for seed in (None, SEED):
                    one(19, 96, 7, elem, mode, swizzled, seed)
        one(19, 96, 40, elem, 0, False, SEED)
    one(19, 96, 7, "e2m1", 0, False, None, strength=-1.0)
    one(19, 96, 7, "e2m1", 1, True, SEED, zero_b=True)


def gen_static_float8(sf8, w: Writer, g) -> None:
    def one(rows, cols, rank, e4m3, seed, dt, strength=1.0, zero_b=False):
        fdt = torch.float8_e4m3fn if e4m3 else torch.float8_e5m2
        limit = torch.finfo(fdt).max
        base = torch.randn(rows, cols, generator=g) * 0.02
        s = (base.abs().amax() / limit).reshape(()).float()
        q = (base / s).clamp(-limit, limit).to(fdt)
        b, a = exact_factors(g, rows, cols, rank, DTYPES[dt], zero_b=zero_b)
        oq, os_ = sf8.merge_static_float8_lora(q.clone(), s.clone(), b, a, strength, rounding_seed=seed)
        w.add({"launcher": "static_float8", "rows": rows, "cols": cols, "rank": rank, "e4m3": e4m3, "seed": seed,
               "dtype": dt, "strength": strength},
              qdata=q, scale=s, b=b, a=a, out_qdata=oq, out_scale=os_)

    for e4m3 in (True, False):
        for seed in (None, SEED):
            one(70, 130, 7, e4m3, seed, "bf16")
    one(70, 130, 7, True, SEED, "f16", strength=-0.75)
    one(70, 130, 7, True, None, "bf16", zero_b=True)


def gen_bnb8(bnb8, w: Writer, g) -> None:
    def one(rows, cols, rank, seed, strength=1.0, zero_b=False, zero_row=False):
        cb = torch.randint(-127, 128, (rows, cols), generator=g, dtype=torch.int8)
        scb = (torch.rand(rows, generator=g) * 0.05 + 0.01).float()
        if zero_row:
            cb[3] = 0
            scb[3] = 0.0
        b, a = exact_factors(g, rows, cols, rank, torch.float16, exp=9, zero_b=zero_b)
        if zero_row:
            b[3] = 0
        ocb, oscb = bnb8.merge_bnb8_lora(cb.clone(), scb.clone(), b, a, strength, rounding_seed=seed)
        w.add({"launcher": "bnb8", "rows": rows, "cols": cols, "rank": rank, "seed": seed, "dtype": "f16",
               "strength": strength},
              qdata=cb, scale=scb, b=b, a=a, out_qdata=ocb, out_scale=oscb)

    for seed in (None, SEED):
        one(35, 69, 7, seed)
        one(35, 69, 19, seed, zero_row=True)
    one(16, 64, 7, SEED, strength=-1.25)
    one(35, 69, 7, None, zero_b=True)


def gen_quanto(qo, w: Writer, g) -> None:
    def one(rows, cols, rank, storage, axis, seed, dt, strength=1.0, zero_scale=False):
        if storage == "int8":
            q = torch.randint(-128, 128, (rows, cols), generator=g, dtype=torch.int8)
            qmax = 127.0
        else:
            fdt = torch.float8_e4m3fn if storage == "e4m3" else torch.float8_e5m2
            qmax = torch.finfo(fdt).max
            q = (torch.randn(rows, cols, generator=g) * qmax / 4).clamp(-qmax, qmax).to(fdt)
        sshape = {None: (), 0: (rows, 1), -1: (1, cols)}[axis]
        scale = (torch.rand(sshape, generator=g) * 2e-4 + 5e-5).to(DTYPES[dt])
        if zero_scale and axis == 0:
            scale[2] = 0.0
        b, a = exact_factors(g, rows, cols, rank, DTYPES[dt], exp=9)
        fn = qo.merge_quanto_qint8_lora if storage == "int8" else qo.merge_quanto_qfloat8_lora
        oq, os_ = fn(q.clone(), scale.clone(), axis, b, a, strength, rounding_seed=seed)
        w.add({"launcher": "quanto", "rows": rows, "cols": cols, "rank": rank, "storage": storage, "axis": axis,
               "seed": seed, "dtype": dt, "strength": strength},
              qdata=q, scale=scale, b=b, a=a, out_qdata=oq, out_scale=os_)

    for storage in ("int8", "e4m3", "e5m2"):
        for axis in (None, 0, -1):
            for seed in (None, SEED):
                one(35, 69, 7, storage, axis, seed, "bf16")
        one(35, 69, 7, storage, 0, SEED, "f16", strength=-0.75, zero_scale=True)


def bnb4_tables(g):
    """Synthetic sorted code tables with few significant bits, so that the
    nested scale ``code * absmax + offset`` is exact with or without a fused
    multiply-add."""
    inner = torch.randperm(2047, generator=g)[:13].sort().values.float() / 1024.0 - 1.0 + 1.0 / 1024.0
    code = torch.cat([torch.tensor([-1.0, 0.0, 1.0]), inner]).unique().sort().values
    while code.numel() < 16:
        code = torch.cat([code, torch.tensor([float(code.numel()) / 4096.0])]).unique().sort().values
    nested = torch.round(torch.linspace(-1.0, 1.0, 256) * 1024.0) / 1024.0
    return code[:16].float().contiguous(), nested.float().contiguous()


def gen_bnb4(bnb4, w: Writer, g) -> None:
    code, nested_code = bnb4_tables(g)

    def one(rows, cols, rank, quant_type, seed, dt, nested=False, strength=1.0, zero_b=False):
        nblk = rows * cols // 64
        packed = torch.randint(0, 256, (rows * cols // 2, 1), generator=g, dtype=torch.uint8)
        if nested:
            absmax = torch.randint(0, 256, (nblk,), generator=g, dtype=torch.uint8)
            nabs = (torch.randint(64, 4096, ((nblk + 255) // 256,), generator=g).float() * 2.0**-14)
            offset = torch.tensor(float(torch.randint(1, 4096, (1,), generator=g)) * 2.0**-16)
        else:
            absmax = torch.rand(nblk, generator=g) * 0.05 + 0.005
            nabs = offset = None
        b, a = exact_factors(g, rows, cols, rank, DTYPES[dt], exp=9, zero_b=zero_b)
        out = bnb4.merge_bnb4_lora(packed.clone(), absmax.clone(), code, nabs, nested_code if nested else None,
                                   offset, (rows, cols), 64, quant_type, b, a, strength, rounding_seed=seed)
        w.add({"launcher": "bnb4", "rows": rows, "cols": cols, "rank": rank, "quant_type": quant_type,
               "nested": nested, "seed": seed, "dtype": dt, "strength": strength},
              qdata=packed, scale=absmax, code=code, nested_absmax=nabs,
              nested_code=nested_code if nested else None, offset=offset, b=b, a=a,
              out_qdata=out[0], out_scale=out[1], out_nested_absmax=out[2], out_offset=out[3])

    for quant_type in ("nf4", "fp4"):
        for seed in (None, SEED):
            one(19, 128, 13, quant_type, seed, "bf16")
            one(24, 256, 40, quant_type, seed, "f16")
        one(40, 512, 7, quant_type, None, "bf16", nested=True)
        one(40, 512, 7, quant_type, None, "f16", nested=True, strength=-0.5)
        one(19, 128, 13, quant_type, SEED, "bf16", zero_b=True)


def gen_f32(mods, w: Writer, g) -> None:
    """fp32 LoRA factors (the launchers' IEEE fp32 ``tl.dot`` path, and fp32
    compute for the adapters' float32 weights): scaled FP8, INT8, NVFP4 and MX."""
    f8, i8, n4, mx = mods["float8"], mods["int8"], mods["nvfp4"], mods["mx"]
    for layout, seed, rank in (("row", SEED, 7), ("row", None, 40), ("tensor", SEED, 19), ("group", None, 7)):
        rows, cols = 70, 130 if layout != "group" else 120
        base = torch.randn(rows, cols, generator=g) * 0.02
        if layout == "row":
            block, s = (1, cols), base.abs().amax(1, keepdim=True) / 448.0
            sx = s
        elif layout == "tensor":
            block, s = (rows, cols), (base.abs().amax() / 448.0).reshape(1, 1)
            sx = s
        else:
            block = (1, 10)
            s = base.reshape(rows, cols // 10, 10).abs().amax(2) / 448.0
            sx = s.repeat_interleave(10, 1)
        s = s.float()
        q = (base / sx).clamp(-448, 448).to(torch.float8_e4m3fn)
        b, a = exact_factors(g, rows, cols, rank, torch.float32)
        oq, os_ = f8.merge_float8_lora(q.clone(), s.clone(), block, b, a, 1.0, rounding_seed=seed)
        w.add({"launcher": "float8", "rows": rows, "cols": cols, "rank": rank, "e4m3": True, "block": list(block),
               "seed": seed, "dtype": "f32", "strength": 1.0},
              qdata=q, scale=s, b=b, a=a, out_qdata=oq, out_scale=os_)
    for asym, seed, sdt in ((False, SEED, "bf16"), (True, None, "f32"), (False, None, "f16")):
        rows, cols, rank = 35, 69, 19
        q = torch.randint(-128, 128, (rows, cols), generator=g, dtype=torch.int8)
        scale = (torch.rand((rows, 1), generator=g) * 2e-4 + 1e-4).to(DTYPES[sdt])
        zp = torch.randint(-10, 10, (rows, 1), generator=g, dtype=torch.int8) if asym else None
        b, a = exact_factors(g, rows, cols, rank, torch.float32, exp=9)
        oq, os_, oz = i8.merge_int8_lora(q.clone(), scale.clone(), None if zp is None else zp.clone(), (1, cols),
                                         b, a, 1.0, asymmetric=asym, reduce_range=False, rounding_seed=seed)
        w.add({"launcher": "int8", "rows": rows, "cols": cols, "rank": rank, "block": [1, cols], "asymmetric": asym,
               "reduce_range": False, "seed": seed, "dtype": "f32", "scale_dtype": sdt, "strength": 1.0},
              qdata=q, scale=scale, zero_point=zp, b=b, a=a, out_qdata=oq, out_scale=os_, out_zero_point=oz)
    for two_level, seed in ((True, SEED), (False, None), (True, None)):
        rows, cols, rank = 19, 80, 13
        q = torch.randint(0, 256, (rows, cols // 2), generator=g, dtype=torch.uint8)
        if two_level:
            scale = (torch.rand((rows, cols // 16), generator=g) * 3 + 0.5).to(torch.float8_e4m3fn)
            pts = torch.tensor(0.003, dtype=torch.float32)
        else:
            scale = (torch.rand((rows, cols // 16), generator=g) * 0.01 + 0.002).to(torch.float8_e4m3fn)
            pts = None
        b, a = exact_factors(g, rows, cols, rank, torch.float32)
        oq, os_, og = n4.merge_nvfp4_lora(q.clone(), scale.clone(), None if pts is None else pts.clone(), 16, False,
                                          b, a, 1.0, rounding_seed=seed)
        w.add({"launcher": "nvfp4", "rows": rows, "cols": cols, "rank": rank, "swizzled": False,
               "two_level": two_level, "seed": seed, "dtype": "f32", "strength": 1.0},
              qdata=q, scale=scale, per_tensor_scale=pts, b=b, a=a, out_qdata=oq, out_scale=os_,
              out_per_tensor_scale=og)
    elem_dtypes = {"e4m3": torch.float8_e4m3fn, "e2m1": torch.float4_e2m1fn_x2}
    for elem, mode, seed in (("e4m3", 0, SEED), ("e4m3", 1, None), ("e2m1", 0, None), ("e2m1", 3, SEED)):
        rows, cols, rank = 19, 96, 7
        if elem == "e2m1":
            q = torch.randint(0, 256, (rows, cols // 2), generator=g, dtype=torch.uint8)
        else:
            q = (torch.randn(rows, cols, generator=g) * 100).clamp(-400, 400).to(elem_dtypes[elem])
        scale = torch.randint(110, 122, (rows, cols // 32), generator=g, dtype=torch.uint8).view(torch.float8_e8m0fnu)
        b, a = exact_factors(g, rows, cols, rank, torch.float32, exp=9)
        oq, os_ = q.clone(), scale.clone()
        mx.merge_mx_lora_(oq, os_, elem_dtypes[elem], 32, torch.float32, b, a, 1.0, scaling_mode=mode,
                          swizzled=False, rounding_seed=seed)
        w.add({"launcher": "mx", "rows": rows, "cols": cols, "rank": rank, "elem": elem, "scaling_mode": mode,
               "swizzled": False, "seed": seed, "dtype": "f32", "strength": 1.0},
              qdata=q, scale=scale, b=b, a=a, out_qdata=oq, out_scale=os_)


def main() -> None:
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PIPER_OFFLOAD_SRC", ""))
    mods = load_reference(ref / "src")
    w = Writer()
    gen_float8(mods["float8"], w, torch.Generator().manual_seed(80))
    gen_int8(mods["int8"], w, torch.Generator().manual_seed(81))
    gen_nvfp4(mods["nvfp4"], w, torch.Generator().manual_seed(82))
    gen_mx(mods["mx"], w, torch.Generator().manual_seed(83))
    gen_static_float8(mods["static_float8"], w, torch.Generator().manual_seed(84))
    gen_bnb8(mods["bnb8"], w, torch.Generator().manual_seed(85))
    gen_quanto(mods["quanto"], w, torch.Generator().manual_seed(86))
    gen_bnb4(mods["bnb4"], w, torch.Generator().manual_seed(87))
    gen_f32(mods, w, torch.Generator().manual_seed(88))
    w.save()
    print(f"{len(w.cases)} reference merge cases written to", HERE)


if __name__ == "__main__":
    main()

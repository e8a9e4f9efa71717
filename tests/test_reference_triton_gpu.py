"""GPU: the sm_100a merge against the reference's own Triton kernels on the B200.

The unmodified reference launchers -- ``merge_float8_lora``
(``_triton_float8_lora.py:486-588``), ``merge_int8_lora``
(``_triton_int8_lora.py:267-407``), ``merge_nvfp4_lora``
(``_triton_nvfp4_lora.py:515-595``) and ``merge_mx_lora_``
(``_triton_mx_lora.py:333-425``) -- run from ``baseline/_ref`` (installed by
``baseline/install_reference.py``; the module is skipped without it) on the
same device inputs as ``piper_offload_b200.kernels``.

Two input kinds:

* exact factors (small-integer multiples of 2**-8): every rank-r dot product
  is exact in any summation order, so the codes and scales must be identical;
  this covers the reference tests' shapes and the RCEIL ``tl.log2`` /
  ``tl.exp2`` scale path on device;
* the BASELINE configs' own factor distributions at full weight sizes, where
  the fp32 summation order of the dot product (tensor core tiles vs Triton's
  ``tl.dot`` tiles) is the one tie class: mismatching codes differ by at most
  one step and number at most ``TIE_FRACTION`` of the elements; scales may
  differ where such a tie moved a block maximum (``SCALE_TIE_FRACTION``).

With ``PIPER_PARITY_LOG`` set, each comparison appends its counts as a JSON
line to that file.

One known exception: the reference's FP8 stochastic rounding
(``_stochastic_float8``, ``_triton_stochastic_quantization.py:132-175``) is
miscompiled by the triton 3.6 in this image on sm_100 (the reference pins
triton >= 3.7). Run on its own over 1M values, every odd-indexed element of a
1-D block decodes to +-2^-9, and where round-to-nearest rounds up (p > 0.5)
the result is always the upper code, as if the fp32 -> fp8 -> fp32 round trip
of ``deterministic_value`` were folded into the identity; 2-D blocks show the
second effect only. Those comparisons (FP8 e4m3/e5m2 and MXFP8 with a seed)
are expected failures under triton < 3.7; the kernels follow the reference
source, which the interpreter-recorded fixtures pin
(``tests/test_reference_fixtures.py``).
"""

from __future__ import annotations

import json
import math
import os

import numpy as np
import pytest
import torch

from merge_cases import Case, compare, f32np, u8np
from piper_offload_b200 import _native

pytestmark = pytest.mark.gpu

TIE_FRACTION = 1e-5
SCALE_TIE_FRACTION = 1e-4
SEED = 0x9C3EA68DBAC91AAD


@pytest.fixture(scope="module")
def ref():
    from baseline import reference

    if not reference.available():
        pytest.skip("reference not installed under baseline/_ref")
    triton = pytest.importorskip("triton")
    mods = {k: reference.load(f"piper_offload._triton_{k}_lora") for k in ("float8", "int8", "nvfp4", "mx")}
    mods["triton_version"] = triton.__version__
    return mods


@pytest.fixture(autouse=True)
def device_status_clean(cuda_device):
    yield
    assert _native.device_status(cuda_device) == 0, "a bounded device wait timed out"


def exact_factors(case: Case, seed: int) -> None:
    g = torch.Generator().manual_seed(seed)
    b = torch.randint(-15, 16, (case.rows, case.rank), generator=g).float() * 2.0**-8
    a = torch.randint(-15, 16, (case.rank, case.cols), generator=g).float() * 2.0**-8
    case.tensors["b"], case.tensors["a"] = b.to(case.factor_dtype), a.to(case.factor_dtype)


def run_reference(ref, case: Case, dev) -> dict:
    """The reference launcher on device copies of the case's inputs."""
    q = case.tensors["q"]
    b = case.tensors["b"].to(dev)
    a = case.tensors["a"].to(dev)
    f = case.fmt
    qd = q.qdata.to(dev)
    sc = q.scale.to(dev) if q.scale is not None else None
    out = {}
    if f.startswith("mx"):
        elem = {"mxfp8": torch.float8_e4m3fn, "mxfp8_e5m2": torch.float8_e5m2,
                "mxfp4": torch.float4_e2m1fn_x2}[f]
        scale_e8 = sc.view(torch.float8_e8m0fnu)
        ref["mx"].merge_mx_lora_(qd, scale_e8, elem, 32, case.factor_dtype, b, a, case.strength,
                                 scaling_mode=case.scale_mode, swizzled=case.swizzled, rounding_seed=case.seed)
        out["q"], out["scale"] = u8np(qd), u8np(scale_e8)
    elif f.startswith("nvfp4"):
        pts = q.per_tensor_scale.to(dev) if q.per_tensor_scale is not None else None
        nq, ns, npts = ref["nvfp4"].merge_nvfp4_lora(qd.view(torch.uint8), sc.view(torch.float8_e4m3fn), pts, 16,
                                                      case.swizzled, b, a, case.strength, rounding_seed=case.seed)
        out["q"], out["scale"] = u8np(nq), u8np(ns)
        out["global"] = None if npts is None else float(npts.reshape(-1)[0].cpu())
    elif f.startswith("fp8"):
        block = {"fp8_row": (1, case.cols), "fp8_tensor": (case.rows, case.cols), "fp8_group": (1, case.group)}[f]
        nq, ns = ref["float8"].merge_float8_lora(qd, sc, block, b, a, case.strength, rounding_seed=case.seed)
        out["q"], out["scale"] = u8np(nq), f32np(ns)
    elif f.startswith("int8"):
        block = {"int8_row": (1, case.cols), "int8_tensor": (case.rows, case.cols), "int8_group": (1, case.group),
                 "int8_asym": (1, case.cols)}[f]
        zp = q.zero_point.to(dev) if q.zero_point is not None else None
        nq, ns, nz = ref["int8"].merge_int8_lora(qd, sc, zp, block, b, a, case.strength, asymmetric=zp is not None,
                                                 reduce_range=False, rounding_seed=case.seed)
        out["q"], out["scale"] = nq.cpu().numpy().copy(), f32np(ns)
        out["zp"] = None if zp is None else nz.cpu().numpy().copy()
    else:
        raise KeyError(f)
    return out


def log_counts(name: str, case: Case, d, ref) -> None:
    path = os.environ.get("PIPER_PARITY_LOG")
    if not path:
        return
    rec = {"case": name, "fmt": case.fmt, "shape": [case.rows, case.cols], "rank": case.rank,
           "sr": case.seed is not None, "scale_mode": case.scale_mode, "elements": d.n,
           "code_mismatch": d.code_mismatch, "max_step": d.max_step, "scale_mismatch": d.scale_mismatch,
           "extra": d.extra, "triton": ref["triton_version"]}
    with open(path, "a") as fh:
        fh.write(json.dumps(rec) + "\n")


FP8_SR_FORMATS = ("fp8_row", "fp8_tensor", "fp8_group", "mxfp8", "mxfp8_e5m2")


def triton_fp8_sr_broken(ref) -> bool:
    major, minor = (int(x) for x in ref["triton_version"].split(".")[:2])
    return (major, minor) < (3, 7)


def versus_reference(ref, case: Case, dev, name: str, *, exact: bool):
    got = case.run_native(dev)
    try:
        want = run_reference(ref, case, dev)
    except RuntimeError as exc:  # a compile failure on the host; nothing ran on the device
        if "PassManager::run failed" in str(exc):
            pytest.skip(f"the reference kernel for {case.fmt} does not compile under triton {ref['triton_version']} "
                        "on sm_100 (MLIR: parent layout must have at least rank >= 2)")
        raise
    torch.cuda.synchronize(dev)
    d = compare(case, got, want)
    log_counts(name, case, d, ref)
    if case.seed is not None and case.fmt in FP8_SR_FORMATS and triton_fp8_sr_broken(ref) and d.code_mismatch:
        pytest.xfail(f"reference FP8 stochastic rounding is miscompiled by triton {ref['triton_version']} "
                     f"on sm_100 ({d.code_mismatch} of {d.n} codes differ)")
    allowed = 0 if exact else math.floor(TIE_FRACTION * d.n)
    assert d.max_step <= (0 if exact else 1), f"{name}: {d}"
    assert d.code_mismatch <= allowed, f"{name}: {d.code_mismatch} > {allowed} ({d})"
    n_scales = max(1, d.n // 16)
    assert d.scale_mismatch <= (0 if exact else max(1, math.floor(SCALE_TIE_FRACTION * n_scales))), f"{name}: {d}"
    return d


# The reference tests' shapes with exact factors: identical results required.
EXACT = [
    ("fp8_row", 70, 130, 7, {}), ("fp8_tensor", 70, 130, 7, {}), ("fp8_group", 70, 128, 7, {"group": 32}),
    ("int8_row", 35, 69, 7, {}), ("int8_tensor", 35, 69, 19, {}), ("int8_group", 35, 128, 7, {"group": 64}),
    ("int8_asym", 35, 69, 7, {}),
    ("nvfp4", 19, 80, 13, {}), ("nvfp4_1l", 19, 80, 13, {}), ("nvfp4", 300, 1024, 64, {"swizzled": True}),
    ("mxfp8", 19, 96, 7, {}), ("mxfp8_e5m2", 19, 96, 7, {}), ("mxfp4", 19, 96, 7, {}),
    ("mxfp8", 300, 1024, 64, {"swizzled": True}),
]


@pytest.mark.parametrize("stochastic", [False, True], ids=["rtn", "sr"])
@pytest.mark.parametrize("fmt,rows,cols,rank,kw", EXACT, ids=[f"{e[0]}-{e[1]}x{e[2]}" for e in EXACT])
def test_reference_shapes_exact_factors(ref, fmt, rows, cols, rank, kw, stochastic, cuda_device):
    case = Case(fmt, rows, cols, rank, seed=SEED if stochastic else None, outliers=0.001, **kw).build()
    exact_factors(case, rows * 131 + cols)
    versus_reference(ref, case, cuda_device, f"exact-{fmt}-{rows}x{cols}", exact=True)


@pytest.mark.parametrize("mode", [0, 1, 2, 3], ids=["floor", "rceil", "ceil", "even"])
@pytest.mark.parametrize("fmt", ["mxfp8", "mxfp8_e5m2", "mxfp4"])
def test_mx_scale_modes_exact_factors(ref, fmt, mode, cuda_device):
    """RCEIL's ``tl.ceil(tl.log2(amax / max_pos))`` and ``tl.exp2`` as the GPU
    evaluates them, against the kernel's exact ceil(log2) (_triton_mx_lora.py:115-131)."""
    case = Case(fmt, 256, 2048, 32, scale_mode=mode, outliers=0.001).build()
    exact_factors(case, 7 + mode)
    versus_reference(ref, case, cuda_device, f"mxmode-{fmt}-{mode}", exact=True)


# One full-size weight per BASELINE config, with that config's factor
# distribution (rank, std) and rounding: the tie-class bound applies.
CONFIG_SIZES = [
    ("config1-int8", Case("int8_row", 4096, 4096, 16, lora_std=0.01)),
    ("config2-fp8-gate-sr", Case("fp8_row", 14336, 4096, 32, seed=SEED, lora_std=0.01)),
    ("config2-fp8-down-sr", Case("fp8_row", 4096, 14336, 32, seed=SEED + 1, lora_std=0.01)),
    ("config3-nvfp4-rtn", Case("nvfp4", 14336, 4096, 64, lora_std=0.005)),
    ("config3-nvfp4-sr", Case("nvfp4", 4096, 14336, 64, seed=SEED, lora_std=0.005)),
    ("config4-mxfp8-floor", Case("mxfp8", 12288, 3072, 128, lora_std=0.005, outliers=0.001)),
    ("config4-mxfp8-rceil", Case("mxfp8", 3072, 12288, 128, scale_mode=1, lora_std=0.005, outliers=0.001)),
    ("config4-mxfp4-floor", Case("mxfp4", 12288, 3072, 128, lora_std=0.005, outliers=0.001)),
]


@pytest.mark.parametrize("name,case", CONFIG_SIZES, ids=[c[0] for c in CONFIG_SIZES])
def test_config_sizes_against_reference(ref, name, case, cuda_device):
    case.build(data_seed=17)
    versus_reference(ref, case, cuda_device, name, exact=False)


def test_reference_exact_at_config_size_with_exact_factors(ref, cuda_device):
    """Full-size FP8 SR weight (config 2's down_proj) with exact factors: no
    tie class remains, so the 58.7 M codes and the row scales are identical."""
    case = Case("fp8_row", 4096, 14336, 32, seed=SEED).build(data_seed=3)
    exact_factors(case, 99)
    versus_reference(ref, case, cuda_device, "exact-fp8-4096x14336-sr", exact=True)


# fp32 factors with the configs' own factor distributions (not exact in any
# summation order): the reference's IEEE fp32 dot is one fused multiply-add per
# rank step in rank order, which the CUDA-core update reproduces, so no tie
# class remains and the codes and scales must be identical. Ranks below and
# above the reference's rank blocks (16, then multiples of 32).
F32_REFERENCE = [
    ("fp8_row", 256, 1024, 48, {}), ("fp8_tensor", 70, 130, 7, {}), ("int8_row", 128, 512, 19, {}),
    ("int8_asym", 35, 69, 7, {}), ("mxfp8", 128, 1024, 64, {}), ("mxfp4", 64, 512, 16, {}),
    ("nvfp4", 128, 1024, 33, {}), ("nvfp4_1l", 19, 80, 13, {}),
]


@pytest.mark.parametrize("stochastic", [False, True], ids=["rtn", "sr"])
@pytest.mark.parametrize("fmt,rows,cols,rank,kw", F32_REFERENCE,
                         ids=[f"{e[0]}-{e[1]}x{e[2]}-r{e[3]}" for e in F32_REFERENCE])
def test_fp32_factors_against_reference(ref, fmt, rows, cols, rank, kw, stochastic, cuda_device):
    case = Case(fmt, rows, cols, rank, seed=SEED if stochastic else None, factor_dtype=torch.float32,
                outliers=0.001, **kw).build(data_seed=rows + rank)
    versus_reference(ref, case, cuda_device, f"f32-{fmt}-{rows}x{cols}-r{rank}", exact=True)


@pytest.mark.parametrize("stochastic", [False, True], ids=["rtn", "sr"])
def test_fp32_factors_int8_fp32_scales_against_reference(ref, stochastic, cuda_device):
    """fp32 scales make ``(q - zp) * scale`` inexact, so the contraction of the
    fp32-compute ``base + acc * strength`` onto that product is visible."""
    case = Case("int8_row", 128, 512, 24, seed=SEED if stochastic else None, factor_dtype=torch.float32,
                outliers=0.001).build(data_seed=5)
    case.tensors["q"].scale = case.tensors["q"].scale.float()
    versus_reference(ref, case, cuda_device, "f32-int8-f32scales", exact=True)

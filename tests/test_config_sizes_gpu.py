"""GPU parity at the BASELINE configs' own sizes, merged exactly as ``bench.py``
batches them.

For each config, one layer of that config's model shapes is built on the
device by ``bench.build_weights`` (same generators, seeds, factor
distributions and rounding as the benchmark) and merged with one
``piper_merge_batch`` call, the benchmark's launch sequence. Four 128-row
strips of every weight (first, last and two inner ones) are then merged by the
CPU oracle from copies of their inputs taken before the merge:

* per-row and per-block layouts are independent per row; a strip starting at
  row r0 is checked with ``offset_base = r0 * N``, which reproduces the
  stochastic-rounding stream of the whole-weight merge exactly;
* the two-level NVFP4 global scale comes from the whole tensor: its maximum
  |merged| is computed over all rows in numpy and passed to the strip merges
  (``oracle.merge.merge_nvfp4(global_amax=...)``), and the device's new global
  scale is checked against it.

Tolerance (the contract): mismatching codes differ by one step at most and
number at most ``TIE_FRACTION`` of the checked elements (fp32 summation order
of the rank-r dot product); scales match except where such a tie moved a
maximum (``SCALE_TIE_FRACTION`` of the checked scales).
"""

from __future__ import annotations

import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import bench
from merge_cases import compare
from oracle import merge as om
from piper_offload_b200 import _native
from piper_offload_b200 import adapters as AD
from piper_offload_b200.seeding import derive_seed

pytestmark = pytest.mark.gpu

TIE_FRACTION = 1e-5
SCALE_TIE_FRACTION = 1e-4
FMT_OF = {"fp8": "fp8_row", "int8": "int8_row", "nvfp4": "nvfp4", "mxfp8": "mxfp8", "mxfp4": "mxfp4",
          "q8_0": "q8_0", "q4_0": "q4_0"}


@pytest.fixture(scope="module", autouse=True)
def triton_division():
    from oracle import gpu_division

    if not torch.cuda.is_available():
        pytest.skip("CUDA device not available")
    gpu_division.install()
    yield
    gpu_division.uninstall()


def strips_of(rows: int) -> list[int]:
    last = (rows - 1) // 128 * 128
    picks = {0, last, (rows // 3) // 128 * 128, (2 * rows // 3) // 128 * 128}
    return sorted(picks)


def u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy().copy()


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float32)


def storage_rows(cfg: str, t, r0: int, r1: int) -> dict:
    """CPU copies of rows r0..r1 of a weight's storage (per-row / per-block layouts)."""
    if cfg == "fp8":
        return {"q": u8(t.qdata[r0:r1]), "scale": f32(t.scale[r0:r1])}
    if cfg == "int8":
        return {"q": t.qdata[r0:r1].cpu().numpy().copy(), "scale": f32(t.scale[r0:r1])}
    if cfg == "nvfp4":
        return {"q": u8(t.qdata[r0:r1]), "scale": u8(t.scale[r0:r1])}
    if cfg in ("mxfp8", "mxfp4"):
        return {"q": u8(t.qdata[r0:r1]), "scale": u8(t.scale[r0:r1])}
    return {"q": u8(t.raw[r0:r1])}


def oracle_strip(cfg: str, inp: dict, b: np.ndarray, a: np.ndarray, seed, offset_base: int, extra: dict) -> dict:
    kw = dict(seed=seed, offset_base=offset_base)
    n = a.shape[1]
    if cfg == "fp8":
        q, s = om.merge_float8(inp["q"], inp["scale"], (1, n), b, a, 1.0, e4m3=True, **kw)
        return {"q": q, "scale": s}
    if cfg == "int8":
        q, s, _ = om.merge_int8(inp["q"], inp["scale"], None, (1, n), b, a, 1.0, asymmetric=False, compute="bf16",
                                qparam="bf16", **kw)
        return {"q": q, "scale": s}
    if cfg == "nvfp4":
        q, s, g = om.merge_nvfp4(inp["q"], inp["scale"], extra["g_in"], b, a, 1.0, global_amax=extra["amax"], **kw)
        return {"q": q, "scale": s, "global": None if g is None else float(g)}
    if cfg in ("mxfp8", "mxfp4"):
        q, s = om.merge_mx(inp["q"], inp["scale"], "e4m3" if cfg == "mxfp8" else "e2m1", b, a, 1.0,
                           scaling_mode=0, **kw)
        return {"q": q, "scale": s}
    return {"q": om.merge_gguf(inp["q"], 8 if cfg == "q8_0" else 2, b, a, 1.0, **kw)}


def nvfp4_tensor_amax(q: np.ndarray, scale: np.ndarray, g_in: float, b: np.ndarray, a: np.ndarray) -> float:
    """max |merged| over the whole two-level NVFP4 tensor, in row chunks."""
    amax = np.float32(0.0)
    for r0 in range(0, b.shape[0], 1024):
        merged, _ = om._nvfp4_merged(q[r0:r0 + 1024], scale[r0:r0 + 1024], np.float32(g_in), False,
                                     b[r0:r0 + 1024], a, 1.0, "bf16")
        amax = max(amax, np.float32(np.nanmax(np.abs(merged))))
    return float(amax)


CONFIGS = [("fp8", False), ("int8", False), ("nvfp4", False), ("nvfp4", True), ("mxfp8", False),
           ("mxfp4", False), ("q8_0", False), ("q8_0", True), ("q4_0", False), ("q4_0", True)]


@pytest.mark.parametrize("cfg,force_sr", CONFIGS, ids=[f"{c}{'-sr' if s else ''}" for c, s in CONFIGS])
def test_config_layer_batch_matches_oracle_on_strips(cfg, force_sr, cuda_device):
    dev = cuda_device
    items = bench.build_weights(cfg, dev, seed_base=0, n_layers=1)
    stochastic = bench.CONFIGS[cfg][5] or force_sr
    checks = []
    for key, rows, cols, t, b, a, _ in items:
        a_np = f32(a)
        extra = {}
        if cfg == "nvfp4":
            g_in = float(t.per_tensor_scale.reshape(-1)[0].cpu())
            extra = {"g_in": g_in, "amax": nvfp4_tensor_amax(u8(t.qdata), u8(t.scale), g_in, f32(b), a_np)}
        for r0 in strips_of(rows):
            r1 = min(rows, r0 + 128)
            checks.append((key, rows, cols, t, r0, storage_rows(cfg, t, r0, r1), f32(b[r0:r1]), a_np, extra))
    seeds = {key: (derive_seed(key, 0) if stochastic else None) for key, *_ in items}
    keep: list = []
    descs = [AD.select_adapter(t).merge_desc(t, b, a, 1.0, rounding_seed=seeds[key], keep=keep)
             for key, rows, cols, t, b, a, _ in items]
    _native.merge_batch(descs, dev)
    torch.cuda.synchronize(dev)
    assert _native.device_status(dev) == 0

    n = mism = scale_mism = n_scales = 0
    worst = 0
    for key, rows, cols, t, r0, inp, b_np, a_np, extra in checks:
        r1 = min(rows, r0 + 128)
        want = oracle_strip(cfg, inp, b_np, a_np, seeds[key], r0 * cols, extra)
        got = storage_rows(cfg, t, r0, r1)
        if cfg == "nvfp4":
            got["global"] = float(t.per_tensor_scale.reshape(-1)[0].cpu())
        d = compare(SimpleNamespace(fmt=FMT_OF[cfg]), got, want)
        n += d.n
        mism += d.code_mismatch
        scale_mism += d.scale_mismatch
        n_scales += max(1, d.n // 16)
        worst = max(worst, d.max_step)
    assert worst <= 1, f"{cfg}: a code differs by {worst} steps"
    assert mism <= math.floor(TIE_FRACTION * n), f"{cfg}: {mism} mismatching codes of {n}"
    assert scale_mism <= max(1, math.floor(SCALE_TIE_FRACTION * n_scales)), f"{cfg}: {scale_mism} scales differ"

"""GPU parity tests: the sm_100a merge against the CPU oracle, code for code.

The oracle's tensor/tensor fp32 quotients are evaluated with Triton's default
division on the device (``oracle.gpu_division``), which makes every quotient
the reference computes with ``/`` bit-identical. What remains is the fp32
summation order of the rank-r dot product (tensor core vs. the oracle's
correctly rounded sum). Tolerance: mismatching
codes differ by at most one code step and number at most 1e-5 of the
elements (``TIE_FRACTION``); scales and zero points must match exactly
except where such a tie moved a block maximum (``SCALE_TIE_FRACTION``).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from merge_cases import FORMATS, SMALL_SHAPES, Case, compare
from piper_offload_b200 import _native
from piper_offload_b200 import kernels as K

pytestmark = pytest.mark.gpu

TIE_FRACTION = 1e-5
SCALE_TIE_FRACTION = 1e-4
SEED = 0x9C3EA68DBAC91AAD  # derive_seed("layer.0.weight", 0)


@pytest.fixture(scope="module", autouse=True)
def triton_division():
    from oracle import gpu_division

    if not torch.cuda.is_available():
        pytest.skip("CUDA device not available")
    gpu_division.install()
    yield
    gpu_division.uninstall()


@pytest.fixture(autouse=True)
def device_status_clean(cuda_device):
    yield
    assert _native.device_status(cuda_device) == 0, "a bounded device wait timed out"


def check(case: Case, dev, *, exact: bool = False):
    case.build()
    got = case.run_native(dev)
    torch.cuda.synchronize(dev)
    want = case.run_oracle()
    d = compare(case, got, want)
    allowed = 0 if exact else math.floor(TIE_FRACTION * d.n)
    assert d.max_step <= 1, f"{case.fmt}: code differs by {d.max_step} steps ({d})"
    assert d.code_mismatch <= allowed, f"{case.fmt}: {d.code_mismatch} > {allowed} tie mismatches ({d})"
    n_scales = max(1, d.n // 16)
    assert d.scale_mismatch <= (0 if exact else math.floor(SCALE_TIE_FRACTION * n_scales)), (
        f"{case.fmt}: scale mismatches {d}"
    )
    return d


def _group(fmt: str, default: int = 32) -> int:
    return default if fmt in ("fp8_group", "int8_group") else 64


@pytest.mark.parametrize("stochastic", [False, True], ids=["rtn", "sr"])
@pytest.mark.parametrize("fmt", FORMATS)
def test_reference_shapes_exact(fmt, stochastic, cuda_device):
    """The reference tests' own shapes (tail rows, ragged columns, odd ranks)."""
    rows, cols, rank = SMALL_SHAPES[fmt]
    check(Case(fmt, rows, cols, rank, seed=SEED if stochastic else None, group=_group(fmt)), cuda_device,
          exact=True)


@pytest.mark.parametrize("stochastic", [False, True], ids=["rtn", "sr"])
@pytest.mark.parametrize("fmt", FORMATS)
def test_medium_shapes(fmt, stochastic, cuda_device):
    check(Case(fmt, 512, 2048, 32, seed=12345 if stochastic else None, group=_group(fmt, 128),
               outliers=0.001), cuda_device)


@pytest.mark.parametrize("stochastic", [False, True], ids=["rtn", "sr"])
@pytest.mark.parametrize("fmt", ["int8_row", "int8_asym", "fp8_row"])
def test_per_row_fused_pass_exact(fmt, stochastic, cuda_device):
    """Per-row weights with more than two 128-row strips per SM (298 strips,
    the last one 12 rows) run the one-launch fused pass and its shortcut
    encoders for all-finite rows; smaller ones run the reduce / encode pair."""
    check(Case(fmt, 297 * 128 + 12, 160, 8, seed=SEED if stochastic else None), cuda_device, exact=True)


@pytest.mark.parametrize("fmt", ["int8_row", "int8_asym"])
def test_per_row_fused_pass_fp32_scales_exact(fmt, cuda_device):
    """fp32 INT8 scales leave no rounding between ``m * inv`` and the
    round-to-integer step, so a fused multiply-add there shows at ties."""
    cs = Case(fmt, 297 * 128 + 12, 160, 8).build(data_seed=5)
    cs.tensors["q"].scale = cs.tensors["q"].scale.float()
    got = cs.run_native(cuda_device)
    torch.cuda.synchronize(cuda_device)
    d = compare(cs, got, cs.run_oracle())
    assert d.code_mismatch == 0 and d.scale_mismatch == 0, d


@pytest.mark.parametrize("mode", [0, 1, 2, 3], ids=["floor", "rceil", "ceil", "even"])
@pytest.mark.parametrize("fmt", ["mxfp8", "mxfp8_e5m2", "mxfp4"])
def test_mx_scale_modes(fmt, mode, cuda_device):
    check(Case(fmt, 256, 1024, 64, scale_mode=mode, outliers=0.001), cuda_device)


@pytest.mark.parametrize("fmt,rows,cols", [("mxfp8", 300, 1024), ("mxfp4", 200, 96 * 4),
                                           ("nvfp4", 300, 1024), ("nvfp4_1l", 130, 1040),
                                           ("nvfp4", 19, 80)])
def test_swizzled_scales(fmt, rows, cols, cuda_device):
    check(Case(fmt, rows, cols, 64, swizzled=True, seed=SEED), cuda_device)


@pytest.mark.parametrize("fmt", ["fp8_row", "int8_row", "int8_tensor", "fp8_tensor", "q8_0", "q4_0",
                                 "fp8_group", "int8_group"])
def test_fp16_factors(fmt, cuda_device):
    check(Case(fmt, 96, 256, 16, factor_dtype=torch.float16, group=_group(fmt)), cuda_device)


# fp32 factors: the reference's IEEE fp32 dot (one fused multiply-add per rank
# step in rank order) has no summation-order tie class, so the CUDA-core update
# matches the oracle's exact chain bit for bit. Ranks below, at and above the
# reference's rank blocks (16, then multiples of 32), ragged shapes included.
F32_CASES = [
    ("fp8_row", 70, 130, 7), ("fp8_row", 256, 1024, 48), ("fp8_tensor", 96, 256, 16), ("fp8_group", 64, 256, 32),
    ("int8_row", 35, 69, 19), ("int8_tensor", 96, 256, 40), ("int8_group", 64, 512, 16), ("int8_asym", 35, 69, 7),
    ("mxfp8", 19, 96, 7), ("mxfp8", 256, 1024, 64), ("mxfp8_e5m2", 64, 256, 33), ("mxfp4", 128, 512, 32),
    ("nvfp4", 19, 80, 13), ("nvfp4", 256, 1024, 64), ("nvfp4_1l", 130, 1040, 20),
    ("q8_0", 96, 256, 16), ("q4_0", 64, 512, 24),
]


@pytest.mark.parametrize("stochastic", [False, True], ids=["rtn", "sr"])
@pytest.mark.parametrize("fmt,rows,cols,rank", F32_CASES, ids=[f"{c[0]}-{c[1]}x{c[2]}-r{c[3]}" for c in F32_CASES])
def test_fp32_factors_exact(fmt, rows, cols, rank, stochastic, cuda_device):
    check(Case(fmt, rows, cols, rank, seed=SEED if stochastic else None, factor_dtype=torch.float32,
               group=_group(fmt), outliers=0.001), cuda_device, exact=True)


@pytest.mark.parametrize("strength", [0.0, -0.75, 3.5])
def test_strengths(strength, cuda_device):
    for fmt in ("mxfp8", "nvfp4", "fp8_row", "int8_row", "q8_0"):
        check(Case(fmt, 64, 256, 16, strength=strength), cuda_device)


@pytest.mark.parametrize("rank", [1, 16, 128, 200, 256])
def test_ranks(rank, cuda_device):
    # GGUF: 256-column TMA tiles up to rank 160 (Q8_0) / 224 (Q4_0), the
    # cp.async fallback on narrower tiles above.
    for fmt in ("mxfp4", "fp8_row", "q8_0", "q4_0"):
        check(Case(fmt, 160, 512, rank), cuda_device)


def test_int8_group_two_pass(cuda_device):
    """Groups that are not a multiple of 32 take the REDUCE/ENCODE path."""
    check(Case("int8_group", 70, 96 * 3, 13, group=48), cuda_device)
    check(Case("int8_group", 70, 1024, 13, group=512, seed=SEED), cuda_device)


def test_fp8_group_256(cuda_device):
    check(Case("fp8_group", 130, 1024, 32, group=256, seed=SEED), cuda_device)


def _nvfp4_special(fmt, *, strength=1.0, zero_b=False, neg_scales=False, nan_row=None, inf_row=None,
                   seed=None):
    cs = Case(fmt, 64, 256, 16, strength=strength, seed=seed).build()
    b = cs.tensors["b"]
    if zero_b:
        b.zero_()
    if nan_row is not None:
        b[nan_row, :] = float("nan")
    if inf_row is not None:
        b[inf_row, :] = 0.0
        b[inf_row, 0] = float("inf")
    if neg_scales:
        sc = cs.tensors["q"].scale.view(torch.uint8)
        sc.view(-1)[::3] |= 0x80  # E4M3 block scales with the sign bit set: -0 bases
    return cs


def _check_built(cs: Case, dev, *, exact_rows=None, exact=False):
    got = cs.run_native(dev)
    torch.cuda.synchronize(dev)
    want = cs.run_oracle()
    d = compare(cs, got, want)
    allowed = 0 if exact else math.floor(TIE_FRACTION * d.n)
    assert d.max_step <= 1 and d.code_mismatch <= allowed, d
    rows = slice(None) if exact else exact_rows
    if rows is not None:
        # Raw bytes: the code comparison above treats +0 and -0 (codes 0 and 8) alike.
        assert np.array_equal(got["q"][rows], want["q"][rows]), "E2M1 bytes differ"
        assert np.array_equal(got["scale"][rows], want["scale"][rows]), "block scales differ"
    if want.get("global") is not None:
        assert np.float32(got["global"]).tobytes() == np.float32(want["global"]).tobytes()


@pytest.mark.parametrize("fmt", ["nvfp4", "nvfp4_1l"])
def test_nvfp4_zero_updates_keep_signed_bases(fmt, cuda_device):
    """acc = 0 everywhere: the reference keeps each base, -0 included (negative block scales)."""
    _check_built(_nvfp4_special(fmt, zero_b=True, neg_scales=True), cuda_device, exact=True)
    _check_built(_nvfp4_special(fmt, zero_b=True, neg_scales=True, seed=SEED), cuda_device, exact=True)


@pytest.mark.parametrize("fmt", ["mxfp4", "mxfp8"])
def test_mx_sr_zero_updates_exact(fmt, cuda_device):
    """Zero updates leave every normalized value on the code grid: no stochastic step."""
    cs = Case(fmt, 64, 256, 16, seed=SEED).build()
    cs.tensors["b"].zero_()
    _check_built(cs, cuda_device, exact=True)


@pytest.mark.parametrize("strength", [2.0 ** 70, 2.0 ** -70, -(2.0 ** 61)])
@pytest.mark.parametrize("fmt", ["nvfp4", "nvfp4_1l"])
def test_nvfp4_extreme_strengths(fmt, strength, cuda_device):
    """Strengths outside [2^-60, 2^60] take the exact update-is-zero test for every block."""
    _check_built(_nvfp4_special(fmt, strength=strength, neg_scales=True), cuda_device)


@pytest.mark.parametrize("fmt", ["nvfp4", "nvfp4_1l"])
def test_nvfp4_nan_and_inf_updates(fmt, cuda_device):
    """A NaN row and an infinite row of B: those rows match the oracle byte for byte."""
    cs = _nvfp4_special(fmt, nan_row=5, inf_row=9, neg_scales=True)
    _check_built(cs, cuda_device, exact_rows=[5, 9])


def test_in_place_identity(cuda_device):
    """Storage tensors keep their data pointers (reference asserts this identity)."""
    c = Case("fp8_row", 64, 256, 16).build()
    q = c.tensors["q"]
    qd = q.qdata.to(cuda_device)
    sc = q.scale.to(cuda_device)
    p0, p1 = qd.data_ptr(), sc.data_ptr()
    b = c.tensors["b"].to(cuda_device)
    a = c.tensors["a"].to(cuda_device)
    out_q, out_s = K.merge_float8_lora(qd, sc, (1, 256), b, a, 1.0)
    assert out_q is qd and out_s is sc
    assert qd.data_ptr() == p0 and sc.data_ptr() == p1


def test_stochastic_replay_and_seed_sensitivity(cuda_device):
    """Same seed -> same bytes; another seed -> other codes, same scales."""
    outs = []
    for seed in (SEED, SEED, SEED + 1):
        c = Case("mxfp8", 128, 1024, 32, seed=seed).build()
        outs.append(c.run_native(cuda_device))
    assert np.array_equal(outs[0]["q"], outs[1]["q"])
    assert not np.array_equal(outs[0]["q"], outs[2]["q"])
    assert np.array_equal(outs[0]["scale"], outs[2]["scale"])


def test_row_shard_offsets_reproduce_unsharded(cuda_device):
    """Merging row shards with their global offset base equals the 1-GPU merge."""
    rows, cols = 256, 512
    full = Case("nvfp4_1l", rows, cols, 32, seed=SEED).build()
    want = full.run_native(cuda_device)
    q = full.tensors["q"]
    parts = []
    for r0, r1 in ((0, 128), (128, 256)):
        qd = q.qdata[r0:r1].clone().to(cuda_device)
        sc = q.scale.view(torch.uint8)[r0:r1].clone().view(torch.float8_e4m3fn).to(cuda_device)
        b = full.tensors["b"][r0:r1].to(cuda_device)
        a = full.tensors["a"].to(cuda_device)
        K.merge_nvfp4_lora(qd, sc, None, 16, False, b, a, 1.0, rounding_seed=SEED, offset_base=r0 * cols)
        parts.append(qd.cpu().numpy())
    assert np.array_equal(np.concatenate(parts), want["q"])


def test_sr_unbiased(cuda_device):
    """Mean of stochastic FP8 merges over seeds approaches the exact merged value."""
    rows, cols, rank = 64, 256, 16
    c = Case("fp8_row", rows, cols, rank, seed=None).build()
    q = c.tensors["q"]
    b = c.tensors["b"].to(cuda_device)
    a = c.tensors["a"].to(cuda_device)
    base = q.qdata.float() * q.scale.float()
    exact = (base.bfloat16().float() + (c.tensors["b"].float() @ c.tensors["a"].float())).to(cuda_device)
    acc = torch.zeros_like(exact)
    n = 64
    for s in range(n):
        qd = q.qdata.to(cuda_device).clone()
        sc = q.scale.to(cuda_device).clone()
        K.merge_float8_lora(qd, sc, (1, cols), b, a, 1.0, rounding_seed=1000 + s)
        acc += qd.float() * sc
    mean = acc / n
    err = (mean - exact).abs().mean() / exact.abs().mean()
    rtn_q = q.qdata.to(cuda_device).clone()
    rtn_s = q.scale.to(cuda_device).clone()
    K.merge_float8_lora(rtn_q, rtn_s, (1, cols), b, a, 1.0)
    rtn_err = ((rtn_q.float() * rtn_s) - exact).abs().mean() / exact.abs().mean()
    assert err < rtn_err * 0.5, (float(err), float(rtn_err))


def test_batched_multi_weight_launch(cuda_device):
    """One piper_merge_batch call over mixed formats equals per-weight calls."""
    specs = [("fp8_row", 300, 512, 32), ("mxfp8", 128, 256, 16), ("fp8_row", 129, 1024, 8),
             ("nvfp4", 64, 256, 16), ("int8_row", 77, 384, 24), ("q4_0", 50, 256, 16)]
    cases = [Case(f, r, c, k, seed=SEED if i % 2 else None).build(data_seed=i) for i, (f, r, c, k) in
             enumerate(specs)]
    wants = [cs.run_oracle() for cs in cases]
    # Build descriptors for one batch call.
    descs, keep = [], []
    for cs in cases:
        d, held = _desc_for(cs, cuda_device)
        descs.append(d)
        keep.append(held)
    _native.merge_batch(descs, cuda_device)
    torch.cuda.synchronize(cuda_device)
    for cs, held, want in zip(cases, keep, wants):
        got = _collect(cs, held)
        d = compare(cs, got, want)
        assert d.code_mismatch <= math.floor(TIE_FRACTION * d.n) and d.max_step <= 1, (cs.fmt, d)
        assert d.scale_mismatch == 0, (cs.fmt, d)


def test_batched_mixed_tma_and_fallback_weights(cuda_device):
    """One fused launch over per-row weights whose codes and factors move by
    bulk tensor copies (aligned rows) and weights that need the cp.async
    fallback (130-column rows, rank 7), alternating, RTN and stochastic."""
    specs = [("fp8_row", 300, 512, 32), ("fp8_row", 70, 130, 7), ("fp8_row", 256, 1024, 16),
             ("fp8_row", 35, 69, 7), ("int8_row", 200, 512, 16), ("int8_row", 35, 69, 7)]
    cases = [Case(f, r, c, k, seed=SEED if i % 3 == 1 else None).build(data_seed=50 + i) for i, (f, r, c, k) in
             enumerate(specs)]
    wants = [cs.run_oracle() for cs in cases]
    descs, keep = [], []
    for cs in cases:
        d, held = _desc_for(cs, cuda_device)
        descs.append(d)
        keep.append(held)
    _native.merge_batch(descs, cuda_device)
    torch.cuda.synchronize(cuda_device)
    assert _native.device_status(cuda_device) == 0
    for cs, held, want in zip(cases, keep, wants):
        d = compare(cs, _collect(cs, held), want)
        assert d.code_mismatch <= math.floor(TIE_FRACTION * d.n) and d.max_step <= 1, (cs.fmt, cs.rows, cs.cols, d)
        assert d.scale_mismatch == 0, (cs.fmt, cs.rows, cs.cols, d)


def _desc_for(cs: Case, dev):
    from merge_cases import f32np  # noqa: F401

    q = cs.tensors["q"]
    held = {"q": q.qdata.to(dev), "b": cs.tensors["b"].to(dev), "a": cs.tensors["a"].to(dev)}
    d = _native.MergeDesc()
    d.rows, d.cols, d.rank = cs.rows, cs.cols, cs.rank
    d.compute_dtype = _native.DT_BF16
    d.strength = cs.strength
    if cs.seed is not None:
        d.seed = cs.seed
        d.flags |= _native.FLAG_STOCHASTIC
    if q.scale is not None:
        held["scale"] = q.scale.to(dev)
        d.scale = held["scale"].data_ptr()
    if cs.fmt == "fp8_row":
        d.format, d.block_rows, d.block_cols = _native.FMT_FP8_E4M3, 1, cs.cols
    elif cs.fmt == "mxfp8":
        d.format = _native.FMT_MXFP8_E4M3
    elif cs.fmt == "nvfp4":
        d.format = _native.FMT_NVFP4
        held["g"] = q.per_tensor_scale.to(dev)
        d.global_scale = held["g"].data_ptr()
    elif cs.fmt == "int8_row":
        d.format, d.block_rows, d.block_cols = _native.FMT_INT8, 1, cs.cols
        d.scale_dtype = _native.DT_BF16
    elif cs.fmt == "q4_0":
        d.format = _native.FMT_GGUF_Q4_0
    d.qdata = held["q"].data_ptr()
    d.b = held["b"].data_ptr()
    d.a = held["a"].data_ptr()
    return d, held


def _collect(cs: Case, held):
    from merge_cases import f32np, u8np

    out = {}
    if cs.fmt.startswith("int8"):
        out["q"] = held["q"].cpu().numpy()
        out["scale"] = f32np(held["scale"])
    else:
        out["q"] = u8np(held["q"])
        if "scale" in held:
            out["scale"] = f32np(held["scale"]) if cs.fmt.startswith("fp8") else u8np(held["scale"])
    if "g" in held:
        out["global"] = float(held["g"].cpu())
    return out


def test_argument_errors_raise_before_mutation(cuda_device):
    c = Case("fp8_row", 64, 256, 16).build()
    q = c.tensors["q"]
    qd = q.qdata.to(cuda_device)
    before = qd.clone()
    b = c.tensors["b"].to(cuda_device)
    a = c.tensors["a"].to(cuda_device)
    with pytest.raises(ValueError):
        K.merge_float8_lora(qd, q.scale.to(cuda_device), (1, 256), b[:, :8], a, 1.0)
    with pytest.raises(ValueError):
        K.merge_float8_lora(qd, q.scale.to(cuda_device), (3, 7), b, a, 1.0)
    big_b = torch.zeros((64, 257), dtype=torch.bfloat16, device=cuda_device)
    big_a = torch.zeros((257, 256), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError, match="rank above 256"):
        K.merge_float8_lora(qd, q.scale.to(cuda_device), (1, 256), big_b, big_a, 1.0)
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(qd, before)

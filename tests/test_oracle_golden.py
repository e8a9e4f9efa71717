"""CPU: pin the oracle (and the product's host seeding) to the reference's golden vectors.

Fixtures in tests/golden were produced by ``tests/golden/make_golden.py`` from
Piper Offload 0.2.5's own code (derive_seed, the Triton ``_random`` stream
under the Triton CPU interpreter, ``gguf_dequant``) and from gguf 0.19.0's
quantizers.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import merge as om
from oracle import numerics as nm
from oracle.philox import philox_uniform
from piper_offload_b200.seeding import derive_seed

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_derive_seed_reference_golden():
    # tests/test_stochastic_rounding.py:25 of the reference
    assert derive_seed("layer.0.weight", 0) == 0x9C3EA68DBAC91AAD


def test_derive_seed_fixture_vectors():
    for entry in json.loads((GOLDEN / "seeds.json").read_text()):
        assert derive_seed(*entry["parts"]) == entry["seed"], entry["parts"]


def test_derive_seed_rejects_bad_parts():
    with pytest.raises(ValueError):
        derive_seed(-1)
    with pytest.raises(ValueError):
        derive_seed(1 << 64)
    with pytest.raises(TypeError):
        derive_seed(True)
    with pytest.raises(TypeError):
        derive_seed(1.5)


def test_philox_matches_reference_stream():
    for entry in json.loads((GOLDEN / "philox.json").read_text()):
        u = philox_uniform(entry["seed"], np.array(entry["offsets"], dtype=np.uint64))
        assert np.array_equal(u.view(np.int32), np.array(entry["uniform_bits"], dtype=np.int32)), hex(entry["seed"])


def test_philox_survey_kat():
    seed = derive_seed("layer.0.weight", 0)
    offs = np.array([0, 1, 2, 3, 4095, 16777215, 2**32 + 5], dtype=np.uint64)
    want = [0.574550986289978, 0.46430733799934387, 0.5867659449577332, 0.17042607069015503,
            0.5754178762435913, 0.8808434009552002, 0.11858648806810379]
    assert philox_uniform(seed, offs).tolist() == want


def test_gguf_dequant_matches_reference():
    g = np.load(GOLDEN / "gguf.npz")
    for name, qt in (("q8_0", om.Q8_0), ("q4_0", om.Q4_0)):
        raw = g[f"{name}_raw"]
        rows = raw.shape[0]
        cols = raw.shape[1] // (34 if qt == om.Q8_0 else 18) * 32
        ours = om.gguf_dequant(raw, qt, rows, cols, "bf16")
        want = (g[f"{name}_dequant_bf16_bits"].astype(np.uint16).astype(np.uint32) << 16).view(np.float32)
        assert np.array_equal(ours.view(np.uint32), want.view(np.uint32)), name


def test_gguf_quantize_matches_gguf_package():
    g = np.load(GOLDEN / "gguf.npz")
    for name, qt in (("q8_0", om.Q8_0), ("q4_0", om.Q4_0)):
        vals = g[f"{name}_values"]
        ours = om.gguf_quantize(vals, qt)
        assert np.array_equal(ours, g[f"{name}_quantized"]), name


def test_gguf_quantize_matches_live_gguf():
    gguf = pytest.importorskip("gguf")
    rng = np.random.default_rng(7)
    vals = (rng.standard_normal((8, 256)) * 0.015).astype(np.float32)
    vals[3, :32] = 0
    for qt in (om.Q8_0, om.Q4_0):
        want = gguf.quants.quantize(vals, gguf.GGMLQuantizationType(qt))
        assert np.array_equal(om.gguf_quantize(vals, qt), want)


def test_fp8_codecs_match_torch():
    codes = np.arange(256, dtype=np.uint8)
    for dt, dec in ((torch.float8_e4m3fn, nm.decode_e4m3), (torch.float8_e5m2, nm.decode_e5m2)):
        ref = torch.from_numpy(codes.copy()).view(dt).float().numpy()
        ours = dec(codes)
        same = (ref == ours) | (np.isnan(ref) & np.isnan(ours))
        assert same.all()
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000) * 50, rng.standard_normal(20000) * 1e-2,
                        np.array([0.0, -0.0, 448.0, -448.0, 1.0625, 0.0009765625 * 1.5])]).astype(np.float32)
    x = np.clip(x, -448, 448)
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(nm.encode_e4m3(x), want)
    y = np.clip(x * 100, -57344, 57344).astype(np.float32)
    want5 = torch.from_numpy(y).to(torch.float8_e5m2).view(torch.uint8).numpy()
    assert np.array_equal(nm.encode_e5m2(y), want5)


def test_fp8_saturates_like_satfinite():
    assert nm.encode_e4m3(np.array([1000.0, -1e30, np.inf], np.float32)).tolist() == [0x7E, 0xFE, 0x7E]
    assert nm.encode_e5m2(np.array([1e6], np.float32)).tolist() == [0x7B]


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(100000) * np.exp(rng.uniform(-30, 30, 100000))).astype(np.float32)
    want = torch.from_numpy(x).bfloat16().float().numpy()
    assert np.array_equal(nm.bf16_round(x), want)


def test_e2m1_ladder_is_rtne_on_grid():
    grid = nm.E2M1_VALUES.astype(np.float64)
    xs = np.linspace(0, 6.5, 6501).astype(np.float32)
    codes = nm.encode_e2m1(xs) & 7
    for x, c in zip(xs, codes):
        xm = min(float(x), 6.0)
        d = np.abs(grid - xm)
        best = np.flatnonzero(d == d.min())
        expect = best[0] if len(best) == 1 else [b for b in best if b % 2 == 0][0]
        assert c == expect, (x, c, expect)
    assert nm.encode_e2m1(np.array([-0.0, -0.1], np.float32)).tolist() == [8, 8]


def test_e8m0_decode_edges():
    v = nm.decode_e8m0(np.array([0, 1, 127, 254, 255], np.uint8))
    assert v[0] == np.float32(2.0 ** -127) and v[1] == np.float32(2.0 ** -126)
    assert v[2] == 1.0 and v[3] == np.float32(2.0 ** 127) and np.isnan(v[4])


def test_mx_zero_update_is_idempotent_on_floor_quantized_weight():
    from piper_offload_b200 import synthetic as S

    w = S.normal((64, 256), 0.02, seed=3, device="cpu", outlier_frac=0.01)
    q = S.quantize_mx(w, "e4m3")
    b = np.zeros((64, 16), np.float32)
    a = np.zeros((16, 256), np.float32)
    qd = q.qdata.view(torch.uint8).numpy()
    nq, ns = om.merge_mx(qd, q.scale.numpy(), "e4m3", b, a, 1.0)
    assert np.array_equal(ns, q.scale.numpy())
    assert np.array_equal(nq, qd)


def test_merge_stays_within_half_step_of_exact_update():
    """Dequantized oracle merge vs. a plain fp32 reference of dequant + s*B@A."""
    from piper_offload_b200 import synthetic as S

    w = S.normal((32, 512), 0.02, seed=5, device="cpu")
    q = S.quantize_fp8(w)
    b, a = S.lora_factors(32, 512, 16, 0.01, seed=6, device="cpu")
    bf, af = b.float().numpy(), a.float().numpy()
    nq, ns = om.merge_float8(q.qdata.view(torch.uint8).numpy(), q.scale.numpy(), (1, 512), bf, af, 1.0)
    deq_new = nm.decode_e4m3(nq) * ns
    exact = (q.qdata.float() * q.scale).bfloat16().float().numpy() + bf @ af
    # half of the largest e4m3 step (2^-3 relative) times the row scale
    tol = 0.0625 * np.abs(exact).max(axis=1, keepdims=True) * 1.01
    assert (np.abs(deq_new - exact) <= tol).all()


def test_sr_int_probability_fixture():
    """INT8 SR probability P(upper) = frac(x/scale) (test_stochastic_quantized_merge.py:711-743)."""
    vals = np.full(200000, 0.3, np.float32)
    det = np.zeros_like(vals)
    offs = np.arange(vals.size, dtype=np.uint64)
    out = om.sr_round_to_int(vals, det, 42, offs, -128, 127)
    assert abs(out.mean() - 0.3) < 0.005


def test_bnb8_decode_multiply_equals_division_for_every_code():
    # The kernel decodes bitsandbytes codes as f16(cb * fp32(1/127)); the reference
    # computes f16(cb / 127.0) (_triton_bnb8_lora.py:67). Equal over the whole int8 domain.
    q = np.arange(-128, 128, dtype=np.float32)
    div = (q / np.float32(127.0)).astype(np.float32).astype(np.float16)
    mul = (q * (np.float32(1.0) / np.float32(127.0))).astype(np.float32).astype(np.float16)
    assert np.array_equal(div.view(np.uint16), mul.view(np.uint16))

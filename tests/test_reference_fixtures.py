"""CPU: the oracle against the reference's own Triton merge kernels, bit for bit.

The fixtures (``tests/golden/merge_reference.*``) were recorded from the
raw-buffer launchers of the reference (``merge_float8_lora``,
``merge_int8_lora``, ``merge_nvfp4_lora``, ``merge_mx_lora_``,
``merge_static_float8_lora``, ``merge_bnb8_lora``, ``merge_quanto_qint8_lora``,
``merge_quanto_qfloat8_lora``) at the
reference tests' shapes, across layouts, scale modes, swizzling, rounding
modes, factor and scale dtypes, negative strengths and zero factors. The
interpreter divides in IEEE fp32, by a tensor and by a constant alike, so the
oracle runs here without its GPU-division hook and with IEEE constant
division (on the GPU, Triton multiplies by the constant's fp32 reciprocal).
"""

from __future__ import annotations

import pytest

import reference_fixtures as rf
from oracle import numerics as onum

CASES = rf.cases()


@pytest.fixture(scope="module", autouse=True)
def interpreter_division():
    # The interpreter divides by constants in IEEE fp32 and rounds every
    # operation on its own (no fp32 contraction).
    onum.set_constant_division("ieee")
    onum.set_fp32_contraction("separate")
    yield
    onum.set_constant_division("reciprocal")
    onum.set_fp32_contraction("gpu")


def test_fixture_coverage():
    launchers = {c["launcher"] for c in CASES}
    assert launchers == {"float8", "int8", "nvfp4", "mx", "static_float8", "bnb8", "quanto", "bnb4"}
    assert {c["elem"] for c in CASES if c["launcher"] == "mx"} == {"e4m3", "e5m2", "e2m1"}
    assert {c["scaling_mode"] for c in CASES if c["launcher"] == "mx"} == {0, 1, 2, 3}
    assert any(c["seed"] is not None for c in CASES) and any(c["seed"] is None for c in CASES)


@pytest.mark.parametrize("case", CASES, ids=[c["id"] + "-" + rf.case_label(c) for c in CASES])
def test_oracle_matches_reference_kernels(case):
    got = rf.oracle(case)
    want = rf.expected(case)
    bad = {k: v[:8].tolist() for k, v in rf.mismatches(got, want).items() if v.size}
    assert not bad, bad

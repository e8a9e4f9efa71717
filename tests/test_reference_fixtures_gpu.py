"""GPU: the sm_100a merge on the inputs the reference's own Triton kernels were recorded on.

Each fixture case (``tests/golden/merge_reference.*``) runs through
``piper_offload_b200.kernels``. Two checks, both exact:

* against the oracle evaluated with the GPU's tensor-by-tensor division
  (``oracle.gpu_division``): every code, scale, zero point and global scale;
* against the reference's recorded outputs: the only differing elements are
  those where the GPU's ``div.full`` quotient and the IEEE quotient of the
  recording differ, i.e. exactly where the GPU-division oracle differs from
  the recording.
"""

from __future__ import annotations

import numpy as np
import pytest

import reference_fixtures as rf

pytestmark = pytest.mark.gpu

CASES = rf.cases()


@pytest.fixture(scope="module", autouse=True)
def _gpu_division(cuda_device):
    from oracle import gpu_division

    gpu_division.install()
    yield
    gpu_division.uninstall()


@pytest.mark.parametrize("case", CASES, ids=[c["id"] + "-" + rf.case_label(c) for c in CASES])
def test_native_matches_reference_kernels(case, cuda_device):
    got = rf.native(case, cuda_device)
    oracle = rf.oracle(case)
    bad = {k: v[:8].tolist() for k, v in rf.mismatches(got, oracle).items() if v.size}
    assert not bad, f"native vs GPU-division oracle: {bad}"
    want = rf.expected(case)
    vs_ref = rf.mismatches(got, want)
    explained = rf.mismatches(oracle, want)
    for k in want:
        assert np.array_equal(vs_ref[k], explained[k]), (k, vs_ref[k][:8].tolist(), explained[k][:8].tolist())


def test_torch_cuda_divides_by_host_scalar_through_its_reciprocal(cuda_device):
    # Quanto's scale recompute, ``(amax / qmax).to(dtype)``, runs in torch on the
    # device; the fixtures and the kernels take it as amax * fp32(1 / qmax).
    import torch

    g = torch.Generator(device=cuda_device).manual_seed(0)
    for dt in (torch.bfloat16, torch.float16, torch.float32):
        x = (torch.rand(1 << 20, generator=g, device=cuda_device) * 4.0).to(dt)
        for qmax in (127.0, 448.0, 57344.0):
            inv = torch.tensor(float(np.float32(1.0) / np.float32(qmax)), dtype=torch.float32, device=cuda_device)
            assert torch.equal(x / qmax, (x.float() * inv).to(dt)), (dt, qmax)


def test_bnb4_unsorted_table_follows_the_binary_search(cuda_device):
    # NF4 code selection is the reference's binary search (_triton_bnb4_lora.py:29-50).
    # For a sorted table the kernel counts entries instead; an unsorted table must
    # still give the binary search's answer.
    case = next(c for c in CASES if c["launcher"] == "bnb4" and c["quant_type"] == "nf4" and not c["nested"]
                and c["seed"] is None)
    code = rf.arr(case, "code").copy()
    code[[3, 11]] = code[[11, 3]]
    arrays = rf._load()[1]
    key = f"{case['id']}.code"
    saved = arrays[key]
    arrays[key] = code
    try:
        got = rf.native(case, cuda_device)
        want = rf.oracle(case)
    finally:
        arrays[key] = saved
    bad = {k: v[:8].tolist() for k, v in rf.mismatches(got, want).items() if v.size}
    assert not bad, bad

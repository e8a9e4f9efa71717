"""GPU: the kernels' bounded waits fail soft. A self-test kernel waits on a
barrier that nothing arrives on; the wait gives up after its limit, the
device status word reports the timeout (and is cleared by reading it), and
the CUDA context stays usable: a merge right afterwards still matches the
oracle. No GPU fault, trap or hang is involved."""

from __future__ import annotations

import time

import pytest
import torch

from merge_cases import Case, compare
from piper_offload_b200 import _native as nat

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu_division(cuda_device):
    # The oracle's tensor-by-tensor quotients use the GPU's division, as in the
    # parity tests, so the follow-up merge is compared exactly.
    from oracle import gpu_division

    gpu_division.install()
    yield
    gpu_division.uninstall()


def test_bounded_wait_times_out_and_reports(cuda_device):
    lib = nat.load()
    assert nat.device_status(cuda_device) in (0, 1, 2, 3)  # clear anything left over
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    t0 = time.monotonic()
    assert lib.piper_merge_selftest_timeout(stream) == nat.OK
    status = nat.device_status(cuda_device)
    elapsed = time.monotonic() - t0
    assert status & 1, status  # kStatusTimeoutLoad
    assert 1.0 < elapsed < 30.0, elapsed
    assert nat.device_status(cuda_device) == 0
    # The context is intact: an ordinary merge still matches the oracle exactly.
    case = Case("fp8_row", 70, 130, 7, seed=None).build(data_seed=3)
    got = case.run_native(cuda_device)
    d = compare(case, got, case.run_oracle())
    assert d.code_mismatch == 0 and d.scale_mismatch == 0, d

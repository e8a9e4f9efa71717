"""GPU: GGUF Q8_0 / Q4_0 stochastic rounding is unbiased.

The reference has no GGUF merge and so no reference noise stream to match;
its own statistical test for counter-based integer rounding
(``tests/test_stochastic_quantized_merge.py:956-980``: all-zero codes, a rank-1
update of 0.3 with one larger element, 64 seeds, mean within 5e-4) is the
model here. Two checks per format:

* known answer: every block holds 31 elements of bf16(0.3) and one of 1.0, so
  the block scale is fixed by the 1.0 and each 0.3 lies strictly between two
  codes (Q8_0: 0.3 * 127 = 38.2 on the grid 1/127; Q4_0: 0.3 / -0.125 + 8 = 5.6);
  over 64 seeds the mean dequantized value of those elements is within a bound
  of the merged value (the bound covers the fp16 rounding of the stored scale
  and the sampling error, ~0.5 code step / sqrt(64 * elements));
* random weights (the config-5 distributions): the mean of 64 stochastic
  merges is closer to the exact merged values than half the round-to-nearest
  error.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import merge as om
from piper_offload_b200 import _native
from piper_offload_b200 import kernels as K
from piper_offload_b200 import synthetic as S
from piper_offload_b200.seeding import derive_seed

pytestmark = pytest.mark.gpu

FORMATS = [(8, "q8_0"), (2, "q4_0")]


def dequant(raw: torch.Tensor, qt: int, rows: int, cols: int) -> np.ndarray:
    return om.gguf_dequant(raw.cpu().numpy(), qt, rows, cols, compute="f32").astype(np.float64)


@pytest.mark.parametrize("qt,name", FORMATS, ids=[f[1] for f in FORMATS])
def test_gguf_sr_known_answer(qt, name, cuda_device):
    rows, cols = 16, 64
    bytes_per_row = cols // 32 * (34 if qt == 8 else 18)
    zero = torch.zeros((rows, bytes_per_row), dtype=torch.uint8, device=cuda_device)  # d = 0: every base is 0
    b = torch.ones((rows, 1), dtype=torch.bfloat16, device=cuda_device)
    a = torch.full((1, cols), 0.3, dtype=torch.bfloat16, device=cuda_device)
    a[0, 31::32] = 1.0
    target = float(torch.tensor(0.3, dtype=torch.bfloat16).float())
    mask = np.ones((rows, cols), bool)
    mask[:, 31::32] = False
    samples = []
    for s in range(64):
        raw = zero.clone()
        K.merge_gguf_lora_(raw, qt, b, a, 1.0, rounding_seed=derive_seed("gguf-statistical", s))
        vals = dequant(raw, qt, rows, cols)
        # the block maximum takes the top code (Q8_0: 127 * fp16(1/127); Q4_0: exactly 1.0)
        assert np.allclose(vals[:, 31::32], 1.0, rtol=2.0**-10, atol=0)
        samples.append(vals[mask])
    observed = float(np.mean(samples))
    # Q8_0 stores d = fp16(1/127): relative error <= 2^-11 of 0.3; Q4_0's d = -0.125 is exact.
    bound = 5e-4 + (0.3 * 2.0**-11 if qt == 8 else 0.0)
    assert abs(observed - target) < bound, (name, observed, target)
    # and it is genuinely stochastic: both neighbouring codes occur
    assert len(np.unique(np.concatenate(samples))) == 2


@pytest.mark.parametrize("qt,name", FORMATS, ids=[f[1] for f in FORMATS])
def test_gguf_sr_mean_beats_rtn(qt, name, cuda_device):
    rows, cols, rank = 64, 1024, 16
    w = S.normal((rows, cols), 0.015, seed=21, device="cpu")
    q = S.quantize_gguf(w, qt)
    b, a = S.lora_factors(rows, cols, rank, 0.01, seed=22, device="cpu")
    base = om.gguf_dequant(q.qdata.numpy(), qt, rows, cols, compute="bf16")
    exact = om.merged_values(base, om.lora_delta(b.float().numpy(), a.float().numpy()), 1.0, "bf16")
    exact = exact.astype(np.float64)
    bd, ad = b.to(cuda_device), a.to(cuda_device)
    acc = np.zeros((rows, cols))
    n = 64
    for s in range(n):
        raw = q.qdata.to(cuda_device).clone()
        K.merge_gguf_lora_(raw, qt, bd, ad, 1.0, rounding_seed=derive_seed("gguf-mean", s))
        acc += dequant(raw, qt, rows, cols)
    assert _native.device_status(cuda_device) == 0
    mean_err = np.abs(acc / n - exact).mean() / np.abs(exact).mean()
    raw = q.qdata.to(cuda_device).clone()
    K.merge_gguf_lora_(raw, qt, bd, ad, 1.0)
    rtn_err = np.abs(dequant(raw, qt, rows, cols) - exact).mean() / np.abs(exact).mean()
    assert mean_err < 0.5 * rtn_err, (name, mean_err, rtn_err)

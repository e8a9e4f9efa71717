"""GPU: batched factor staging (one host-to-device copy per device) and its merge results."""

from __future__ import annotations

import pytest
import torch

from piper_offload_b200 import synthetic as S
from piper_offload_b200 import transform as TR
from piper_offload_b200 import weights as WT


def _fp8_weight(shape, seed, device):
    q = S.quantize_fp8(S.normal(shape, 0.02, seed=seed, device=device))
    return WT.Float8Weight(q.qdata, q.scale, (1, shape[1]))

pytestmark = pytest.mark.gpu


def _factors(g, rows, cols, rank, strength):
    return TR.LoRAFactor(torch.randn(rank, cols, generator=g) * 0.01, torch.randn(rows, rank, generator=g) * 0.01,
                         strength=strength)


def test_stage_factors_one_copy_and_equal_values(cuda_device):
    g = torch.Generator().manual_seed(5)
    shapes = [(256, 512), (384, 256), (128, 1024)]
    pairs = []
    for i, (rows, cols) in enumerate(shapes):
        w = _fp8_weight((rows, cols), i, cuda_device)
        fs = [_factors(g, rows, cols, 16, 1.0)] if i != 1 else [_factors(g, rows, cols, 8, 0.75),
                                                                 _factors(g, rows, cols, 4, -1.25)]
        pairs.append((TR.LoRATransform(fs), w))
    staged = TR.stage_factors(pairs)
    storages = {b.untyped_storage().data_ptr() for b, _, _ in staged} | {a.untyped_storage().data_ptr()
                                                                          for _, a, _ in staged}
    assert len(storages) == 1  # every factor of the batch came over in one copy
    for (tr, x), (b, a, s) in zip(pairs, staged):
        assert b.device == x.qdata.device and a.data_ptr() % 16 == 0 and b.data_ptr() % 16 == 0
        rb, ra, rs = tr._stage(x, tr._make_plan(x))
        assert s == rs and torch.equal(b, rb) and torch.equal(a, ra)


def test_merge_lora_with_host_factors_equals_per_weight_merges(cuda_device):
    g = torch.Generator().manual_seed(6)
    shapes = {"q": (256, 512), "k": (128, 512), "o": (512, 256)}
    lora1 = {n: (torch.randn(16, c, generator=g) * 0.01, torch.randn(r, 16, generator=g) * 0.01)
             for n, (r, c) in shapes.items()}
    lora2 = {"q": (torch.randn(8, 512, generator=g) * 0.01, torch.randn(256, 8, generator=g) * 0.01)}

    def build():
        return {n: _fp8_weight(sh, j, cuda_device) for j, (n, sh) in enumerate(shapes.items())}

    batched = build()
    TR.merge_lora(batched, [(lora1, 1.0), (lora2, 0.5)], stochastic_rounding=True)
    single = build()
    grouped = {n: [TR.LoRAFactor(lora1[n][0], lora1[n][1], 1.0)] for n in shapes}
    grouped["q"].append(TR.LoRAFactor(lora2["q"][0], lora2["q"][1], 0.5))
    for n, fs in grouped.items():
        tr = TR.LoRATransform(fs, stochastic_rounding=True, target_key=n)
        tr.validate_target(single[n])
        tr.apply_weight(single[n])
    torch.cuda.synchronize()
    for n in shapes:
        assert torch.equal(batched[n].qdata.view(torch.uint8), single[n].qdata.view(torch.uint8)), n
        assert torch.equal(batched[n].scale, single[n].scale), n

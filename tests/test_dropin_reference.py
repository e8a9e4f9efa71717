"""The B200 launchers as a drop-in for the reference's own API.

CPU: the launchers of ``piper_offload_b200.kernels`` take exactly the
reference launchers' parameters (names, kinds, defaults), plus the keyword
``offset_base``; and ``integration.install`` rebinds the names each reference
adapter imported and registers the GGUF merge adapter, and its undo restores
both.

GPU: the reference's unchanged ``merge_lora()`` (``merge.py:54``) merges a
LoRA built by its own ``LoRA.from_state_dict`` into a module whose weight is
the reference's own ``GGUFWeight`` (``gguf_adapter.py:61-105``), through the
registered B200 GGUF adapter; the raw blocks equal the oracle's merge with the
seed the reference derives (``lora.py:356-359``: ``derive_seed(key, 0)``).

The reference is imported from ``baseline/_ref`` (``baseline/reference.py``);
the module is skipped without it.
"""

from __future__ import annotations

import inspect

import numpy as np
import pytest
import torch

from piper_offload_b200 import integration
from piper_offload_b200 import kernels as K

PAIRS = [("merge_float8_lora", "_triton_float8_lora"), ("merge_int8_lora", "_triton_int8_lora"),
         ("merge_nvfp4_lora", "_triton_nvfp4_lora"), ("merge_mx_lora_", "_triton_mx_lora"),
         ("merge_static_float8_lora", "_triton_static_float8_lora"), ("merge_bnb8_lora", "_triton_bnb8_lora"),
         ("merge_bnb4_lora", "_triton_bnb4_lora"), ("merge_quanto_qint8_lora", "_triton_quanto_lora"),
         ("merge_quanto_qfloat8_lora", "_triton_quanto_lora")]


@pytest.fixture(scope="module")
def po():
    from baseline import reference

    if not reference.available():
        pytest.skip("reference not installed under baseline/_ref")
    pytest.importorskip("triton")
    pytest.importorskip("gguf")
    return reference.load("piper_offload")


def _params(fn):
    return [(p.name, p.kind, p.default) for p in inspect.signature(fn).parameters.values() if p.name != "offset_base"]


@pytest.mark.parametrize("name,module", PAIRS, ids=[p[0] for p in PAIRS])
def test_launcher_signatures_match_the_reference(po, name, module):
    ref = getattr(__import__(f"{po.__name__}.{module}", fromlist=[name]), name)
    ours = getattr(K, name)
    assert _params(ours) == _params(ref)
    extra = inspect.signature(ours).parameters["offset_base"]
    assert extra.kind is inspect.Parameter.KEYWORD_ONLY and extra.default == 0


def test_install_binds_and_undo_restores(po):
    from piper_offload import float8_adapter, int8_adapter, mx_adapter, nvfp4_adapter
    from piper_offload.tensor_adapter_registry import _REGISTERED_ADAPTERS

    before = (float8_adapter._triton_merge_float8_lora, int8_adapter._triton_merge_int8_lora,
              mx_adapter._triton_merge_mx_lora_, nvfp4_adapter._triton_merge_nvfp4_lora, list(_REGISTERED_ADAPTERS))
    undo = integration.install(po)
    try:
        assert float8_adapter._triton_merge_float8_lora is K.merge_float8_lora
        assert int8_adapter._triton_merge_int8_lora is K.merge_int8_lora
        assert mx_adapter._triton_merge_mx_lora_ is K.merge_mx_lora_
        assert nvfp4_adapter._triton_merge_nvfp4_lora is K.merge_nvfp4_lora
        assert float8_adapter._TRITON_MAX_GROUP_SIZE == K.MAX_GROUP_SIZE
        assert _REGISTERED_ADAPTERS[0].__name__ == "B200GgufAdapter"
    finally:
        undo()
    after = (float8_adapter._triton_merge_float8_lora, int8_adapter._triton_merge_int8_lora,
             mx_adapter._triton_merge_mx_lora_, nvfp4_adapter._triton_merge_nvfp4_lora, list(_REGISTERED_ADAPTERS))
    assert after == before


@pytest.mark.gpu
@pytest.mark.parametrize("stochastic", [False, True], ids=["rtn", "sr"])
@pytest.mark.parametrize("quant_type", [8, 2], ids=["q8_0", "q4_0"])
def test_reference_merge_lora_drives_the_b200_gguf_merge(po, cuda_device, quant_type, stochastic):
    from oracle import merge as om
    from piper_offload import LoRA, merge_lora
    from piper_offload.gguf_adapter import GGUFWeight
    from piper_offload.seeding import derive_seed
    from piper_offload_b200 import synthetic as S

    rows, cols, rank = 96, 512, 8
    w = S.normal((rows, cols), 0.015, seed=31, device="cpu")
    raw = S.quantize_gguf(w, quant_type).qdata
    # Small-integer multiples of 2^-8: every dot product is exact in any
    # summation order, so the blocks must equal the oracle's bit for bit.
    g = torch.Generator().manual_seed(32)
    b = torch.randint(-15, 16, (rows, rank), generator=g).float() * 2.0**-8
    a = torch.randint(-15, 16, (rank, cols), generator=g).float() * 2.0**-8

    class M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = torch.nn.Module()
            self.lin.weight = torch.nn.Parameter(GGUFWeight(raw.to(cuda_device), quant_type=quant_type),
                                                 requires_grad=False)

    model = M()
    lora = LoRA.from_state_dict({"lin.lora_A.weight": a, "lin.lora_B.weight": b})
    undo = integration.install(po)
    try:
        assert merge_lora(model, [(lora, 0.5)], stochastic_rounding=stochastic) == 1
    finally:
        undo()
    torch.cuda.synchronize(cuda_device)
    got = model.lin.weight.as_subclass(torch.Tensor).cpu().numpy()
    # LoRATransform stages the factors in the adapter's compute dtype (bf16).
    b16 = b.to(torch.bfloat16).float().numpy()
    a16 = a.to(torch.bfloat16).float().numpy()
    seed = derive_seed("lin.weight", 0) if stochastic else None
    want = om.merge_gguf(raw.numpy(), quant_type, b16, a16, 0.5, seed=seed)
    assert np.array_equal(got, want)

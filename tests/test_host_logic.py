"""CPU: host-side logic of the merge path (no device compute)."""

from __future__ import annotations

import pytest
import torch

from piper_offload_b200 import adapters as AD
from piper_offload_b200 import kernels as K
from piper_offload_b200 import sharding as SH
from piper_offload_b200 import transform as TR
from piper_offload_b200 import weights as WT
from piper_offload_b200.seeding import derive_seed


# ----------------------------------------------------------- DTensor rules
def test_local_shape_and_offsets_matches_dtensor_rules():
    from torch.distributed.tensor import Replicate, Shard

    g = (10, 7)
    shapes = [SH.local_shape_and_offsets(g, (4,), (i,), (Shard(0),)) for i in range(4)]
    assert shapes == [((3, 7), (0, 0)), ((3, 7), (3, 0)), ((3, 7), (6, 0)), ((1, 7), (9, 0))]
    assert SH.local_shape_and_offsets(g, (2, 2), (1, 1), (Shard(0), Shard(1))) == ((5, 3), (5, 4))
    assert SH.local_shape_and_offsets(g, (2,), (1,), (Replicate(),)) == ((10, 7), (0, 0))
    # repeated sharding of one dimension, and an empty shard anchored at the end
    assert SH.local_shape_and_offsets((3, 4), (4,), (3,), (Shard(0),)) == ((0, 4), (3, 0))
    assert SH.local_shape_and_offsets(g, (2, 2), (1, 1), (Shard(0), Shard(0))) == ((2, 7), (8, 0))
    with pytest.raises(ValueError):
        SH.local_shape_and_offsets(g, (2,), (0, 1), (Shard(0),))
    with pytest.raises(ValueError):
        SH.local_shape_and_offsets(g, (2,), (0,), (("partial",),))


def test_seed_localisation_and_modes():
    assert SH.localize_rounding_seed(None, (4, 0)) is None
    assert SH.localize_rounding_seed(5, (4, 0)) == derive_seed(5, 4, 0)
    seed, base = SH.shard_merge_args(5, global_shape=(100, 64), offsets=(40, 0), mode="dtensor")
    assert (seed, base) == (derive_seed(5, 40, 0), 0)
    assert SH.shard_merge_args(5, global_shape=(100, 64), offsets=(40, 0), mode="global") == (5, 40 * 64)
    with pytest.raises(ValueError):
        SH.shard_merge_args(5, global_shape=(100, 64), offsets=(40, 8), mode="global")


def test_local_lora_factors():
    b = torch.arange(20.0).reshape(10, 2)
    a = torch.arange(14.0).reshape(2, 7)
    lb, la = SH.local_lora_factors(b, a, global_shape=(10, 7), local_shape=(3, 4), offsets=(6, 3))
    assert torch.equal(lb, b[6:9]) and torch.equal(la, a[:, 3:7])
    lb2, la2 = SH.local_lora_factors(lb, la, global_shape=(10, 7), local_shape=(3, 4), offsets=(6, 3))
    assert torch.equal(lb2, lb)
    with pytest.raises(ValueError):
        SH.local_lora_factors(b[:5], a, global_shape=(10, 7), local_shape=(3, 4), offsets=(6, 3))


# ------------------------------------------------------------- partition
def _llama_items(layers=32):
    shapes = [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
              ("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)]
    return [SH.WorkItem(f"l{i}.{n}", r, c, c) for i in range(layers) for n, r, c in shapes]


@pytest.mark.parametrize("world", [1, 2, 4, 8, 3])
def test_partition_covers_each_row_once_and_balances(world):
    items = _llama_items()
    parts = SH.partition(items, world)
    covered = {}
    for shards in parts:
        for s in shards:
            covered.setdefault(s.key, []).append((s.row_begin, s.row_end))
    for it in items:
        spans = sorted(covered[it.key])
        assert spans[0][0] == 0 and spans[-1][1] == it.rows
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert all((r0 % 128) == 0 for r0, _ in spans)
    loads = [sum(s.bytes for s in shards) for shards in parts]
    assert max(loads) <= 1.1 * (sum(loads) / world)


def test_partition_keeps_per_tensor_weights_whole():
    items = [SH.WorkItem("big", 8192, 8192, 8192, row_splittable=False), SH.WorkItem("small", 128, 128, 128)]
    parts = SH.partition(items, 4)
    assert sum(1 for p in parts for s in p if s.key == "big") == 1
    shard = next(s for p in parts for s in p if s.key == "big")
    assert (shard.row_begin, shard.row_end) == (0, 8192) and shard.offset_base == 0


# ---------------------------------------------------------- raw launchers
def test_raw_launchers_reject_cpu_tensors():
    q = torch.zeros(4, 32, dtype=torch.float8_e4m3fn)
    with pytest.raises(ValueError, match="CUDA"):
        K.merge_float8_lora(q, torch.ones(4, 1), (1, 32), torch.zeros(4, 2, dtype=torch.bfloat16),
                            torch.zeros(2, 32, dtype=torch.bfloat16), 1.0)
    with pytest.raises(ValueError, match="CUDA"):
        K.merge_int8_lora(torch.zeros(4, 32, dtype=torch.int8), torch.ones(4, 1, dtype=torch.bfloat16), None,
                          (1, 32), torch.zeros(4, 2, dtype=torch.bfloat16),
                          torch.zeros(2, 32, dtype=torch.bfloat16), 1.0, asymmetric=False, reduce_range=False)


def test_layout_helpers():
    assert K.mx_expected_scale_shape(19, 96, swizzled=False) == (19, 3)
    assert K.mx_expected_scale_shape(300, 1024, swizzled=True) == (96, 128)
    assert K.nvfp4_expected_scale_shape(300, 1040, swizzled=True) == (96, 272)
    assert K.int8_block_numel((35, 69), (1, 69)) == 69
    assert K.int8_block_numel((35, 69), (35, 69)) == 35 * 69
    with pytest.raises(ValueError, match="per-group"):
        K.int8_block_numel((35, 69), (1, 10))
    q = torch.zeros(8, 512, dtype=torch.float8_e4m3fn)
    assert K.float8_layout(q, torch.ones(8, 1), (1, 512))[2] is True
    with pytest.raises(ValueError, match="up to 256"):
        K.float8_layout(torch.zeros(8, 1024, dtype=torch.float8_e4m3fn), torch.ones(8, 2), (1, 512))
    assert K.gguf_logical_cols(34 * 4, 8) == 128
    with pytest.raises(ValueError):
        K.gguf_logical_cols(35, 8)


def test_seed_fields():
    assert K._seed_fields(None) == (0, 0)
    assert K._seed_fields(5)[0] == 5
    assert K._seed_fields(-1)[0] == (1 << 64) - 1  # signed launch form of the same bits


# --------------------------------------------------------------- adapters
def test_adapter_selection_and_shapes():
    i8 = WT.Int8Weight(torch.zeros(4, 32, dtype=torch.int8), torch.ones(4, 1), (1, 32))
    f8 = WT.Float8Weight(torch.zeros(4, 32, dtype=torch.float8_e4m3fn), torch.ones(4, 1), (1, 32))
    nv = WT.NVFP4Weight(torch.zeros(4, 16, dtype=torch.uint8), torch.zeros(4, 2, dtype=torch.float8_e4m3fn))
    mx = WT.MXWeight(torch.zeros(4, 32, dtype=torch.float8_e4m3fn), torch.zeros(4, 1, dtype=torch.uint8),
                     torch.float8_e4m3fn)
    gg = WT.GGUFWeight(torch.zeros(4, 34, dtype=torch.uint8), 8)
    assert AD.select_adapter(i8) is AD.Int8Adapter
    assert AD.select_adapter(f8) is AD.Float8Adapter
    assert AD.select_adapter(nv) is AD.Nvfp4Adapter and AD.Nvfp4Adapter.logical_shape(nv) == (4, 32)
    assert AD.select_adapter(mx) is AD.MxAdapter
    assert AD.select_adapter(gg) is AD.GgufAdapter and AD.GgufAdapter.logical_shape(gg) == (4, 32)
    with pytest.raises(NotImplementedError):
        AD.select_adapter(torch.zeros(3))


def test_static_float8_adapter_selection_and_layout_rules():
    q = torch.zeros(4, 32, dtype=torch.float8_e4m3fn)
    st = WT.StaticFloat8Weight(q, torch.ones(()), torch.ones(()))
    assert AD.select_adapter(st) is AD.StaticFloat8Adapter  # ahead of the dynamic Float8Tensor adapter
    assert st.block_size == (4, 32) and AD.StaticFloat8Adapter.logical_shape(st) == (4, 32)
    b, a = torch.zeros(4, 2, dtype=torch.bfloat16), torch.zeros(2, 32, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="exactly one value"):
        AD.StaticFloat8Adapter.validate_lora_merge(WT.StaticFloat8Weight(q, torch.ones(()), torch.ones(2)), b, a, 1.0)
    with pytest.raises(ValueError, match="per-tensor FP8 weight layout"):
        AD.StaticFloat8Adapter.validate_lora_merge(WT.StaticFloat8Weight(q, torch.ones(()), torch.ones(()), (1, 32)),
                                                   b, a, 1.0)
    with pytest.raises(ValueError, match="CUDA"):
        AD.StaticFloat8Adapter.validate_lora_merge(st, b, a, 1.0)
    with pytest.raises(ValueError, match="CUDA"):
        K.merge_static_float8_lora(q, torch.ones(()), b, a, 1.0)


def test_bnb8_and_quanto_adapter_rules():
    cb = torch.zeros(4, 32, dtype=torch.int8)
    bnb = WT.Bnb8Weight(cb, torch.ones(4))
    assert AD.select_adapter(bnb) is AD.Bnb8Adapter and AD.Bnb8Adapter.compute_dtype(bnb) is torch.float16
    f16 = (torch.zeros(4, 2, dtype=torch.float16), torch.zeros(2, 32, dtype=torch.float16))
    bf16 = (torch.zeros(4, 2, dtype=torch.bfloat16), torch.zeros(2, 32, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="float16 LoRA factors"):
        AD.Bnb8Adapter.validate_lora_merge(bnb, *bf16, 1.0)
    with pytest.raises(ValueError, match="one SCB value per row"):
        AD.Bnb8Adapter.validate_lora_merge(WT.Bnb8Weight(cb, torch.ones(3)), *f16, 1.0)
    with pytest.raises(ValueError, match="CUDA"):
        AD.Bnb8Adapter.validate_lora_merge(bnb, *f16, 1.0)
    qrow = WT.QuantoWeight(cb, torch.ones(4, 1, dtype=torch.bfloat16), 0, WT.QINT8)
    assert AD.select_adapter(qrow) is AD.QuantoAdapter and AD.QuantoAdapter.compute_dtype(qrow) is torch.bfloat16
    with pytest.raises(ValueError, match="CUDA"):
        AD.QuantoAdapter.validate_lora_merge(qrow, *bf16, 1.0)
    qcol = WT.QuantoWeight(cb, torch.ones(1, 32, dtype=torch.bfloat16), -1, WT.QINT8)
    with pytest.raises(ValueError, match="CUDA"):
        AD.QuantoAdapter.validate_lora_merge(qcol, *bf16, 1.0)
    assert K.QUANTO_BLOCK["column"](4, 32) == (4, 1) and K.QUANTO_BLOCK["row"](4, 32) == (1, 32)
    with pytest.raises(ValueError, match="matching scale and factor dtypes"):
        AD.QuantoAdapter.validate_lora_merge(qrow, *f16, 1.0)
    with pytest.raises(ValueError, match="qtype metadata"):
        AD.QuantoAdapter.validate_lora_merge(WT.QuantoWeight(cb, torch.ones(4, 1, dtype=torch.bfloat16), 0,
                                                             WT.QFLOAT8_E4M3), *bf16, 1.0)
    with pytest.raises(ValueError, match="scalar scale, one scale per row"):
        K.quanto_scale_axis(0, torch.ones(3), 4, 32)
    assert K.quanto_scale_axis(None, torch.ones(()), 4, 32) == "tensor"
    assert K.quanto_scale_axis(-1, torch.ones(1, 32), 4, 32) == "column"


def test_bnb4_adapter_rules():
    code = torch.linspace(-1, 1, 16)
    qs = WT.Bnb4State(torch.ones(8), code, (4, 128))
    w4 = WT.Bnb4Weight(torch.zeros(256, 1, dtype=torch.uint8), qs)
    assert AD.select_adapter(w4) is AD.Bnb4Adapter and AD.Bnb4Adapter.logical_shape(w4) == (4, 128)
    b, a = torch.zeros(4, 2, dtype=torch.bfloat16), torch.zeros(2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        AD.Bnb4Adapter.validate_lora_merge(w4, b, a, 1.0)
    with pytest.raises(ValueError, match="CUDA"):
        K.merge_bnb4_lora(w4.data, qs.absmax, code, None, None, None, (4, 128), 64, "nf4", b, a, 1.0)


def test_mx_scaling_mode_resolution():
    mx = WT.MXWeight(torch.zeros(1, 32, dtype=torch.float8_e4m3fn), torch.zeros(1, 1), torch.float8_e4m3fn)
    assert AD.mx_scaling_mode_id(mx) == 0
    mx.act_quant_kwargs = WT.MXActQuantKwargs(WT.MXScalingMode("rceil"))
    assert AD.mx_scaling_mode_id(mx) == 1
    mx.act_quant_kwargs = WT.MXActQuantKwargs(WT.MXScalingMode("weird"))
    assert AD.mx_scaling_mode_id(mx) is None


def test_int8_act_pre_scale_folding():
    t = WT.Int8Weight(torch.zeros(4, 8, dtype=torch.int8), torch.ones(4, 1), (1, 8))
    a = torch.ones(2, 8, dtype=torch.bfloat16)
    same, s = AD.Int8Adapter.stored_factors(t, a, 0.5)
    assert same is a and s == 0.5
    t.act_pre_scale = torch.full((1, 8), 2.0)
    stored, s = AD.Int8Adapter.stored_factors(t, a, 0.5)
    assert s == 1.0 and torch.all(stored.float() == 0.25)
    t.act_pre_scale = torch.zeros(8)
    with pytest.raises(ValueError, match="non-zero"):
        AD.Int8Adapter.stored_factors(t, a, 0.5)
    t.act_pre_scale = torch.ones(3, 8)
    with pytest.raises(ValueError, match="scalar or one value per input feature"):
        AD.Int8Adapter.stored_factors(t, a, 0.5)


def test_nvfp4_rejects_grouped_global_scale():
    nv = WT.NVFP4Weight(torch.zeros(4, 16, dtype=torch.uint8), torch.zeros(4, 2, dtype=torch.float8_e4m3fn),
                        per_tensor_scale=torch.ones(2))
    with pytest.raises(ValueError, match="non-scalar per_tensor_scale"):
        AD.Nvfp4Adapter.validate_lora_merge(nv, torch.zeros(4, 2), torch.zeros(2, 32), 1.0)


# ------------------------------------------------------- transform (fake)
class FakeTarget:
    def __init__(self, rows, cols, dtype=torch.bfloat16, bad=False):
        self.rows, self.cols, self.dtype, self.bad = rows, cols, dtype, bad
        self.calls = []
        self.qdata = torch.zeros(1)


class FakeAdapter:
    @staticmethod
    def matches(t):
        return isinstance(t, FakeTarget)

    @staticmethod
    def logical_shape(t):
        return (t.rows, t.cols)

    @staticmethod
    def compute_dtype(t):
        return t.dtype

    @staticmethod
    def validate_lora_merge(t, b, a, s, *, rounding_seed=None):
        if t.bad:
            raise ValueError("fake layout rejected")

    @staticmethod
    def merge_desc(t, b, a, s, *, rounding_seed=None, offset_base=0, keep=None):
        t.calls.append((b.clone(), a.clone(), s, rounding_seed))
        return None

    @staticmethod
    def merge_lora_(t, b, a, s, *, rounding_seed=None, offset_base=0):
        t.calls.append((b.clone(), a.clone(), s, rounding_seed))


@pytest.fixture
def fake_adapter(monkeypatch):
    AD.register_adapter(FakeAdapter)
    monkeypatch.setattr(AD.nat, "merge_batch", lambda descs, dev, ws=None: None)
    yield
    AD._ADAPTERS.remove(FakeAdapter)


def test_transform_seeds_follow_merge_index(fake_adapter):
    t = FakeTarget(4, 6)
    f = TR.LoRAFactor(torch.ones(2, 6), torch.ones(4, 2))
    tr = TR.LoRATransform([f], stochastic_rounding=True, target_key="layer.0.weight")
    with pytest.raises(RuntimeError):
        tr.apply_weight(t)
    tr.validate_target(t)
    tr.apply_weight(t)
    tr.apply_weight(t)
    assert [c[3] for c in t.calls] == [derive_seed("layer.0.weight", 0), derive_seed("layer.0.weight", 1)]
    assert t.calls[0][0].dtype is torch.bfloat16


def test_transform_requires_key_for_sr_and_matching_shapes(fake_adapter):
    with pytest.raises(ValueError, match="target_key"):
        TR.LoRATransform([TR.LoRAFactor(torch.ones(2, 6), torch.ones(4, 2))], stochastic_rounding=True)
    tr = TR.LoRATransform([TR.LoRAFactor(torch.ones(2, 5), torch.ones(4, 2))])
    with pytest.raises(ValueError, match="shape mismatch"):
        tr.validate_target(FakeTarget(4, 6))


def test_transform_packs_multiple_factors(fake_adapter):
    t = FakeTarget(3, 4)
    f1 = TR.LoRAFactor(torch.full((2, 4), 1.0), torch.full((3, 2), 2.0), strength=0.5)
    f2 = TR.LoRAFactor(torch.full((1, 4), 3.0), torch.full((3, 1), 4.0), strength=2.0)
    tr = TR.LoRATransform([f1, f2])
    tr.validate_target(t)
    tr.apply_weight(t)
    b, a, s, seed = t.calls[-1]
    assert s == 1.0 and seed is None
    assert a.shape == (3, 4) and b.shape == (3, 3)
    assert torch.all(a[:2].float() == 0.5) and torch.all(a[2].float() == 6.0)
    assert torch.all(b[:, :2].float() == 2.0) and torch.all(b[:, 2].float() == 4.0)


def test_merge_lora_preflight_rejects_before_mutation(fake_adapter):
    good, bad = FakeTarget(4, 6), FakeTarget(4, 6, bad=True)
    lora = {"good": (torch.ones(2, 6), torch.ones(4, 2)), "bad": (torch.ones(2, 6), torch.ones(4, 2))}
    with pytest.raises(ValueError, match="fake layout rejected"):
        TR.merge_lora({"good": good, "bad": bad}, [(lora, 1.0)])
    assert good.calls == [] and bad.calls == []


def test_merge_lora_driver_rules(fake_adapter):
    w = {"a": FakeTarget(4, 6), "b": FakeTarget(4, 6)}
    l1 = {"a": (torch.ones(2, 6), torch.ones(4, 2))}
    with pytest.raises(ValueError, match="more than once"):
        TR.merge_lora(w, [(l1, 1.0), (l1, 1.0)])
    with pytest.raises(ValueError, match="missing"):
        TR.merge_lora(w, [({"zzz": (torch.ones(2, 6), torch.ones(4, 2))}, 1.0)])
    assert TR.merge_lora(w, [(l1, 0.0)]) == 0
    n = TR.merge_lora(w, [(l1, 1.0), ({"a": (torch.ones(1, 6), torch.ones(4, 1)), "b": (torch.ones(1, 6),
                                                                                          torch.ones(4, 1))}, 2.0)])
    assert n == 2
    b, a, s, seed = w["a"].calls[-1]
    assert a.shape == (3, 6) and seed == derive_seed("a", 0)


def test_validated_transform_stages_once(fake_adapter, monkeypatch):
    t = FakeTarget(4, 6)
    tr = TR.LoRATransform([TR.LoRAFactor(torch.ones(2, 6), torch.ones(4, 2))])
    calls = []
    orig = TR.LoRATransform._stage
    monkeypatch.setattr(TR.LoRATransform, "_stage", lambda self, x, plan: calls.append(1) or orig(self, x, plan))
    tr.validate_target(t)
    tr.apply_weight(t)
    assert len(calls) == 1  # validation's staging is reused by the application
    tr.apply_weight(t)
    assert len(calls) == 2  # a further application stages afresh


def test_stage_factors_matches_per_weight_staging(fake_adapter):
    g = torch.Generator().manual_seed(3)
    f1 = TR.LoRAFactor(torch.randn(2, 6, generator=g), torch.randn(4, 2, generator=g), strength=0.7)
    f2 = TR.LoRAFactor(torch.randn(3, 6, generator=g), torch.randn(4, 3, generator=g), strength=-1.5)
    pairs = [(TR.LoRATransform([f1]), FakeTarget(4, 6)), (TR.LoRATransform([f1, f2]), FakeTarget(4, 6)),
             (TR.LoRATransform([f2]), FakeTarget(4, 6, dtype=torch.float16))]
    staged = TR.stage_factors(pairs)
    for (tr, x), (b, a, s) in zip(pairs, staged):
        rb, ra, rs = tr._stage(x, tr._make_plan(x))
        assert s == rs and b.dtype == rb.dtype and a.dtype == ra.dtype
        assert torch.equal(b, rb) and torch.equal(a, ra)

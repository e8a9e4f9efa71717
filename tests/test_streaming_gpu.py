"""GPU: the streamed-block pipeline (host-resident weights merged through a
ring of device slots on upload / merge / download streams) gives the same
codes and scales as merging the same weights on the device with
``adapters.merge_lora_batch``, for mixed formats, stochastic rounding and a
ring shorter than the block count."""

from __future__ import annotations

import copy

import pytest
import torch

from piper_offload_b200 import adapters as AD
from piper_offload_b200 import synthetic as S
from piper_offload_b200 import weights as WT
from piper_offload_b200.seeding import derive_seed
from piper_offload_b200.streaming import StreamedOp, merge_streamed, storages

pytestmark = pytest.mark.gpu


def _weights(device, seed):
    out = []
    w = S.normal((256, 512), 0.02, seed=seed, device=device)
    q = S.quantize_fp8(w)
    out.append(WT.Float8Weight(q.qdata, q.scale, (1, 512)))
    w = S.normal((128, 256), 0.02, seed=seed + 1, device=device)
    q = S.quantize_mx(w, "e4m3")
    out.append(WT.MXWeight(q.qdata, q.scale.view(torch.float8_e8m0fnu), torch.float8_e4m3fn))
    w = S.normal((96, 512), 0.02, seed=seed + 2, device=device)
    q = S.quantize_gguf(w, 8)
    out.append(WT.GGUFWeight(q.qdata, 8))
    return out


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_streamed_merge_equals_device_batch(cuda_device, depth):
    blocks_dev, blocks_host = [], []
    for blk in range(5):
        dev_ops, host_ops = [], []
        for j, t in enumerate(_weights(cuda_device, 100 * blk)):
            key = f"model.layers.{blk}.w{j}.weight"
            rows = storages(t)[0][1].shape[0]
            cols = {0: 512, 1: 256, 2: 512}[j]
            b, a = S.lora_factors(rows, cols, 16, 0.01, seed=7 * blk + j, device=cuda_device)
            seed = derive_seed(key, 3) if j != 1 else None
            ht = copy.copy(t)
            for name, d in storages(t):
                setattr(ht, name, d.detach().cpu().pin_memory())
            host_ops.append(StreamedOp(ht, b.cpu().pin_memory(), a.cpu().pin_memory(), 1.0, seed))
            dev_ops.append((t, b, a, 1.0, seed))
        blocks_dev.append(dev_ops)
        blocks_host.append(host_ops)
    for ops in blocks_dev:
        AD.merge_lora_batch(ops)
    merge_streamed(blocks_host, cuda_device, depth=depth)
    torch.cuda.synchronize(cuda_device)
    for ops_d, ops_h in zip(blocks_dev, blocks_host):
        for (t, *_), op in zip(ops_d, ops_h):
            for (name, d), (_, h) in zip(storages(t), storages(op.target)):
                assert torch.equal(d.cpu().view(torch.uint8), h.view(torch.uint8)), name


def test_streamed_merge_rejects_device_storages(cuda_device):
    t = _weights(cuda_device, 1)[0]
    b, a = S.lora_factors(256, 512, 16, 0.01, seed=1, device=cuda_device)
    with pytest.raises(ValueError, match="host storages"):
        merge_streamed([[StreamedOp(t, b, a, 1.0)]], cuda_device)

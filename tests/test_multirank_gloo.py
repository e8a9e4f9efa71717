"""CPU, world_size 2 over gloo: the multi-GPU partition of a merge workload.

Each rank plans the same partition, merges its row shards with the oracle
(global-offset stochastic mode, so shards reproduce the unsharded stream) and
the results are all-gathered; rank 0 checks them against a single-process
merge of every weight. A second scenario drops one rank before it joins a
collective and checks that the survivor's collective fails instead of hanging.
Pattern follows the reference's tests/test_dtensor_lora_slicing.py:24-60
(``mp.spawn``, gloo over a FileStore).
"""

from __future__ import annotations

import os
import tempfile
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import merge as om
from piper_offload_b200 import sharding as SH
from piper_offload_b200 import synthetic as S

SEED = 0x9C3EA68DBAC91AAD
SHAPES = [("w0", 300, 256), ("w1", 128, 512), ("w2", 520, 128), ("w3", 64, 96)]


def _inputs(key: str, rows: int, cols: int):
    s = sum(map(ord, key))
    w = S.normal((rows, cols), 0.02, seed=s, device="cpu")
    q = S.quantize_fp8(w)
    b, a = S.lora_factors(rows, cols, 16, 0.01, seed=s + 1, device="cpu")
    return q.qdata.view(torch.uint8).numpy(), q.scale.numpy(), b.float().numpy(), a.float().numpy()


def _merge_shard(key, rows, cols, r0, r1):
    q, s, b, a = _inputs(key, rows, cols)
    nq, ns = om.merge_float8(q[r0:r1], s[r0:r1], (1, cols), b[r0:r1], a, 1.0, seed=SEED, offset_base=r0 * cols)
    return nq, ns


def _worker(rank: int, world: int, store_path: str, result_path: str):
    store = dist.FileStore(store_path, world)
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world, timeout=timedelta(seconds=60))
    items = [SH.WorkItem(k, r, c, c) for k, r, c in SHAPES]
    parts = SH.partition(items, world, granularity=128)
    mine = []
    for shard in parts[rank]:
        rows, cols = next((r, c) for k, r, c in SHAPES if k == shard.key)
        nq, ns = _merge_shard(shard.key, rows, cols, shard.row_begin, shard.row_end)
        mine.append((shard.key, shard.row_begin, shard.row_end, nq, ns))
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    if rank == 0:
        ok = True
        for key, rows, cols in SHAPES:
            q, s, b, a = _inputs(key, rows, cols)
            want_q, want_s = om.merge_float8(q, s, (1, cols), b, a, 1.0, seed=SEED)
            got_q = np.zeros_like(want_q)
            got_s = np.zeros_like(want_s)
            covered = np.zeros(rows, np.int32)
            for lst in gathered:
                for k, r0, r1, nq, ns in lst:
                    if k == key:
                        got_q[r0:r1] = nq
                        got_s[r0:r1] = ns
                        covered[r0:r1] += 1
            ok &= bool((covered == 1).all() and np.array_equal(got_q, want_q) and np.array_equal(got_s, want_s))
        with open(result_path, "w") as f:
            f.write("ok" if ok else "mismatch")
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_partitioned_merge_equals_single_process():
    with tempfile.TemporaryDirectory() as d:
        store = os.path.join(d, "store")
        result = os.path.join(d, "result")
        mp.spawn(_worker, args=(2, store, result), nprocs=2, join=True)
        assert open(result).read() == "ok"


def _dropout_worker(rank: int, world: int, store_path: str, result_path: str):
    store = dist.FileStore(store_path, world)
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        # This rank leaves between steps: it never enters the next collective.
        os._exit(0)
    try:
        t = torch.ones(1)
        dist.all_reduce(t)
        outcome = "completed"
    except Exception as exc:  # noqa: BLE001 - gloo raises RuntimeError subclasses
        outcome = "error:" + type(exc).__name__
    with open(result_path, "w") as f:
        f.write(outcome)
    os._exit(0)


def test_departed_rank_surfaces_as_collective_error():
    with tempfile.TemporaryDirectory() as d:
        store = os.path.join(d, "store")
        result = os.path.join(d, "result")
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_dropout_worker, args=(r, 2, store, result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=90)
            if p.is_alive():
                p.kill()
                pytest.fail("a rank did not exit")
        assert open(result).read().startswith("error:")

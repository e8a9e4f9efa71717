"""Benchmark of the fused quantized LoRA merge on B200.

Default workload: scaled-FP8 e4m3 per-row weights of a
Llama-3-8B-shaped stack (32 layers x {q,o 4096x4096; k,v 1024x4096; gate,up
14336x4096; down 4096x14336}), base N(0, 0.02) quantized per row, rank-32
bf16 LoRA N(0, 0.01), strength 1.0, stochastic rounding seeded per weight with
``derive_seed(f"model.layers.{i}.{proj}.weight", merge_index)``. One step
merges every weight once (in place). Inputs total ~7 GB of codes, far larger
than the 126 MB L2, so no flush is needed between steps.

Metric: weight GB/s = (codes + scales read + codes + scales written) / time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
                    [--config fp8|int8|nvfp4|mxfp8|mxfp4|q8_0|q4_0|static_fp8|bnb8|
                              quanto_int8|quanto_fp8|nf4|nf4_nested] [--rtn] [--staging]

The last six configs run the reference's other Triton merges (static FP8,
bitsandbytes 8- and 4-bit, Quanto) on the same Llama-3-8B-shaped stack; they
are not BASELINE configs. ``nf4*`` report no ``e2e`` (the 4-bit quant state is
not streamed).

Under ``torch.distributed.run`` each rank merges its own copy of the model
(weak scaling, no data-path collective); the step time is the max over ranks.
``--impl reference`` times the reference algorithm's CPU restatement
(``oracle``) on the host cores on a bounded sample (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LLAMA3_8B = [("q_proj", 4096, 4096), ("k_proj", 1024, 4096), ("v_proj", 1024, 4096),
             ("o_proj", 4096, 4096), ("gate_proj", 14336, 4096), ("up_proj", 14336, 4096),
             ("down_proj", 4096, 14336)]
DIT_12B = [("attn_q", 3072, 3072), ("attn_k", 3072, 3072), ("attn_v", 3072, 3072), ("attn_o", 3072, 3072),
           ("mlp_up", 12288, 3072), ("mlp_down", 3072, 12288)]
LLAMA_70B = [("attn_qo", 8192, 8192), ("attn_kv", 1024, 8192), ("mlp_gate", 28672, 8192),
             ("mlp_down", 8192, 28672)]

CONFIGS = {
    # name: (layer list, layers, rank, lora std, base std, stochastic, description)
    "fp8": (LLAMA3_8B, 32, 32, 0.01, 0.02, True, "scaled-FP8 e4m3 per-row, Llama-3-8B x32, r32, SR"),
    "int8": (LLAMA3_8B, 32, 16, 0.01, 0.02, False, "INT8 per-row symmetric, Llama-3-8B x32, r16, RTN"),
    "nvfp4": ([("up", 14336, 4096), ("down", 4096, 14336)], 32, 64, 0.005, 0.02, False,
              "NVFP4 two-level, 14336x4096 + 4096x14336 x32, r64, RTN"),
    "mxfp8": (DIT_12B, 57, 128, 0.005, 0.02, False, "MXFP8 e4m3 FLOOR, DiT-12B 57 blocks, r128, RTN"),
    "mxfp4": (DIT_12B, 57, 128, 0.005, 0.02, False, "MXFP4 FLOOR, DiT-12B 57 blocks, r128, RTN"),
    "q8_0": (LLAMA_70B, 80, 16, 0.01, 0.015, False, "GGUF Q8_0, 70B-shaped x80, r16, RTN"),
    "q4_0": (LLAMA_70B, 80, 16, 0.01, 0.015, False, "GGUF Q4_0, 70B-shaped x80, r16, RTN"),
    # one 4096 x 4096 INT8 per-row weight (launch-bound: ~5 us of HBM time per merge).
    "int8_4096": ([("proj", 4096, 4096)], 1, 16, 0.01, 0.02, False, "INT8 per-row symmetric, one 4096x4096, r16, RTN"),
    # Formats beyond BASELINE's configs (the reference's other Triton merges), on the config-2 stack.
    "static_fp8": (LLAMA3_8B, 32, 32, 0.01, 0.02, True, "static per-tensor FP8 e4m3, Llama-3-8B x32, r32, SR"),
    "bnb8": (LLAMA3_8B, 32, 16, 0.01, 0.02, False, "bitsandbytes LLM.int8, Llama-3-8B x32, r16, fp16, RTN"),
    "quanto_int8": (LLAMA3_8B, 32, 32, 0.01, 0.02, False, "Quanto qint8 per-row, Llama-3-8B x32, r32, RTN"),
    "quanto_fp8": (LLAMA3_8B, 32, 32, 0.01, 0.02, False, "Quanto qfloat8 e4m3 per-row, Llama-3-8B x32, r32, RTN"),
    "nf4": (LLAMA3_8B, 32, 64, 0.005, 0.02, False, "bitsandbytes NF4, plain absmax, Llama-3-8B x32, r64, RTN"),
    "nf4_nested": (LLAMA3_8B, 32, 64, 0.005, 0.02, False,
                   "bitsandbytes NF4, nested absmax, Llama-3-8B x32, r64, RTN"),
}


def apply_rank(rank: int) -> None:
    """Run every config at LoRA rank ``rank`` (``--rank``); spawned CPU-baseline
    workers re-import this module and read it from ``PIPER_BENCH_RANK``."""
    import re

    os.environ["PIPER_BENCH_RANK"] = str(rank)
    for k, v in list(CONFIGS.items()):
        CONFIGS[k] = (v[0], v[1], rank, *v[3:6], re.sub(r"\br\d+\b", f"r{rank}", v[6]))


if os.environ.get("PIPER_BENCH_RANK"):
    apply_rank(int(os.environ["PIPER_BENCH_RANK"]))
# Algorithmic bytes per element (read + write) and per-row scale bytes.
BYTES_PER_ELEM = {"fp8": 2.0, "int8": 2.0, "int8_4096": 2.0, "nvfp4": 1.125, "mxfp8": 2.0625, "mxfp4": 1.0625,
                  "q8_0": 2.125, "q4_0": 1.125, "static_fp8": 2.0, "bnb8": 2.0, "quanto_int8": 2.0,
                  "quanto_fp8": 2.0, "nf4": 1.125, "nf4_nested": 1.03125}
# fp32 / bf16 row scale read + written
ROW_SCALE_BYTES = {"fp8": 8, "int8": 4, "int8_4096": 4, "bnb8": 8, "quanto_int8": 4, "quanto_fp8": 4}

FALLBACK_HBM_GBS = 6650.0


def weight_list(cfg: str, model_copies: int = 1, n_layers: int | None = None):
    layers, cfg_layers, *_ = CONFIGS[cfg]
    n_layers = cfg_layers if n_layers is None else n_layers
    out = []
    for copy in range(model_copies):
        for i in range(n_layers):
            for name, rows, cols in layers:
                prefix = f"model{copy}." if copy else ""
                out.append((f"{prefix}model.layers.{i}.{name}.weight", rows, cols))
    return out


def algorithmic_bytes(cfg: str, rows: int, cols: int) -> int:
    return int(rows * cols * BYTES_PER_ELEM[cfg]) + rows * ROW_SCALE_BYTES.get(cfg, 0)


def measured_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return FALLBACK_HBM_GBS, "fallback"


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi during the timed region (recipe's clocks line)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for _, _, parts in rows:
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows)}


# --------------------------------------------------------------- workload
def build_weights(cfg: str, device, seed_base: int, n_layers: int | None = None, shards: dict | None = None):
    """Quantized weights + factors on `device` (torch ops, seeded per weight).

    ``shards`` maps a weight key to the (row_begin, row_end) ranges this rank
    merges (multi-GPU partition): the full weight is generated with the same
    seed on every rank and only those rows are kept, so the shards of all
    ranks are exactly the single-GPU weight's rows. Weights absent from
    ``shards`` are skipped. Items are (key, rows, cols, weight, b, a,
    row_begin)."""
    import torch

    from piper_offload_b200 import synthetic as S

    _, _, rank, lora_std, base_std, _, _ = CONFIGS[cfg]
    items = []
    for k, (key, rows, cols) in enumerate(weight_list(cfg, n_layers=n_layers)):
        if shards is not None and key not in shards:
            continue
        s = seed_base + 7919 * k
        w_full = S.normal((rows, cols), base_std, seed=s, device=device,
                          outlier_frac=0.001 if cfg.startswith("mx") else 0.0)
        for r0, r1 in ([(0, rows)] if shards is None else shards[key]):
            items.append(_quantized_item(cfg, key, rows, cols, w_full, r0, r1, s, rank, lora_std, device))
        del w_full
    torch.cuda.synchronize(device)
    return items


def _quantized_item(cfg: str, key: str, rows: int, cols: int, w_full, r0: int, r1: int, s: int, rank: int,
                    lora_std: float, device):
    """One weight (or rows r0..r1 of it) quantized in the config's format, with its LoRA factors."""
    import torch

    from piper_offload_b200 import synthetic as S
    from piper_offload_b200 import weights as WT

    w = w_full if (r0, r1) == (0, rows) else w_full[r0:r1].contiguous()
    rows_here = r1 - r0
    if cfg == "fp8":
        q = S.quantize_fp8(w)
        t = WT.Float8Weight(q.qdata, q.scale, (1, cols))
    elif cfg in ("int8", "int8_4096"):
        q = S.quantize_int8_per_row(w)
        t = WT.Int8Weight(q.qdata, q.scale, (1, cols))
    elif cfg == "nvfp4":
        q = S.quantize_nvfp4(w, two_level=True)
        t = WT.NVFP4Weight(q.qdata, q.scale, q.per_tensor_scale)
    elif cfg in ("mxfp8", "mxfp4"):
        elem = "e4m3" if cfg == "mxfp8" else "e2m1"
        q = S.quantize_mx(w, elem)
        edt = torch.float8_e4m3fn if cfg == "mxfp8" else torch.float4_e2m1fn_x2
        t = WT.MXWeight(q.qdata, q.scale.view(torch.float8_e8m0fnu), edt)
    elif cfg == "static_fp8":
        q = S.quantize_fp8(w, per_tensor=True)
        t = WT.StaticFloat8Weight(q.qdata, q.scale.reshape(()), torch.ones((), device=device))
    elif cfg == "bnb8":
        t = WT.Bnb8Weight(*S.quantize_bnb8(w))
    elif cfg in ("quanto_int8", "quanto_fp8"):
        storage = "int8" if cfg == "quanto_int8" else "e4m3"
        data, qscale = S.quantize_quanto(w, storage, axis=0)
        t = WT.QuantoWeight(data, qscale, 0, WT.QINT8 if storage == "int8" else WT.QFLOAT8_E4M3)
    elif cfg in ("nf4", "nf4_nested"):
        packed, absmax, code, nabs, ncode, off = S.quantize_bnb4(w, nested=cfg == "nf4_nested")
        st2 = None if nabs is None else WT.Bnb4State(nabs, ncode, (1, 1), blocksize=256, dtype=torch.float32)
        t = WT.Bnb4Weight(packed, WT.Bnb4State(absmax, code, (rows_here, cols), "nf4", 64, torch.bfloat16, st2, off))
    else:
        q = S.quantize_gguf(w, 8 if cfg == "q8_0" else 2)
        t = WT.GGUFWeight(q.qdata, 8 if cfg == "q8_0" else 2)
    del w
    fdt = torch.float16 if cfg == "bnb8" else torch.bfloat16
    b, a = S.lora_factors(rows, cols, rank, lora_std, seed=s + 1, device=device, dtype=fdt)
    if (r0, r1) != (0, rows):
        b = b[r0:r1].contiguous()
    return (key, rows_here, cols, t, b, a, r0)


def storage_tensors(t):
    out = []
    for name in ("qdata", "scale", "zero_point", "per_tensor_scale", "raw"):
        v = getattr(t, name, None)
        if v is not None:
            out.append(v)
    return out


# ------------------------------------------------------------ CPU baseline
def _gguf_reference_chunk(raw, quant_type: int, b, a, strength: float) -> None:
    """The reference's own GGUF path on CPU tensors: ``gguf_dequant.dequantize``
    (``gguf_dequant.py:303-331``) to bf16, the update added in fp32 by
    ``torch.addmm`` and rounded to bf16, and re-encoding by the pinned ``gguf``
    package (``gguf.quants.quantize``, 0.19.0)."""
    import gguf
    import torch

    from baseline import reference

    gd = reference.load("piper_offload.gguf_dequant")
    base = gd.dequantize(torch.from_numpy(raw), quant_type, dtype=torch.bfloat16)
    merged = torch.addmm(base.float(), torch.from_numpy(b), torch.from_numpy(a), alpha=strength).to(torch.bfloat16)
    qtype = gguf.GGMLQuantizationType.Q8_0 if quant_type == 8 else gguf.GGMLQuantizationType.Q4_0
    gguf.quants.quantize(merged.float().numpy(), qtype)


def _oracle_chunk(args):
    """One row chunk of the CPU baseline (runs in a spawned worker)."""
    import numpy as np
    import torch

    torch.set_num_threads(1)
    from oracle import merge as om

    cfg, q, scale, b, a, seed, offset_base, extra = args
    t0 = time.perf_counter()
    if cfg == "fp8":
        om.merge_float8(q, scale, (1, a.shape[1]), b, a, 1.0, seed=seed, offset_base=offset_base)
    elif cfg == "static_fp8":
        om.merge_static_float8(q, scale, b, a, 1.0, seed=seed, offset_base=offset_base)
    elif cfg in ("int8", "int8_4096"):
        om.merge_int8(q, scale, None, (1, a.shape[1]), b, a, 1.0, seed=seed, offset_base=offset_base)
    elif cfg == "bnb8":
        om.merge_bnb8(q, scale.reshape(-1), b, a, 1.0, seed=seed, offset_base=offset_base)
    elif cfg in ("quanto_int8", "quanto_fp8"):
        om.merge_quanto(q, scale, "row", b, a, 1.0, storage="int8" if cfg == "quanto_int8" else "e4m3", seed=seed,
                        offset_base=offset_base)
    elif cfg in ("nf4", "nf4_nested"):
        code, nabs, ncode, off = extra
        om.merge_bnb4(q, scale, code, b, a, 1.0, nested_absmax=nabs, nested_code=ncode, offset=off, seed=seed,
                      offset_base=offset_base)
    elif cfg == "nvfp4":
        om.merge_nvfp4(q, scale, extra, b, a, 1.0, seed=seed, offset_base=offset_base)
    elif cfg in ("mxfp8", "mxfp4"):
        om.merge_mx(q, scale, "e4m3" if cfg == "mxfp8" else "e2m1", b, a, 1.0, seed=seed, offset_base=offset_base)
    elif cfg in ("q8_0", "q4_0"):
        qt = 8 if cfg == "q8_0" else 2
        if extra == "reference":
            _gguf_reference_chunk(q, qt, b, a, 1.0)
        else:
            om.merge_gguf(q, qt, b, a, 1.0, seed=seed, offset_base=offset_base)
    else:
        raise ValueError(cfg)
    return time.perf_counter() - t0, int(np.asarray(q).size)


def _gguf_reference_ready() -> bool:
    try:
        import gguf  # noqa: F401

        from baseline import reference

        return reference.available()
    except ImportError:
        return False


def cpu_baseline(cfg: str, steps: int, warmup: int, rows_per_step: int = 1024, cols: int = 4096,
                 stochastic: bool | None = None):
    """Time the reference's CPU path for ``cfg`` on the host cores: for GGUF the
    reference's own code (``kind: reference``), for the other formats the numpy
    restatement of the reference's kernels (``kind: port``; TorchAO, which holds
    the reference's portable CPU fallbacks, is not installed)."""
    import multiprocessing as mp

    import numpy as np
    import torch

    from piper_offload_b200 import synthetic as S

    _, _, rank, lora_std, base_std, cfg_sr, _ = CONFIGS[cfg]
    stochastic = cfg_sr if stochastic is None else stochastic
    cores = max(1, min(os.cpu_count() or 1, 32))
    chunk = max(16, rows_per_step // cores)
    w = S.normal((rows_per_step, cols), base_std, seed=11, device="cpu",
                 outlier_frac=0.001 if cfg.startswith("mx") else 0.0)
    b, a = S.lora_factors(rows_per_step, cols, rank, lora_std, seed=12, device="cpu")
    extra = None
    kind, what = "port", "numpy restatement of the reference kernels, not reference code"
    per_chunk_extra = None
    if cfg in ("fp8", "static_fp8"):
        q = S.quantize_fp8(w, per_tensor=cfg == "static_fp8")
        qn, sn = q.qdata.view(torch.uint8).numpy(), q.scale.float().numpy()
    elif cfg in ("int8", "int8_4096"):
        q = S.quantize_int8_per_row(w)
        qn, sn = q.qdata.numpy(), q.scale.float().numpy()
    elif cfg == "bnb8":
        cb, scb = S.quantize_bnb8(w)
        qn, sn = cb.numpy(), scb.numpy().reshape(-1, 1)
    elif cfg in ("quanto_int8", "quanto_fp8"):
        data, qs = S.quantize_quanto(w, "int8" if cfg == "quanto_int8" else "e4m3", axis=0)
        qn = data.numpy() if cfg == "quanto_int8" else data.view(torch.uint8).numpy()
        sn = qs.float().numpy()
    elif cfg in ("mxfp8", "mxfp4"):
        q = S.quantize_mx(w, "e4m3" if cfg == "mxfp8" else "e2m1")
        qn, sn = q.qdata.view(torch.uint8).numpy(), q.scale.numpy()
    elif cfg in ("q8_0", "q4_0"):
        q = S.quantize_gguf(w, 8 if cfg == "q8_0" else 2)
        qn, sn = q.qdata.numpy(), np.zeros((rows_per_step, 1), np.float32)
        if _gguf_reference_ready() and not stochastic:
            extra = "reference"
            kind = "reference"
            what = ("the reference's gguf_dequant.dequantize + torch.addmm + gguf 0.19.0 quants.quantize "
                    "(reference code and its pinned dependency)")
    elif cfg in ("nvfp4", "nf4", "nf4_nested"):
        # Each row chunk is merged as its own weight, so a chunk carries its own
        # per-tensor state (NVFP4 global scale, bitsandbytes nested absmax).
        qn, sn, per_chunk_extra = [], [], []
        for r in range(0, rows_per_step, chunk):
            if cfg == "nvfp4":
                q = S.quantize_nvfp4(w[r:r + chunk], two_level=True)
                qn.append(q.qdata.numpy())
                sn.append(q.scale.view(torch.uint8).numpy())
                per_chunk_extra.append(float(q.per_tensor_scale))
            else:
                packed, absmax, code, nabs, ncode, off = S.quantize_bnb4(w[r:r + chunk], nested=cfg == "nf4_nested")
                qn.append(packed.numpy().reshape(-1, cols // 2))
                sn.append(absmax.numpy().reshape(-1))
                per_chunk_extra.append((code.numpy(), None if nabs is None else nabs.numpy(),
                                        None if ncode is None else ncode.numpy(), None if off is None else float(off)))
    else:
        raise ValueError(cfg)
    bn, an = b.float().numpy(), a.float().numpy()
    seed = 0x9C3EA68DBAC91AAD if stochastic else None
    if cfg == "static_fp8":
        sn = np.repeat(sn.reshape(1, 1), rows_per_step, axis=0)  # one scale per chunk
    if per_chunk_extra is not None:
        tasks = [(cfg, qn[j], sn[j], bn[r:r + chunk], an, seed, r * cols, per_chunk_extra[j])
                 for j, r in enumerate(range(0, rows_per_step, chunk))]
    else:
        tasks = [(cfg, qn[r:r + chunk], sn[r] if cfg == "static_fp8" else sn[r:r + chunk], bn[r:r + chunk],
                  an, seed, r * cols, extra) for r in range(0, rows_per_step, chunk)]
    ctx = mp.get_context("spawn")
    times = []
    with ctx.Pool(cores) as pool:
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            pool.map(_oracle_chunk, tasks)
            dt = time.perf_counter() - t0
            if i >= warmup:
                times.append(dt)
    nbytes = algorithmic_bytes(cfg, rows_per_step, cols)
    t = statistics.median(times)
    return {"value": nbytes / t / 1e9, "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": f"{rows_per_step}x{cols} {cfg}{' SR' if stochastic else ' RTN'} rows of one weight, "
                      f"{len(tasks)} row chunks over {cores} spawned processes ({what})",
            "ms_per_sample": t * 1e3}


# -------------------------------------------------------------- triton bar
TRITON_BAR_CONFIGS = ("fp8", "int8", "int8_4096", "nvfp4", "mxfp8", "mxfp4")


def triton_bar(cfg: str, items, seeds, steps: int, warmup: int, device, stream) -> dict | None:
    """The reference's own Triton merge launchers (unmodified, from
    ``baseline/_ref``) over the same weights, as each reference adapter runs
    them: the launcher, then the copy of its out-of-place buffers back into the
    weight's storage (``int8_adapter.py:397-400``, ``float8_adapter.py:252-265``,
    ``nvfp4_adapter.py:265-282``; the MX launcher merges in place,
    ``mx_adapter.py:284-300``). Timed like the native step: CUDA events over
    ``steps`` passes after ``warmup``."""
    import torch

    if cfg not in TRITON_BAR_CONFIGS:
        return None
    try:
        import triton

        from baseline import reference

        if not reference.available():
            return {"unavailable": "reference not installed under baseline/_ref"}
        f8 = reference.load("piper_offload._triton_float8_lora")
        i8 = reference.load("piper_offload._triton_int8_lora")
        n4 = reference.load("piper_offload._triton_nvfp4_lora")
        mx = reference.load("piper_offload._triton_mx_lora")
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": f"reference import failed: {exc!r}"[:200]}

    def one(i: int, key: str, t, b, a, seed) -> None:
        if cfg == "fp8":
            nq, ns = f8.merge_float8_lora(t.qdata, t.scale, tuple(t.block_size), b, a, 1.0, rounding_seed=seed)
            t.qdata.copy_(nq)
            t.scale.copy_(ns)
        elif cfg in ("int8", "int8_4096"):
            nq, ns, _ = i8.merge_int8_lora(t.qdata, t.scale, None, tuple(t.block_size), b, a, 1.0, asymmetric=False,
                                           reduce_range=False, rounding_seed=seed)
            t.qdata.copy_(nq)
            t.scale.copy_(ns)
        elif cfg == "nvfp4":
            nq, ns, npts = n4.merge_nvfp4_lora(t.qdata, t.scale, t.per_tensor_scale, 16, False, b, a, 1.0,
                                               rounding_seed=seed)
            t.qdata.copy_(nq)
            t.scale.copy_(ns)
            t.per_tensor_scale.copy_(npts.reshape(t.per_tensor_scale.shape))
        else:
            mx.merge_mx_lora_(t.qdata, t.scale, t.elem_dtype, 32, torch.bfloat16, b, a, 1.0, scaling_mode=0,
                              swizzled=False, rounding_seed=seed)

    def step(s: int) -> None:
        for i, (key, rows, cols, t, b, a, _) in enumerate(items):
            one(i, key, t, b, a, None if seeds is None else seeds[s][i])

    try:
        for s in range(warmup):
            step(s)
        torch.cuda.synchronize(device)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for s in range(steps):
            step(warmup + s)
        e1.record(stream)
        torch.cuda.synchronize(device)
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": f"reference Triton launch failed: {exc!r}"[:200]}
    ms = e0.elapsed_time(e1) / steps
    total = sum(algorithmic_bytes(cfg, r, c) for _, r, c, *_ in items)
    return {"value": round(total / (ms / 1e3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "triton": triton.__version__, "steps": steps, "warmup": warmup,
            "what": "reference Triton launchers from baseline/_ref (unmodified) + the adapters' copy-back, same "
                    "weights, seeds and step as `value`"}


# ------------------------------------------------------------------ main
def staging_bench(cfg: str, n_layers: int | None, steps: int, warmup: int) -> dict:
    """``merge_lora()`` end to end with the LoRA factors in host memory (bf16,
    pageable, as a checkpoint loader leaves them) and the weights on the GPU.

    ``per_weight`` is the reference driver's sequence: for each weight, stage
    for validation, validate, stage again, merge (``lora.py:406-413``,
    ``:543-549``), four host-to-device copies and one launch per weight.
    ``batched`` is ``transform.merge_lora``: one staging copy for the batch,
    validation of every weight, one batched launch. Wall-clock per call, with
    the device synchronized on both sides; median of ``steps`` calls.
    """
    import torch

    from piper_offload_b200 import transform as TR

    dev = torch.device("cuda", 0)
    items = build_weights(cfg, dev, 0, n_layers)
    weights = {key: t for key, _, _, t, _, _, _ in items}
    lora = {key: (a.cpu(), b.cpu()) for key, _, _, _, b, a, _ in items}
    stochastic = CONFIGS[cfg][5]
    del items

    def per_weight():
        for key, target in weights.items():
            tr = TR.LoRATransform([TR.LoRAFactor(*lora[key])], stochastic_rounding=stochastic, target_key=key)
            plan = tr._make_plan(target)
            b, a, s = tr._stage(target, plan)
            plan.adapter.validate_lora_merge(target, b, a, s, rounding_seed=tr._rounding_seed())
            b, a, s = tr._stage(target, plan)
            plan.adapter.merge_lora_(target, b, a, s, rounding_seed=tr._rounding_seed())

    def batched():
        TR.merge_lora(weights, [(lora, 1.0)], stochastic_rounding=stochastic)

    def timed(fn):
        for _ in range(warmup):
            fn()
        out = []
        for _ in range(steps):
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            fn()
            torch.cuda.synchronize(dev)
            out.append((time.perf_counter() - t0) * 1e3)
        return statistics.median(out)

    factor_bytes = sum((a.numel() + b.numel()) * a.element_size() for a, b in lora.values())
    pw, bt = timed(per_weight), timed(batched)
    return {"mode": "staging", "config": {"workload": CONFIGS[cfg][6], "weights": len(weights),
                                          "factor_bytes": factor_bytes},
            "per_weight_ms": round(pw, 3), "batched_ms": round(bt, 3),
            "h2d_copies": {"per_weight": 4 * len(weights), "batched": 1}, "steps": steps, "warmup": warmup}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--config", default="fp8", choices=sorted(CONFIGS))
    ap.add_argument("--rtn", action="store_true", help="round-to-nearest instead of the config's rounding")
    ap.add_argument("--sr", action="store_true", help="stochastic rounding instead of the config's rounding")
    ap.add_argument("--rank", type=int, default=None, help="LoRA rank instead of the config's")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--layers", type=int, default=None,
                    help="override the layer count (small profiling case; the headline uses the config's)")
    ap.add_argument("--kernel-reps", type=int, default=3,
                    help="timed repetitions of the roofline leg (the step's launches, each timed)")
    ap.add_argument("--no-triton-bar", action="store_true", help="skip timing the reference's Triton launchers")
    ap.add_argument("--partition", action="store_true",
                    help="multi-GPU: ONE model split over the ranks by sharding.partition (whole weights and "
                         "128-row output shards, global-offset seeds; strong scaling) instead of one model per rank")
    ap.add_argument("--staging", action="store_true",
                    help="time merge_lora() with host-resident factors: batched staging vs the per-weight driver")
    args = ap.parse_args()
    if args.rank:
        apply_rank(args.rank)
    warmup = max(3, args.warmup)
    if args.staging:
        print(json.dumps(staging_bench(args.config, args.layers, args.steps, warmup)), flush=True)
        return 0

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = args.config
    _, _, lrank, _, _, cfg_sr, desc = CONFIGS[cfg]
    stochastic = (cfg_sr or args.sr) and not args.rtn
    if stochastic != cfg_sr:
        desc = desc.rsplit(", ", 1)[0] + (", SR" if stochastic else ", RTN")
    metric = "LoRA-merge weight GB/s (read+write)"

    if args.impl == "reference":
        if rank != 0:
            return 0
        res = cpu_baseline(cfg, args.steps, warmup, stochastic=stochastic)
        line = {"metric": metric, "value": res["value"], "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
                "warmup": warmup, "ms_per_step": res["ms_per_sample"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "impl": "reference",
                "config": {"workload": desc, "rank": lrank, "stochastic": stochastic},
                "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": res["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    import torch.distributed as dist

    from piper_offload_b200 import _native
    from piper_offload_b200 import adapters as AD
    from piper_offload_b200.seeding import derive_seed

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # CPU baseline first (spawned pool, before heavy GPU allocations), rank 0 only.
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(cfg, steps=1, warmup=1, stochastic=stochastic)

    shards = None
    job_bytes_model = sum(algorithmic_bytes(cfg, r, c) for _, r, c in weight_list(cfg, n_layers=args.layers))
    if args.partition:
        from piper_offload_b200.sharding import WorkItem, partition

        # Per-tensor scales (two-level NVFP4, static FP8) span all rows: those weights move whole.
        row_split = cfg not in ("nvfp4", "static_fp8", "nf4_nested")
        witems = [WorkItem(key, r, c, algorithmic_bytes(cfg, 1, c), row_splittable=row_split)
                  for key, r, c in weight_list(cfg, n_layers=args.layers)]
        shards = {}
        for sh in partition(witems, world)[rank]:
            shards.setdefault(sh.key, []).append((sh.row_begin, sh.row_end))
    items = build_weights(cfg, device, seed_base=0 if args.partition else 1000 * rank, n_layers=args.layers,
                          shards=shards)
    total_bytes = sum(algorithmic_bytes(cfg, r, c) for _, r, c, *_ in items)
    # Whole-job bytes per step: one model per rank (weak), or one model split over the ranks (strong).
    job_bytes = job_bytes_model if args.partition else total_bytes * world

    # Device-resident path: descriptors built once through the adapters, then
    # one piper_merge_batch call per step with that step's seeds.
    stream = torch.cuda.current_stream(device)
    keep: list = []
    descs = [AD.select_adapter(t).merge_desc(t, b, a, 1.0, rounding_seed=0 if stochastic else None,
                                             offset_base=r0 * cols, keep=keep)
             for key, rows, cols, t, b, a, r0 in items]
    arr = (_native.MergeDesc * len(descs))(*descs)
    need = _native.workspace_bytes(descs)
    ws = torch.empty(max(64 << 20, need), dtype=torch.uint8, device=device)
    ws_ptr, ws_len = ws.data_ptr(), ws.numel()
    lib = _native.load()
    total_steps = warmup + args.steps
    seeds = [[derive_seed(key, s) for key, *_ in items] for s in range(total_steps + args.e2e_steps + 2)] \
        if stochastic else None

    def run_step(s: int) -> None:
        if seeds is not None:
            for i, sd in enumerate(seeds[s]):
                arr[i].seed = sd
        _native.check(lib.piper_merge_batch(arr, len(descs), ws_ptr, ws_len, stream.cuda_stream))

    step = 0
    for _ in range(warmup):
        run_step(step)
        step += 1
    torch.cuda.synchronize(device)
    assert _native.device_status(device) == 0

    launches0 = _native.launches()
    barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local_rank) as clk:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            run_step(step)
            step += 1
        end.record(stream)
        torch.cuda.synchronize(device)
    barrier()
    launches = _native.launches() - launches0
    ms = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms)
    value = job_bytes / (ms / 1e3) / 1e9
    clocks = clk.summary()
    status = _native.device_status(device)

    # Roofline leg: the step's own merge_kernel launches. The step's
    # descriptors are issued in calls of at most MAX_WEIGHTS_PER_LAUNCH (the
    # library packs at most that many weights into one launch), with CUDA
    # events on the launching stream around each call, `kernel_reps` times.
    # Per launch = the calls' algorithmic bytes and event time divided by the
    # launches they made (every launch of a step is the same kernel).
    chunks = [list(range(i, min(i + _native.MAX_WEIGHTS_PER_LAUNCH, len(descs))))
              for i in range(0, len(descs), _native.MAX_WEIGHTS_PER_LAUNCH)]
    chunk_arrs = [(_native.MergeDesc * len(ch))(*[arr[i] for i in ch]) for ch in chunks]
    chunk_bytes = [sum(algorithmic_bytes(cfg, items[i][1], items[i][2]) for i in ch) for ch in chunks]

    def run_chunk(j: int, s: int) -> None:
        if seeds is not None:
            for pos, i in enumerate(chunks[j]):
                chunk_arrs[j][pos].seed = seeds[s][i]
        _native.check(lib.piper_merge_batch(chunk_arrs[j], len(chunks[j]), ws_ptr, ws_len, stream.cuda_stream))

    for j in range(len(chunks)):
        run_chunk(j, 0)
    torch.cuda.synchronize(device)
    l0 = _native.launches()
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in chunks]
           for _ in range(args.kernel_reps)]
    for rep in range(args.kernel_reps):
        for j in range(len(chunks)):
            evs[rep][j][0].record(stream)
            run_chunk(j, 1 + rep)
            evs[rep][j][1].record(stream)
    torch.cuda.synchronize(device)
    n_launch = (_native.launches() - l0) / args.kernel_reps
    call_ms = sum(a.elapsed_time(b) for rep in evs for a, b in rep) / args.kernel_reps
    launch_ms = call_ms / n_launch
    launch_bytes = sum(chunk_bytes) / n_launch

    peak, peak_kind = measured_peak()
    achieved = launch_bytes / (launch_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} (hbm_gbs copy)",
                "kernel": f"merge_kernel, the step's {n_launch:g} launches ({len(descs)} weights, calls of at most "
                          f"{_native.MAX_WEIGHTS_PER_LAUNCH} weights, each timed by CUDA events)",
                "algorithmic_bytes_per_launch": int(launch_bytes), "launch_ms": round(launch_ms, 5),
                "step_achieved": round(value / world, 1), "traffic": None}
    tfile = ROOT / "profiles" / f"traffic_{cfg}.json"
    if tfile.exists():
        try:
            tj = json.loads(tfile.read_text())
            ratio = float(tj["dram_bytes_per_algorithmic_byte"])
            roofline["traffic"] = int(ratio * launch_bytes)
            roofline["traffic_source"] = tj.get("note")
        except Exception:  # noqa: BLE001
            pass

    # Host cost per call: wall clock over back-to-back calls of the whole step
    # (one batched C-ABI call) and of the reference driver's per-weight loop
    # (merge.py:124: one call per weight), each synchronised once at the end.
    def wall_us(fn, reps: int) -> float:
        fn()
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        torch.cuda.synchronize(device)
        return (time.perf_counter() - t0) / reps * 1e6

    singles = [(_native.MergeDesc * 1)(arr[i]) for i in range(len(descs))]

    def per_weight_loop() -> None:
        for one_arr in singles:
            _native.check(lib.piper_merge_batch(one_arr, 1, ws_ptr, ws_len, stream.cuda_stream))

    reps = max(3, min(200, int(2000 / max(ms, 0.01))))
    host = {"batched_call_us": round(wall_us(lambda: run_step(step), reps), 2),
            "per_weight_loop_us": round(wall_us(per_weight_loop, max(3, reps // 4)), 2),
            "device_step_us": round(ms * 1e3, 2), "weights": len(descs),
            "what": "wall clock per step over back-to-back calls, one sync at the end: one batched call vs one C-ABI "
                    "call per weight (the reference's per-weight loop)"}

    bar = None
    if world == 1 and not args.no_triton_bar:
        bar = triton_bar(cfg, items, seeds, args.steps, warmup, device, stream)

    # End to end through the public API: every weight starts and ends in pinned
    # host memory; streaming.merge_streamed moves each layer through a ring of
    # three device slots, overlapping upload, merge and download on three streams.
    e2e = None
    if not args.no_e2e and not cfg.startswith("nf4"):  # bitsandbytes 4-bit state is not streamed
        import copy

        from piper_offload_b200.streaming import StreamedOp, merge_streamed, storages

        host_ops = []
        h2d = d2h = 0
        for key, rows, cols, t, b, a, r0 in items:
            ht = copy.copy(t)
            for name, dt in storages(t):
                setattr(ht, name, dt.detach().cpu().pin_memory())
            hb, ha = b.cpu().pin_memory(), a.cpu().pin_memory()
            host_ops.append((key, ht, hb, ha))
            st = [x for _, x in storages(ht)]
            h2d += sum(x.numel() * x.element_size() for x in st + [hb, ha])
            d2h += sum(x.numel() * x.element_size() for x in st)
        per_layer = len(CONFIGS[cfg][0])
        layer_ops = [host_ops[i:i + per_layer] for i in range(0, len(host_ops), per_layer)]
        torch.cuda.synchronize(device)

        def e2e_step(stp: int):
            blocks = [[StreamedOp(ht, hb, ha, 1.0, derive_seed(key, stp) if stochastic else None)
                       for key, ht, hb, ha in layer] for layer in layer_ops]
            merge_streamed(blocks, device, depth=3, workspace=ws)

        e2e_step(step)
        torch.cuda.synchronize(device)
        barrier()
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        for i in range(args.e2e_steps):
            e2e_step(step + 1 + i)
        e_end.record(stream)
        torch.cuda.synchronize(device)
        barrier()
        e_ms = max_over_ranks(e_start.elapsed_time(e_end) / args.e2e_steps)
        e2e = {"value": job_bytes / (e_ms / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e_ms, "steps": args.e2e_steps,
               "path": "pinned host -> streaming.merge_streamed (per layer: upload / merge via C ABI / download "
                       "on three streams, 3 device slots) -> pinned host"}

    if rank == 0:
        line = {
            "metric": metric, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong" if args.partition else "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": desc, "weights_per_gpu": len(items), "rank": lrank, "stochastic": stochastic,
                       "weight_bytes_per_gpu": total_bytes, "l2": "inputs (~GBs) exceed the 126 MB L2; no flush",
                       "layers": args.layers or CONFIGS[cfg][1],
                       "parallelism": (f"partition x{world}: one model split by whole weights and 128-row shards "
                                       f"(sharding.partition), global-offset seeds, no collective")
                       if args.partition else f"weak x{world}: one model per GPU, no collective"},
            "roofline": roofline,
            "cpu_baseline": None if cpu is None else {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": e2e, "gpu_launches": launches, "clocks": clocks, "device_status": status,
            "host": host, "triton_bar": bar,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

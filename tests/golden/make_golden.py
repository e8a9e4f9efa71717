"""Generate golden vectors from the reference implementation (run in the build container).

Usage: ``TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/piper-offload``

Imports Piper Offload 0.2.5 from its source tree (Python 3.12 needs the
module-level ``from __future__ import annotations`` flag, applied by a small
import hook) and records, as small JSON / NPZ fixtures:

* ``seeds.json``  -- ``piper_offload.seeding.derive_seed`` on typed part lists;
* ``philox.json`` -- the reference stochastic stream ``_random(seed, offsets)``
  (``_triton_stochastic_quantization.py:18-21``) evaluated by the Triton CPU
  interpreter, whose integer Philox arithmetic is exact;
* ``gguf.npz``    -- ``piper_offload.gguf_dequant.dequantize`` (bf16) of random
  Q8_0 / Q4_0 blocks, and ``gguf.quants.quantize`` (gguf 0.19.0, the pinned
  dependency range) of random fp32 rows.

The reference tree is only needed to regenerate; tests read the fixtures.
"""

from __future__ import annotations

import __future__
import importlib.abc
import importlib.machinery
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def install_reference(src: Path) -> None:
    class _Loader(importlib.machinery.SourceFileLoader):
        def source_to_code(self, data, path, *, _optimize=-1):  # noqa: ANN001
            return compile(data, path, "exec", flags=__future__.annotations.compiler_flag,
                           dont_inherit=True, optimize=_optimize)

    class _Finder(importlib.abc.MetaPathFinder):
        def find_spec(self, name, path, target=None):  # noqa: ANN001, ARG002
            if not name.startswith("piper_offload"):
                return None
            spec = importlib.machinery.PathFinder.find_spec(name, path or [str(src)])
            if spec and spec.origin and spec.origin.endswith(".py"):
                spec.loader = _Loader(name, spec.origin)
            return spec

    sys.meta_path.insert(0, _Finder())


SEED_PARTS = [
    ["layer.0.weight", 0],
    ["layer.0.weight", 1],
    ["model.layers.0.self_attn.q_proj.weight", 0],
    ["model.layers.31.mlp.down_proj.weight", 7],
    [123456789, 0, 4096],
    ["", 0],
    ["unicodé-κλειδί", 18446744073709551615],
    [0],
]
PHILOX_SEEDS = [0x9C3EA68DBAC91AAD, 0, 1, 0xFFFFFFFFFFFFFFFF, 0x0123456789ABCDEF]
PHILOX_OFFSETS = [0, 1, 2, 3, 31, 32, 4095, 4096, 65535, 16777215, 2**31 - 1, 2**31, 2**32 - 1,
                  2**32, 2**32 + 5, 2**40 + 12345, 2**63 - 1]


def gen_seeds() -> None:
    from piper_offload.seeding import derive_seed

    out = [{"parts": p, "seed": derive_seed(*p)} for p in SEED_PARTS]
    (HERE / "seeds.json").write_text(json.dumps(out, indent=1, ensure_ascii=False))


def gen_philox() -> None:
    import torch
    import triton
    import triton.language as tl

    from piper_offload._triton_stochastic_quantization import _random, _seed_argument

    globals()["_random"] = _random  # the jitted kernel resolves helpers from module globals

    @triton.jit
    def kernel(seed, off_ptr, out_ptr, N: tl.constexpr):
        i = tl.arange(0, N)
        tl.store(out_ptr + i, _random(seed, tl.load(off_ptr + i)))

    n = 32
    offs = PHILOX_OFFSETS + [0] * (n - len(PHILOX_OFFSETS))
    out = []
    for seed in PHILOX_SEEDS:
        off_t = torch.tensor(offs, dtype=torch.int64)
        res = torch.empty(n, dtype=torch.float32)
        kernel[(1,)](_seed_argument(seed), off_t, res, N=n)
        out.append({"seed": seed, "offsets": PHILOX_OFFSETS,
                    "uniform_bits": [int(x) for x in res.view(torch.int32)[: len(PHILOX_OFFSETS)].tolist()]})
    (HERE / "philox.json").write_text(json.dumps(out, indent=1))


def gen_gguf() -> None:
    import gguf
    import torch

    from piper_offload import gguf_dequant

    rng = np.random.default_rng(0)
    arrays = {}
    for name, qt, ts in (("q8_0", 8, 34), ("q4_0", 2, 18)):
        rows, blocks = 6, 4
        raw = rng.integers(0, 256, size=(rows, blocks * ts), dtype=np.uint8)
        # keep the fp16 scales finite and moderate
        d = (rng.standard_normal((rows, blocks)) * 0.01).astype(np.float16).view(np.uint8).reshape(rows, blocks, 2)
        raw = raw.reshape(rows, blocks, ts)
        raw[:, :, :2] = d
        raw = raw.reshape(rows, blocks * ts)
        deq = gguf_dequant.dequantize(torch.from_numpy(raw.copy()), qt, dtype=torch.bfloat16)
        arrays[f"{name}_raw"] = raw
        arrays[f"{name}_dequant_bf16_bits"] = deq.view(torch.int16).numpy()
        vals = (rng.standard_normal((5, 128)) * 0.015).astype(np.float32)
        vals[0, :32] = 0.0  # an all-zero block
        vals[1, 5] = 0.2  # a single outlier
        vals[2, 40] = -0.3
        arrays[f"{name}_values"] = vals
        arrays[f"{name}_quantized"] = gguf.quants.quantize(vals, gguf.GGMLQuantizationType(qt))
    np.savez_compressed(HERE / "gguf.npz", **arrays)


def main() -> None:
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PIPER_OFFLOAD_SRC", ""))
    install_reference(ref / "src")
    gen_seeds()
    gen_philox()
    gen_gguf()
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()

"""Optional device hook for the oracle's tensor/tensor fp32 quotients (TEST INFRASTRUCTURE ONLY).

The reference kernels divide fp32 tensors with Triton's default ``/``. On
sm_100 that lowers to the approximate ``div.full.f32`` (probed on a B200 with
triton 3.6: ``tensor / tensor`` is bit-identical to ``div.full.f32`` and
differs from IEEE division in ~30% of random operand pairs, while division by
a constexpr or literal is IEEE-exact). The oracle cannot restate NVIDIA's
instruction, so on a GPU box the parity tests install this hook: it evaluates
exactly the oracle's tensor/tensor quotients with a one-line Triton kernel,
i.e. with the reference's own compiler and instruction. Without the hook the
oracle uses IEEE division and these quotients form a documented tie class.
"""

from __future__ import annotations

import numpy as np

_kernel = None


def _build():
    import triton
    import triton.language as tl

    @triton.jit
    def _div(a_ptr, b_ptr, o_ptr, n, BLOCK: tl.constexpr):
        offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
        mask = offs < n
        a = tl.load(a_ptr + offs, mask=mask, other=1.0)
        b = tl.load(b_ptr + offs, mask=mask, other=1.0)
        tl.store(o_ptr + offs, a / b, mask=mask)

    return _div


def triton_tensor_division(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Elementwise fp32 ``a / b`` computed by Triton's default division on CUDA."""
    import torch
    import triton

    global _kernel
    if _kernel is None:
        _kernel = _build()
    n = a.size
    if n == 0:
        return np.zeros(0, np.float32)
    ta = torch.from_numpy(np.array(a, dtype=np.float32, copy=True)).cuda()
    tb = torch.from_numpy(np.array(b, dtype=np.float32, copy=True)).cuda()
    out = torch.empty_like(ta)
    _kernel[(triton.cdiv(n, 1024),)](ta, tb, out, n, BLOCK=1024)
    return out.cpu().numpy()


def install() -> None:
    from .numerics import set_tensor_division

    set_tensor_division(triton_tensor_division)


def uninstall() -> None:
    from .numerics import set_tensor_division

    set_tensor_division(None)

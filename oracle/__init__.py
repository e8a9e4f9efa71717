"""CPU oracle for the quantized LoRA merge (TEST INFRASTRUCTURE ONLY).

This package is a plain numpy restatement of Piper Offload's fused LoRA-merge
kernels (``src/piper_offload/_triton_{int8,float8,nvfp4,mx}_lora.py``), its
counter-based stochastic-rounding helpers
(``src/piper_offload/_triton_stochastic_quantization.py``) and of the GGUF
Q8_0/Q4_0 codecs (``src/piper_offload/gguf_dequant.py`` plus the ``gguf``
package's ``quants.Q8_0``/``quants.Q4_0`` quantizers, gguf 0.19.0).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` may import it, and only as the checker or the timed CPU baseline.
The product path (``piper_offload_b200``) never imports anything from here.

Each function cites the reference file:line whose arithmetic it restates. The
restatement keeps every rounding point of the GPU kernels: RTNE casts to
bf16/fp16/e4m3/e5m2, fused multiply-add of ``base + acc * strength``, and the
fp32 quotient of each ``/``. Two documented tie classes remain between this
oracle and any GPU implementation (including the reference's own Triton
kernels): the fp32 summation order of the rank-r ``B @ A`` dot product and the
last-ulp behaviour of the GPU's approximate ``div.full.f32`` / ``lg2.approx``.
The oracle uses a correctly rounded dot product and IEEE division.
"""

from .numerics import (  # noqa: F401
    bf16_round,
    decode_e4m3,
    decode_e5m2,
    encode_e4m3,
    encode_e5m2,
    f16_round,
)
from .philox import philox_uniform  # noqa: F401

"""Drop-in replacement for the reference module `kernels.py` (Vaibhav1067/specdec-quant-triton).

Put this directory first on PYTHONPATH and the reference's scripts run unchanged against the
B200 kernels:

    PYTHONPATH=specdec-quant-triton_b200 python correctness.py

`from kernels import *` yields the same public names as the reference module (kernels.py:58,
65, 71, 138, 150, 239, 265, 289); `from kernels import _w8a8_kernel, _w4a16_kernel`
(correctness.py:5) yields registries whose `device_caches` count the kernel binaries used.
"""
from specq import (make_paged_kv, paged_attention, paged_attention_ref, quantize_act_int8,  # noqa: F401
                   quantize_weight_int4, quantize_weight_int8, w4a16_matmul, w8a8_matmul)
from specq.ops import _paged_attn_kernel, _w4a16_kernel, _w8a8_kernel  # noqa: F401

__all__ = ["w8a8_matmul", "w4a16_matmul", "paged_attention", "quantize_act_int8", "quantize_weight_int8",
           "quantize_weight_int4", "make_paged_kv", "paged_attention_ref"]

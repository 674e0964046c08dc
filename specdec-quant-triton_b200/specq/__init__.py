"""specq -- B200 (sm_100a) verification-shape kernels behind the reference's Python API.

    from specq import w8a8_matmul, w4a16_matmul, paged_attention

Everything runs as hand-written CUDA in libspecq.so (see include/specq.h); importing this
package fails loudly if the library has not been built.
"""
from . import _lib
from .fixtures import (make_paged_kv, paged_attention_ref, quantize_act_int8, quantize_weight_int4,
                       quantize_weight_int8)
from .ops import (QUANT_PLAIN, QUANT_RESIDUAL, QUANT_SILU_MUL, KernelHandle, _paged_attn_kernel, _w4a16_kernel,
                  _w8a8_kernel, kv_append, paged_attention, paged_attention_packed, quant_rows, w4a16_matmul,
                  w8a8_accumulator, w8a8_matmul)

_lib.load()

get_status = _lib.get_status
SpecqError = _lib.SpecqError

__all__ = [
    "w8a8_matmul", "w4a16_matmul", "paged_attention", "w8a8_accumulator",
    "quantize_act_int8", "quantize_weight_int8", "quantize_weight_int4", "make_paged_kv", "paged_attention_ref",
    "KernelHandle", "get_status", "SpecqError",
    "quant_rows", "kv_append", "paged_attention_packed", "QUANT_PLAIN", "QUANT_RESIDUAL", "QUANT_SILU_MUL",
]

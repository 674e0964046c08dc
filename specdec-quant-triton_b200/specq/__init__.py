"""specq -- B200 (sm_100a) verification-shape kernels behind the reference's Python API.

    from specq import w8a8_matmul, w4a16_matmul, paged_attention

Everything runs as hand-written CUDA in libspecq.so (see include/specq.h); importing this
package fails loudly if the library has not been built.
"""
import torch

from . import _lib
from . import fixtures
from .fixtures import make_paged_kv, paged_attention_ref, quantize_weight_int8
from .ops import (QUANT_PLAIN, QUANT_RESIDUAL, QUANT_SILU_MUL, KernelHandle, _paged_attn_kernel, _w4a16_kernel,
                  _w8a8_kernel, kv_append, pack_int4, paged_attention, paged_attention_packed, quant_rows,
                  w4a16_matmul, w8a8_accumulator, w8a8_matmul)

_lib.load()



def quantize_act_int8(x):
    """Per-token symmetric INT8 (kernels.py:58-62) -> (int8 like x, fp32 scales x.shape[:-1]).

    A float16 CUDA tensor is quantised by the device kernel (quant_rows), bit-exact with the
    reference's torch function on the GPU; any other tensor by that same torch formula, on
    its own device, as the reference's function runs."""
    if x.is_cuda and x.dtype == torch.float16 and x.dim() >= 1 and x.numel() > 0:
        x2 = x.reshape(-1, x.shape[-1])
        q, s = quant_rows(x2)
        return q.view(x.shape), s.view(x.shape[:-1])
    return fixtures.quantize_act_int8(x)


def quantize_weight_int4(w, group=128):
    """Group-wise INT4 with split-half packing (kernels.py:138-147) -> (packed uint8 [N, K/2],
    fp16 scales [N, K/group], fp16 dequantised [N, K]).

    A 2-D float16 / float32 / bfloat16 CUDA tensor is packed by the device kernel (pack_int4),
    bit-exact with the reference's torch function on the GPU; a CPU tensor by that same torch
    formula, as the reference's function runs there."""
    if w.is_cuda and w.dim() == 2 and w.dtype in (torch.float16, torch.float32, torch.bfloat16):
        return pack_int4(w, group, deq=True)
    return fixtures.quantize_weight_int4(w, group)


get_status = _lib.get_status
SpecqError = _lib.SpecqError

__all__ = [
    "w8a8_matmul", "w4a16_matmul", "paged_attention", "w8a8_accumulator",
    "quantize_act_int8", "quantize_weight_int8", "quantize_weight_int4", "make_paged_kv", "paged_attention_ref",
    "KernelHandle", "get_status", "SpecqError",
    "quant_rows", "kv_append", "pack_int4", "fixtures", "paged_attention_packed", "QUANT_PLAIN", "QUANT_RESIDUAL", "QUANT_SILU_MUL",
]

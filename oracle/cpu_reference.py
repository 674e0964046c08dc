"""Timed CPU baseline: the reference's own exact PyTorch path, restated on CPU tensors
(TEST / BENCH INFRASTRUCTURE ONLY -- never on the product path).

`bench.py` times these as `cpu_baseline` (and as its `--impl reference` arm) on the GPU box's
host cores.  They are the functions the reference checks its kernels against:

  w8a8:   ((a_q.float() @ w_q.float().T) * sa[:, None] * sw[None, :]).half()   (correctness.py:37)
  w4a16:  (x.float() @ deq.float().T).half(),  deq from the packed weights   (correctness.py:76,
          with the dequantisation of kernels.py:117-127)
  attn:   paged_attention_ref                                                (kernels.py:289-309)

Parity of these formulas with the reference is pinned by tests/test_oracle_golden.py (the
numpy oracle) and tests/test_cpu_reference.py (this module against the same goldens).
"""
from __future__ import annotations

import torch


def w8a8(a_q, sa, w_q, sw):
    return ((a_q.float() @ w_q.float().T) * sa[:, None] * sw[None, :]).half()


def dequant_int4(wp, sc, group=128):
    """fp16(q * fp16 scale) from the split-half packing (low nibble: k < K/2, high: k >= K/2)."""
    lo = (wp & 0xF).to(torch.int16) - 8
    hi = ((wp >> 4) & 0xF).to(torch.int16) - 8
    q = torch.cat([lo, hi], dim=1).to(torch.float16)
    return q * sc.repeat_interleave(group, dim=1)[:, : q.shape[1]]


def w4a16(x, deq):
    return (x.float() @ deq.float().T).half()


def paged_attention(q, kc, vc, ks, vs, block_tbl, ctx_len, q_len):
    n_b, _, h, d = q.shape
    page, h_kv = kc.shape[1], kc.shape[2]
    g = h // h_kv
    out = torch.zeros(q.shape, dtype=torch.float32)
    for b in range(n_b):
        L = int(ctx_len[b])
        t = torch.arange(L)
        phys = block_tbl[b].long()[t // page]
        slot = t % page
        k = (kc[phys, slot].float() * ks[phys, slot].float()[..., None]).repeat_interleave(g, dim=1)
        v = (vc[phys, slot].float() * vs[phys, slot].float()[..., None]).repeat_interleave(g, dim=1)
        qq = q[b, :q_len].float()
        s = torch.einsum("qhd,khd->hqk", qq, k) / d ** 0.5
        last = L - q_len + torch.arange(q_len)
        s = s.masked_fill(t[None, None, :] > last[None, :, None], float("-inf"))
        out[b, :q_len] = torch.einsum("hqk,khd->qhd", s.softmax(-1), v)
    return out.half()

"""Host-side helpers of the reference module's public API, in PyTorch.

The reference's `kernels.py` exports these next to its three kernels, and its scripts import
them through `from kernels import *` (correctness.py:4, bench_*.py), so the drop-in module
keeps them with the same names, arguments and results:

  quantize_act_int8     per-token symmetric INT8              (kernels.py:58-62)
  quantize_weight_int8  per-output-channel symmetric INT8     (kernels.py:65-68)
  quantize_weight_int4  group-wise INT4, split-half packing   (kernels.py:138-147)
  make_paged_kv         random INT8 paged KV cache fixture    (kernels.py:265-286)
  paged_attention_ref   PyTorch attention reference           (kernels.py:289-309)

The quantisers' rounding steps and the fixture's random-number call order are part of the
data format (the same seed must give the same cache), so they follow the reference step by
step.  They run as ordinary torch ops on whatever device their input lives on and are not
on any kernel path: `ops.py` never calls them.
"""
from __future__ import annotations

import torch


def _symmetric_quant(x: torch.Tensor, qmax: int, scale_dtype=torch.float32):
    """Symmetric quantisation along the last dim: s = max|x| / qmax (floored at 1e-8),
    q = clamp(round_half_even(x / s), -qmax, qmax) as int8."""
    s = x.abs().amax(dim=-1).float().clamp(min=1e-8) / float(qmax)
    q = torch.round(x.float() / s.unsqueeze(-1)).clamp(-qmax, qmax).to(torch.int8)
    return q, s.to(scale_dtype)


def quantize_act_int8(x):
    """Dynamic per-token symmetric INT8: returns (int8 [M, K], fp32 scales [M])."""
    return _symmetric_quant(x, 127)


def quantize_weight_int8(w):
    """Per-output-channel symmetric INT8: returns (int8 [N, K], fp32 scales [N])."""
    return _symmetric_quant(w, 127)


def quantize_weight_int4(w, group=128):
    """Group-wise symmetric INT4 in [-8, 7].

    Returns (packed uint8 [N, K/2], scales fp16 [N, K/group], dequantised fp16 [N, K]).
    Byte j of row n holds q[n, j] + 8 in its low nibble and q[n, j + K/2] + 8 in its high
    nibble.  The dequantised copy uses the fp32 scale before rounding to fp16.
    """
    n, k = w.shape
    assert k % 2 == 0 and (k // 2) % group == 0
    groups = w.float().reshape(n, k // group, group)
    scale = groups.abs().amax(dim=-1).clamp(min=1e-8) / 7.0
    q = torch.round(groups / scale.unsqueeze(-1)).clamp(-8, 7)
    deq = (q * scale.unsqueeze(-1)).reshape(n, k).to(torch.float16)
    nib = (q.reshape(n, k) + 8).to(torch.int16)
    packed = (nib[:, : k // 2] | (nib[:, k // 2:] << 4)).to(torch.uint8).contiguous()
    return packed, scale.to(torch.float16).contiguous(), deq


def make_paged_kv(B, ctx_len, H_KV, D, PAGE=16, device="cuda", seed=0):
    """Random INT8 KV cache [P, PAGE, H_KV, D] with per-(token, head) fp16 scales.

    Pages are assigned to sequences through a shuffled block table [B, max_pages] (int32);
    ctx_len [B] (int32) is returned as given.  A CPU generator seeded with `seed` draws, in
    this order, the page permutation, the K values and the V values.
    """
    gen = torch.Generator(device="cpu").manual_seed(seed)
    n_pages = [-(-int(n) // PAGE) for n in ctx_len]
    perm = torch.randperm(sum(n_pages), generator=gen).to(torch.int32)
    table = torch.zeros((B, max(n_pages)), dtype=torch.int32)
    offsets = [0]
    for n in n_pages:
        offsets.append(offsets[-1] + n)
    for b, n in enumerate(n_pages):
        table[b, :n] = perm[offsets[b]:offsets[b] + n]
    shape = (sum(n_pages), PAGE, H_KV, D)
    k_src = torch.randn(shape, generator=gen).half()
    v_src = torch.randn(shape, generator=gen).half()
    kc, ks = _symmetric_quant(k_src, 127, torch.float16)
    vc, vs = _symmetric_quant(v_src, 127, torch.float16)
    return tuple(t.to(device).contiguous() for t in (kc, vc, ks, vs, table)) + (
        torch.tensor(ctx_len, dtype=torch.int32, device=device),)


def paged_attention_ref(q, kc, vc, ks, vs, block_tbl, ctx_len, q_len):
    """PyTorch reference of the verification attention, in fp32, returned as fp16.

    For sequence b with context L = ctx_len[b], query token qi < q_len of head h attends to
    tokens t <= L - q_len + qi through the block table; K/V are dequantised with their
    per-(token, kv-head) scales and kv-head h // (H / H_KV) serves head h.  Query slots
    >= q_len are zero.
    """
    n_b, _, h, d = q.shape
    page, h_kv = kc.shape[1], kc.shape[2]
    group = h // h_kv
    out = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    for b in range(n_b):
        L = int(ctx_len[b])
        t = torch.arange(L, device=q.device)
        phys = block_tbl[b].long()[t // page]
        slot = t % page
        k = (kc[phys, slot].float() * ks[phys, slot].float().unsqueeze(-1))     # [L, H_KV, D]
        v = (vc[phys, slot].float() * vs[phys, slot].float().unsqueeze(-1))
        qq = q[b, :q_len].float().reshape(q_len, h_kv, group, d)               # [ql, H_KV, G, D]
        scores = torch.einsum("qkgd,tkd->kgqt", qq, k) * (1.0 / d ** 0.5)
        last = L - q_len + torch.arange(q_len, device=q.device)                 # last visible token
        scores = scores.masked_fill(t.view(1, 1, 1, L) > last.view(1, 1, q_len, 1), float("-inf"))
        o = torch.einsum("kgqt,tkd->qkgd", torch.softmax(scores, dim=-1), v)
        out[b, :q_len] = o.reshape(q_len, h, d)
    return out.half()

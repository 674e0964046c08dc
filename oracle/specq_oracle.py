"""CPU oracle for the three verification-shape kernels (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only `tests/`, `__graft_entry__.smoke()`
and the `cpu_baseline` / `--impl reference` legs of `bench.py` may import it.  The CUDA
path in `specdec-quant-triton_b200/` never imports it and has no CPU fallback.

Every function restates the arithmetic of the reference repository
(Vaibhav1067/specdec-quant-triton) in numpy, with the file:line it follows.  Integer
work is exact (int64 / float64 accumulation); floating-point steps keep the reference's
dtype at every rounding point so that outputs can be compared bit for bit where the
reference itself is deterministic.

Parity pin: the restatement is checked against golden vectors produced by the
reference's own code (its quantizers, `make_paged_kv`, `paged_attention_ref` and its
Triton kernels executed by the Triton CPU interpreter) in `tests/golden/`, made by
`tests/golden/make_golden.py`.
"""
from __future__ import annotations

import numpy as np

# ----------------------------------------------------------------------------------
# Quantizers  (kernels.py:58-68, kernels.py:138-147)
# ----------------------------------------------------------------------------------


def _amax_rows(x: np.ndarray) -> np.ndarray:
    # kernels.py:60 -- x.abs().amax(dim=-1).float(); |fp16| and its max are exact.
    return np.abs(x).max(axis=-1).astype(np.float32)


def _div_scalar(x: np.ndarray, d: float, on_cuda: bool) -> np.ndarray:
    """`tensor / d` for a Python scalar d, as torch evaluates it: an IEEE fp32 division on a CPU
    tensor, a multiplication by the fp32 reciprocal fp32(1/d) on a CUDA tensor."""
    if on_cuda:
        return (x * np.float32(1.0 / d)).astype(np.float32)
    return (x / np.float32(d)).astype(np.float32)


def quantize_act_int8(x: np.ndarray, on_cuda: bool = False):
    """Per-token symmetric INT8 (kernels.py:58-62). Returns (q int8 [M,K], s fp32 [M]).

    on_cuda: the scale's division by 127 as torch evaluates it on a GPU tensor."""
    s = _div_scalar(np.maximum(_amax_rows(x), np.float32(1e-8)), 127.0, on_cuda)
    q = np.rint(x.astype(np.float32) / s[:, None])          # torch.round: half to even
    q = np.clip(q, -127, 127).astype(np.int8)
    return q, s.astype(np.float32)


def quantize_weight_int8(w: np.ndarray, on_cuda: bool = False):
    """Per-output-channel symmetric INT8 (kernels.py:65-68)."""
    return quantize_act_int8(w, on_cuda)


def quantize_weight_int4(w: np.ndarray, group: int = 128, on_cuda: bool = False):
    """Group-wise INT4 with split-half packing (kernels.py:138-147).

    Returns (packed uint8 [N, K/2], sc fp16 [N, K/group], deq fp16 [N, K]).
    Byte j of row n holds q[n, j] + 8 in its low nibble and q[n, j + K/2] + 8 in its high
    nibble (kernels.py:143-145).  `deq` uses the fp32 scale before the fp16 cast
    (kernels.py:146), exactly as the reference does.  on_cuda: the division of the group
    maximum by 7 as torch evaluates it on a GPU tensor.
    """
    n, k = w.shape
    assert k % 2 == 0 and (k // 2) % group == 0
    wg = w.astype(np.float32).reshape(n, k // group, group)
    sc = _div_scalar(np.maximum(np.abs(wg).max(axis=-1), np.float32(1e-8)), 7.0, on_cuda)
    q = np.clip(np.rint(wg / sc[..., None]), -8, 7).reshape(n, k).astype(np.int16) + 8
    lo, hi = q[:, : k // 2], q[:, k // 2:]
    packed = (lo | (hi << 4)).astype(np.uint8)
    deq = ((q - 8).astype(np.float32).reshape(n, k // group, group) * sc[..., None]).reshape(n, k)
    return packed, sc.astype(np.float16), deq.astype(np.float16)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """Inverse of the split-half packing (kernels.py:90-92, 117-118): int8 [N, K] in [-8, 7]."""
    lo = (packed & 0xF).astype(np.int16) - 8
    hi = ((packed >> 4) & 0xF).astype(np.int16) - 8
    return np.concatenate([lo, hi], axis=1).astype(np.int8)


def dequant_int4_kernel(packed: np.ndarray, sc16: np.ndarray, group: int = 128) -> np.ndarray:
    """Dequantised weights exactly as the reference kernel forms them (kernels.py:117-127).

    `lo.to(fp16) * sc_lo` with the fp16 scale: one fp16 rounding of the product.  The product
    of two fp16 values is exact in fp32, so rounding it to fp16 reproduces fp16 multiplication.
    """
    q = unpack_int4(packed).astype(np.float32)
    n, k = q.shape
    s = np.repeat(sc16.astype(np.float32), group, axis=1)[:, :k]
    return (q * s).astype(np.float16)


# ----------------------------------------------------------------------------------
# W8A8 GEMM  (kernels.py:27-55, reference oracle correctness.py:37)
# ----------------------------------------------------------------------------------


def w8a8_acc(a_q: np.ndarray, w_q: np.ndarray) -> np.ndarray:
    """Exact integer accumulator acc[m, n] = sum_k a[m,k] * w[n,k] as int64.

    float64 BLAS is exact here: every partial sum is an integer below 2**53.
    """
    acc = a_q.astype(np.float64) @ w_q.astype(np.float64).T
    return acc.astype(np.int64)


def w8a8_epilogue(acc: np.ndarray, sa: np.ndarray, sw: np.ndarray) -> np.ndarray:
    """out = fp16((fp32(acc) * sa[m]) * sw[n]) -- kernels.py:53-55, left-to-right in fp32."""
    c = acc.astype(np.float32)
    c = c * sa.astype(np.float32)[:, None]
    c = c * sw.astype(np.float32)[None, :]
    return c.astype(np.float16)


def w8a8_ref(a_q, sa, w_q, sw) -> np.ndarray:
    """Reference W8A8 output with an exact accumulator (correctness.py:37 with int64)."""
    return w8a8_epilogue(w8a8_acc(a_q, w_q), sa, sw)


# ----------------------------------------------------------------------------------
# W4A16 GEMM  (kernels.py:95-135, reference oracle correctness.py:76)
# ----------------------------------------------------------------------------------


def w4a16_ref(x: np.ndarray, packed: np.ndarray, sc16: np.ndarray, group: int = 128) -> np.ndarray:
    """Kernel-semantics W4A16: fp16 dequant with the fp16 scale, float64 dot, fp16 out."""
    deq = dequant_int4_kernel(packed, sc16, group)
    return (x.astype(np.float64) @ deq.astype(np.float64).T).astype(np.float16)


def w4a16_ref_from_deq(x: np.ndarray, deq: np.ndarray) -> np.ndarray:
    """correctness.py:76 -- x.float() @ deq.float().T, as fp32 (before any cast)."""
    return (x.astype(np.float64) @ deq.astype(np.float64).T).astype(np.float32)


# ----------------------------------------------------------------------------------
# INT8 paged verification attention  (kernels.py:178-236, oracle kernels.py:289-309)
# ----------------------------------------------------------------------------------


def paged_attention_ref(q, kc, vc, ks, vs, block_tbl, ctx_len, q_len) -> np.ndarray:
    """Restatement of paged_attention_ref (kernels.py:289-309) in float64.

    q [B, QL, H, D] fp16; kc/vc [P, PAGE, H_KV, D] int8; ks/vs [P, PAGE, H_KV] (fp16 or fp32);
    block_tbl [B, max_pages] int32; ctx_len [B] int32 (includes the q_len query tokens).
    Row qi attends to tokens t <= L - q_len + qi (kernels.py:306-307).  Rows >= q_len stay 0.
    """
    b_, _, h, d = q.shape
    h_kv = kc.shape[2]
    g = h // h_kv
    page = kc.shape[1]
    out = np.zeros(q.shape, dtype=np.float64)
    for b in range(b_):
        L = int(ctx_len[b])
        idx = np.arange(L)
        pg = block_tbl[b, idx // page].astype(np.int64)
        off = idx % page
        k = kc[pg, off].astype(np.float64) * ks[pg, off].astype(np.float64)[..., None]
        v = vc[pg, off].astype(np.float64) * vs[pg, off].astype(np.float64)[..., None]
        k = np.repeat(k, g, axis=1)                              # repeat_interleave, dim=1
        v = np.repeat(v, g, axis=1)
        qq = q[b, :q_len].astype(np.float64)                     # [ql, H, D]
        s = np.einsum("qhd,khd->hqk", qq, k) / np.sqrt(d)
        qpos = L - q_len + np.arange(q_len)
        s = np.where(idx[None, None, :] > qpos[None, :, None], -np.inf, s)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p = p / p.sum(axis=-1, keepdims=True)
        out[b, :q_len] = np.einsum("hqk,khd->qhd", p, v)
    return out.astype(np.float16)


# ----------------------------------------------------------------------------------
# Verification-layer glue (the plan-graph stack of bench_graphs.py:49-64, extended with a
# connected data flow): KV-cache append, SiLU-mul quantisation, fp16 residual add
# ----------------------------------------------------------------------------------


def kv_quant_rows(x: np.ndarray, on_cuda: bool = True):
    """INT8 of K or V rows [T, H_KV, D] with one scale per (token, head), the cache format of
    make_paged_kv's q8 (kernels.py:276-283): s = max(amax, 1e-8) / 127 (fp32; stored fp16),
    q = clamp(rint(x / s), -127, 127) with the fp32 s.  on_cuda: `/ 127.0` as torch evaluates
    it on a GPU tensor (the device append runs there)."""
    xf = x.astype(np.float32)
    s = _div_scalar(np.maximum(np.abs(xf).max(axis=-1), np.float32(1e-8)), 127.0, on_cuda)
    q = np.clip(np.rint(xf / s[..., None]), -127, 127).astype(np.int8)
    return q, s.astype(np.float16)


def kv_append(x_rows, k_col, v_col, kc, vc, ks, vs, block_tbl, ctx_len, q_len, n_seqs, h_kv, d, page):
    """Write the K / V of the q_len newest tokens of each sequence into copies of the caches.
    x_rows: packed token rows (sequence b's token t at row b*q_len + t), K of head h at columns
    k_col + h*d, V at v_col + h*d; token t goes to position ctx_len[b] - q_len + t."""
    kc, vc, ks, vs = kc.copy(), vc.copy(), ks.copy(), vs.copy()
    for b in range(n_seqs):
        for t in range(q_len):
            pos = int(ctx_len[b]) - q_len + t
            pg, slot = int(block_tbl[b, pos // page]), pos % page
            row = x_rows[b * q_len + t]
            for col, c, sc in ((k_col, kc, ks), (v_col, vc, vs)):
                q, s = kv_quant_rows(row[col:col + h_kv * d].reshape(1, h_kv, d))
                c[pg, slot] = q[0]
                sc[pg, slot] = s[0]
    return kc, vc, ks, vs


def silu_mul(gu: np.ndarray) -> np.ndarray:
    """silu(gate) * up in fp32 for fp16 rows [M, 2N] (gate = first half): the MLP activation of
    the stack's gate_up projection, torch.nn.functional.silu(g.float()) * u.float()."""
    n = gu.shape[1] // 2
    g = gu[:, :n].astype(np.float32)
    u = gu[:, n:].astype(np.float32)
    return (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32) * u


def residual_add(x: np.ndarray, r: np.ndarray) -> np.ndarray:
    """fp16(x + r) of two fp16 tensors (one rounding: the fp32 sum of two fp16 values rounds to
    the same fp16 value as the exact sum, 24 >= 2 * 11 + 2 bits)."""
    return (x.astype(np.float32) + r.astype(np.float32)).astype(np.float16)


# ----------------------------------------------------------------------------------
# Error metrics used by the reference's correctness script
# ----------------------------------------------------------------------------------


def max_rel_err_plus1(out, ref) -> float:
    """correctness.py:38 -- max |out - ref| / (|ref| + 1)."""
    o = np.asarray(out, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    return float((np.abs(o - r) / (np.abs(r) + 1.0)).max()) if r.size else 0.0


def rel_fro_err(out, ref) -> float:
    """correctness.py:77 -- ||out - ref||_F / ||ref||_F."""
    o = np.asarray(out, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    n = np.linalg.norm(r)
    return float(np.linalg.norm(o - r) / n) if n > 0 else float(np.linalg.norm(o - r))


def max_abs_err(out, ref) -> float:
    """correctness.py:98 -- max |out - ref|."""
    o = np.asarray(out, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    return float(np.abs(o - r).max()) if r.size else 0.0

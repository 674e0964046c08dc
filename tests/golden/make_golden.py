"""Generate the golden vectors in this folder from the reference implementation itself.

Run in a container that has the reference checkout (read-only is fine) and Triton:

    TRITON_INTERPRET=1 python tests/golden/make_golden.py [--ref /path/to/reference]

The script imports the reference's `kernels.py` and, for every case, records its inputs
together with what the reference produces for them:
  * its quantizers (`quantize_act_int8`, `quantize_weight_int8`, `quantize_weight_int4`,
    kernels.py:58-68, 138-147) and its paged-KV fixture (`make_paged_kv`, kernels.py:265-286);
  * its exact PyTorch oracles (correctness.py:37, correctness.py:76, kernels.py:289-309);
  * the outputs of its three Triton kernels (`w8a8_matmul`, `w4a16_matmul`,
    `paged_attention`, kernels.py:71, 150, 239), executed by Triton's CPU interpreter,
    including their plan mode on sentinel-filled outputs (correctness.py:50-65, 103-120).

All inputs come from seeded CPU generators.  Nothing at run time of the tests reads the
reference: the `.npz` files are the fixtures.
"""
from __future__ import annotations

import argparse
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
SEEDS = {"w8a8_small": 11, "w8a8_ragged": 12, "w8a8_m1": 13, "w4a16_small": 21, "w4a16_mid": 22}


def _np(t):
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.numpy().copy()


def _save(name, **arrays):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **{k: (_np(v) if torch.is_tensor(v) else np.asarray(v)) for k, v in arrays.items()})
    print("wrote", os.path.relpath(path), {k: tuple(np.asarray(_np(v) if torch.is_tensor(v) else v).shape)
                                            for k, v in arrays.items()})


def _uniform(g, shape, lo, hi):
    return torch.rand(shape, generator=g) * (hi - lo) + lo


def _int8_uniform(g, shape):
    # int8 uniform in [-127, 127], the value distribution of the W8A8 benchmark config.
    return torch.randint(-127, 128, shape, generator=g, dtype=torch.int16).to(torch.int8)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    import kernels as R  # the reference module

    # ------------------------------------------------------------------ quantizers
    g = torch.Generator().manual_seed(1234)
    x = torch.randn(7, 256, generator=g).half()
    w = (torch.randn(48, 256, generator=g) * 0.02).half()
    w4 = torch.randn(40, 512, generator=g).half()
    a_q, sa = R.quantize_act_int8(x)
    w_q, sw = R.quantize_weight_int8(w)
    wp, sc, deq = R.quantize_weight_int4(w4, group=128)
    x_edge = torch.zeros(3, 64).half()                 # all-zero row exercises the 1e-8 clamp
    x_edge[1] = torch.linspace(-2, 2, 64).half()
    x_edge[2, 5] = 65504.0
    e_q, e_s = R.quantize_act_int8(x_edge)
    _save("quant", x=x, w=w, w4=w4, a_q=a_q, sa=sa, w_q=w_q, sw=sw, wp=wp, sc=sc, deq=deq,
          x_edge=x_edge, e_q=e_q, e_s=e_s)

    # ------------------------------------------------------------------ W8A8
    cases = [("w8a8_small", 5, 96, 256), ("w8a8_ragged", 19, 72, 200), ("w8a8_m1", 1, 40, 128)]
    for name, M, N, K in cases:
        g = torch.Generator().manual_seed(SEEDS[name])
        aq = _int8_uniform(g, (M, K))
        wq = _int8_uniform(g, (N, K))
        sa_ = _uniform(g, (M,), 0.001, 0.02).float()
        sw_ = _uniform(g, (N,), 0.001, 0.02).float()
        out, _ = R.w8a8_matmul(aq, sa_, wq, sw_, BLOCK_M=16, BLOCK_N=32, BLOCK_K=64)
        ref = (aq.float() @ wq.float().T) * sa_[:, None] * sw_[None, :]   # correctness.py:37
        _save(name, a_q=aq, sa=sa_, w_q=wq, sw=sw_, out=out, ref=ref)

    # plan mode: fixed grid at M_MAX, active M from the device plan, sentinel rows untouched
    g = torch.Generator().manual_seed(77)
    MMAX, N, K = 40, 64, 256
    aq = _int8_uniform(g, (MMAX, K))
    wq = _int8_uniform(g, (N, K))
    sa_ = _uniform(g, (MMAX,), 0.001, 0.02).float()
    sw_ = _uniform(g, (N,), 0.001, 0.02).float()
    plan = torch.zeros(8, dtype=torch.int32)
    plan[0] = 13
    out = torch.full((MMAX, N), 12345.0).half()
    R.w8a8_matmul(aq, sa_, wq, sw_, out=out, plan=plan, grid_m_max=MMAX, BLOCK_M=16, BLOCK_N=32, BLOCK_K=64)
    _save("w8a8_plan", a_q=aq, sa=sa_, w_q=wq, sw=sw_, plan=plan, out=out)

    # ------------------------------------------------------------------ W4A16
    for name, M, N, K in [("w4a16_small", 3, 64, 512), ("w4a16_mid", 20, 48, 1024)]:
        g = torch.Generator().manual_seed(SEEDS[name])
        xa = torch.randn(M, K, generator=g).half()
        ww = torch.randn(N, K, generator=g).half()
        wp_, sc_, deq_ = R.quantize_weight_int4(ww, group=128)
        out, _ = R.w4a16_matmul(xa, wp_, sc_, BLOCK_M=16, BLOCK_N=32, BLOCK_K=64)
        ref = xa.float() @ deq_.float().T                                    # correctness.py:76
        _save(name, x=xa, wp=wp_, sc=sc_, deq=deq_, out=out, ref=ref)

    g = torch.Generator().manual_seed(88)
    MMAX, N, K = 24, 32, 512
    xa = torch.randn(MMAX, K, generator=g).half()
    ww = torch.randn(N, K, generator=g).half()
    wp_, sc_, deq_ = R.quantize_weight_int4(ww, group=128)
    plan = torch.zeros(8, dtype=torch.int32)
    plan[0] = 7
    out = torch.full((MMAX, N), 12345.0).half()
    R.w4a16_matmul(xa, wp_, sc_, out=out, plan=plan, grid_m_max=MMAX, BLOCK_M=16, BLOCK_N=32, BLOCK_K=64)
    _save("w4a16_plan", x=xa, wp=wp_, sc=sc_, plan=plan, out=out)

    # ------------------------------------------------------------------ paged attention
    H, H_KV, D = 8, 2, 128
    B, ql = 2, 3
    ctx = [37, 70]                                   # not page aligned
    kc, vc, ks, vs, bt, cl = R.make_paged_kv(B, ctx, H_KV, D, device="cpu", seed=5)
    g = torch.Generator().manual_seed(6)
    q = torch.randn(B, ql, H, D, generator=g).half()
    ref = R.paged_attention_ref(q, kc, vc, ks, vs, bt, cl, ql)
    o_fused, _ = R.paged_attention(q, kc, vc, ks, vs, bt, cl, ql, QPP=ql, BLOCK_N=32)
    o_tok, _ = R.paged_attention(q, kc, vc, ks, vs, bt, cl, ql, QPP=1, BLOCK_N=32)
    _save("attn_small", q=q, kc=kc, vc=vc, ks=ks, vs=vs, bt=bt, cl=cl, q_len=ql,
          ref=ref, out_fused=o_fused, out_tok=o_tok)

    # fp32 scales (the value type of the attention benchmark config) through the same kernel
    ks32, vs32 = ks.float(), vs.float()
    o32, _ = R.paged_attention(q, kc, vc, ks32, vs32, bt, cl, ql, QPP=ql, BLOCK_N=32)
    ref32 = R.paged_attention_ref(q, kc, vc, ks32, vs32, bt, cl, ql)
    _save("attn_f32scales", q=q, kc=kc, vc=vc, ks=ks32, vs=vs32, bt=bt, cl=cl, q_len=ql,
          ref=ref32, out_fused=o32)

    # plan mode: fixed grid (BMAX, QLMAX), active (n_seqs, q_len) = (2, 3), sentinel 7.0
    BMAX, QLMAX = 3, 4
    ctxp = [20, 45, 33]
    kc, vc, ks, vs, bt, cl = R.make_paged_kv(BMAX, ctxp, H_KV, D, device="cpu", seed=9)
    qf = torch.randn(BMAX, QLMAX, H, D, generator=g).half()
    plan = torch.zeros(8, dtype=torch.int32)
    plan[0], plan[1] = 2, 3
    out = torch.full_like(qf, 7.0)
    R.paged_attention(qf, kc, vc, ks, vs, bt, cl, QLMAX, QPP=QLMAX, plan=plan, out=out, BLOCK_N=32)
    refp = R.paged_attention_ref(qf[:2], kc, vc, ks, vs, bt[:2], cl[:2], 3)
    _save("attn_plan", q=qf, kc=kc, vc=vc, ks=ks, vs=vs, bt=bt, cl=cl, plan=plan, out=out, ref=refp)


if __name__ == "__main__":
    main()

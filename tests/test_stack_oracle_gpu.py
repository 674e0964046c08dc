"""One layer of the plan-graph verification stack (specq.stack) against the oracle.

The reference checks its plan graph only against its own eager run (bench_graphs.py:144-159);
this pins every kernel call of a stack layer to the oracle as well:

  1. stage by stage, each call recomputed by the oracle from the stack's own inputs to that call
     (so a wrong buffer, column offset, scale or mode in the wiring shows up at the call that
     has it): the quantiser, the four W8A8 GEMMs, the KV append and the residual adds
     bit-exact; attention within the reference's 2e-2 max-abs bar (correctness.py:100) and
     1e-3 Frobenius-relative; the SiLU-mul quantiser within one int8 unit (the kernel's fast
     exponential may move a rounding tie) and 1e-6 relative on the scales;
  2. end to end, the whole layer composed from oracle functions alone from the initial
     residual stream: the final residual stream within 1e-2 Frobenius-relative (attention's
     error moves a few int8 roundings of the next quantiser, and those propagate).

Both eager execution and the single plan-buffer graph captured at the maximum shape.
"""
import numpy as np
import pytest
import torch

from oracle import specq_oracle as O

pytestmark = pytest.mark.gpu

H, H_KV, D, HID, FF, PAGE = 4, 2, 128, 512, 1024, 16


def _np(t):
    return t.detach().cpu().numpy()


def _quant(x):
    return O.quantize_act_int8(x, on_cuda=True)


def _oracle_layer(h0, w, kv0, bt, cl, B, ql):
    """The layer from oracle functions alone -> (final residual stream, appended caches)."""
    kc, vc, ks, vs = kv0
    x8, sx = _quant(h0)
    qkv = O.w8a8_ref(x8, sx, *w["qkv"])
    kc, vc, ks, vs = O.kv_append(qkv, H * D, (H + H_KV) * D, kc, vc, ks, vs, bt, cl, ql, B, H_KV, D, PAGE)
    q = qkv[:, : H * D].reshape(B, ql, H, D)
    attn = O.paged_attention_ref(q, kc, vc, ks, vs, bt, cl, ql).reshape(B * ql, H * D)
    o = O.w8a8_ref(*_quant(attn), *w["o"])
    h1 = O.residual_add(o, h0)
    gu = O.w8a8_ref(*_quant(h1), *w["gu"])
    f8, sf = O.quantize_act_int8(O.silu_mul(gu), on_cuda=True)
    down = O.w8a8_ref(f8, sf, *w["down"])
    return O.residual_add(down, h1), (kc, vc, ks, vs)


@pytest.mark.parametrize("use_plan", [False, True])
@pytest.mark.parametrize("B,ql", [(3, 5), (2, 3)])
def test_stack_layer_matches_oracle(cuda, use_plan, B, ql):
    from specq.stack import Stack
    st = Stack(layers=1, hid=HID, ff=FF, heads=H, kv_heads=H_KV, head_dim=D, ctx=96, b_max=3, ks=(0, 2, 4),
               seed=7)
    st.snapshot()
    st.reset()
    kv0 = tuple(_np(t) for t in st.kv[0][:4])
    bt, cl = _np(st.kv[0][4]), _np(st.kv[0][5])
    w = {k: (_np(v[0]), _np(v[1])) for k, v in st.w[0].items()}
    M = B * ql
    if use_plan:
        st.set_plan(st.b_max, st.ql_max)
        g = st.capture(lambda: st.step(st.b_max, st.ql_max, use_plan=True))
        st.reset()
        st.set_plan(B, ql)
        g.replay()
    else:
        st.step(B, ql)
    torch.cuda.synchronize()
    h0 = _np(st.h0[:M])

    # ---- 1. stage by stage, each call from the stack's own inputs -----------------------
    qkv = _np(st.qkv[:M])
    x8, sx = _quant(h0)
    assert np.array_equal(qkv.view(np.uint16), O.w8a8_ref(x8, sx, *w["qkv"]).view(np.uint16)), "qkv projection"
    kc, vc, ks, vs = O.kv_append(qkv, H * D, (H + H_KV) * D, *kv0, bt, cl, ql, B, H_KV, D, PAGE)
    for got, want, name in zip(st.kv[0][:4], (kc, vc, ks, vs), ("kc", "vc", "ks", "vs")):
        assert np.array_equal(_np(got).view(np.uint8), want.view(np.uint8)), f"KV append: {name}"
    attn = _np(st.attn[:M])
    ref_attn = O.paged_attention_ref(qkv[:, : H * D].reshape(B, ql, H, D), kc, vc, ks, vs, bt, cl, ql)
    assert O.max_abs_err(attn, ref_attn.reshape(M, -1)) < 2e-2, "attention"
    assert O.rel_fro_err(attn, ref_attn.reshape(M, -1)) < 1e-3, "attention"
    o = _np(st.o[:M])
    assert np.array_equal(o.view(np.uint16), O.w8a8_ref(*_quant(attn), *w["o"]).view(np.uint16)), "o projection"
    h1 = O.residual_add(o, h0)
    gu = _np(st.gu[:M])
    assert np.array_equal(gu.view(np.uint16), O.w8a8_ref(*_quant(h1), *w["gu"]).view(np.uint16)), "gate_up"
    f8, sf = _np(st.f8[:M]), _np(st.sf[:M])
    rf8, rsf = O.quantize_act_int8(O.silu_mul(gu), on_cuda=True)
    assert np.allclose(sf, rsf, rtol=1e-6, atol=0), "SiLU-mul scales"
    d = np.abs(f8.astype(np.int32) - rf8.astype(np.int32))
    assert d.max() <= 1 and (d > 0).mean() < 1e-3, "SiLU-mul int8"
    down = _np(st.down[:M])
    assert np.array_equal(down.view(np.uint16), O.w8a8_ref(f8, sf, *w["down"]).view(np.uint16)), "down projection"
    h2 = _np(st.h[:M])
    assert np.array_equal(h2.view(np.uint16), O.residual_add(down, h1).view(np.uint16)), "final residual add"
    q_last, s_last = _quant(h2)
    assert np.array_equal(_np(st.x8[:M]), q_last) and np.array_equal(_np(st.sx[:M]), s_last), "last quantiser"
    # rows past the active M (plan graph at the maximum grid) are untouched
    if use_plan and M < st.m_max:
        assert bool((st.h[M:] == st.h0[M:]).all()), "inactive residual rows"

    # ---- 2. end to end from the oracle alone ----------------------------------------------
    h_ref, _ = _oracle_layer(h0, w, kv0, bt, cl, B, ql)
    err = O.rel_fro_err(h2, h_ref)
    assert err < 1e-2, f"layer output rel-fro {err}"

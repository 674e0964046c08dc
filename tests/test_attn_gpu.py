"""GPU parity of the INT8 paged verification attention against the oracle (a float64
restatement of paged_attention_ref, kernels.py:289-309) and the reference kernel's own
outputs.  Tolerances: max |err| < 2e-2 (correctness.py:100) and Frobenius-relative < 1e-3
(north-star bar); plan mode is bit-exact against eager mode and never writes inactive slots."""
import numpy as np
import pytest
import torch

from oracle import specq_oracle as O

pytestmark = pytest.mark.gpu


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _np(t):
    return t.detach().cpu().numpy()


def _check(out, ref, mask_rows=None):
    o = _np(out).astype(np.float64)
    r = ref.astype(np.float64)
    assert np.isfinite(o).all()
    assert O.max_abs_err(o, r) < 2e-2
    assert O.rel_fro_err(o, r) < 1e-3


def _ref(q, kc, vc, ks, vs, bt, cl, ql):
    return O.paged_attention_ref(_np(q), _np(kc), _np(vc), _np(ks), _np(vs), _np(bt), _np(cl), ql)


@pytest.mark.parametrize("name", ["attn_small", "attn_f32scales"])
def test_golden(cuda, golden, name):
    import specq
    g = golden(name)
    ql = int(g["q_len"])
    t = {k: _dev(g[k]) for k in ("q", "kc", "vc", "ks", "vs", "bt", "cl")}
    for qpp, key in ((ql, "out_fused"), (1, "out_tok")):
        out, ck = specq.paged_attention(t["q"], t["kc"], t["vc"], t["ks"], t["vs"], t["bt"], t["cl"], ql, QPP=qpp)
        torch.cuda.synchronize()
        _check(out, g["ref"])
        if key in g:
            assert O.max_abs_err(_np(out), g[key]) < 2e-2
            assert O.rel_fro_err(_np(out), g[key]) < 1e-3


def test_golden_plan_mode(cuda, golden):
    import specq
    g = golden("attn_plan")
    t = {k: _dev(g[k]) for k in ("q", "kc", "vc", "ks", "vs", "bt", "cl", "plan")}
    b_act, ql = int(g["plan"][0]), int(g["plan"][1])
    qlmax = g["q"].shape[1]
    out = torch.full_like(t["q"], 7.0)
    specq.paged_attention(t["q"], t["kc"], t["vc"], t["ks"], t["vs"], t["bt"], t["cl"], qlmax, QPP=qlmax,
                          plan=t["plan"], out=out)
    torch.cuda.synchronize()
    o = _np(out)
    assert O.max_abs_err(o[:b_act, :ql], g["ref"][:, :ql]) < 2e-2
    assert O.max_abs_err(o[:b_act, :ql], g["out"][:b_act, :ql]) < 2e-2
    assert np.all(o[b_act:] == np.float16(7.0)) and np.all(o[:b_act, ql:] == np.float16(7.0))


def test_correctness_sweep(cuda):
    """correctness.py:86-101: B in {1,3,8} x k in {2,4,8}, random non-page-aligned contexts,
    QPP in {1, k+1}."""
    import specq
    H, H_KV, D = 32, 8, 128
    gen = torch.Generator().manual_seed(0)
    for B in (1, 3, 8):
        for k in (2, 4, 8):
            ql = k + 1
            ctx = [int(x) for x in torch.randint(ql, 700, (B,), generator=gen)]
            kc, vc, ks, vs, bt, cl = specq.make_paged_kv(B, ctx, H_KV, D, device="cuda", seed=B * 10 + k)
            q = torch.randn(B, ql, H, D, generator=gen).half().cuda()
            ref = _ref(q, kc, vc, ks, vs, bt, cl, ql)
            for qpp in (1, ql):
                out, _ = specq.paged_attention(q, kc, vc, ks, vs, bt, cl, ql, QPP=qpp)
                _check(out, ref)


def _config2(B=8, ctx=4096, H=32, H_KV=8, D=128, page=16, ql=9, seed=0, scale_dtype=torch.float32):
    """Config 2 value distributions: Q ~ N(0,1); K/V int8 uniform in [-127, 127]; per-token /
    per-head scales uniform in [0.005, 0.02]; block table = seeded permutation of the pages."""
    g = torch.Generator().manual_seed(seed)
    n_pages = B * ((ctx + page - 1) // page)
    kc = torch.randint(-127, 128, (n_pages, page, H_KV, D), generator=g, dtype=torch.int16).to(torch.int8)
    vc = torch.randint(-127, 128, (n_pages, page, H_KV, D), generator=g, dtype=torch.int16).to(torch.int8)
    ks = (torch.rand(n_pages, page, H_KV, generator=g) * 0.015 + 0.005).to(scale_dtype)
    vs = (torch.rand(n_pages, page, H_KV, generator=g) * 0.015 + 0.005).to(scale_dtype)
    bt = torch.randperm(n_pages, generator=g).to(torch.int32).view(B, -1)
    cl = torch.full((B,), ctx, dtype=torch.int32)
    q = torch.randn(B, ql, H, D, generator=g).half()
    return [t.cuda() for t in (q, kc, vc, ks, vs, bt, cl)]


@pytest.mark.parametrize("scale_dtype", [torch.float32, torch.float16])
def test_config2_full_size(cuda, scale_dtype):
    import specq
    q, kc, vc, ks, vs, bt, cl = _config2(scale_dtype=scale_dtype)
    out, ck = specq.paged_attention(q, kc, vc, ks, vs, bt, cl, 9, QPP=9)
    _check(out, _ref(q, kc, vc, ks, vs, bt, cl, 9))
    assert ck.cluster >= 1


@pytest.mark.parametrize("ctx,cluster", [([1, 17, 128, 129, 2048, 8192 - 3], 4),   # 8192-token table
                                         ([5, 300, 6000], 4),                       # 6000: 3 -> 4 splits
                                         ([2, 3000, 4100], 4),
                                         ([16000, 40, 1], 8)])
def test_context_lengths_and_splits(cuda, ctx, cluster):
    import specq
    B, H, H_KV, D, ql = len(ctx), 16, 4, 128, 4
    kc, vc, ks, vs, bt, cl = specq.make_paged_kv(B, [max(c, ql) for c in ctx], H_KV, D, device="cuda", seed=3)
    q = torch.randn(B, ql, H, D, generator=torch.Generator().manual_seed(4)).half().cuda()
    out, ck = specq.paged_attention(q, kc, vc, ks, vs, bt, cl, ql)
    _check(out, _ref(q, kc, vc, ks, vs, bt, cl, ql))
    assert ck.cluster == cluster   # the context split across a cluster: a power of two


@pytest.mark.parametrize("H,H_KV,page,qpp", [(64, 8, 16, 9), (8, 8, 16, 5), (32, 8, 8, 4), (32, 8, 32, 2),
                                             (16, 2, 64, 9), (32, 8, 24, 9), (16, 4, 256, 9)])
def test_gqa_page_and_qpp_variants(cuda, H, H_KV, page, qpp):
    import specq
    B, D, ql = 3, 128, 9
    ctx = [300, 45, 777]
    kc, vc, ks, vs, bt, cl = specq.make_paged_kv(B, ctx, H_KV, D, PAGE=page, device="cuda", seed=H + page)
    q = torch.randn(B, ql, H, D, generator=torch.Generator().manual_seed(qpp)).half().cuda()
    out, _ = specq.paged_attention(q, kc, vc, ks, vs, bt, cl, ql, QPP=qpp)
    _check(out, _ref(q, kc, vc, ks, vs, bt, cl, ql))


def test_context_shorter_than_window_writes_zeros(cuda):
    """ctx_len < q_len: the first query rows see no key; the kernel writes 0 (l = 0 guard of
    kernels.py:234), the rest match the oracle."""
    import specq
    B, H, H_KV, D, ql = 1, 8, 2, 128, 4
    kc, vc, ks, vs, bt, cl = specq.make_paged_kv(B, [2], H_KV, D, device="cuda", seed=8)
    q = torch.randn(B, ql, H, D, generator=torch.Generator().manual_seed(8)).half().cuda()
    out, _ = specq.paged_attention(q, kc, vc, ks, vs, bt, cl, ql)
    o = _np(out)
    assert np.all(o[0, :2] == 0)
    with np.errstate(invalid="ignore"):
        ref = _ref(q, kc, vc, ks, vs, bt, cl, ql)
    assert O.max_abs_err(o[0, 2:], ref[0, 2:]) < 2e-2


def test_plan_mode_inactive_untouched_and_bit_exact(cuda):
    """correctness.py:103-120 plus plan == eager bit for bit (bench_graphs.py:144-159)."""
    import specq
    H, H_KV, D = 32, 8, 128
    BMAX, QLMAX = 8, 9
    gen = torch.Generator().manual_seed(99)
    ctx = [int(x) for x in torch.randint(QLMAX, 700, (BMAX,), generator=gen)]
    kc, vc, ks, vs, bt, cl = specq.make_paged_kv(BMAX, ctx, H_KV, D, device="cuda", seed=99)
    qfull = torch.randn(BMAX, QLMAX, H, D, generator=gen).half().cuda()
    plan = torch.zeros(8, dtype=torch.int32, device="cuda")
    for b_act, ql in ((1, 3), (3, 5), (8, 9), (5, 3), (8, 5)):
        plan[0], plan[1] = b_act, ql
        out = torch.full_like(qfull, 7.0)
        specq.paged_attention(qfull, kc, vc, ks, vs, bt, cl, QLMAX, QPP=QLMAX, plan=plan, out=out)
        eager = torch.zeros_like(qfull)
        specq.paged_attention(qfull[:b_act], kc, vc, ks, vs, bt[:b_act], cl[:b_act], ql, QPP=ql,
                              out=eager[:b_act])
        torch.cuda.synchronize()
        o = _np(out)
        ref = _ref(qfull[:b_act], kc, vc, ks, vs, bt[:b_act], cl[:b_act], ql)
        assert O.max_abs_err(o[:b_act, :ql], ref[:, :ql]) < 2e-2
        assert np.all(o[b_act:] == np.float16(7.0)) and np.all(o[:b_act, ql:] == np.float16(7.0))
        assert torch.equal(out[:b_act, :ql], eager[:b_act, :ql]), (b_act, ql)


def test_cuda_graph_plan_replay(cuda):
    import specq
    H, H_KV, D, BMAX, QLMAX = 32, 8, 128, 4, 9
    kc, vc, ks, vs, bt, cl = specq.make_paged_kv(BMAX, [1024] * BMAX, H_KV, D, device="cuda", seed=5)
    q = torch.randn(BMAX, QLMAX, H, D, generator=torch.Generator().manual_seed(5)).half().cuda()
    plan = torch.tensor([BMAX, QLMAX, 0, 0, 0, 0, 0, 0], dtype=torch.int32, device="cuda")
    out = torch.zeros_like(q)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        specq.paged_attention(q, kc, vc, ks, vs, bt, cl, QLMAX, QPP=QLMAX, plan=plan, out=out)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        specq.paged_attention(q, kc, vc, ks, vs, bt, cl, QLMAX, QPP=QLMAX, plan=plan, out=out)
    for b_act, ql in ((2, 3), (4, 9), (1, 5)):
        out.zero_()
        plan[0], plan[1] = b_act, ql
        graph.replay()
        eager, _ = specq.paged_attention(q[:b_act], kc, vc, ks, vs, bt[:b_act], cl[:b_act], ql, QPP=ql)
        torch.cuda.synchronize()
        assert torch.equal(out[:b_act, :ql], eager[:, :ql])
        assert bool((out[b_act:] == 0).all()) and bool((out[:b_act, ql:] == 0).all())


def test_status_clean_after_attention(cuda):
    import specq
    q, kc, vc, ks, vs, bt, cl = _config2(B=2, ctx=1024)
    specq.get_status(clear=True)
    specq.paged_attention(q, kc, vc, ks, vs, bt, cl, 9)
    torch.cuda.synchronize()
    assert specq.get_status(clear=True) == 0


def test_failure_detection_selftest_wait_times_out(cuda):
    """A wait on a barrier nothing completes gives up after its limit, records the timeout bit
    in the status word and returns; the context stays usable."""
    import specq
    from specq import _lib
    specq.get_status(clear=True)
    _lib.check(_lib.load().specq_selftest_wait_timeout(2_000_000, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert specq.get_status(clear=True) & _lib.SPECQ_STATUS_TIMEOUT_TEST
    x = torch.ones(4, device="cuda")
    assert float(x.sum()) == 4.0

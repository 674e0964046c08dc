"""Per-token INT8 quantiser, paged-KV append and packed-row attention on the GPU.

The quantiser's plain and residual modes equal the reference's quantize_act_int8 formula
(kernels.py:58-62) bit for bit; the KV append writes the reference cache format
(kernels.py:280-283) for the new tokens; packed-row attention equals the strided call."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref_quant(y):
    """kernels.py:58-62 on float32 rows."""
    s = y.abs().amax(dim=-1).clamp(min=1e-8) / 127.0
    q = torch.round(y / s[:, None]).clamp(-127, 127).to(torch.int8)
    return q, s


@pytest.mark.parametrize("M,N", [(1, 4096), (40, 4096), (72, 6144), (288, 14336), (5, 130)])
def test_quant_plain_bit_exact(cuda, M, N):
    import specq
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    x = (torch.randn(M, N, device="cuda", generator=g) * 3).half()
    x[0, :7] = 0                                      # a few exact zeros
    q, s = specq.quant_rows(x)
    rq, rs = _ref_quant(x.float())
    assert torch.equal(s, rs)
    assert torch.equal(q, rq)
    # the reference's torch function evaluated on the same fp16 rows on the GPU
    fq, fs = specq.fixtures.quantize_act_int8(x)
    assert torch.equal(q, fq.to(q.device)) and torch.equal(s, fs.to(s.device))
    # the public drop-in name routes a CUDA fp16 tensor to the kernel
    pq, ps = specq.quantize_act_int8(x)
    assert torch.equal(pq, q) and torch.equal(ps, s)


def test_quant_zero_row_and_plan(cuda):
    import specq
    x = torch.randn(16, 256, device="cuda").half()
    x[3] = 0
    plan = torch.tensor([9], dtype=torch.int32, device="cuda")
    q = torch.full((16, 256), 55, dtype=torch.int8, device="cuda")
    s = torch.full((16,), -1.0, device="cuda")
    specq.quant_rows(x, q=q, s=s, plan=plan)
    rq, rs = _ref_quant(x[:9].float())
    assert torch.equal(q[:9], rq) and torch.equal(s[:9], rs)
    assert s[3].item() == pytest.approx(1e-8 / 127.0)
    assert bool((q[9:] == 55).all()) and bool((s[9:] == -1.0).all())   # inactive rows untouched


def test_quant_residual(cuda):
    import specq
    M, N = 24, 4096
    x = torch.randn(M, N, device="cuda").half()
    r = torch.randn(M, N, device="cuda").half()
    h = x + r                                          # fp16 add, one rounding
    q, s = specq.quant_rows(x, mode=specq.QUANT_RESIDUAL, residual=r)
    assert torch.equal(r, h)
    rq, rs = _ref_quant(h.float())
    assert torch.equal(q, rq) and torch.equal(s, rs)


def test_quant_silu_mul(cuda):
    import specq
    M, N = 18, 14336
    x = torch.randn(M, 2 * N, device="cuda").half()
    q, s = specq.quant_rows(x, mode=specq.QUANT_SILU_MUL)
    y = torch.nn.functional.silu(x[:, :N].float()) * x[:, N:].float()
    rq, rs = _ref_quant(y)
    assert torch.allclose(s, rs, rtol=1e-6, atol=0)
    d = (q.int() - rq.int()).abs()
    assert int(d.max()) <= 1                           # silu's last bit may move a rounding tie
    assert float((d > 0).float().mean()) < 1e-3


def _cache(B, ctx, H_KV, seed):
    import specq
    return specq.make_paged_kv(B, ctx, H_KV, 128, device="cuda", seed=seed)


@pytest.mark.parametrize("use_plan", [False, True])
def test_kv_append(cuda, use_plan):
    import specq
    B, H_KV, ql, ql_max, cols = 3, 4, 5, 9, 3 * 4 * 128
    ctx = [40, 17, 64]
    kc, vc, ks, vs, bt, cl = _cache(B, ctx, H_KV, 5)
    kc0, vc0, ks0, vs0 = kc.clone(), vc.clone(), ks.clone(), vs.clone()
    x = torch.randn(B * ql_max, 4 * H_KV * 128, device="cuda").half()
    k_col, v_col = 2 * H_KV * 128, 3 * H_KV * 128
    if use_plan:
        plan = torch.tensor([B, ql], dtype=torch.int32, device="cuda")
        specq.kv_append(x, k_col, v_col, kc, vc, ks, vs, bt, cl, ql, plan=plan, B=B, ql_max=ql_max)
    else:
        specq.kv_append(x, k_col, v_col, kc, vc, ks, vs, bt, cl, ql)
    ek, ev, eks, evs = kc0.clone(), vc0.clone(), ks0.clone(), vs0.clone()
    for b in range(B):
        for t in range(ql):
            pos = ctx[b] - ql + t
            pg, slot = int(bt[b, pos // 16]), pos % 16
            row = x[b * ql + t].float()
            for src, c, sc, col in ((row, ek, eks, k_col), (row, ev, evs, v_col)):
                kv = src[col:col + H_KV * 128].view(H_KV, 128)
                s = kv.abs().amax(-1).clamp(min=1e-8) / 127.0
                c[pg, slot] = torch.round(kv / s[:, None]).clamp(-127, 127).to(torch.int8)
                sc[pg, slot] = s.half()
    assert torch.equal(kc, ek) and torch.equal(vc, ev)
    assert torch.equal(ks, eks) and torch.equal(vs, evs)


def test_packed_attention_equals_strided(cuda):
    import specq
    B, H, H_KV, ql = 3, 16, 4, 6
    kc, vc, ks, vs, bt, cl = _cache(B, [300, 129, 64], H_KV, 9)
    qkv = torch.randn(B * ql, (H + 2 * H_KV) * 128, device="cuda").half()
    q4 = qkv[:, : H * 128].reshape(B, ql, H, 128)
    ref, _ = specq.paged_attention(q4, kc, vc, ks, vs, bt, cl, ql)
    out = torch.zeros(B * ql, H * 128, device="cuda").half()
    specq.paged_attention_packed(qkv, 0, out, kc, vc, ks, vs, bt, cl, ql, H)
    assert torch.equal(out.view(B, ql, H, 128), ref)
    # under a plan graph grid: the packed stride follows plan[1]
    plan = torch.tensor([B, ql], dtype=torch.int32, device="cuda")
    out2 = torch.zeros(B * 9, H * 128, device="cuda").half()
    specq.paged_attention_packed(qkv, 0, out2, kc, vc, ks, vs, bt, cl, ql, H, B=B, ql_max=9, plan=plan)
    assert torch.equal(out2[: B * ql].view(B, ql, H, 128), ref)
    assert bool((out2[B * ql:] == 0).all())


@pytest.mark.parametrize("mode", [0, 2])
def test_quant_sharded_rows_match_whole_rows(cuda, mode):
    """A row split across two shards: amax_out per shard, the maximum as amax_in -- each shard's
    int8 values and scale equal those of the whole row (the tensor-parallel stack relies on it)."""
    import specq
    M, N = 24, 4096
    g = torch.Generator(device="cuda").manual_seed(mode + 11)
    if mode == 0:
        x = (torch.randn(M, N, device="cuda", generator=g) * 2).half()
        halves = [x[:, : N // 2], x[:, N // 2:]]
    else:   # gate | up; shard r holds [gate_r | up_r]
        x = torch.randn(M, 2 * N, device="cuda", generator=g).half()
        halves = [torch.cat([x[:, :N // 2], x[:, N:N + N // 2]], 1), torch.cat([x[:, N // 2:N], x[:, N + N // 2:]], 1)]
    q, s = specq.quant_rows(x, mode=mode)
    amax = [torch.empty(M, device="cuda") for _ in halves]
    for h, a in zip(halves, amax):
        assert specq.quant_rows(h, mode=mode, amax_out=a) is None
    whole = torch.maximum(amax[0], amax[1])
    parts = [specq.quant_rows(h, mode=mode, amax_in=whole) for h in halves]
    assert torch.equal(parts[0][1], s) and torch.equal(parts[1][1], s)
    assert torch.equal(torch.cat([parts[0][0], parts[1][0]], 1), q)

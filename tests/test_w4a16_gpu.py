"""GPU parity of the W4A16 kernel against the oracle (kernel-semantics dequant: fp16(q * fp16
scale), kernels.py:117-127) and against the reference's own kernel outputs and exact
reference (correctness.py:76-79).  Tolerances: Frobenius-relative 1e-3 against the oracle
and 2e-3 against the fp32-scale reference (correctness.py:79); plan mode
is bit-exact against non-plan mode."""
import numpy as np
import pytest
import torch

from oracle import specq_oracle as O

pytestmark = pytest.mark.gpu


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _weights(N, K, seed, group=128):
    import specq
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g).half()
    wp, sc, deq = specq.quantize_weight_int4(w, group)
    return wp, sc, deq


def _config1_weights(N, K, seed, group=128):
    """Config 1 value distribution: int4 uniform in [-8, 7], fp16 scales uniform in [0.005, 0.02]."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-8, 8, (N, K), generator=g, dtype=torch.int16)
    nib = q + 8
    wp = (nib[:, : K // 2] | (nib[:, K // 2:] << 4)).to(torch.uint8)
    sc = (torch.rand(N, K // group, generator=g) * 0.015 + 0.005).half()
    return wp, sc


@pytest.mark.parametrize("name", ["w4a16_small", "w4a16_mid"])
def test_golden(cuda, golden, name):
    import specq
    g = golden(name)
    out, ck = specq.w4a16_matmul(_dev(g["x"]), _dev(g["wp"]), _dev(g["sc"]))
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    assert O.rel_fro_err(o, O.w4a16_ref(g["x"], g["wp"], g["sc"])) < 1e-3
    assert O.rel_fro_err(o, g["out"]) < 1e-3          # the reference's own kernel output
    assert O.rel_fro_err(o, g["ref"]) < 2e-3          # correctness.py:79


def test_golden_plan_mode(cuda, golden):
    import specq
    g = golden("w4a16_plan")
    M = int(g["plan"][0])
    out = torch.full(g["out"].shape, 12345.0, dtype=torch.float16, device="cuda")
    specq.w4a16_matmul(_dev(g["x"]), _dev(g["wp"]), _dev(g["sc"]), out=out, plan=_dev(g["plan"]),
                       grid_m_max=g["x"].shape[0])
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    assert O.rel_fro_err(o[:M], g["out"][:M]) < 1e-3
    assert np.all(o[M:] == np.float16(12345.0))


def test_correctness_sweep(cuda):
    """correctness.py:67-84: N=1000, K=1024, M = 1..64 and edge cases up to 300."""
    import specq
    wp, sc, deq = _weights(1000, 1024, 11)
    x = torch.randn(300, 1024, generator=torch.Generator().manual_seed(12)).half()
    xd, wpd, scd = x.cuda(), wp.cuda(), sc.cuda()
    for M in list(range(1, 65)) + [72, 99, 128, 129, 200, 288, 300]:
        out, _ = specq.w4a16_matmul(xd[:M], wpd, scd)
        o = out.cpu().numpy()
        assert O.rel_fro_err(o, O.w4a16_ref(x[:M].numpy(), wp.numpy(), sc.numpy())) < 1e-3, M
        assert O.rel_fro_err(o, O.w4a16_ref_from_deq(x[:M].numpy(), deq.numpy())) < 2e-3, M


@pytest.mark.parametrize("M", [1, 8, 9, 24, 40, 72, 144, 288])
def test_config1_gate_proj(cuda, M):
    """Config 1: K=4096, N=14336 at verification widths M = B*(k+1)."""
    import specq
    N, K = 14336, 4096
    wp, sc = _config1_weights(N, K, 21)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).half()
    out, ck = specq.w4a16_matmul(x.cuda(), wp.cuda(), sc.cuda())
    o = out.cpu().numpy()
    ref = O.w4a16_ref(x.numpy(), wp.numpy(), sc.numpy())
    assert O.rel_fro_err(o, ref) < 1e-3
    assert O.max_rel_err_plus1(o, ref) < 2e-3


def test_plan_mode_bit_exact_and_inactive_rows_untouched(cuda):
    import specq
    MMAX, N, K = 288, 1000, 1024
    wp, sc, _ = _weights(N, K, 31)
    x = torch.randn(MMAX, K, generator=torch.Generator().manual_seed(32)).half().cuda()
    wpd, scd = wp.cuda(), sc.cuda()
    plan = torch.zeros(8, dtype=torch.int32, device="cuda")
    for M in (1, 3, 9, 16, 17, 45, 81, 144, 288):
        plan[0] = M
        out = torch.full((MMAX, N), 12345.0, device="cuda", dtype=torch.float16)
        specq.w4a16_matmul(x, wpd, scd, out=out, plan=plan, grid_m_max=MMAX)
        ref, _ = specq.w4a16_matmul(x[:M], wpd, scd)
        torch.cuda.synchronize()
        assert torch.equal(out[:M], ref), f"M={M}"
        assert bool((out[M:] == 12345.0).all()), f"M={M}"


def test_group_256(cuda):
    import specq
    wp, sc, _ = _weights(256, 2048, 41, group=256)
    x = torch.randn(19, 2048, generator=torch.Generator().manual_seed(42)).half()
    out, _ = specq.w4a16_matmul(x.cuda(), wp.cuda(), sc.cuda(), group=256)
    o = out.cpu().numpy()
    assert O.rel_fro_err(o, O.w4a16_ref(x.numpy(), wp.numpy(), sc.numpy(), 256)) < 1e-3


def test_cuda_graph_plan_replay(cuda):
    import specq
    MMAX, N, K = 72, 1024, 2048
    wp, sc, _ = _weights(N, K, 51)
    x = torch.randn(MMAX, K, generator=torch.Generator().manual_seed(52)).half().cuda()
    wpd, scd = wp.cuda(), sc.cuda()
    plan = torch.full((8,), MMAX, dtype=torch.int32, device="cuda")
    out = torch.zeros(MMAX, N, dtype=torch.float16, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        specq.w4a16_matmul(x, wpd, scd, out=out, plan=plan, grid_m_max=MMAX)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        specq.w4a16_matmul(x, wpd, scd, out=out, plan=plan, grid_m_max=MMAX)
    for M in (9, 72, 3):
        out.zero_()
        plan[0] = M
        graph.replay()
        ref, _ = specq.w4a16_matmul(x[:M], wpd, scd)
        torch.cuda.synchronize()
        assert torch.equal(out[:M], ref) and bool((out[M:] == 0).all())


@pytest.mark.parametrize("K,group", [(1408, 192), (1664, 192), (2176, 256), (1536, 192)])
def test_partial_last_group(cuda, K, group):
    """K % group != 0: each row has ceil(K/group) scale columns, the last one covering a partial
    group that the high-half K-blocks near the end read (column (k + K/2) // group, as
    kernels.py:119-120 indexes it).  (1408, 192) takes the TMA scale tile (8 columns),
    (1664, 192) and (2176, 256) the per-block scale loads (9 columns); (1536, 192) divides
    evenly and is the control."""
    import specq
    N, M = 200, 24
    G = -(-K // group)
    g = torch.Generator().manual_seed(K + group)
    nib = torch.randint(0, 16, (N, K), generator=g, dtype=torch.int16)
    wp = (nib[:, : K // 2] | (nib[:, K // 2:] << 4)).to(torch.uint8)
    sc = (torch.rand(N, G, generator=g) * 0.015 + 0.005).half()
    x = torch.randn(M, K, generator=g).half()
    out, _ = specq.w4a16_matmul(x.cuda(), wp.cuda(), sc.cuda(), group=group)
    torch.cuda.synchronize()
    ref = O.w4a16_ref(x.numpy(), wp.numpy(), sc.numpy(), group)
    assert O.rel_fro_err(out.cpu().numpy(), ref) < 1e-3
    # a scale tile that read the wrong column of the last group would be off by far more
    sc_bad = sc.clone()
    sc_bad[:, G - 1] *= 2
    assert O.rel_fro_err(O.w4a16_ref(x.numpy(), wp.numpy(), sc_bad.numpy(), group), ref) > 1e-2

"""GPU parity of the W8A8 kernel (through the C ABI) against the oracle and the reference's own
outputs.  The kernel's epilogue is the reference's arithmetic (fp32(acc) * sa * sw -> fp16,
kernels.py:53-55) on an exact INT32 accumulator, so every comparison here is bit for bit."""
import numpy as np
import pytest
import torch

from oracle import specq_oracle as O

pytestmark = pytest.mark.gpu


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _bits(t):
    return t.detach().cpu().numpy().view(np.uint16)


def _inputs(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int16).to(torch.int8)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int16).to(torch.int8)
    sa = torch.rand(M, generator=g) * 0.019 + 0.001
    sw = torch.rand(N, generator=g) * 0.019 + 0.001
    return a, sa, w, sw


@pytest.mark.parametrize("name", ["w8a8_small", "w8a8_ragged", "w8a8_m1"])
def test_golden_bit_exact(cuda, golden, name):
    import specq
    g = golden(name)
    out, ck = specq.w8a8_matmul(_dev(g["a_q"]), _dev(g["sa"]), _dev(g["w_q"]), _dev(g["sw"]))
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out), g["out"].view(np.uint16))
    assert ck.n_regs > 0


def test_golden_plan_mode(cuda, golden):
    import specq
    g = golden("w8a8_plan")
    out = torch.full(g["out"].shape, 12345.0, dtype=torch.float16, device="cuda")
    specq.w8a8_matmul(_dev(g["a_q"]), _dev(g["sa"]), _dev(g["w_q"]), _dev(g["sw"]), out=out, plan=_dev(g["plan"]),
                      grid_m_max=g["a_q"].shape[0])
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out), g["out"].view(np.uint16))


def test_config0_accumulator_and_output_bit_exact(cuda):
    """Config 0 (o_proj, M = 8*(4+1) = 40, K = N = 4096): INT32 accumulator and fp16 output."""
    import specq
    a, sa, w, sw = _inputs(40, 4096, 4096, 0)
    acc = specq.w8a8_accumulator(a.cuda(), w.cuda())
    out, ck = specq.w8a8_matmul(a.cuda(), sa.cuda(), w.cuda(), sw.cuda())
    torch.cuda.synchronize()
    ref_acc = O.w8a8_acc(a.numpy(), w.numpy())
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), ref_acc)
    assert np.array_equal(_bits(out), O.w8a8_epilogue(ref_acc, sa.numpy(), sw.numpy()).view(np.uint16))


def test_accumulator_beyond_exact_fp32_range(cuda):
    """|acc| up to 127*127*14336 > 2**24: an fp32 accumulation would round; INT32 must not."""
    import specq
    M, N, K = 16, 256, 14336
    g = torch.Generator().manual_seed(9)
    a = torch.full((M, K), 127, dtype=torch.int8)
    a[1::2] = -127
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int16).to(torch.int8)
    w[:8] = 127
    w[8:16] = -127
    acc = specq.w8a8_accumulator(a.cuda(), w.cuda())
    ref = O.w8a8_acc(a.numpy(), w.numpy())
    assert np.abs(ref).max() == 127 * 127 * K > 2 ** 24
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), ref)


@pytest.mark.parametrize("N,K", [(6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336)])
@pytest.mark.parametrize("M", [1, 9, 40, 72, 288])
def test_llama_linear_set_accumulator(cuda, N, K, M):
    """Config 3 shapes (qkv, o, gate_up, down) over verification widths M = B*(k+1)."""
    import specq
    a, sa, w, sw = _inputs(M, N, K, M + N + K)
    acc = specq.w8a8_accumulator(a.cuda(), w.cuda())
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), O.w8a8_acc(a.numpy(), w.numpy()))


@pytest.mark.parametrize("K", [520, 512, 200, 1000, 524, 522, 521])
def test_exhaustive_dynamic_M(cuda, K):
    """correctness.py:27-42: every M in 1..300 at N=1000 (not tile multiples); K=520 and
    K=200 have row strides that are not 16-byte aligned (register-staged loader)."""
    import specq
    N = 1000
    a, _, w, sw = _inputs(300, N, K, 1)
    x = torch.randn(300, K, generator=torch.Generator().manual_seed(2)).half()
    a, sa = specq.quantize_act_int8(x)
    ad, sad, wd, swd = a.cuda(), sa.cuda(), w.cuda(), sw.cuda()
    acc_all = O.w8a8_acc(a.numpy(), w.numpy())
    step = 1 if K == 520 else 7
    for M in range(1, 301, step):
        out, _ = specq.w8a8_matmul(ad[:M], sad[:M], wd, swd)
        ref = O.w8a8_epilogue(acc_all[:M], sa.numpy()[:M], sw.numpy())
        assert np.array_equal(_bits(out), ref.view(np.uint16)), f"M={M}"


def test_plan_mode_inactive_rows_untouched_and_bit_exact(cuda):
    """correctness.py:50-65, plus plan == non-plan bit for bit."""
    import specq
    MMAX, N, K = 288, 1000, 512
    a, sa, w, sw = (t.cuda() for t in _inputs(MMAX, N, K, 3))
    plan = torch.zeros(8, dtype=torch.int32, device="cuda")
    for M in (1, 3, 5, 9, 15, 16, 17, 27, 45, 81, 144, 288):
        plan[0] = M
        out = torch.full((MMAX, N), 12345.0, device="cuda", dtype=torch.float16)
        specq.w8a8_matmul(a, sa, w, sw, out=out, plan=plan, grid_m_max=MMAX, BLOCK_M=16)
        ref, _ = specq.w8a8_matmul(a[:M], sa[:M], w, sw)
        torch.cuda.synchronize()
        assert torch.equal(out[:M], ref), f"M={M}"
        assert bool((out[M:] == 12345.0).all()), f"M={M}"


def test_plan_value_out_of_range_is_clamped_and_flagged(cuda):
    import specq
    MMAX, N, K = 32, 256, 256
    a, sa, w, sw = (t.cuda() for t in _inputs(MMAX, N, K, 4))
    specq.get_status(clear=True)
    plan = torch.tensor([MMAX + 100, 0, 0, 0, 0, 0, 0, 0], dtype=torch.int32, device="cuda")
    out = torch.full((MMAX, N), 7.0, device="cuda", dtype=torch.float16)
    specq.w8a8_matmul(a, sa, w, sw, out=out, plan=plan, grid_m_max=MMAX)
    ref, _ = specq.w8a8_matmul(a, sa, w, sw)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert specq.get_status(clear=True) & 0x100


@pytest.mark.parametrize("M,chunks", [(257, 2), (288, 2), (289, 2), (600, 3)])
def test_token_chunks_eager(cuda, M, chunks):
    """Eager calls of a narrow shape (fewer channel tiles than SMs) split the tokens into chunks
    of at most 256 (smaller split-K partials); every split gives the exact int32 sums."""
    import specq
    a, sa, w, sw = _inputs(M, 384, 768, M)
    out, ck = specq.w8a8_matmul(a.cuda(), sa.cuda(), w.cuda(), sw.cuda())
    torch.cuda.synchronize()
    assert ck.grid[1] == chunks      # grid = (split, token chunk, channel tile)
    assert np.array_equal(_bits(out), O.w8a8_ref(a.numpy(), sa.numpy(), w.numpy(), sw.numpy()).view(np.uint16))


def test_plan_grid_of_288_tokens_is_one_chunk(cuda):
    """A plan-buffer grid sized for 288 tokens (32 sequences x 9) keeps them in one CTA per
    channel tile: past 256 tokens a second MMA per K step covers tokens 256.. at TMEM column
    256.  Checked against the oracle at active M on both sides of 256."""
    import specq
    MMAX, N, K = 288, 384, 768
    a, sa, w, sw = _inputs(MMAX, N, K, 31)
    ad, sad, wd, swd = a.cuda(), sa.cuda(), w.cuda(), sw.cuda()
    plan = torch.zeros(8, dtype=torch.int32, device="cuda")
    for M in (288, 272, 257, 256, 40):
        plan[0] = M
        out = torch.full((MMAX, N), 7.0, dtype=torch.float16, device="cuda")
        _, ck = specq.w8a8_matmul(ad, sad, wd, swd, out=out, plan=plan, grid_m_max=MMAX)
        torch.cuda.synchronize()
        assert ck.grid[1] == 1
        ref = O.w8a8_ref(a[:M].numpy(), sa[:M].numpy(), w.numpy(), sw.numpy())
        assert np.array_equal(_bits(out[:M]), ref.view(np.uint16)), M
        assert bool((out[M:] == 7.0).all())


def test_strided_and_transposed_outputs(cuda):
    import specq
    M, N, K = 24, 320, 384
    a, sa, w, sw = (t.cuda() for t in _inputs(M, N, K, 5))
    ref, _ = specq.w8a8_matmul(a, sa, w, sw)
    big = torch.zeros(M, N + 64, dtype=torch.float16, device="cuda")
    specq.w8a8_matmul(a, sa, w, sw, out=big[:, 32:32 + N])
    outT = torch.zeros(N, M, dtype=torch.float16, device="cuda").t()      # column-major [M, N]
    specq.w8a8_matmul(a, sa, w, sw, out=outT)
    torch.cuda.synchronize()
    assert torch.equal(big[:, 32:32 + N], ref) and bool((big[:, :32] == 0).all())
    assert torch.equal(outT, ref)


def test_empty_m(cuda):
    import specq
    a = torch.zeros(0, 128, dtype=torch.int8, device="cuda")
    w = torch.zeros(64, 128, dtype=torch.int8, device="cuda")
    out, _ = specq.w8a8_matmul(a, torch.zeros(0, device="cuda"), w, torch.ones(64, device="cuda"))
    assert out.shape == (0, 64)


def test_cuda_graph_plan_replay(cuda):
    """One graph captured at the maximum grid serves every M (bench_graphs.py:72-82)."""
    import specq
    MMAX, N, K = 96, 512, 1024
    a, sa, w, sw = (t.cuda() for t in _inputs(MMAX, N, K, 6))
    plan = torch.zeros(8, dtype=torch.int32, device="cuda")
    out = torch.zeros(MMAX, N, dtype=torch.float16, device="cuda")
    plan[0] = MMAX
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        specq.w8a8_matmul(a, sa, w, sw, out=out, plan=plan, grid_m_max=MMAX)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        specq.w8a8_matmul(a, sa, w, sw, out=out, plan=plan, grid_m_max=MMAX)
    for M in (5, 40, 96, 17):
        out.zero_()
        plan[0] = M
        graph.replay()
        ref, _ = specq.w8a8_matmul(a[:M], sa[:M], w, sw)
        torch.cuda.synchronize()
        assert torch.equal(out[:M], ref) and bool((out[M:] == 0).all())


def test_compiled_kernel_registry_counts_binaries(cuda):
    import kernels
    import specq
    a, sa, w, sw = (t.cuda() for t in _inputs(8, 128, 512, 7))
    _, ck = kernels.w8a8_matmul(a, sa, w, sw)
    dev = torch.cuda.current_device()
    assert ck.variant in kernels._w8a8_kernel.device_caches[dev][0]
    assert ck.metadata.shared > 0 and ck.n_spills == 0


def test_no_status_flags_after_normal_runs(cuda):
    import specq
    a, sa, w, sw = (t.cuda() for t in _inputs(40, 4096, 4096, 8))
    specq.get_status(clear=True)
    specq.w8a8_matmul(a, sa, w, sw)
    torch.cuda.synchronize()
    assert specq.get_status(clear=True) == 0

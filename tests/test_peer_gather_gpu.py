"""specq_peer_gather on one GPU: the copy into every rank's full buffer, the epoch protocol and
the max reduction, with the peer's side emulated by buffers on the same GPU whose signal is
set before the launch (one launch, nothing waits on another launch), and the bounded wait
running out when no peer ever signals (status bit, no hang).  The two-rank exchange over
NVLink is covered by test_stack_tp_gpu.py."""
import ctypes as C

import pytest
import torch

from specq import _lib

pytestmark = pytest.mark.gpu


def _call(src, rows, dsts, ld_dst, dst_off, flags, state, rank, world, plan=None, max_out=None):
    lib = _lib.load()
    esz = src.element_size()
    _lib.check(lib.specq_peer_gather(
        src.data_ptr(), src.stride(0) * esz, src.shape[1] * esz, None if plan is None else plan.data_ptr(), rows,
        (C.c_void_p * world)(*[d.data_ptr() for d in dsts]), ld_dst, dst_off,
        (C.c_void_p * world)(*[f.data_ptr() for f in flags]), state.data_ptr(),
        None if max_out is None else max_out.data_ptr(), rank, world, torch.cuda.current_stream().cuda_stream))


def test_single_rank_copy_and_plan_rows(cuda):
    g = torch.Generator(device="cuda").manual_seed(0)
    for dtype, n in ((torch.float16, 2048), (torch.int8, 7168), (torch.float16, 6)):
        src = torch.randint(-100, 100, (40, n), generator=g, device="cuda").to(dtype)
        full = torch.full((40, n), 7, dtype=dtype, device="cuda")
        flags = torch.zeros(1, dtype=torch.int32, device="cuda")
        state = torch.zeros(2, dtype=torch.int32, device="cuda")
        plan = torch.tensor([29], dtype=torch.int32, device="cuda")
        _call(src, 40, [full], full.stride(0) * full.element_size(), 0, [flags], state, 0, 1, plan=plan)
        torch.cuda.synchronize()
        assert torch.equal(full[:29], src[:29])
        assert (full[29:] == 7).all()                      # rows past the plan's are not touched
        assert state[0].item() >= 1 and state[1].item() == 0   # the launch's CTAs counted
    assert _lib.get_status() == 0


def test_two_rank_emulation_copy_signal_and_max(cuda):
    g = torch.Generator(device="cuda").manual_seed(1)
    rows, n, world = 24, 512, 2
    src = torch.randn(rows, n, generator=g, device="cuda").half()
    full = [torch.zeros(rows, world * n, dtype=torch.float16, device="cuda") for _ in range(world)]
    flags = [torch.zeros(world, dtype=torch.int32, device="cuda") for _ in range(world)]
    flags[0][1] = 1 << 20     # rank 1's CTAs have all signalled already
    state = torch.zeros(2, dtype=torch.int32, device="cuda")
    ld = full[0].stride(0) * 2
    # rank 0 writes columns [0, n) of both full buffers and signals flags[1][0]
    _call(src, rows, full, ld, 0, flags, state, 0, world)
    torch.cuda.synchronize()
    for f in full:
        assert torch.equal(f[:, :n], src)
        assert (f[:, n:] == 0).all()
    # one release-add per CTA of rank 0 in rank 1's flag array; rank 0's running total matches
    assert flags[1][1].item() == 0 and flags[1][0].item() == state[0].item() >= 1
    # max mode: rank 0's amax column against a pre-filled peer column
    a0 = torch.rand(rows, generator=g, device="cuda")
    fm = [torch.zeros(rows, world, dtype=torch.float32, device="cuda") for _ in range(world)]
    fm[0][:, 1] = torch.rand(rows, generator=g, device="cuda")
    fl = [torch.zeros(world, dtype=torch.int32, device="cuda") for _ in range(world)]
    fl[0][1] = 1 << 20
    st = torch.zeros(2, dtype=torch.int32, device="cuda")
    out = torch.zeros(rows, dtype=torch.float32, device="cuda")
    _call(a0.view(-1, 1), rows, fm, 4 * world, 0, fl, st, 0, world, max_out=out)
    torch.cuda.synchronize()
    assert torch.equal(out, torch.maximum(a0, fm[0][:, 1]))
    assert torch.equal(fm[1][:, 0], a0)
    assert _lib.get_status() == 0


def test_missing_peer_signal_times_out_with_status(cuda):
    rows, n, world = 8, 64, 2
    src = torch.ones(rows, n, dtype=torch.float16, device="cuda")
    full = [torch.zeros(rows, world * n, dtype=torch.float16, device="cuda") for _ in range(world)]
    flags = [torch.zeros(world, dtype=torch.int32, device="cuda") for _ in range(world)]   # nobody signals
    state = torch.zeros(2, dtype=torch.int32, device="cuda")
    _lib.get_status()
    _call(src, rows, full, full[0].stride(0) * 2, 0, flags, state, 0, world)
    torch.cuda.synchronize()                               # returns after the 1 s limit
    assert _lib.get_status() & _lib.SPECQ_STATUS_TIMEOUT_PEER
    assert torch.equal(full[0][:, :n], src)
    torch.zeros(1, device="cuda").add_(1)                  # the context is still usable
    torch.cuda.synchronize()


def test_w8a8_peer_output_and_counts_two_rank_emulation(cuda):
    """specq_w8a8_peer as rank 0 of 2: its output block lands in column block 0 of both 'ranks''
    full buffers (same GPU here), equal to the plain GEMM, and every CTA counts itself into slot 0
    of both flag arrays; a consumer then waits for rank 1's count to reach rank 0's own."""
    import specq
    g = torch.Generator(device="cuda").manual_seed(2)
    M, N, K, world = 40, 512, 1024, 2
    a = torch.randint(-127, 128, (M, K), generator=g, device="cuda", dtype=torch.int16).to(torch.int8)
    w = torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int16).to(torch.int8)
    sa = torch.rand(M, generator=g, device="cuda") * 0.02 + 0.001
    sw = torch.rand(N, generator=g, device="cuda") * 0.02 + 0.001
    ref, _ = specq.w8a8_matmul(a, sa, w, sw)
    full = [torch.full((M, world * N), 3.0, dtype=torch.float16, device="cuda") for _ in range(world)]
    flags = [torch.zeros(world, dtype=torch.int32, device="cuda") for _ in range(world)]
    lib = _lib.load()
    _lib.check(lib.specq_w8a8_peer(
        a.data_ptr(), a.stride(0), sa.data_ptr(), w.data_ptr(), w.stride(0), sw.data_ptr(),
        (C.c_void_p * world)(*[f.data_ptr() for f in full]), full[0].stride(0), None, M, N, K,
        (C.c_void_p * world)(*[f.data_ptr() for f in flags]), 0, world, torch.cuda.current_stream().cuda_stream))
    ctas = _lib.last_launch()["grid"]
    torch.cuda.synchronize()
    n_ctas = ctas[0] * ctas[1] * ctas[2]
    for f in full:
        assert torch.equal(f[:, :N], ref)                    # bit-exact with the plain epilogue
        assert (f[:, N:] == 3.0).all()                       # the other rank's block untouched
    assert flags[0].tolist() == [n_ctas, 0] and flags[1].tolist() == [n_ctas, 0]
    # consumer on rank 0: rank 1's count preset to the same total -> no wait, same result
    flags[0][1] = n_ctas
    q, s = specq.quant_rows(full[0], wait=(flags[0], 0, world))
    torch.cuda.synchronize()
    q_full, s_full = specq.quant_rows(full[0])
    assert torch.equal(q, q_full) and torch.equal(s, s_full)
    assert _lib.get_status() == 0


def test_consumer_wait_times_out_without_the_peer_count(cuda):
    import specq
    M, N, world = 4, 256, 2
    x = torch.ones(M, N, dtype=torch.float16, device="cuda")
    flags = torch.tensor([5, 0], dtype=torch.int32, device="cuda")   # rank 1 never counts in
    _lib.get_status()
    q, s = specq.quant_rows(x, wait=(flags, 0, world))
    torch.cuda.synchronize()                                          # each CTA gives up after 1 s
    assert _lib.get_status() & _lib.SPECQ_STATUS_TIMEOUT_PEER
    assert (q == 127).all()                                           # it still quantised its row

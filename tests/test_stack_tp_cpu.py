"""Tensor-parallel stack, host side on CPU: the weight / KV-head ranges partition every
projection, and the all-gather reassembly puts each rank's column shard where the unsharded
tensor has it -- checked with two gloo ranks exchanging real column shards."""
from __future__ import annotations

import os
import socket
import sys

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "specdec-quant-triton_b200"))

from specq.stack_tp import gathered_to_rows, shard_rows, tp_slices  # noqa: E402


def test_slices_partition_every_projection():
    H, H_KV, D, hid, ff = 32, 8, 128, 4096, 14336
    for world in (1, 2, 4, 8):
        sl = [tp_slices(world, r, H, H_KV, D, hid, ff) for r in range(world)]
        for name, total in (("qkv", (H + 2 * H_KV) * D), ("o", hid), ("gu", 2 * ff), ("down", hid)):
            rows = sorted(i for s in sl for a, b in s[name] for i in range(a, b))
            assert rows == list(range(total)), (world, name)
        heads = sorted(i for s in sl for i in range(*s["kv_heads"]))
        assert heads == list(range(H_KV))
        # rank r's Q heads are the query heads of its KV heads (GQA groups stay whole)
        G = H // H_KV
        for r, s in enumerate(sl):
            q0, q1 = s["qkv"][0]
            k0, k1 = s["kv_heads"]
            assert (q0 // D, q1 // D) == (k0 * G, k1 * G)


def test_gate_and_up_ranges_match():
    ff = 14336
    for world in (2, 4):
        for r in range(world):
            (g0, g1), (u0, u1) = tp_slices(world, r, 32, 8, 128, 4096, ff)["gu"]
            assert (u0 - ff, u1 - ff) == (g0, g1)


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        M, N = 7, 24
        full = torch.arange(M * N, dtype=torch.float32).view(M, N)
        n = N // world
        local = full[:, rank * n:(rank + 1) * n].contiguous()
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local)
        buf = torch.cat(parts, 0)               # the layout all_gather_into_tensor produces
        out = torch.zeros(M + 3, N)
        gathered_to_rows(buf, world, M, out)
        if rank == 0:
            q.put(bool(torch.equal(out[:M], full)) and bool((out[M:] == 0).all()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # surfaced to the test through the queue
        q.put(repr(e))


def test_two_gloo_ranks_reassemble_column_shards():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
    assert res is True, res


def test_shard_rows_concatenates_ranges():
    t = torch.arange(20).view(10, 2)
    assert torch.equal(shard_rows(t, [(0, 2), (5, 6)]), torch.tensor([[0, 1], [2, 3], [10, 11]]))

"""Multi-GPU decomposition on CPU: two `gloo` ranks each compute their shard of the
verification step with the CPU restatement of the reference path, and the shards, gathered
here only to check them, must equal the unsharded step.  Also checks the max-over-ranks
reduction the benchmark uses for its timings."""
from __future__ import annotations

import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "specdec-quant-triton_b200"))

from specq.sharding import shard_inputs, shard_plan  # noqa: E402


def _inputs(seed=0):
    g = torch.Generator().manual_seed(seed)
    M, K, N = 8, 256, 512
    x = {"a8": torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int16).to(torch.int8),
         "w8": torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int16).to(torch.int8),
         "sa": torch.rand(M, generator=g) * 0.019 + 0.001,
         "sw": torch.rand(N, generator=g) * 0.019 + 0.001,
         "a4": torch.randn(M, K, generator=g).half()}
    nib = torch.randint(0, 16, (N, K), generator=g, dtype=torch.int16)
    x["wp"] = (nib[:, : K // 2] | (nib[:, K // 2:] << 4)).to(torch.uint8)
    x["sc"] = (torch.rand(N, K // 128, generator=g) * 0.015 + 0.005).half()
    B, ctx, page, D, H_KV, H, ql = 2, 64, 16, 128, 4, 8, 3
    n_pages = B * ctx // page
    x["kc"] = torch.randint(-127, 128, (n_pages, page, H_KV, D), generator=g, dtype=torch.int16).to(torch.int8)
    x["vc"] = torch.randint(-127, 128, (n_pages, page, H_KV, D), generator=g, dtype=torch.int16).to(torch.int8)
    x["ks"] = torch.rand(n_pages, page, H_KV, generator=g) * 0.015 + 0.005
    x["vs"] = torch.rand(n_pages, page, H_KV, generator=g) * 0.015 + 0.005
    x["bt"] = torch.randperm(n_pages, generator=g).to(torch.int32).view(B, -1)
    x["cl"] = torch.full((B,), ctx, dtype=torch.int32)
    x["q"] = torch.randn(B, ql, H, D, generator=g).half()
    x["ql"] = ql
    return x


def _step(x):
    from oracle import cpu_reference as R
    return (R.w8a8(x["a8"], x["sa"], x["w8"], x["sw"]),
            R.w4a16(x["a4"], R.dequant_int4(x["wp"], x["sc"])),
            R.paged_attention(x["q"], x["kc"], x["vc"], x["ks"], x["vs"], x["bt"], x["cl"], x["ql"]))


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        x = _inputs()
        plan = shard_plan(world, rank, n_w8a8=x["w8"].shape[0], n_w4a16=x["wp"].shape[0],
                          h_kv=x["kc"].shape[2], h=x["q"].shape[2])
        o8, o4, oa = _step(shard_inputs(x, plan))
        parts = []
        for t in (o8.float().contiguous(), o4.float().contiguous(), oa.float().contiguous()):
            g = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(g, t)
            parts.append(g)
        # the benchmark reports the slowest rank's time: MAX over ranks
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            f8, f4, fa = _step(x)
            ok8 = torch.equal(torch.cat(parts[0], dim=1), f8.float())
            ok4 = torch.equal(torch.cat(parts[1], dim=1), f4.float())
            oka = torch.equal(torch.cat(parts[2], dim=2), fa.float())
            q.put((ok8, ok4, oka, float(t.item())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # surfaced to the test through the queue
        q.put(("error", repr(e)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_plan_partitions_every_unit():
    world = 4
    plans = [shard_plan(world, r, n_w8a8=4096, n_w4a16=14336, h_kv=8, h=32) for r in range(world)]
    for key, total in (("w8a8_cols", 4096), ("w4a16_cols", 14336), ("kv_heads", 8), ("q_heads", 32)):
        covered = sorted(i for p in plans for i in range(p[key].start, p[key].stop))
        assert covered == list(range(total)), key
    with pytest.raises(ValueError):
        shard_plan(3, 0, n_w8a8=4096, n_w4a16=14336, h_kv=8, h=32)   # 8 KV heads over 3 ranks


def test_two_gloo_ranks_reassemble_the_step():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
    assert res[0] != "error", res
    ok8, ok4, oka, tmax = res
    assert ok8 and ok4 and oka
    assert tmax == 2.0

"""The plan-graph verification stack across GPUs: tensor parallel, one process per GPU, NCCL.

Rank r of g holds (survey config 4 extended to g GPUs):

  qkv   the Q heads [r H/g, (r+1) H/g) and the K / V heads [r H_KV/g, (r+1) H_KV/g) -- its KV
        cache holds those KV heads only, so the KV append and attention stay local;
  o     output channels [r hid/g, (r+1) hid/g);
  gu    gate and up channels with matching ranges, so silu(gate) * up stays local;
  down  output channels [r hid/g, (r+1) hid/g).

The residual stream h is replicated.  Per layer the ranks all-gather the attention output
(fp16), the o-projection output (fp16), the quantised MLP activation (int8) and the
down-projection output (fp16), plus one all-reduce (MAX) of the MLP activation's per-token
amax, so every rank quantises its slice with the whole row's scale.  With exchange="peer" (the
command line's default) each of these is one `specq_peer_gather` launch that stores the rank's
block over NVLink straight into every rank's symmetric full buffer (specq/peer.py); with
exchange="nccl" they are NCCL collectives followed by a re-layout copy.
Every kernel computes each output column exactly as the single-GPU stack does (W8A8 sums in
int32 whatever the column split), so the tensor-parallel residual stream equals the single-GPU
one bit for bit whenever the attention splits each context the same way on both (the split
count follows the context length and the KV heads a GPU holds; at the stack's 1024-token
contexts it is 2 on one GPU and on a 2-way shard).

Under the plan graph the NCCL collectives move the maximum grid's rows (a graph fixes their
sizes) while the peer-store kernel reads the active rows from the plan buffer; eager steps move
the active rows.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m specq.stack_tp [--layers 4] [--steps 200] [--exchange peer|nccl] [--check]
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import random

import torch
import torch.distributed as dist

from . import ops
from .fixtures import make_paged_kv
from .stack import make_model


def shard_rows(t: torch.Tensor, parts) -> torch.Tensor:
    """Concatenate row ranges `parts` ([(start, stop), ...]) of t into one contiguous tensor."""
    return torch.cat([t[a:b] for a, b in parts], dim=0).contiguous()


def tp_slices(world: int, rank: int, heads: int, kv_heads: int, head_dim: int, hid: int, ff: int) -> dict:
    """Row ranges of each full weight that rank `rank` of `world` owns (see the module text)."""
    for n, what in ((heads, "heads"), (kv_heads, "kv_heads"), (hid, "hid"), (ff, "ff")):
        if n % world:
            raise ValueError(f"{what}={n} does not split over {world} ranks")
    hl, kl, D = heads // world, kv_heads // world, head_dim
    q0, k0, v0 = 0, heads * D, (heads + kv_heads) * D
    hs, fs = hid // world, ff // world
    return {
        "qkv": [(q0 + rank * hl * D, q0 + (rank + 1) * hl * D), (k0 + rank * kl * D, k0 + (rank + 1) * kl * D),
                (v0 + rank * kl * D, v0 + (rank + 1) * kl * D)],
        "o": [(rank * hs, (rank + 1) * hs)],
        "gu": [(rank * fs, (rank + 1) * fs), (ff + rank * fs, ff + (rank + 1) * fs)],
        "down": [(rank * hs, (rank + 1) * hs)],
        "kv_heads": (rank * kl, (rank + 1) * kl),
    }


def gathered_to_rows(buf: torch.Tensor, world: int, rows: int, out: torch.Tensor) -> None:
    """out[:rows] <- the all-gathered column shards: buf holds rank r's [rows, n] block at
    buf[r * rows: (r + 1) * rows]; out's columns [r n, (r+1) n) take it."""
    n = buf.shape[-1]
    out[:rows].view(rows, world, n).copy_(buf[: world * rows].view(world, rows, n).transpose(0, 1))


class StackTP:
    def __init__(self, world, rank, layers=4, hid=4096, ff=14336, heads=32, kv_heads=8, head_dim=128, ctx=1024,
                 b_max=32, ks=(0, 2, 4, 8), page=16, seed=0, device="cuda", group=None, exchange="nccl"):
        if exchange not in ("nccl", "peer", "fused"):
            raise ValueError(f"exchange {exchange!r}: 'nccl', 'peer' or 'fused'")
        self.g, self.r, self.group, self.exchange = world, rank, group, exchange
        self.L, self.hid, self.ff, self.H, self.H_KV, self.D = layers, hid, ff, heads, kv_heads, head_dim
        self.b_max, self.ks = b_max, tuple(ks)
        self.ql_max = max(ks) + 1
        self.m_max = b_max * self.ql_max
        self.Hl, self.Kl = heads // world, kv_heads // world
        sl = tp_slices(world, rank, heads, kv_heads, head_dim, hid, ff)
        w, self.h0 = make_model(layers, hid, ff, heads, kv_heads, head_dim, self.m_max, seed, device)
        self.w = [{name: (shard_rows(q, sl[name]), shard_rows(s, sl[name])) for name, (q, s) in lw.items()}
                  for lw in w]
        del w
        k0, k1 = sl["kv_heads"]
        self.kv = []
        for i in range(layers):
            kc, vc, ks_, vs, bt, cl = make_paged_kv(b_max, [ctx] * b_max, kv_heads, head_dim, PAGE=page,
                                                    device=device, seed=seed + i)
            self.kv.append((kc[:, :, k0:k1].contiguous(), vc[:, :, k0:k1].contiguous(),
                            ks_[:, :, k0:k1].contiguous(), vs[:, :, k0:k1].contiguous(), bt, cl))
        M, D, g = self.m_max, head_dim, world
        mk = lambda *shape, dtype=torch.float16: torch.zeros(shape, dtype=dtype, device=device)  # noqa: E731
        self.h = self.h0.clone()
        self.x8, self.sx = mk(M, hid, dtype=torch.int8), mk(M, dtype=torch.float32)
        self.qkv = mk(M, (self.Hl + 2 * self.Kl) * D)
        self.attn_l, self.attn = mk(M, self.Hl * D), mk(M, heads * D)
        self.o_l, self.o = mk(M, hid // g), mk(M, hid)
        self.gu_l = mk(M, 2 * ff // g)
        self.amax = mk(M, dtype=torch.float32)
        self.f8_l, self.f8, self.sf = mk(M, ff // g, dtype=torch.int8), mk(M, ff, dtype=torch.int8), mk(M, dtype=torch.float32)
        self.down_l, self.down = mk(M, hid // g), mk(M, hid)
        self.bufs = {n: torch.empty(g * t.numel(), dtype=t.dtype, device=device).view(g * M, t.shape[1])
                     for n, t in (("attn", self.attn_l), ("o", self.o_l), ("f8", self.f8_l), ("down", self.down_l))}
        if exchange in ("peer", "fused"):
            # the gathered rows land in symmetric full buffers written by every rank's kernel
            # (with "fused", the O and down projections' own epilogues store them)
            from .peer import PeerExchange
            self.px = PeerExchange(group)
            self.attn = self.px.add("attn", M, self.Hl * D, torch.float16)
            self.o = self.px.add("o", M, hid // g, torch.float16)
            self.f8 = self.px.add("f8", M, ff // g, torch.int8)
            self.down = self.px.add("down", M, hid // g, torch.float16)
            self.px.add("amax", M, 1, torch.float32)
            self.bufs = {}
        self.plan = torch.zeros(4, dtype=torch.int32, device=device)
        self.plan_host = torch.zeros(1024, 4, dtype=torch.int32).pin_memory()
        self._slot = 0
        self._kv0 = None

    # ---- state (as the single-GPU stack) ------------------------------------------------------
    def snapshot(self):
        self._kv0 = [tuple(t.clone() for t in kv[:4]) for kv in self.kv]

    def reset(self):
        self.h.copy_(self.h0)
        for kv, kv0 in zip(self.kv, self._kv0):
            for t, t0 in zip(kv[:4], kv0):
                t.copy_(t0)

    def set_plan(self, B, ql):
        if self._slot == self.plan_host.shape[0]:
            torch.cuda.current_stream().synchronize()
            self._slot = 0
        h = self.plan_host[self._slot]
        self._slot += 1
        h[0], h[1], h[2] = B * ql, B, ql
        self.plan.copy_(h, non_blocking=True)

    def _gather(self, name, local, full, rows, plan=None):
        if self.exchange in ("peer", "fused"):
            self.px.gather(name, local, rows, plan=plan)   # lands in `full` (the symmetric buffer)
            return
        buf = self.bufs[name]
        dist.all_gather_into_tensor(buf[: self.g * rows], local[:rows], group=self.group)
        gathered_to_rows(buf, self.g, rows, full)

    def _amax_all_ranks(self, rows, plan=None):
        if self.exchange in ("peer", "fused"):
            self.px.all_max("amax", self.amax, self.amax, rows, plan=plan)
        else:
            dist.all_reduce(self.amax[:rows], op=dist.ReduceOp.MAX, group=self.group)

    # ---- one verification pass ----------------------------------------------------------------
    def step(self, B, ql, use_plan=False):
        if use_plan:
            M, Bg, qlg = self.m_max, self.b_max, self.ql_max
            pl, pa = self.plan, self.plan[1:]
        else:
            M, Bg, qlg = B * ql, B, ql
            pl = pa = None
        gm = dict(plan=pl, grid_m_max=M) if use_plan else {}
        rows = slice(0, M)
        D, Hl, Kl = self.D, self.Hl, self.Kl
        for i, (lw, kv) in enumerate(zip(self.w, self.kv)):
            kc, vc, ks, vs, bt, cl = kv
            if i == 0:
                ops.quant_rows(self.h[rows], q=self.x8[rows], s=self.sx[rows], plan=pl)
            else:
                ops.quant_rows(self.down[rows], mode=ops.QUANT_RESIDUAL, residual=self.h[rows], q=self.x8[rows],
                               s=self.sx[rows], plan=pl, wait=self._wait("down"))
            ops.w8a8_matmul(self.x8[rows], self.sx[rows], *lw["qkv"], out=self.qkv[rows], **gm)
            ops.kv_append(self.qkv, Hl * D, (Hl + Kl) * D, kc, vc, ks, vs, bt[:Bg], cl[:Bg], ql, plan=pa, B=Bg,
                          ql_max=qlg)
            ops.paged_attention_packed(self.qkv, 0, self.attn_l, kc, vc, ks, vs, bt[:Bg], cl[:Bg], ql, Hl, B=Bg,
                                       ql_max=qlg, QPP=self.ql_max, plan=pa)
            self._gather("attn", self.attn_l, self.attn, M, pl)
            ops.quant_rows(self.attn[rows], q=self.x8[rows], s=self.sx[rows], plan=pl)
            self._gemm_out("o", self.x8, self.sx, lw["o"], self.o_l, self.o, M, pl, gm)
            ops.quant_rows(self.o[rows], mode=ops.QUANT_RESIDUAL, residual=self.h[rows], q=self.x8[rows],
                           s=self.sx[rows], plan=pl, wait=self._wait("o"))
            ops.w8a8_matmul(self.x8[rows], self.sx[rows], *lw["gu"], out=self.gu_l[rows], **gm)
            ops.quant_rows(self.gu_l[rows], mode=ops.QUANT_SILU_MUL, amax_out=self.amax[rows], plan=pl)
            self._amax_all_ranks(M, pl)
            ops.quant_rows(self.gu_l[rows], mode=ops.QUANT_SILU_MUL, q=self.f8_l[rows], s=self.sf[rows], plan=pl,
                           amax_in=self.amax[rows])
            self._gather("f8", self.f8_l, self.f8, M, pl)
            self._gemm_out("down", self.f8, self.sf, lw["down"], self.down_l, self.down, M, pl, gm)
        ops.quant_rows(self.down[rows], mode=ops.QUANT_RESIDUAL, residual=self.h[rows], q=self.x8[rows],
                       s=self.sx[rows], plan=pl, wait=self._wait("down"))

    def _gemm_out(self, name, a, sa, w, local, full, M, pl, gm):
        """A row-sharded projection whose output columns every rank needs: with exchange="fused"
        the GEMM's epilogue stores them into every rank's full buffer; otherwise the GEMM writes
        its block locally and an all-gather follows."""
        rows = slice(0, M)
        if self.exchange == "fused":
            self.px.w8a8(name, a[rows], sa[rows], *w, M, plan=pl)
            return
        ops.w8a8_matmul(a[rows], sa[rows], *w, out=local[rows], **gm)
        self._gather(name, local, full, M, pl)

    def _wait(self, name):
        return self.px.wait_args(name) if self.exchange == "fused" else None

    def capture(self, fn):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g


def _max_over_ranks(x: float, group=None) -> float:
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def run(world, rank, layers=4, steps=200, b_max=32, ks=(0, 2, 4, 8), ctx=1024, seed=0, check=False, exchange="nccl"):
    """Eager and plan-graph latency of the tensor-parallel stack over a seeded (B, k) trace;
    times are device times (CUDA events) per step, the max over ranks.  check: rank 0 also runs
    the single-GPU stack and reports the largest difference of the residual streams."""
    st = StackTP(world, rank, layers=layers, b_max=b_max, ks=ks, ctx=ctx, seed=seed, exchange=exchange)
    st.snapshot()
    ql_max = st.ql_max
    rng = random.Random(seed)
    trace = [(rng.randint(1, b_max), rng.choice(ks)) for _ in range(steps)]
    res = {"config": dict(world=world, layers=layers, b_max=b_max, ks=list(ks), ctx=ctx, m_max=st.m_max,
                          steps=steps, parallelism=f"tp{world}", exchange=exchange)}
    for B, k in sorted(set(trace))[:4]:
        st.step(B, k + 1)
    torch.cuda.synchronize()
    st.set_plan(b_max, ql_max)
    graph = st.capture(lambda: st.step(b_max, ql_max, use_plan=True))
    torch.cuda.synchronize()
    useful = sum(B * (k + 1) for B, k in trace)
    strategies = {"eager": lambda B, k: st.step(B, k + 1),
                  "plan": lambda B, k: (st.set_plan(B, k + 1), graph.replay())}
    for name, fn in strategies.items():
        for B, k in trace[:10]:
            fn(B, k)
        torch.cuda.synchronize()
        dist.barrier(group=st.group)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in trace]
        for (B, k), (a, b) in zip(trace, ev):
            a.record()
            fn(B, k)
            b.record()
        torch.cuda.synchronize()
        lat = [a.elapsed_time(b) for a, b in ev]
        total = _max_over_ranks(sum(lat), st.group)
        lat.sort()
        res[name] = dict(p50_ms=_max_over_ranks(lat[len(lat) // 2], st.group), mean_ms=total / len(lat),
                         tok_per_s=useful / (total / 1e3))
    # plan graph vs eager, and (check) vs the single-GPU stack, on a few shapes
    worst_plan, worst_single = 0.0, 0.0
    single = None
    if check and rank == 0:
        from .stack import Stack
        single = Stack(layers=layers, b_max=b_max, ks=ks, ctx=ctx, seed=seed)
        single.snapshot()
    for B, ql in [(1, 1), (b_max, ql_max), (3, 3), (b_max // 2 + 1, min(5, ql_max))]:
        st.reset()
        st.step(B, ql)
        ref = st.h[: B * ql].clone()
        st.reset()
        st.set_plan(B, ql)
        graph.replay()
        torch.cuda.synchronize()
        worst_plan = max(worst_plan, (st.h[: B * ql].float() - ref.float()).abs().max().item())
        if single is not None:
            single.reset()
            single.step(B, ql)
            worst_single = max(worst_single, (single.h[: B * ql].float() - ref.float()).abs().max().item())
    res["plan_vs_eager_max_abs_diff"] = _max_over_ranks(worst_plan, st.group)
    if check:
        res["tp_vs_single_gpu_max_abs_diff"] = _max_over_ranks(worst_single, st.group)
    st.reset()
    del graph
    return res


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--b-max", type=int, default=32)
    ap.add_argument("--ks", default="0,2,4,8")
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--check", action="store_true", help="compare with the single-GPU stack on rank 0")
    ap.add_argument("--exchange", choices=("nccl", "peer", "fused"), default="peer",
                    help="all-gathers by NCCL, by the library's peer-store kernel, or (fused) with the O and "
                         "down projections storing into every rank's buffer from their epilogues")
    args = ap.parse_args()
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        res = run(world, rank, layers=args.layers, steps=args.steps, b_max=args.b_max,
                  ks=tuple(int(k) for k in args.ks.split(",")), ctx=args.ctx, seed=args.seed, check=args.check,
                  exchange=args.exchange)
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

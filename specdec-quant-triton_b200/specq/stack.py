"""Plan-buffer CUDA graph of an INT8 Llama-3-8B-shaped verification stack.

The reference's graph benchmark (bench_graphs.py:17-114) drives L W8A8 + INT8-attention
layers with a random (B, k) trace and compares four strategies:

  eager      exact shapes, one launch per kernel
  allshapes  one graph per (B, k)
  maxpad     one graph per B, always verifying k_max + 1 tokens (padding waste)
  plan       ONE graph captured at (B_max, k_max + 1); the active (M, B, q_len) are copied into
             a device plan buffer before each replay and the kernels leave early outside them

Here a layer has a connected data flow (the reference's layers read static buffers):

  x8 = quant(h) [or quant(h += down of the previous layer)]
  qkv = W8A8(x8, Wqkv)                         -> K/V of the new tokens appended to the cache
  a = attention(q rows of qkv) ; o = W8A8(quant(a), Wo)
  gu = W8A8(quant(h += o), Wgu) ; down = W8A8(quant(silu(g) * u), Wdown)

with fp16 residual adds fused into the quantiser.  Token rows are packed (sequence b's token t
at row b * q_len + t), so under the plan graph every kernel finds the active rows from the
plan alone.  `run` reports per-strategy latency, throughput and padding waste, and the largest
difference between the plan graph and eager execution (0: bit-exact).

    python -m specq.stack [--layers 4] [--steps 200] [--b-max 32] [--ks 0,2,4,8]
"""
from __future__ import annotations

import argparse
import os
import json
import random
import time

import torch

from . import ops
from .fixtures import make_paged_kv


def make_model(layers, hid, ff, heads, kv_heads, head_dim, m_max, seed, device):
    """Random INT8 weights of every layer ({"qkv", "o", "gu", "down"}: (int8 [N, K], fp32 scales
    [N])) and the initial residual stream [m_max, hid], drawn in a fixed order from one seed:
    the single-GPU and the tensor-parallel stacks build the same model."""
    g = torch.Generator(device=device).manual_seed(seed)

    def w8(n, k):   # int8 weights uniform in [-127, 127], per-channel scales ~ 1/sqrt(k)
        q = torch.randint(-127, 128, (n, k), generator=g, device=device, dtype=torch.int16).to(torch.int8)
        s = (torch.rand(n, generator=g, device=device) * 0.5 + 0.5) / (127.0 * k ** 0.5)
        return q, s

    n_qkv = (heads + 2 * kv_heads) * head_dim
    w = [{"qkv": w8(n_qkv, hid), "o": w8(hid, hid), "gu": w8(2 * ff, hid), "down": w8(hid, ff)}
         for _ in range(layers)]
    h0 = (torch.randn(m_max, hid, generator=g, device=device) * 0.5).half()
    return w, h0


class Stack:
    def __init__(self, layers=4, hid=4096, ff=14336, heads=32, kv_heads=8, head_dim=128, ctx=1024, b_max=32,
                 ks=(0, 2, 4, 8), page=16, seed=0, device="cuda"):
        self.L, self.hid, self.ff, self.H, self.H_KV, self.D = layers, hid, ff, heads, kv_heads, head_dim
        self.ctx, self.b_max, self.ks, self.page = ctx, b_max, tuple(ks), page
        self.ql_max = max(ks) + 1
        self.m_max = b_max * self.ql_max
        self.n_qkv = (heads + 2 * kv_heads) * head_dim
        self.w, self.h0 = make_model(layers, hid, ff, heads, kv_heads, head_dim, self.m_max, seed, device)
        self.kv = [make_paged_kv(b_max, [ctx] * b_max, kv_heads, head_dim, PAGE=page, device=device, seed=seed + i)
                   for i in range(layers)]
        mk = lambda *shape, dtype=torch.float16: torch.zeros(shape, dtype=dtype, device=device)  # noqa: E731
        self.h = self.h0.clone()
        self.x8, self.sx = mk(self.m_max, hid, dtype=torch.int8), mk(self.m_max, dtype=torch.float32)
        self.f8, self.sf = mk(self.m_max, ff, dtype=torch.int8), mk(self.m_max, dtype=torch.float32)
        self.qkv, self.attn = mk(self.m_max, self.n_qkv), mk(self.m_max, hid)
        self.o, self.gu, self.down = mk(self.m_max, hid), mk(self.m_max, 2 * ff), mk(self.m_max, hid)
        self.plan = torch.zeros(4, dtype=torch.int32, device=device)   # [M, B, q_len]
        # one pinned slot per enqueued step: a slot must not be rewritten while its
        # asynchronous copy may still be pending
        self.plan_host = torch.zeros(1024, 4, dtype=torch.int32).pin_memory()
        self._slot = 0
        self._kv0 = None

    # ---- state ------------------------------------------------------------------------------
    def snapshot(self):
        """Remember the residual stream and caches (appends change them)."""
        self._kv0 = [tuple(t.clone() for t in kv[:4]) for kv in self.kv]

    def reset(self):
        self.h.copy_(self.h0)
        for kv, kv0 in zip(self.kv, self._kv0):
            for t, t0 in zip(kv[:4], kv0):
                t.copy_(t0)

    def set_plan(self, B, ql):
        if self._slot == self.plan_host.shape[0]:   # every slot used: let the copies drain
            torch.cuda.current_stream().synchronize()
            self._slot = 0
        h = self.plan_host[self._slot]
        self._slot += 1
        h[0], h[1], h[2] = B * ql, B, ql
        self.plan.copy_(h, non_blocking=True)

    # ---- one verification pass --------------------------------------------------------------
    def step(self, B, ql, use_plan=False):
        """B sequences x ql tokens through every layer (use_plan: the grid is the maximum shape
        and the active shape comes from the plan buffer)."""
        if use_plan:
            M, Bg, qlg = self.m_max, self.b_max, self.ql_max
            pl, pa = self.plan, self.plan[1:]
        else:
            M, Bg, qlg = B * ql, B, ql
            pl = pa = None
        gm = dict(plan=pl, grid_m_max=M) if use_plan else {}
        rows = slice(0, M)
        hid, kvd = self.hid, self.H_KV * self.D
        for i, (lw, kv) in enumerate(zip(self.w, self.kv)):
            kc, vc, ks, vs, bt, cl = kv
            if i == 0:
                ops.quant_rows(self.h[rows], q=self.x8[rows], s=self.sx[rows], plan=pl)
            else:   # h += down of the previous layer, then quantise
                ops.quant_rows(self.down[rows], mode=ops.QUANT_RESIDUAL, residual=self.h[rows], q=self.x8[rows],
                               s=self.sx[rows], plan=pl)
            ops.w8a8_matmul(self.x8[rows], self.sx[rows], *lw["qkv"], out=self.qkv[rows], **gm)
            ops.kv_append(self.qkv, self.H * self.D, self.H * self.D + kvd, kc, vc, ks, vs, bt[:Bg], cl[:Bg], ql,
                          plan=pa, B=Bg, ql_max=qlg)
            # one CTA schedule (QPP = the graph's q_len) in every mode: identical bits
            ops.paged_attention_packed(self.qkv, 0, self.attn, kc, vc, ks, vs, bt[:Bg], cl[:Bg], ql, self.H, B=Bg,
                                       ql_max=qlg, QPP=self.ql_max, plan=pa)
            ops.quant_rows(self.attn[rows], q=self.x8[rows], s=self.sx[rows], plan=pl)
            ops.w8a8_matmul(self.x8[rows], self.sx[rows], *lw["o"], out=self.o[rows], **gm)
            ops.quant_rows(self.o[rows], mode=ops.QUANT_RESIDUAL, residual=self.h[rows], q=self.x8[rows],
                           s=self.sx[rows], plan=pl)
            ops.w8a8_matmul(self.x8[rows], self.sx[rows], *lw["gu"], out=self.gu[rows], **gm)
            ops.quant_rows(self.gu[rows], mode=ops.QUANT_SILU_MUL, q=self.f8[rows], s=self.sf[rows], plan=pl)
            ops.w8a8_matmul(self.f8[rows], self.sf[rows], *lw["down"], out=self.down[rows], **gm)
        # the last layer's residual add (its quantised output is not used)
        ops.quant_rows(self.down[rows], mode=ops.QUANT_RESIDUAL, residual=self.h[rows], q=self.x8[rows],
                       s=self.sx[rows], plan=pl)

    def capture(self, fn, pool=None):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=pool):
            fn()
        return g


def plan_vs_eager(stack: Stack, shapes) -> float:
    """Largest |difference| of the residual stream and the appended caches between eager
    execution and the plan graph over `shapes` (0.0: bit-exact)."""
    stack.snapshot()
    stack.reset()
    stack.set_plan(stack.b_max, stack.ql_max)
    g = stack.capture(lambda: stack.step(stack.b_max, stack.ql_max, use_plan=True))
    worst = 0.0
    for B, ql in shapes:
        stack.reset()
        stack.step(B, ql)
        ref_h = stack.h[: B * ql].clone()
        ref_kv = [tuple(t.clone() for t in kv[:4]) for kv in stack.kv]
        stack.reset()
        stack.set_plan(B, ql)
        g.replay()
        torch.cuda.synchronize()
        worst = max(worst, (stack.h[: B * ql].float() - ref_h.float()).abs().max().item())
        for kv, rk in zip(stack.kv, ref_kv):
            for t, r in zip(kv[:4], rk):
                worst = max(worst, (t.float() - r.float()).abs().max().item())
    stack.reset()
    del g
    return worst


def run(layers=4, steps=200, b_max=32, ks=(0, 2, 4, 8), ctx=1024, seed=0, allshapes=True):
    stack = Stack(layers=layers, b_max=b_max, ks=ks, ctx=ctx, seed=seed)
    stack.snapshot()
    ql_max = stack.ql_max
    rng = random.Random(seed)
    trace = [(rng.randint(1, b_max), rng.choice(ks)) for _ in range(steps)]
    res = {"config": dict(layers=layers, b_max=b_max, ks=list(ks), ctx=ctx, m_max=stack.m_max, steps=steps)}

    pool = torch.cuda.graph_pool_handle()
    for B, k in set(trace):   # warm up every eager shape
        stack.step(B, k + 1)
    torch.cuda.synchronize()
    graphs = {}
    t0 = time.perf_counter()
    stack.set_plan(b_max, ql_max)
    graphs["plan"] = stack.capture(lambda: stack.step(b_max, ql_max, use_plan=True), pool)
    torch.cuda.synchronize()
    res["plan_build_s"], res["plan_graphs"] = time.perf_counter() - t0, 1
    t0 = time.perf_counter()
    g_pad = {B: stack.capture(lambda B=B: stack.step(B, ql_max), pool) for B in sorted({b for b, _ in trace})}
    torch.cuda.synchronize()
    res["maxpad_build_s"], res["maxpad_graphs"] = time.perf_counter() - t0, len(g_pad)
    g_all = {}
    if allshapes:
        t0 = time.perf_counter()
        g_all = {(B, k): stack.capture(lambda B=B, k=k: stack.step(B, k + 1), pool) for B, k in sorted(set(trace))}
        torch.cuda.synchronize()
        res["allshapes_build_s"], res["allshapes_graphs"] = time.perf_counter() - t0, len(g_all)

    strategies = {
        "eager": lambda B, k: stack.step(B, k + 1),
        "maxpad": lambda B, k: g_pad[B].replay(),
        "plan": lambda B, k: (stack.set_plan(B, k + 1), graphs["plan"].replay()),
    }
    if allshapes:
        strategies["allshapes"] = lambda B, k: g_all[(B, k)].replay()
    useful = sum(B * (k + 1) for B, k in trace)
    for name, fn in strategies.items():
        for B, k in trace[:10]:
            fn(B, k)
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in trace]
        for (B, k), (a, b) in zip(trace, ev):
            a.record()
            fn(B, k)
            b.record()
        torch.cuda.synchronize()
        lat = sorted(a.elapsed_time(b) for a, b in ev)   # device time per step, ms
        total = sum(lat)
        computed = sum(B * ql_max for B, _ in trace) if name == "maxpad" else useful
        res[name] = dict(p50_ms=lat[len(lat) // 2], p99_ms=lat[min(len(lat) - 1, int(0.99 * len(lat)))],
                         mean_ms=total / len(lat), tok_per_s=useful / (total / 1e3),
                         waste_pct=100.0 * (computed - useful) / useful)
    stack.reset()
    shapes = [(1, 1), (b_max, ql_max), (3, 3), (b_max // 2 + 1, 5)]
    res["plan_vs_eager_max_abs_diff"] = plan_vs_eager(stack, [(B, ql) for B, ql in shapes if ql <= ql_max])
    res["plan_overhead_vs_allshapes_pct"] = (100.0 * (res["plan"]["mean_ms"] / res["allshapes"]["mean_ms"] - 1)
                                            if allshapes else None)
    return res


def _event_us(fn, reps=50):
    """Mean device time of fn() in µs: `reps` calls captured in one CUDA graph (so the host's
    launch cost is not what is timed), CUDA events around a replay."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        with torch.cuda.graph(graph, stream=st):
            for _ in range(reps):
                fn()
    torch.cuda.current_stream().wait_stream(st)
    graph.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / reps


def measure_rowops(hbm_gbs=None):
    """Device time and algorithmic bandwidth of the row kernels at the stack's largest shapes:
    the quantiser (M=288 rows of 4096 / 14336), the KV append (32 sequences x 9 tokens) and
    the INT4 packer (the W4A16 config's 14336 x 4096 weight).  The quantiser's and the
    append's inputs fit in L2, so theirs are L2-warm figures; the packer's 117 MB input
    streams from HBM."""
    import specq
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    res = {}

    def rec(name, us, nbytes):
        res[name] = {"us": round(us, 3), "bytes": int(nbytes), "gbs": round(nbytes / us / 1e3, 1)}
        if hbm_gbs:
            res[name]["hbm_frac"] = round(nbytes / us / 1e3 / hbm_gbs, 4)

    M = 288
    for N, mode, name in ((4096, specq.QUANT_PLAIN, "quant_rows_plain_4096"),
                          (4096, specq.QUANT_RESIDUAL, "quant_rows_residual_4096"),
                          (14336, specq.QUANT_SILU_MUL, "quant_rows_silu_14336")):
        x = torch.randn(M, 2 * N if mode == specq.QUANT_SILU_MUL else N, device=dev, generator=g).half()
        r = torch.randn(M, N, device=dev, generator=g).half() if mode == specq.QUANT_RESIDUAL else None
        q = torch.empty(M, N, dtype=torch.int8, device=dev)
        sc = torch.empty(M, device=dev)
        us = _event_us(lambda: specq.quant_rows(x, mode=mode, residual=r, q=q, s=sc))
        nbytes = x.numel() * 2 + M * N + 4 * M + (2 * 2 * M * N if r is not None else 0)
        rec(name, us, nbytes)
    B, ql, H_KV, D = 32, 9, 8, 128
    kc, vc, ks, vs, bt, cl = specq.make_paged_kv(B, [1024] * B, H_KV, D, device=dev, seed=1)
    x = torch.randn(B * ql, (32 + 2 * H_KV) * D, device=dev, generator=g).half()
    us = _event_us(lambda: specq.kv_append(x, 32 * D, (32 + H_KV) * D, kc, vc, ks, vs, bt, cl, ql))
    rec("kv_append_b32_q9", us, B * ql * 2 * H_KV * (2 * D + D + 2))
    w = (torch.randn(14336, 4096, device=dev, generator=g) * 0.02).half()
    us = _event_us(lambda: specq.pack_int4(w, 128, deq=False), reps=20)
    rec("pack_int4_14336x4096", us, w.numel() * 2 + w.numel() // 2 + 2 * w.numel() // 128)
    us = _event_us(lambda: specq.pack_int4(w, 128, deq=True), reps=20)
    rec("pack_int4_14336x4096_with_deq", us, w.numel() * 4 + w.numel() // 2 + 2 * w.numel() // 128)
    return res


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--b-max", type=int, default=32)
    ap.add_argument("--ks", default="0,2,4,8")
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-allshapes", action="store_true")
    ap.add_argument("--rowops", action="store_true", help="time the row kernels instead of the stack")
    args = ap.parse_args()
    if args.rowops:
        peaks = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                             "MEASURED_PEAKS.json")
        hbm = json.load(open(peaks)).get("hbm_gbs") if os.path.exists(peaks) else None
        print(json.dumps({"rowops": measure_rowops(hbm), "hbm_gbs_peak": hbm}), flush=True)
        return
    res = run(layers=args.layers, steps=args.steps, b_max=args.b_max, ks=tuple(int(k) for k in args.ks.split(",")),
              ctx=args.ctx, seed=args.seed, allshapes=not args.no_allshapes)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

"""Timing sweep of the GEMMs over the verification grid M = B * (k + 1).

  W8A8  the Llama-3-8B linear set (qkv 4096->6144, o 4096->4096, gate_up 4096->28672,
        down 14336->4096) with N sharded over g GPUs (the per-GPU shape N/g is timed; survey
        config 3)
  W4A16 gate_proj 4096->14336 (config 1)

for B in {1, 2, 4, 8, 16, 32} and k in {0, 2, 4, 8}.  Each point is the mean device time of one
launch (CUDA events around a captured chain of >= 30 launches over rotating input copies,
together larger than L2, so the weights stream from HBM), with the algorithmic bytes, achieved GB/s and
the fraction of the measured HBM bandwidth, and the tensor throughput against the dense peak
(INT8: 4500 TOPS nominal, no measured figure; FP16: the measured burst peak).

    PYTHONPATH=specdec-quant-triton_b200 python -m specq.sweep [--shards 1,2,4,8] [--reps 20]
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from . import ops

L2_BYTES = 126 * 1024 * 1024
INT8_TOPS_NOMINAL = 4500.0
LINEAR_SET = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336)}
W4A16_SHAPE = (14336, 4096)
BS, KS = (1, 2, 4, 8, 16, 32), (0, 2, 4, 8)


def _peaks():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"])
    return 6650.0, 1590.0


def _time(fns, reps, chain=30):
    """Mean device time of one launch: a captured chain of at least `chain` launches rotating
    over `fns` (consecutive launches overlap their prologue as in a serving loop), replayed."""
    for f in fns:
        f()
    torch.cuda.synchronize()
    fns = [fns[i % len(fns)] for i in range(len(fns) * max(1, -(-chain // len(fns))))]
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / (reps * len(fns))


def w8a8_points(shards=(1,), reps=20, seed=0):
    hbm, _ = _peaks()
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(seed)
    out = []
    for g in shards:
        for name, (N_full, K) in LINEAR_SET.items():
            N = N_full // g
            w_bytes = N * K
            copies = max(2, math.ceil(2 * L2_BYTES / w_bytes))
            ws = [torch.randint(-127, 128, (N, K), generator=gen, device=dev, dtype=torch.int16).to(torch.int8)
                  for _ in range(copies)]
            sws = [torch.rand(N, generator=gen, device=dev) * 0.019 + 0.001 for _ in range(copies)]
            for B in BS:
                for k in KS:
                    M = B * (k + 1)
                    a = torch.randint(-127, 128, (M, K), generator=gen, device=dev, dtype=torch.int16).to(torch.int8)
                    sa = torch.rand(M, generator=gen, device=dev) * 0.019 + 0.001
                    outs = [torch.empty(M, N, dtype=torch.float16, device=dev) for _ in range(copies)]
                    us = _time([lambda i=i: ops.w8a8_matmul(a, sa, ws[i], sws[i], out=outs[i]) for i in range(copies)],
                               reps)
                    nbytes = M * K + N * K + 4 * M + 4 * N + 2 * M * N
                    tops = 2.0 * M * N * K / us / 1e6
                    out.append({"kernel": "w8a8", "shape": name, "shards": g, "N": N, "K": K, "B": B, "k": k, "M": M,
                                "us": round(us, 3), "gbs": round(nbytes / us / 1e3, 1),
                                "hbm_frac": round(nbytes / us / 1e3 / hbm, 4), "tops": round(tops, 1),
                                "int8_frac_nominal": round(tops / INT8_TOPS_NOMINAL, 4)})
            del ws, sws
    return out


def w4a16_points(reps=20, seed=0):
    hbm, fp16_tf = _peaks()
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(seed)
    N, K = W4A16_SHAPE
    copies = max(2, math.ceil(2 * L2_BYTES / (N * K // 2)))
    wps = [torch.randint(0, 256, (N, K // 2), generator=gen, device=dev, dtype=torch.int32).to(torch.uint8)
           for _ in range(copies)]
    scs = [(torch.rand(N, K // 128, generator=gen, device=dev) * 0.015 + 0.005).half() for _ in range(copies)]
    out = []
    for B in BS:
        for k in KS:
            M = B * (k + 1)
            x = torch.randn(M, K, generator=gen, device=dev).half()
            outs = [torch.empty(M, N, dtype=torch.float16, device=dev) for _ in range(copies)]
            us = _time([lambda i=i: ops.w4a16_matmul(x, wps[i], scs[i], out=outs[i]) for i in range(copies)], reps)
            nbytes = N * K // 2 + 2 * N * K // 128 + 2 * M * K + 2 * M * N
            tf = 2.0 * M * N * K / us / 1e6
            out.append({"kernel": "w4a16", "N": N, "K": K, "B": B, "k": k, "M": M, "us": round(us, 3),
                        "gbs": round(nbytes / us / 1e3, 1), "hbm_frac": round(nbytes / us / 1e3 / hbm, 4),
                        "tflops": round(tf, 1), "fp16_frac": round(tf / fp16_tf, 4)})
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--shards", default="1,2,4,8")
    ap.add_argument("--reps", type=int, default=20)
    args = ap.parse_args()
    shards = tuple(int(s) for s in args.shards.split(","))
    res = {"w8a8": w8a8_points(shards, args.reps), "w4a16": w4a16_points(args.reps), "peaks": _peaks()}
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

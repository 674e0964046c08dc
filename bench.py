#!/usr/bin/env python
"""Benchmark of the verification step on B200: W8A8 GEMM + W4A16 GEMM + INT8 paged attention.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One "step" is one pass of the hot path over one batch of synthetic inputs with the BASELINE
configs' shapes and value distributions:
  * W8A8 GEMM, Llama-3-8B o_proj, M = B*(k+1) = 40 (B=8, k=4), K = N = 4096      (config 0)
  * W4A16 GEMM, Llama-3-8B gate_proj, M = 72 (B=8, k=8), K = 4096, N = 14336     (config 1)
  * INT8 paged verification attention, B=8, ctx 4096, k=8, QPP=k+1, 32/8 heads   (config 2)
With N GPUs (torchrun, one process per GPU) the step is sharded as the north star describes:
GEMM output columns and attention KV heads are split across ranks (strong scaling, no
data-path collective); the step time is the max over ranks.

Printed (rank 0, one JSON line): value = device microseconds per step (inputs resident in HBM,
captured CUDA graph replays, rotating input copies larger than L2), per-kernel times with
their roofline fractions, e2e = the same step through the public Python API with pinned
host buffers and host<->device copies inside the timed region (each call's H2D -> call -> D2H
chain on its own stream), and cpu_baseline = the
reference's exact PyTorch path timed on this host's CPU cores.

`--impl reference` times the reference's own CPU implementation of the path (the oracle port
of its exact PyTorch functions; the reference cannot be installed: it is a Triton/Windows
research repo with no package metadata) on this host's cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "specdec-quant-triton_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
INT8_DENSE_TOPS_NOMINAL = 4500.0   # datasheet dense INT8, used only when no measured figure exists

# per-GPU workload at N = 1
W8 = dict(M=40, K=4096, N=4096)
W4 = dict(M=72, K=4096, N=14336, group=128)
AT = dict(B=8, ctx=4096, H=32, H_KV=8, D=128, page=16, k=8)


def _metric():
    try:
        with open(os.path.join(REPO, "BASELINE.json")) as f:
            return json.load(f)["metric"]
    except Exception:
        return "us & % roofline vs M=B*(k+1) for W8A8/W4A16 GEMM and INT8 paged attn"


def _peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def _int8_peak():
    """Dense INT8 tensor peak in TOPS: the figure `bench.py --mma-peak` measured on this pool
    (committed in profiles/int8_mma_peak.md as `int8_dense_tops_burst:` / `..._sustained:`), else
    the datasheet value.  Returns (burst, sustained, source)."""
    path = os.path.join(REPO, "profiles", "int8_mma_peak.md")
    vals = {}
    try:
        for line in open(path):
            for key in ("int8_dense_tops_burst", "int8_dense_tops_sustained"):
                if line.startswith(key + ":"):
                    vals[key] = float(line.split(":", 1)[1].strip())
    except Exception:
        pass
    if "int8_dense_tops_burst" in vals:
        return (vals["int8_dense_tops_burst"], vals.get("int8_dense_tops_sustained", vals["int8_dense_tops_burst"]),
                "measured (bench.py --mma-peak)")
    return INT8_DENSE_TOPS_NOMINAL, INT8_DENSE_TOPS_NOMINAL, "nominal datasheet"


def _traffic_from_profiles():
    """DRAM bytes per launch of the attention kernel from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", "paged_attn_config2.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except Exception:
        pass
    return None


# ----------------------------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------------------------
@contextlib.contextmanager
def _stdout_to_stderr():
    """Route what native libraries print on file descriptor 1 (NCCL's version banner when a
    communicator is created) to stderr, so rank 0's stdout carries only the JSON line."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        yield
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def _dist_init(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        with _stdout_to_stderr():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
    else:
        torch.cuda.set_device(0)
    return rank, world


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------------------------
# clocks during the timed region
# ----------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap,utilization.gpu")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, busy_sm, mx, reasons = [], [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                clk = float(parts[0])
                mx = float(parts[1])
                util = float(parts[7])
            except ValueError:
                continue
            sm.append(clk)
            if util > 0:
                busy_sm.append(clk)
            for name, val in zip(names, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        use = busy_sm or sm
        return {"sm_mhz": statistics.median(use) if use else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "samples_busy": len(busy_sm)}


# ----------------------------------------------------------------------------------------------
# workload
# ----------------------------------------------------------------------------------------------
def _shard_sizes(world):
    """Per-rank sizes of the step under the decomposition of specq.sharding (the same for
    every rank: the ranges split evenly)."""
    from specq.sharding import shard_plan
    try:
        plan = shard_plan(world, 0, n_w8a8=W8["N"], n_w4a16=W4["N"], h_kv=AT["H_KV"], h=AT["H"])
    except ValueError as e:
        raise SystemExit(f"--gpus {world}: {e}")
    size = lambda s: s.stop - s.start  # noqa: E731
    return dict(n8=size(plan["w8a8_cols"]), n4=size(plan["w4a16_cols"]), h_kv=size(plan["kv_heads"]),
                h=size(plan["q_heads"]))


def _make_inputs(sh, seed, dev):
    """One copy of the step's inputs with the BASELINE value distributions, built on the device."""
    g = torch.Generator(device=dev).manual_seed(seed)

    def i8(shape):
        return torch.randint(-127, 128, shape, generator=g, device=dev, dtype=torch.int16).to(torch.int8)

    def uni(shape, lo, hi, dtype=torch.float32):
        return (torch.rand(shape, generator=g, device=dev) * (hi - lo) + lo).to(dtype)

    x = {}
    x["a8"], x["w8"] = i8((W8["M"], W8["K"])), i8((sh["n8"], W8["K"]))
    x["sa"], x["sw"] = uni((W8["M"],), 0.001, 0.02), uni((sh["n8"],), 0.001, 0.02)
    x["a4"] = torch.randn((W4["M"], W4["K"]), generator=g, device=dev).half()
    nib = torch.randint(0, 16, (sh["n4"], W4["K"]), generator=g, device=dev, dtype=torch.int16)
    x["wp"] = (nib[:, : W4["K"] // 2] | (nib[:, W4["K"] // 2:] << 4)).to(torch.uint8)
    x["sc"] = uni((sh["n4"], W4["K"] // W4["group"]), 0.005, 0.02, torch.float16)
    B, ctx, page, D, ql = AT["B"], AT["ctx"], AT["page"], AT["D"], AT["k"] + 1
    n_pages = B * ((ctx + page - 1) // page)
    x["kc"], x["vc"] = i8((n_pages, page, sh["h_kv"], D)), i8((n_pages, page, sh["h_kv"], D))
    x["ks"], x["vs"] = uni((n_pages, page, sh["h_kv"]), 0.005, 0.02), uni((n_pages, page, sh["h_kv"]), 0.005, 0.02)
    x["bt"] = torch.randperm(n_pages, generator=g, device=dev).to(torch.int32).view(B, -1)
    x["cl"] = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    x["q"] = torch.randn((B, ql, sh["h"], D), generator=g, device=dev).half()
    x["o8"] = torch.empty((W8["M"], sh["n8"]), device=dev, dtype=torch.float16)
    x["o4"] = torch.empty((W4["M"], sh["n4"]), device=dev, dtype=torch.float16)
    x["oa"] = torch.zeros_like(x["q"])
    return x


def _bytes(sh):
    """Algorithmic HBM bytes per launch of each kernel (each input read once, output written once)."""
    M, K, N = W8["M"], W8["K"], sh["n8"]
    b8 = M * K + N * K + 4 * M + 4 * N + 2 * M * N
    M4, K4, N4 = W4["M"], W4["K"], sh["n4"]
    b4 = N4 * K4 // 2 + N4 * (K4 // W4["group"]) * 2 + 2 * M4 * K4 + 2 * M4 * N4
    B, ctx, D, ql = AT["B"], AT["ctx"], AT["D"], AT["k"] + 1
    ba = (2 * B * ctx * sh["h_kv"] * D + 2 * B * ctx * sh["h_kv"] * 4 + 2 * (B * ql * sh["h"] * D * 2)
          + B * (ctx // AT["page"]) * 4 + 4 * B)
    return {"w8a8": b8, "w4a16": b4, "paged_attention": ba}


def _flops(sh):
    return {"w8a8": 2 * W8["M"] * sh["n8"] * W8["K"], "w4a16": 2 * W4["M"] * sh["n4"] * W4["K"],
            "paged_attention": 4 * AT["B"] * (AT["k"] + 1) * sh["h"] * AT["ctx"] * AT["D"]}


def _kernels(x):
    import specq
    ql = AT["k"] + 1
    return {
        "w8a8": lambda: specq.w8a8_matmul(x["a8"], x["sa"], x["w8"], x["sw"], out=x["o8"]),
        "w4a16": lambda: specq.w4a16_matmul(x["a4"], x["wp"], x["sc"], out=x["o4"]),
        "paged_attention": lambda: specq.paged_attention(x["q"], x["kc"], x["vc"], x["ks"], x["vs"], x["bt"], x["cl"],
                                                         ql, QPP=ql, out=x["oa"]),
    }


def _capture(fns):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for fn in fns:
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for fn in fns:
            fn()
    return g


# ----------------------------------------------------------------------------------------------
# CPU baseline: the reference's exact PyTorch path on host cores
# ----------------------------------------------------------------------------------------------
def _cpu_inputs(seed=0):
    g = torch.Generator().manual_seed(seed)
    from oracle import cpu_reference as R  # noqa: F401
    x = {}
    x["a8"] = torch.randint(-127, 128, (W8["M"], W8["K"]), generator=g, dtype=torch.int16).to(torch.int8)
    x["w8"] = torch.randint(-127, 128, (W8["N"], W8["K"]), generator=g, dtype=torch.int16).to(torch.int8)
    x["sa"] = torch.rand(W8["M"], generator=g) * 0.019 + 0.001
    x["sw"] = torch.rand(W8["N"], generator=g) * 0.019 + 0.001
    x["a4"] = torch.randn(W4["M"], W4["K"], generator=g).half()
    nib = torch.randint(0, 16, (W4["N"], W4["K"]), generator=g, dtype=torch.int16)
    x["wp"] = (nib[:, : W4["K"] // 2] | (nib[:, W4["K"] // 2:] << 4)).to(torch.uint8)
    x["sc"] = (torch.rand(W4["N"], W4["K"] // 128, generator=g) * 0.015 + 0.005).half()
    B, ctx, page, D, H_KV, H = AT["B"], AT["ctx"], AT["page"], AT["D"], AT["H_KV"], AT["H"]
    n_pages = B * ctx // page
    x["kc"] = torch.randint(-127, 128, (n_pages, page, H_KV, D), generator=g, dtype=torch.int16).to(torch.int8)
    x["vc"] = torch.randint(-127, 128, (n_pages, page, H_KV, D), generator=g, dtype=torch.int16).to(torch.int8)
    x["ks"] = torch.rand(n_pages, page, H_KV, generator=g) * 0.015 + 0.005
    x["vs"] = torch.rand(n_pages, page, H_KV, generator=g) * 0.015 + 0.005
    x["bt"] = torch.randperm(n_pages, generator=g).to(torch.int32).view(B, -1)
    x["cl"] = torch.full((B,), ctx, dtype=torch.int32)
    x["q"] = torch.randn(B, AT["k"] + 1, H, D, generator=g).half()
    return x


def _cpu_step(x, frac_seqs=1.0):
    """One verification step of the reference's exact path, in seconds, scaled to the full
    workload.  `frac_seqs` < 1 samples the attention over a prefix of the sequences (all have
    the same context, so its cost is linear in their number) and scales that part back."""
    from oracle import cpu_reference as R
    t0 = time.perf_counter()
    R.w8a8(x["a8"], x["sa"], x["w8"], x["sw"])
    R.w4a16(x["a4"], R.dequant_int4(x["wp"], x["sc"]))
    t1 = time.perf_counter()
    nb = max(1, int(round(AT["B"] * frac_seqs)))
    R.paged_attention(x["q"][:nb], x["kc"], x["vc"], x["ks"], x["vs"], x["bt"][:nb], x["cl"][:nb], AT["k"] + 1)
    t2 = time.perf_counter()
    return (t1 - t0) + (t2 - t1) * AT["B"] / nb


def _cpu_threads():
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_baseline(budget_s=12.0):
    """Time the reference path on a bounded sample: whole steps until `budget_s` is used."""
    cores = _cpu_threads()
    x = _cpu_inputs()
    _cpu_step(x)                      # warm-up (allocations, MKL init)
    t0 = time.perf_counter()
    n, total = 0, 0.0
    while True:
        total += _cpu_step(x)
        n += 1
        if time.perf_counter() - t0 > budget_s or n >= 50:
            break
    per = total / n
    return {"value": per * 1e6, "unit": "us", "cores": cores, "kind": "port",
            "sample": f"{n} full verification steps (W8A8 M=40 4096x4096, W4A16 M=72 14336x4096, "
                      f"attention B=8 ctx 4096 k=8) of the reference's exact PyTorch path on CPU"}


def _config(world):
    """The workload both arms report (the reference arm runs it on the host cores)."""
    return {
        "workload": ("verification step = W8A8 o_proj M=40 K=N=4096 (config 0) + W4A16 gate_proj M=72 "
                     "K=4096 N=14336 (config 1) + INT8 paged attention B=8 ctx=4096 k=8 QPP=9 H=32/8 "
                     "D=128 page 16 fp32 scales (config 2)"),
        "sharding": f"GEMM columns and attention KV heads split {world} ways" if world > 1 else "none",
        "l2": "rotating input copies > 2x L2 between timed steps (device arm)",
        "parallelism": f"dp{world}-shard" if world > 1 else "single-gpu",
    }


# ----------------------------------------------------------------------------------------------
# arms
# ----------------------------------------------------------------------------------------------
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = _cpu_threads()
    x = _cpu_inputs()
    one = _cpu_step(x)
    # bounded sample so that warmup + steps stay within ~3 minutes
    total = (args.warmup + args.steps) * one
    frac = 1.0 if total < 180 else max(1.0 / AT["B"], 180.0 / total)
    for _ in range(args.warmup):
        _cpu_step(x, frac)
    ts = [_cpu_step(x, frac) for _ in range(args.steps)]
    nb = max(1, int(round(AT["B"] * frac)))
    per_us = statistics.mean(ts) * 1e6
    sample = ("full verification step" if nb == AT["B"] else
              f"verification step with attention timed over {nb} of {AT['B']} sequences and scaled "
              f"to {AT['B']} (attention cost is linear in the sequences)")
    line = {"impl": "reference", "metric": _metric(), "value": per_us, "unit": "us", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_us / 1e3, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (reference PyTorch path)",
            "data": "synthetic",
            "config": _config(args.gpus),
            "cpu_baseline": {"value": per_us, "unit": "us", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": per_us, "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    rank, world = _dist_init(args.gpus)
    dev = torch.device("cuda", torch.cuda.current_device())
    import specq
    sh = _shard_sizes(world)
    bytes_per = _bytes(sh)
    copy_bytes = sum(v.numel() * v.element_size() for v in _make_inputs(sh, 0, dev).values())
    n_copies = max(2, math.ceil(2 * L2_BYTES / copy_bytes))
    inputs = [_make_inputs(sh, 1000 * rank + i, dev) for i in range(n_copies)]
    # The timed region is ONE replay of a graph that holds exactly `steps` consecutive steps
    # (inputs rotating over the copies): the host's launches do not pace the device and
    # consecutive kernels overlap their launch (programmatic dependent launch) as in a serving
    # loop.  The warm-up replays a graph of exactly `warmup` steps; the timed graph is replayed
    # once before that, untimed, so its upload to the device is not in the timed region.
    def _steps_graph(n):
        return _capture([f for i in range(n) for f in _kernels(inputs[i % n_copies]).values()])

    warm_steps = max(3, args.warmup)
    g_warm, g_timed = _steps_graph(warm_steps), _steps_graph(args.steps)
    chain_len = n_copies * max(1, 30 // n_copies)   # per-kernel chains below
    torch.cuda.synchronize()

    sampler = ClockSampler(dev.index)
    sampler.start()
    time.sleep(0.3)
    g_timed.replay()      # upload (untimed)
    g_warm.replay()       # warm-up steps
    torch.cuda.synchronize()
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    g_timed.replay()
    e1.record()
    torch.cuda.synchronize()
    _barrier(world)
    step_ms = _max_over_ranks(e0.elapsed_time(e1) / args.steps, world)

    # per-kernel launch durations (CUDA events around captured chains of chain_len launches of
    # one kernel over the rotating copies, like the step chains), for the roofline of each kernel
    per_kernel = {}
    for name in ("w8a8", "w4a16", "paged_attention"):
        g = _capture([_kernels(inputs[i % n_copies])[name] for i in range(chain_len)])
        g.replay()
        torch.cuda.synchronize()
        # long enough (~0.7 s) for the clock sampler to see the GPU under load
        reps = max(5, min(20000, int(700.0 / max(step_ms, 1e-3) / chain_len)))
        if args.per_kernel_reps:
            reps = args.per_kernel_reps
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        per_kernel[name] = _max_over_ranks(a.elapsed_time(b) * 1e3 / (reps * chain_len), world)   # us
        del g
    clocks = sampler.stop()

    # e2e: public API, pinned host inputs, H2D + 3 calls + D2H every step.  A step's inputs (the
    # activations, token scales and queries of its three calls) sit in one pinned host block and
    # land with one copy in one device block whose views are the tensors the calls take; the
    # three calls write their outputs into views of one device output block, which comes back
    # with one copy.  Consecutive steps rotate over three such buffer sets, each on its own
    # stream, so one step's result copy overlaps the next steps' input copies and kernels, as a
    # serving loop would pipeline them.
    in_keys, out_keys = ("a8", "sa", "a4", "q"), ("o8", "o4", "oa")

    def _stage(x, keys):
        offs, tot = [], 0
        for k in keys:
            offs.append(tot)
            tot += -(-x[k].numel() * x[k].element_size() // 256) * 256
        dev_blk = torch.empty(tot, dtype=torch.uint8, device=dev)
        host_blk = torch.empty(tot, dtype=torch.uint8).pin_memory()
        for k, o in zip(keys, offs):
            t = x[k].contiguous()
            nb = t.numel() * t.element_size()
            view = dev_blk[o:o + nb].view(t.dtype).view(t.shape)
            view.copy_(t)
            host_blk[o:o + nb].copy_(t.reshape(-1).view(torch.uint8).cpu())
            x[k] = view
        return host_blk, dev_blk

    def _buffer_set():
        x = dict(inputs[0])
        for o in out_keys:
            x[o] = torch.empty_like(x[o])
        h_in, d_in = _stage(x, in_keys)
        h_out, d_out = _stage(x, out_keys)
        return dict(h_in=h_in, d_in=d_in, h_out=h_out, d_out=d_out, fns=list(_kernels(x).values()),
                    stream=torch.cuda.Stream())

    sets = [_buffer_set() for _ in range(3)]
    h2d = sets[0]["h_in"].numel()
    d2h = sets[0]["d_out"].numel()

    def e2e_step(bs):
        torch.cuda.set_stream(bs["stream"])
        bs["d_in"].copy_(bs["h_in"], non_blocking=True)
        for f in bs["fns"]:
            f()
        bs["h_out"].copy_(bs["d_out"], non_blocking=True)

    def e2e_run(n):
        main = torch.cuda.current_stream()
        for bs in sets:
            bs["stream"].wait_stream(main)
        for i in range(n):
            e2e_step(sets[i % len(sets)])
        torch.cuda.set_stream(main)
        for bs in sets:
            main.wait_stream(bs["stream"])

    e2e_run(max(3, args.warmup))
    torch.cuda.synchronize()
    _barrier(world)
    n_e2e = max(20, min(args.steps, 200))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    e2e_run(n_e2e)
    b.record()
    torch.cuda.synchronize()
    e2e_us = _max_over_ranks(a.elapsed_time(b) * 1e3 / n_e2e, world)
    status = specq.get_status(clear=True)

    if world > 1:
        import torch.distributed as dist
        _barrier(world)
        del g_warm, g_timed
        dist.destroy_process_group()
    if rank != 0:
        return 0

    peaks, peaks_kind = _peaks()
    flops = _flops(sh)
    kern = {}
    for name, us in per_kernel.items():
        gbs = bytes_per[name] / (us * 1e-6) / 1e9
        entry = {"us": round(us, 3), "bytes": bytes_per[name], "gbs": round(gbs, 1),
                 "hbm_frac": round(gbs / peaks["hbm_gbs"], 4)}
        tflops = flops[name] / (us * 1e-6) / 1e12
        entry["tflops_or_tops"] = round(tflops, 1)
        if name == "w8a8":
            i8_burst, _, i8_src = _int8_peak()
            entry["int8_tensor_frac"] = round(tflops / i8_burst, 4)
            entry["int8_peak_tops"] = i8_burst
            entry["int8_peak_source"] = i8_src
        else:
            entry["fp16_tensor_frac"] = round(tflops / peaks["bf16_tflops"], 4)
        kern[name] = entry
    dom = max(per_kernel, key=per_kernel.get)
    ach = bytes_per[dom] / (per_kernel[dom] * 1e-6) / 1e9
    traffic = _traffic_from_profiles() if dom == "paged_attention" and world == 1 else None
    line = {
        "metric": _metric(),
        "value": round(step_ms * 1e3, 3),
        "unit": "us",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_ms,
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8 (W8A8, int32 accumulate) + fp16 (W4A16, attention; fp32 accumulate)",
        "data": "synthetic (BASELINE config value distributions, seeded, generated on device)",
        "config": _config(world),
        "timing": {"l2": f"{n_copies} rotating input copies of {copy_bytes / 1e6:.1f} MB (> 2x L2)",
                   "method": f"CUDA events around one replay of a captured graph of exactly {args.steps} steps "
                             f"(3 launches each, programmatic dependent launch), after {warm_steps} warm-up steps "
                             "from a graph of their own; per-kernel: events around replays of captured chains "
                             f"of {chain_len} launches of that kernel over the copies",
                   "e2e": "steps back to back through the public API: per step one H2D copy of the three "
                          "calls' inputs (one pinned block), the three calls, one D2H copy of their outputs "
                          "(one device block); consecutive steps rotate over three streams and buffer sets"},
        "kernels": kern,
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(ach / peaks["hbm_gbs"], 4), "traffic": traffic,
                     "peak_source": peaks_kind},
        "e2e": {"value": round(e2e_us, 3), "unit": "us", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": 3 * args.steps,
        "clocks": clocks,
        "device_status": status,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------------------------
# tensor-pipe peak (tcgen05 microbenchmark) and the GEMM sweep over the verification grid
# ----------------------------------------------------------------------------------------------
def run_mma_peak(args):
    """Dense tensor-pipe throughput of this GPU: kind::i8 (the INT8 peak the W8A8 large-M
    roofline needs) and kind::f16 (a cross-check against the measured cuBLAS bf16 figure), each
    as a burst (one launch of ~1 ms, best of 10) and sustained (back to back for ~3 s, clocks
    sampled).  One CTA per SM issues M=128 x N=256 MMAs from resident shared-memory tiles."""
    import specq
    from specq import _lib
    torch.cuda.set_device(0)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    sink = torch.zeros(sms, dtype=torch.int32, device="cuda")
    lib = _lib.load()
    res = {"sms": sms}
    for kind, name, k_per in ((0, "int8", 32), (1, "fp16", 16)):
        iters = 4096
        ops_per_launch = sms * iters * 4 * 2 * 128 * 256 * k_per

        def launch():
            _lib.check(lib.specq_mma_peak(kind, 256, 0, 0, 0, 0, 0, iters, sms, sink.data_ptr(),
                                          torch.cuda.current_stream().cuda_stream))

        for _ in range(3):
            launch()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(10):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            launch()
            b.record()
            torch.cuda.synchronize()
            best = min(best, a.elapsed_time(b))
        per = best / 1e3
        n_sus = max(10, int(3.0 / per))
        sampler = ClockSampler(0)
        sampler.start()
        time.sleep(0.3)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n_sus):
            launch()
        b.record()
        torch.cuda.synchronize()
        clocks = sampler.stop()
        sus = a.elapsed_time(b) / 1e3 / n_sus
        res[name] = {"burst_t": round(ops_per_launch / per / 1e12, 1), "sustained_t": round(ops_per_launch / sus / 1e12, 1),
                     "launch_ms_best": round(best, 4), "launches_sustained": n_sus, "clocks": clocks,
                     "unit": "TOPS" if kind == 0 else "TFLOP/s"}
    res["device_status"] = specq.get_status(clear=True)
    peaks, src = _peaks()
    res["cublas_bf16_tflops_measured"] = {"burst": peaks["bf16_tflops"], "sustained": peaks["bf16_tflops_sustained"],
                                          "source": src}
    print(json.dumps({"mma_peak": res}), flush=True)
    return 0


LINEAR_SET = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336)}
SWEEP_BS, SWEEP_KS = (1, 2, 4, 8, 16, 32), (0, 2, 4, 8)


def _sweep_time(fns, reps, chain=30):
    """Mean device time of one launch: a captured chain of at least `chain` launches rotating
    over `fns` (input copies together larger than L2), replayed `reps` times, CUDA events."""
    for f in fns:
        f()
    torch.cuda.synchronize()
    fns = [fns[i % len(fns)] for i in range(len(fns) * max(1, -(-chain // len(fns))))]
    g = _capture(fns)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / (reps * len(fns))


def run_sweep(args):
    """The GEMMs over the verification grid M = B*(k+1), B in {1,2,4,8,16,32}, k in {0,2,4,8}:
    W8A8 on the Llama-3-8B linear set with N sharded g ways (the per-GPU shard is timed, as each
    rank of `--gpus g` runs it; survey config 3) and W4A16 on gate_proj (config 1).  One JSON
    line: per point us, algorithmic GB/s and fraction of the measured HBM bandwidth, and the
    tensor throughput against the INT8 peak (measured when profiles/int8_mma_peak.md has it) or
    the measured FP16 burst peak."""
    import specq
    torch.cuda.set_device(0)
    dev = torch.device("cuda")
    peaks, _ = _peaks()
    i8_peak, _, i8_src = _int8_peak()
    gen = torch.Generator(device=dev).manual_seed(0)
    shards = tuple(int(x) for x in args.shards.split(","))
    reps = args.sweep_reps
    pts = []
    for g in shards:
        for name, (n_full, K) in LINEAR_SET.items():
            N = n_full // g
            copies = max(2, math.ceil(2 * L2_BYTES / (N * K)))
            ws = [torch.randint(-127, 128, (N, K), generator=gen, device=dev, dtype=torch.int16).to(torch.int8)
                  for _ in range(copies)]
            sws = [torch.rand(N, generator=gen, device=dev) * 0.019 + 0.001 for _ in range(copies)]
            for B in SWEEP_BS:
                for k in SWEEP_KS:
                    M = B * (k + 1)
                    a = torch.randint(-127, 128, (M, K), generator=gen, device=dev, dtype=torch.int16).to(torch.int8)
                    sa = torch.rand(M, generator=gen, device=dev) * 0.019 + 0.001
                    outs = [torch.empty(M, N, dtype=torch.float16, device=dev) for _ in range(copies)]
                    us = _sweep_time([lambda i=i: specq.w8a8_matmul(a, sa, ws[i], sws[i], out=outs[i])
                                      for i in range(copies)], reps)
                    nbytes = M * K + N * K + 4 * M + 4 * N + 2 * M * N
                    tops = 2.0 * M * N * K / us / 1e6
                    pts.append({"kernel": "w8a8", "shape": name, "shards": g, "N": N, "K": K, "B": B, "k": k, "M": M,
                                "us": round(us, 3), "gbs": round(nbytes / us / 1e3, 1),
                                "hbm_frac": round(nbytes / us / 1e3 / peaks["hbm_gbs"], 4), "tops": round(tops, 1),
                                "int8_frac": round(tops / i8_peak, 4)})
            del ws, sws
    N, K = 14336, 4096
    copies = max(2, math.ceil(2 * L2_BYTES / (N * K // 2)))
    wps = [torch.randint(0, 256, (N, K // 2), generator=gen, device=dev, dtype=torch.int32).to(torch.uint8)
           for _ in range(copies)]
    scs = [(torch.rand(N, K // 128, generator=gen, device=dev) * 0.015 + 0.005).half() for _ in range(copies)]
    for B in SWEEP_BS:
        for k in SWEEP_KS:
            M = B * (k + 1)
            x = torch.randn(M, K, generator=gen, device=dev).half()
            outs = [torch.empty(M, N, dtype=torch.float16, device=dev) for _ in range(copies)]
            us = _sweep_time([lambda i=i: specq.w4a16_matmul(x, wps[i], scs[i], out=outs[i]) for i in range(copies)],
                             reps)
            nbytes = N * K // 2 + 2 * N * K // 128 + 2 * M * K + 2 * M * N
            tf = 2.0 * M * N * K / us / 1e6
            pts.append({"kernel": "w4a16", "N": N, "K": K, "B": B, "k": k, "M": M, "us": round(us, 3),
                        "gbs": round(nbytes / us / 1e3, 1), "hbm_frac": round(nbytes / us / 1e3 / peaks["hbm_gbs"], 4),
                        "tflops": round(tf, 1), "fp16_frac": round(tf / peaks["bf16_tflops"], 4)})
    print(json.dumps({"sweep": pts, "hbm_gbs": peaks["hbm_gbs"], "int8_peak_tops": i8_peak, "int8_peak_source": i8_src,
                      "fp16_peak_tflops": peaks["bf16_tflops"], "status": specq.get_status(clear=True)}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--per-kernel-reps", type=int, default=0,
                    help="replays per kernel for the per-kernel durations (0: ~0.7 s each); small values "
                         "keep the launch count low for a profiler's launch list")
    ap.add_argument("--sweep", action="store_true",
                    help="time the GEMMs over the B x k verification grid (1 GPU) instead of the step")
    ap.add_argument("--shards", default="1,2,4,8", help="--sweep: N-shard counts of the W8A8 linear set")
    ap.add_argument("--sweep-reps", type=int, default=20)
    ap.add_argument("--mma-peak", action="store_true",
                    help="measure the dense tcgen05 INT8 / FP16 tensor-pipe peak (1 GPU) instead of the step")
    args = ap.parse_args()
    if args.mma_peak:
        return run_mma_peak(args)
    if args.sweep:
        return run_sweep(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

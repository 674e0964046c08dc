"""The three verification-shape operators, with the reference's Python signatures.

    w8a8_matmul(a_q, sa, w_q, sw, out=None, BLOCK_M=16, BLOCK_N=64, BLOCK_K=128,
                num_warps=4, num_stages=3, plan=None, grid_m_max=None) -> (out, ck)
    w4a16_matmul(a, wp, sc, group=128, out=None, BLOCK_M=16, BLOCK_N=64, BLOCK_K=64,
                 num_warps=4, num_stages=3, plan=None, grid_m_max=None) -> (out, ck)
    paged_attention(q, kc, vc, ks, vs, block_tbl, ctx_len, q_len, QPP=None, BLOCK_N=64,
                    num_warps=4, num_stages=2, plan=None, n_seqs=None, out=None) -> (out, ck)

(reference: kernels.py:71-86, kernels.py:150-166, kernels.py:239-262).  Each call validates
its tensors, then launches the sm_100a kernel through libspecq.so on
`torch.cuda.current_stream()`; nothing is synchronised or allocated beyond `out`, so the
calls can be captured in a CUDA graph.  The tile keyword arguments are scheduling hints of
the Triton original; the B200 kernels choose their own geometry (recorded in `ck`) and give
the same result for any value.  `ck` mirrors the compiled-kernel handle the reference
returns: `ck.n_regs`, `ck.n_spills`, `ck.metadata.shared` (read by regs.py:29-32).
"""
from __future__ import annotations

import ctypes as C
from types import SimpleNamespace

import torch

from . import _lib

# kernel ids of specq_kernel_info
W8A8, W4A16, PAGED_ATTN = 0, 1, 2


class KernelHandle:
    """What a launch used: variant, registers, local (spill) bytes, shared memory, grid.

    Built after every call from the raw launch record; the compiled-kernel attributes are
    looked up only when read, so the handle costs the caller almost nothing."""

    _NO_INFO = {"n_regs": 0, "local_bytes": 0, "static_smem": 0}

    def __init__(self, which: int, launch: tuple, hints: dict, device: int):
        self._which, self._launch, self._device = which, launch, device
        self.hints = hints

    def _info(self):
        # variant < 0: the call launched nothing (an empty problem)
        v = self._launch[0]
        return _kernel_info_cached(self._device, self._which, v) if v >= 0 else self._NO_INFO

    kernel = property(lambda self: ("w8a8", "w4a16", "paged_attention")[self._which])
    variant = property(lambda self: self._launch[0])
    grid = property(lambda self: tuple(self._launch[1:4]))
    cluster = property(lambda self: self._launch[4])
    num_warps = property(lambda self: self._launch[5] // 32)
    n_regs = property(lambda self: self._info()["n_regs"])
    n_spills = property(lambda self: self._info()["local_bytes"])

    @property
    def metadata(self):
        return SimpleNamespace(shared=self._info()["static_smem"] + self._launch[6], num_warps=self._launch[5] // 32)

    def __repr__(self):
        return (f"KernelHandle({self.kernel} v{self.variant}, grid={self.grid}, cluster={self.cluster}, "
                f"regs={self.n_regs}, spill_bytes={self.n_spills}, smem={self.metadata.shared})")


_info_cache: dict = {}


def _kernel_info_cached(device: int, which: int, variant: int) -> dict:
    key = (device, which, variant)
    if key not in _info_cache:
        with torch.cuda.device(device):
            _info_cache[key] = _lib.kernel_info(which, variant)
    return _info_cache[key]


class CompiledKernelRegistry:
    """Stands in for the reference's `_w8a8_kernel` / `_w4a16_kernel` JIT objects.

    correctness.py:18-24 counts compiled binaries through `device_caches` (or `cache`).  The
    B200 kernels are compiled ahead of time; the registry counts the distinct kernel variants
    this process has launched, per device, so the count means the same thing: how many
    binaries served the shapes seen so far.
    """

    def __init__(self, name: str):
        self.__name__ = name
        self.device_caches: dict = {}
        self.cache: dict = {}

    def record(self, variant: int, dev: int):
        entry = self.device_caches.setdefault(dev, ({},))
        entry[0][variant] = True
        self.cache.setdefault(dev, {})[variant] = True


_w8a8_kernel = CompiledKernelRegistry("_w8a8_kernel")
_w4a16_kernel = CompiledKernelRegistry("_w4a16_kernel")
_paged_attn_kernel = CompiledKernelRegistry("_paged_attn_kernel")


if hasattr(torch._C, "_cuda_getCurrentRawStream") and hasattr(torch._C, "_cuda_getDevice"):
    def _stream() -> int:
        """The current stream's cudaStream_t (without building a Stream object: ~0.3 us, not ~3)."""
        return torch._C._cuda_getCurrentRawStream(torch._C._cuda_getDevice())
else:
    def _stream() -> int:
        return torch.cuda.current_stream().cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("specq kernels take CUDA tensors (there is no CPU path)")


def _unit_inner(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def _plan_ptr(plan):
    if plan is None:
        return None
    if plan.dtype != torch.int32:
        raise TypeError(f"plan must be int32, got {plan.dtype}")
    _require_cuda(plan)
    return plan.data_ptr()


def _check_out(name: str, out, dtype, n_cols: int, n_rows: int):
    """A caller-supplied output must have the kernel's dtype, at least n_cols columns (and, without
    a plan, n_rows rows) and positive strides: the kernel writes through the pointer and strides,
    so a smaller buffer would be written past its end."""
    if out.dtype != dtype:
        raise TypeError(f"{name}: out must be {dtype}, got {out.dtype}")
    if out.dim() != 2 or out.shape[1] < n_cols or out.shape[0] < n_rows:
        raise ValueError(f"{name}: out must be 2-D with >= {n_rows} rows and >= {n_cols} columns, "
                         f"got {tuple(out.shape)}")
    if out.stride(0) < 1 or out.stride(1) < 1:
        raise ValueError(f"{name}: out strides {tuple(out.stride())} must be positive")


def _row_extent(n_rows: int, plan, grid_m_max, *tensors_rows) -> int:
    """Rows the kernel may touch: the tensor extent, or the plan grid's maximum."""
    if plan is None:
        return n_rows
    m = grid_m_max if grid_m_max is not None else n_rows
    return min([m, *tensors_rows])


# ----------------------------------------------------------------------------------------------
# W8A8  (kernels.py:71-86)
# ----------------------------------------------------------------------------------------------
def w8a8_matmul(a_q, sa, w_q, sw, out=None, BLOCK_M=16, BLOCK_N=64, BLOCK_K=128, num_warps=4, num_stages=3,
                plan=None, grid_m_max=None):
    M, K = a_q.shape
    N = w_q.shape[0]
    if w_q.shape[1] != K:
        raise ValueError(f"w8a8_matmul: a_q is [M, {K}] but w_q is {tuple(w_q.shape)}")
    if a_q.dtype != torch.int8 or w_q.dtype != torch.int8:
        raise TypeError("w8a8_matmul: a_q and w_q must be int8")
    if out is None:
        out = torch.empty((M, N), device=a_q.device, dtype=torch.float16)
    _check_out("w8a8_matmul", out, torch.float16, N, M if plan is None else 0)
    if sa.numel() < M or sw.numel() < N:
        raise ValueError(f"w8a8_matmul: scales have {sa.numel()} / {sw.numel()} entries for M={M}, N={N}")
    _require_cuda(a_q, sa, w_q, sw, out)
    a_q, w_q = _unit_inner(a_q), _unit_inner(w_q)
    sa = sa if sa.dtype == torch.float32 else sa.float()
    sw = sw if sw.dtype == torch.float32 else sw.float()
    sa, sw = sa.contiguous(), sw.contiguous()
    m_rows = _row_extent(M, plan, grid_m_max, M, out.shape[0], sa.shape[0])
    lib = _lib.load()
    _lib.check(lib.specq_w8a8(a_q.data_ptr(), a_q.stride(0), sa.data_ptr(), w_q.data_ptr(), w_q.stride(0),
                              sw.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1), _plan_ptr(plan),
                              m_rows, N, K, _stream()))
    launch = _lib.last_launch_raw()
    dev = a_q.device.index
    if launch[0] >= 0:
        _w8a8_kernel.record(launch[0], dev)
    ck = KernelHandle(W8A8, launch, dict(BLOCK_M=BLOCK_M, BLOCK_N=BLOCK_N, BLOCK_K=BLOCK_K, num_warps=num_warps,
                                         num_stages=num_stages), dev)
    return out, ck


def w8a8_accumulator(a_q, w_q, plan=None, grid_m_max=None, out=None):
    """Raw INT32 accumulator acc[m, n] = sum_k a_q[m,k] * w_q[n,k] from the same tensor-core
    kernel (the `acc` of kernels.py:44-50, before the scale epilogue)."""
    M, K = a_q.shape
    N = w_q.shape[0]
    if w_q.shape[1] != K:
        raise ValueError(f"w8a8_accumulator: a_q is [M, {K}] but w_q is {tuple(w_q.shape)}")
    if a_q.dtype != torch.int8 or w_q.dtype != torch.int8:
        raise TypeError("w8a8_accumulator: a_q and w_q must be int8")
    if out is None:
        out = torch.empty((M, N), device=a_q.device, dtype=torch.int32)
    _check_out("w8a8_accumulator", out, torch.int32, N, M if plan is None else 0)
    if out.stride(1) != 1:
        raise ValueError("w8a8_accumulator: out must have unit column stride")
    _require_cuda(a_q, w_q, out)
    a_q, w_q = _unit_inner(a_q), _unit_inner(w_q)
    m_rows = _row_extent(M, plan, grid_m_max, M, out.shape[0])
    lib = _lib.load()
    _lib.check(lib.specq_w8a8_acc(a_q.data_ptr(), a_q.stride(0), w_q.data_ptr(), w_q.stride(0), out.data_ptr(),
                                  out.stride(0), _plan_ptr(plan), m_rows, N, K, _stream()))
    return out


# ----------------------------------------------------------------------------------------------
# W4A16  (kernels.py:150-166)
# ----------------------------------------------------------------------------------------------
def w4a16_matmul(a, wp, sc, group=128, out=None, BLOCK_M=16, BLOCK_N=64, BLOCK_K=64, num_warps=4, num_stages=3,
                 plan=None, grid_m_max=None):
    M, K = a.shape
    N = wp.shape[0]
    assert BLOCK_K <= group and group % BLOCK_K == 0      # same contract as kernels.py:154
    if wp.shape[1] * 2 != K:
        raise ValueError(f"w4a16_matmul: a is [M, {K}] but wp is {tuple(wp.shape)} (expected [N, K/2])")
    if a.dtype != torch.float16:
        raise TypeError("w4a16_matmul: activations must be float16")
    if wp.dtype != torch.uint8:
        raise TypeError("w4a16_matmul: wp must be uint8")
    if out is None:
        out = torch.empty((M, N), device=a.device, dtype=torch.float16)
    _check_out("w4a16_matmul", out, torch.float16, N, M if plan is None else 0)
    n_groups = -(-K // group)
    if sc.dim() != 2 or sc.shape[0] < N or sc.shape[1] < n_groups:
        raise ValueError(f"w4a16_matmul: sc is {tuple(sc.shape)}, needs [>= {N}, >= {n_groups}] (ceil(K/group))")
    _require_cuda(a, wp, sc, out)
    sc = sc if sc.dtype == torch.float16 else sc.half()
    a, wp, sc = _unit_inner(a), _unit_inner(wp), _unit_inner(sc)
    if a.data_ptr() % 16 or (a.stride(0) * 2) % 16:
        a = a.contiguous() if (a.stride(0) * 2) % 16 == 0 else a.clone(memory_format=torch.contiguous_format)
    m_rows = _row_extent(M, plan, grid_m_max, M, out.shape[0])
    lib = _lib.load()
    _lib.check(lib.specq_w4a16(a.data_ptr(), a.stride(0), wp.data_ptr(), wp.stride(0), sc.data_ptr(), sc.stride(0),
                               group, out.data_ptr(), out.stride(0), out.stride(1), _plan_ptr(plan), m_rows, N, K,
                               _stream()))
    launch = _lib.last_launch_raw()
    dev = a.device.index
    if launch[0] >= 0:
        _w4a16_kernel.record(launch[0], dev)
    ck = KernelHandle(W4A16, launch, dict(BLOCK_M=BLOCK_M, BLOCK_N=BLOCK_N, BLOCK_K=BLOCK_K, num_warps=num_warps,
                                          num_stages=num_stages), dev)
    return out, ck


# ----------------------------------------------------------------------------------------------
# INT8 paged verification attention  (kernels.py:239-262)
# ----------------------------------------------------------------------------------------------
def paged_attention(q, kc, vc, ks, vs, block_tbl, ctx_len, q_len, QPP=None, BLOCK_N=64, num_warps=4, num_stages=2,
                    plan=None, n_seqs=None, out=None):
    B, QLMAX, H, D = q.shape
    H_KV = kc.shape[2]
    PAGE = kc.shape[1]
    if H % H_KV != 0:
        raise ValueError(f"paged_attention: H={H} is not a multiple of H_KV={H_KV}")
    if QPP is None:
        QPP = q_len
    if out is None:
        out = torch.zeros_like(q)
    n_seqs = B if n_seqs is None else n_seqs
    if q.dtype != torch.float16 or out.dtype != torch.float16:
        raise TypeError("paged_attention: q and out must be float16")
    if kc.dtype != torch.int8 or vc.dtype != torch.int8:
        raise TypeError("paged_attention: kc and vc must be int8")
    if ks.dtype not in (torch.float16, torch.float32) or vs.dtype != ks.dtype:
        raise TypeError("paged_attention: ks and vs must both be float16 or both float32")
    if block_tbl.dtype != torch.int32 or ctx_len.dtype != torch.int32:
        raise TypeError("paged_attention: block_tbl and ctx_len must be int32")
    _require_cuda(q, kc, vc, ks, vs, block_tbl, ctx_len, out)
    q, kc, vc, out_k = _unit_inner(q), _unit_inner(kc), _unit_inner(vc), out
    if kc.stride() != vc.stride():
        vc = vc.contiguous()
        kc = kc.contiguous()
    if ks.stride() != vs.stride():
        ks, vs = ks.contiguous(), vs.contiguous()
    if out.stride(-1) != 1:
        raise ValueError("paged_attention: out must have unit stride along D")
    scale_dtype = _lib.SPECQ_DTYPE_F16 if ks.dtype == torch.float16 else _lib.SPECQ_DTYPE_F32
    lib = _lib.load()
    _lib.check(lib.specq_paged_attention(
        q.data_ptr(), q.stride(0), q.stride(1), q.stride(2),
        kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1), kc.stride(2), kc.shape[0],
        ks.data_ptr(), vs.data_ptr(), ks.stride(0), ks.stride(1), ks.stride(2), scale_dtype,
        block_tbl.data_ptr(), block_tbl.stride(0), block_tbl.shape[1], ctx_len.data_ptr(),
        out_k.data_ptr(), out_k.stride(0), out_k.stride(1), out_k.stride(2),
        _plan_ptr(plan), B, n_seqs, q_len, QLMAX, H, H_KV, D, PAGE, QPP, _stream()))
    launch = _lib.last_launch_raw()
    dev = q.device.index
    if launch[0] >= 0:
        _paged_attn_kernel.record(launch[0], dev)
    ck = KernelHandle(PAGED_ATTN, launch, dict(QPP=QPP, BLOCK_N=BLOCK_N, num_warps=num_warps,
                                               num_stages=num_stages), dev)
    return out, ck


# ----------------------------------------------------------------------------------------------
# Verification-layer glue on the device: per-token INT8 quantisation, paged-KV append and
# attention over packed token rows.  No reference counterparts as kernels (the reference runs
# quantize_act_int8 as a torch function and builds its KV cache with a fixture).
# ----------------------------------------------------------------------------------------------
QUANT_PLAIN, QUANT_RESIDUAL, QUANT_SILU_MUL = 0, 1, 2


def quant_rows(x, mode=QUANT_PLAIN, residual=None, q=None, s=None, plan=None, grid_m_max=None, amax_in=None,
               amax_out=None, wait=None):
    """Per-token symmetric INT8 of fp16 rows on the device -> (q int8 [M, N], s fp32 [M]).

    mode QUANT_PLAIN: quantise x [M, N] (kernels.py:58-62 bit for bit).
    mode QUANT_RESIDUAL: residual <- fp16(x + residual), then quantise that sum.
    mode QUANT_SILU_MUL: quantise silu(x[:, :N]) * x[:, N:] for x [M, 2N].
    With `plan`, only the first plan[0] rows are computed (a plan-buffer graph).
    Rows split across GPUs: `amax_out` (fp32 [M]) receives each row's amax and nothing is
    quantised (returns None); `amax_in` quantises with the given whole-row amax.
    `wait` = (flags, rank, world): x is a full buffer that every rank's `specq_w8a8_peer` writes
    (specq.peer.PeerExchange.wait_args); each CTA first waits until all ranks' blocks landed."""
    if x.dtype != torch.float16 or x.dim() != 2:
        raise TypeError("quant_rows: x must be a 2-D float16 tensor")
    _require_cuda(x, residual, q, s)
    x = _unit_inner(x)
    M = x.shape[0]
    N = x.shape[1] // 2 if mode == QUANT_SILU_MUL else x.shape[1]
    if mode == QUANT_RESIDUAL:
        if residual is None or residual.shape != (M, N) or residual.dtype != torch.float16 or residual.stride(-1) != 1:
            raise ValueError("quant_rows: QUANT_RESIDUAL needs a float16 residual [M, N] with unit inner stride")
    for t, name in ((amax_in, "amax_in"), (amax_out, "amax_out")):
        if t is not None and (t.dtype != torch.float32 or t.dim() != 1 or t.shape[0] < M or not t.is_cuda):
            raise ValueError(f"quant_rows: {name} must be a CUDA float32 vector of >= {M} rows")
    lib = _lib.load()
    if amax_out is not None:
        m_rows = _row_extent(M, plan, grid_m_max, amax_out.shape[0])
        _lib.check(lib.specq_quant_rows(x.data_ptr(), x.stride(0), None, 0, None, 0, None, _plan_ptr(plan), None,
                                        amax_out.data_ptr(), m_rows, N, mode, _stream()))
        return None
    q = torch.empty((M, N), dtype=torch.int8, device=x.device) if q is None else q
    s = torch.empty((M,), dtype=torch.float32, device=x.device) if s is None else s
    m_rows = _row_extent(M, plan, grid_m_max, q.shape[0], s.shape[0])
    if wait is not None:
        flags, rank, world = wait
        _lib.check(lib.specq_quant_rows_peer(x.data_ptr(), x.stride(0), _ptr(residual),
                                             residual.stride(0) if residual is not None else 0, q.data_ptr(),
                                             q.stride(0), s.data_ptr(), _plan_ptr(plan), _ptr(amax_in), None, m_rows,
                                             N, mode, flags.data_ptr(), rank, world, _stream()))
        return q, s
    _lib.check(lib.specq_quant_rows(x.data_ptr(), x.stride(0), _ptr(residual),
                                    residual.stride(0) if residual is not None else 0, q.data_ptr(), q.stride(0),
                                    s.data_ptr(), _plan_ptr(plan), _ptr(amax_in), None, m_rows, N, mode,
                                    _stream()))
    return q, s


def kv_append(x, k_col, v_col, kc, vc, ks, vs, block_tbl, ctx_len, q_len, n_seqs=None, plan=None, B=None,
              ql_max=None):
    """Write the K/V of the q_len newest tokens of each sequence (packed rows of x, sequence b's
    token t at row b * q_len + t; K at columns k_col + h*D, V at v_col + h*D) into the INT8
    paged cache at positions ctx_len[b] - q_len + t (scales fp16, as the reference's cache)."""
    if x.dtype != torch.float16 or kc.dtype != torch.int8 or vc.dtype != torch.int8:
        raise TypeError("kv_append: x float16, kc/vc int8")
    if ks.dtype != torch.float16 or vs.dtype != torch.float16:
        raise TypeError("kv_append: the cache scales must be float16")
    _require_cuda(x, kc, vc, ks, vs, block_tbl, ctx_len)
    B = block_tbl.shape[0] if B is None else B
    n_seqs = B if n_seqs is None else n_seqs
    ql_max = q_len if ql_max is None else ql_max
    lib = _lib.load()
    _lib.check(lib.specq_kv_append(
        x.data_ptr(), x.stride(0), k_col, v_col, kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1),
        kc.stride(2), kc.shape[0], ks.data_ptr(), vs.data_ptr(), ks.stride(0), ks.stride(1), ks.stride(2),
        block_tbl.data_ptr(), block_tbl.stride(0), block_tbl.shape[1], ctx_len.data_ptr(), _plan_ptr(plan),
        B, n_seqs, q_len, ql_max, kc.shape[2], kc.shape[3], kc.shape[1], _stream()))


def paged_attention_packed(x, q_col, out, kc, vc, ks, vs, block_tbl, ctx_len, q_len, H, B=None, ql_max=None,
                           QPP=None, plan=None, n_seqs=None):
    """paged_attention with the queries read from, and the result written to, packed token rows:
    sequence b's token t is row b * q_len + t of x (heads at columns q_col + h*D) and of out
    (heads at columns h*D), for the active q_len (plan[1] under a plan-buffer graph)."""
    if x.dtype != torch.float16 or out.dtype != torch.float16:
        raise TypeError("paged_attention_packed: x and out must be float16")
    _require_cuda(x, out, kc, vc, ks, vs, block_tbl, ctx_len)
    H_KV, PAGE, D = kc.shape[2], kc.shape[1], kc.shape[3]
    B = block_tbl.shape[0] if B is None else B
    n_seqs = B if n_seqs is None else n_seqs
    ql_max = q_len if ql_max is None else ql_max
    QPP = ql_max if QPP is None else QPP
    scale_dtype = _lib.SPECQ_DTYPE_F16 if ks.dtype == torch.float16 else _lib.SPECQ_DTYPE_F32
    esz = x.element_size()
    lib = _lib.load()
    _lib.check(lib.specq_paged_attention(
        x.data_ptr() + q_col * esz, 0, x.stride(0), D,
        kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1), kc.stride(2), kc.shape[0],
        ks.data_ptr(), vs.data_ptr(), ks.stride(0), ks.stride(1), ks.stride(2), scale_dtype,
        block_tbl.data_ptr(), block_tbl.stride(0), block_tbl.shape[1], ctx_len.data_ptr(),
        out.data_ptr(), 0, out.stride(0), D,
        _plan_ptr(plan), B, n_seqs, q_len, ql_max, H, H_KV, D, PAGE, QPP, _stream()))
    return out


_W_DTYPES = {torch.float16: 0, torch.float32: 1, torch.bfloat16: 2}


def pack_int4(w, group=128, deq=True):
    """Group-wise INT4 quantisation and split-half packing of w [N, K] on the device
    (kernels.py:138-147, bit-exact with the reference's torch function on a CUDA tensor).

    Returns (packed uint8 [N, K/2], scales fp16 [N, K/group], dequantised fp16 [N, K] or None
    when deq=False)."""
    if w.dim() != 2 or w.dtype not in _W_DTYPES:
        raise TypeError("pack_int4: w must be a 2-D float16 / float32 / bfloat16 tensor")
    _require_cuda(w)
    w = _unit_inner(w)
    N, K = w.shape
    if K % 2 or (K // 2) % group:
        raise ValueError(f"pack_int4: K={K} needs K % 2 == 0 and (K/2) % group == 0 (group {group})")
    wp = torch.empty((N, K // 2), dtype=torch.uint8, device=w.device)
    sc = torch.empty((N, K // group), dtype=torch.float16, device=w.device)
    dq = torch.empty((N, K), dtype=torch.float16, device=w.device) if deq else None
    lib = _lib.load()
    _lib.check(lib.specq_pack_int4(w.data_ptr(), _W_DTYPES[w.dtype], w.stride(0), N, K, group, wp.data_ptr(),
                                   wp.stride(0), sc.data_ptr(), sc.stride(0), _ptr(dq),
                                   dq.stride(0) if dq is not None else 0, _stream()))
    return wp, sc, dq

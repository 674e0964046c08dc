"""Peer-store all-gather for the tensor-parallel stack (no reference counterpart: the reference
runs on one GPU).

`PeerExchange` owns, for each named exchange, a "full" buffer [rows, world * slice] in
symmetric memory (every rank's copy mapped into every rank's address space through
torch.distributed's symmetric-memory rendezvous), a symmetric flag array [world] and a local
[2] state word.  `gather(name, local, rows)` launches `specq_peer_gather`: one kernel that writes
this rank's [rows, slice] block straight into its column range of every rank's full buffer over
NVLink (plain peer stores; no NCCL kernel, no re-layout copy) and returns once every peer's
block has landed in this rank's copy.  `all_max(name, local, out, rows)` does the same for one
float per row and reduces the gathered row to its maximum (the per-token amax of a row-split
activation).

Every rank must call the exchanges in the same order; calls are stream-ordered and may be
captured in a CUDA graph (the epochs live on the device).
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib


class PeerExchange:
    def __init__(self, group=None, device=None):
        import torch.distributed._symmetric_memory as symm_mem

        self._symm = symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        if self.world > 8:
            raise ValueError("peer exchange: at most 8 ranks")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self._ex = {}

    def _symmetric(self, shape, dtype):
        if hasattr(self._symm, "enable_symm_mem_for_group") and not self._symm.is_symm_mem_enabled_for_group(
                self.group.group_name):
            self._symm.enable_symm_mem_for_group(self.group.group_name)
        t = self._symm.empty(*shape, dtype=dtype, device=self.device)
        hdl = self._symm.rendezvous(t, self.group)
        base = hdl.buffer_ptrs[self.rank]
        off = t.data_ptr() - base
        nbytes = t.numel() * t.element_size()
        # a peer's copy of this tensor sits at the same offset in that peer's buffer: every rank
        # must have allocated it there, inside the mapped range
        offs = [None] * self.world
        dist.all_gather_object(offs, (off, int(hdl.buffer_size)), group=self.group)
        if any(o != offs[0][0] or o < 0 or o + nbytes > size for o, size in offs):
            raise RuntimeError(f"peer exchange: symmetric tensors at different offsets {offs}")
        return t, [int(p) + off for p in hdl.buffer_ptrs], hdl

    def add(self, name: str, rows: int, slice_cols: int, dtype) -> torch.Tensor:
        """Register exchange `name`: returns this rank's full buffer [rows, world * slice_cols]."""
        full, ptrs, h1 = self._symmetric((rows, self.world * slice_cols), dtype)
        flags, fptrs, h2 = self._symmetric((self.world,), torch.int32)
        flags.zero_()
        state = torch.zeros(2, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)   # every rank's flags are zero before any signal
        esz = full.element_size()
        self._ex[name] = dict(full=full, flags=flags, state=state, handles=(h1, h2), esz=esz, cols=slice_cols,
                              dst=(C.c_void_p * self.world)(*ptrs), fl=(C.c_void_p * self.world)(*fptrs))
        return full

    def gather(self, name: str, local: torch.Tensor, rows: int, plan=None, max_out=None) -> torch.Tensor:
        """Gather this rank's block local[:rows] ([rows, slice], unit inner stride) into column
        block `rank` of every rank's full buffer; returns this rank's full buffer."""
        e = self._ex[name]
        if local.dtype != e["full"].dtype or local.shape[1] != e["cols"] or local.stride(1) != 1:
            raise ValueError(f"peer exchange {name}: block {tuple(local.shape)} {local.dtype} does not fit")
        if rows > e["full"].shape[0] or rows > local.shape[0]:
            raise ValueError(f"peer exchange {name}: {rows} rows")
        esz, cols = e["esz"], e["cols"]
        lib = _lib.load()
        _lib.check(lib.specq_peer_gather(
            local.data_ptr(), local.stride(0) * esz, cols * esz, None if plan is None else plan.data_ptr(), rows,
            e["dst"], e["full"].stride(0) * esz, self.rank * cols * esz, e["fl"], e["state"].data_ptr(),
            None if max_out is None else max_out.data_ptr(), self.rank, self.world,
            torch.cuda.current_stream().cuda_stream))
        return e["full"]

    def w8a8(self, name: str, a_q, sa, w_q, sw, rows: int, plan=None) -> torch.Tensor:
        """W8A8 GEMM (this rank's [N_local, K] weight shard) whose output block lands straight in
        column block `rank` of every rank's full buffer of exchange `name` (`specq_w8a8_peer`: the
        GEMM's epilogue stores over NVLink, then counts its CTAs into every rank's flags); a
        consumer of the full buffer waits with `wait_args(name)`.  `rows` is the launch's row
        extent (with a plan, the maximum; plan[0] the active rows).  Returns the full buffer."""
        e = self._ex[name]
        M, K = a_q.shape
        N = w_q.shape[0]
        if N != e["cols"] or e["full"].dtype != torch.float16:
            raise ValueError(f"peer exchange {name}: a [{N}]-column fp16 block does not fit")
        if rows > e["full"].shape[0] or rows > M or a_q.stride(1) != 1 or w_q.stride(1) != 1:
            raise ValueError(f"peer exchange {name}: {rows} rows / strides")
        outs = e.get("outs")
        if outs is None:
            off = self.rank * e["cols"] * e["esz"]
            outs = e["outs"] = (C.c_void_p * self.world)(*[p + off for p in e["dst"]])
        lib = _lib.load()
        _lib.check(lib.specq_w8a8_peer(
            a_q.data_ptr(), a_q.stride(0), sa.data_ptr(), w_q.data_ptr(), w_q.stride(0), sw.data_ptr(), outs,
            e["full"].stride(0), None if plan is None else plan.data_ptr(), rows, N, K, e["fl"], self.rank,
            self.world, torch.cuda.current_stream().cuda_stream))
        return e["full"]

    def wait_args(self, name: str) -> tuple:
        """(flags, rank, world) for `ops.quant_rows(..., wait=...)` on exchange `name`'s full buffer."""
        return (self._ex[name]["flags"], self.rank, self.world)

    def all_max(self, name: str, local: torch.Tensor, out: torch.Tensor, rows: int, plan=None) -> torch.Tensor:
        """out[:rows] <- the maximum over the ranks of local[:rows] (float32 [rows])."""
        if local.dtype != torch.float32 or out.dtype != torch.float32 or not local.is_contiguous():
            raise ValueError("peer exchange all_max: contiguous float32 rows")
        self.gather(name, local.view(-1, 1), rows, plan=plan, max_out=out)
        return out

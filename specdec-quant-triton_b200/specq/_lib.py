"""ctypes binding of libspecq.so (the C ABI declared in include/specq.h).

The library is built in-tree by `specdec-quant-triton_b200/build.py`.  Importing this module
fails loudly when it is missing: there is no CPU or Triton fallback for any kernel.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

# SPECQ_LIB selects another build of the same ABI (e.g. libspecq_trace.so, built with
# `build.py --trace`, whose kernels record pipeline timestamps).
LIB_PATH = os.environ.get("SPECQ_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)), "libspecq.so")

SPECQ_OK = 0
SPECQ_ERR_INVALID_ARG = 1
SPECQ_ERR_UNSUPPORTED = 2
SPECQ_ERR_CUDA = 3
SPECQ_ERR_NO_DEVICE = 4

SPECQ_STATUS_TIMEOUT_PIPELINE = 0x01
SPECQ_STATUS_TIMEOUT_MMA = 0x02
SPECQ_STATUS_TIMEOUT_TEST = 0x04
SPECQ_STATUS_TIMEOUT_PEER = 0x08
SPECQ_STATUS_PLAN_CLAMPED = 0x100

SPECQ_DTYPE_F16 = 0
SPECQ_DTYPE_F32 = 1

_i32, _i64, _u64, _vp = C.c_int, C.c_int64, C.c_uint64, C.c_void_p
_pi32 = C.POINTER(C.c_int)

# name -> (restype, argtypes); must match include/specq.h exactly (a CPU test checks it)
SIGNATURES = {
    "specq_version": (_i32, []),
    "specq_last_error": (C.c_char_p, []),
    "specq_w8a8": (_i32, [_vp, _i64, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _vp, _i32, _i32, _i32, _vp]),
    "specq_w8a8_acc": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _i32, _i32, _i32, _vp]),
    "specq_w4a16": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _vp, _i64, _i64, _vp, _i32, _i32, _i32, _vp]),
    "specq_quant_rows": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "specq_kv_append": (_i32, [_vp, _i64, _i32, _i32, _vp, _vp, _i64, _i64, _i64, _i32, _vp, _vp, _i64, _i64, _i64,
                               _vp, _i64, _i32, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp]),
    "specq_paged_attention": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i32, _vp, _vp, _i64, _i64,
                                     _i64, _i32, _vp, _i64, _i32, _vp, _vp, _i64, _i64, _i64, _vp, _i32, _i32, _i32,
                                     _i32, _i32, _i32, _i32, _i32, _i32, _vp]),
    "specq_pack_int4": (_i32, [_vp, _i32, _i64, _i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp, _i64, _vp]),
    "specq_kernel_info": (_i32, [_i32, _i32, _pi32, _pi32, _pi32, _pi32, _pi32]),
    "specq_last_launch": (_i32, [_pi32, _pi32, _pi32, _pi32, _pi32, _pi32, _pi32]),
    "specq_last_launch_packed": (_i32, [_vp]),
    "specq_get_status": (_i32, [_pi32, _i32]),
    "specq_selftest_wait_timeout": (_i32, [_u64, _vp]),
    "specq_mma_peak": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp]),
    "specq_peer_gather": (_i32, [_vp, _i64, _i32, _vp, _i32, _vp, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _vp]),
    "specq_peer_gather_noalloc": (_i32, [_vp, _i64, _i32, _vp, _i32, _vp, _i64, _i64, _vp, _i32, _i32, _vp, _i32,
                                         _i32, _vp]),
    "specq_w8a8_peer": (_i32, [_vp, _i64, _vp, _vp, _i64, _vp, _vp, _i64, _vp, _i32, _i32, _i32, _vp, _i32, _i32,
                               _vp]),
    "specq_quant_rows_peer": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp,
                                     _i32, _i32, _vp]),
    "specq_trace_configure": (_i32, [_vp, _i32]),
}

_lock = threading.Lock()
_lib = None


class SpecqError(RuntimeError):
    """A libspecq call returned an error code."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"libspecq error {code}: {msg}")
        self.code = code


def load():
    """Load libspecq.so once and declare every entry point's signature."""
    global _lib
    if _lib is not None:   # loaded: no lock on the per-call path
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"libspecq.so not found at {LIB_PATH}; build it with "
                    "`python specdec-quant-triton_b200/build.py` (there is no fallback path)")
            lib = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int):
    if rc != SPECQ_OK:
        msg = load().specq_last_error().decode(errors="replace")
        if rc == SPECQ_ERR_INVALID_ARG:
            raise ValueError(f"libspecq: {msg}")
        raise SpecqError(rc, msg)


def get_status(clear: bool = True) -> int:
    """Read (and by default clear) the device status word of the current device."""
    v = C.c_int(0)
    check(load().specq_get_status(C.byref(v), 1 if clear else 0))
    return v.value


_launch_buf = threading.local()


def last_launch_raw() -> tuple:
    """(variant, grid x, y, z, cluster, threads, dynamic smem) of this thread's last launch, read
    in one call into a buffer allocated once per thread (it runs after every operator call)."""
    b = getattr(_launch_buf, "b", None)
    if b is None:
        b = _launch_buf.b = (C.c_int * 7)()
    (_lib or load()).specq_last_launch_packed(b)
    return tuple(b)


def last_launch() -> dict:
    variant, gx, gy, gz, cx, threads, smem = last_launch_raw()
    return {"variant": variant, "grid": (gx, gy, gz), "cluster": cx, "threads": threads, "dynamic_smem": smem}


def kernel_info(which: int, variant: int) -> dict:
    vals = [C.c_int(0) for _ in range(5)]
    check(load().specq_kernel_info(which, variant, *[C.byref(v) for v in vals]))
    regs, local, static_smem, dyn, max_threads = (v.value for v in vals)
    return {"n_regs": regs, "local_bytes": local, "static_smem": static_smem, "max_dynamic_smem": dyn,
            "max_threads": max_threads}

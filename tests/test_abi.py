"""CPU: the C-ABI library loads without a GPU, exports every symbol include/specq.h declares,
its ctypes signatures agree with the header, and host-side checks reject bad calls before
any device work (no compute call is made here)."""
import ctypes as C
import os
import re

import pytest
import torch

from conftest import REPO

HEADER = os.path.join(REPO, "include", "specq.h")


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    decls = {}
    for m in re.finditer(r"(?:int|const char\*)\s+(specq_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.S):
        args = [a.strip() for a in m.group(2).split(",") if a.strip() and a.strip() != "void"]
        decls[m.group(1)] = len(args)
    return decls


def test_header_declares_the_entry_points():
    decls = _declared_functions()
    for name in ("specq_w8a8", "specq_w4a16", "specq_paged_attention", "specq_kernel_info", "specq_get_status"):
        assert name in decls


def test_library_exports_every_declared_symbol():
    from specq import _lib
    lib = _lib.load()
    for name in _declared_functions():
        assert hasattr(lib, name), name


def test_ctypes_signatures_match_header():
    from specq import _lib
    decls = _declared_functions()
    assert set(decls) == set(_lib.SIGNATURES), set(decls) ^ set(_lib.SIGNATURES)
    for name, nargs in decls.items():
        assert len(_lib.SIGNATURES[name][1]) == nargs, name


def test_library_has_no_driver_link_dependency():
    # libcuda is reached through cudaGetDriverEntryPoint, so the .so loads on a CPU-only host
    from specq import _lib
    maps = open("/proc/self/maps").read() if os.path.exists("/proc/self/maps") else ""
    _lib.load()
    assert os.path.exists(_lib.LIB_PATH)
    assert "libcuda.so" not in maps or torch.cuda.is_available()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_no_device_is_reported_not_crashed():
    from specq import _lib
    lib = _lib.load()
    v = C.c_int(0)
    assert lib.specq_get_status(C.byref(v), 0) == _lib.SPECQ_ERR_NO_DEVICE
    assert b"device" in lib.specq_last_error()


def test_invalid_shapes_rejected_on_host():
    from specq import _lib
    lib = _lib.load()
    rc = lib.specq_w8a8(None, 0, None, None, 0, None, None, 0, 1, None, -1, 16, 16, None)
    assert rc == _lib.SPECQ_ERR_INVALID_ARG
    rc = lib.specq_w8a8(1, 8, 1, 1, 8, 1, 1, 16, 1, None, 4, 16, 16, None)      # lda < K
    assert rc == _lib.SPECQ_ERR_INVALID_ARG
    rc = lib.specq_w4a16(16, 100, 16, 50, 16, 1, 128, 16, 16, 1, None, 4, 16, 100, None)  # K/2 % 64
    assert rc == _lib.SPECQ_ERR_UNSUPPORTED
    rc = lib.specq_w4a16(16, 101, 16, 50, 16, 1, 128, 16, 16, 1, None, 4, 16, 101, None)  # odd K
    assert rc == _lib.SPECQ_ERR_INVALID_ARG


def test_peer_gather_arguments_rejected_on_host():
    from specq import _lib
    lib = _lib.load()
    ptrs = (C.c_void_p * 2)(16, 32)
    ok = dict(src=16, ld_src=64, row_bytes=64, plan=None, rows=4, dst=ptrs, ld_dst=128, dst_off=0, flags=ptrs,
              state=16, max_out=None, rank=0, world=2, stream=None)

    def call(**kw):
        a = dict(ok, **kw)
        return lib.specq_peer_gather(a["src"], a["ld_src"], a["row_bytes"], a["plan"], a["rows"], a["dst"],
                                     a["ld_dst"], a["dst_off"], a["flags"], a["state"], a["max_out"], a["rank"],
                                     a["world"], a["stream"])

    assert call(world=9) == _lib.SPECQ_ERR_INVALID_ARG          # more ranks than the kernel holds
    assert call(rank=2) == _lib.SPECQ_ERR_INVALID_ARG
    assert call(row_bytes=6) == _lib.SPECQ_ERR_INVALID_ARG      # not a multiple of 4
    assert call(dst_off=96) == _lib.SPECQ_ERR_INVALID_ARG       # block past the full row
    assert call(state=None) == _lib.SPECQ_ERR_INVALID_ARG
    assert call(max_out=16) == _lib.SPECQ_ERR_INVALID_ARG       # max mode takes one float per rank


def test_python_wrappers_reject_cpu_tensors():
    import specq
    a = torch.zeros(4, 128, dtype=torch.int8)
    w = torch.zeros(8, 128, dtype=torch.int8)
    s4, s8 = torch.ones(4), torch.ones(8)
    with pytest.raises(ValueError, match="CUDA"):
        specq.w8a8_matmul(a, s4, w, s8, out=torch.empty(4, 8, dtype=torch.float16))
    with pytest.raises(TypeError):
        specq.w8a8_matmul(a.float(), s4, w, s8)


def test_w4a16_block_k_contract_kept():
    import specq
    x = torch.zeros(2, 256, dtype=torch.float16)
    wp = torch.zeros(8, 128, dtype=torch.uint8)
    sc = torch.ones(8, 2, dtype=torch.float16)
    with pytest.raises(AssertionError):                     # kernels.py:154
        specq.w4a16_matmul(x, wp, sc, group=128, BLOCK_K=256)


def test_drop_in_module_exports_reference_names():
    import kernels
    for name in ("w8a8_matmul", "w4a16_matmul", "paged_attention", "quantize_act_int8", "quantize_weight_int8",
                 "quantize_weight_int4", "make_paged_kv", "paged_attention_ref", "_w8a8_kernel", "_w4a16_kernel"):
        assert hasattr(kernels, name), name
    assert kernels._w8a8_kernel.device_caches == {} or isinstance(kernels._w8a8_kernel.device_caches, dict)


def test_kernel_handle_reads_the_launch_record():
    """The `ck` handle each operator returns carries what regs.py reads (n_regs, n_spills,
    metadata.shared) and the launch geometry; a call that launched nothing (variant -1) needs
    no kernel lookup."""
    from specq.ops import KernelHandle, W8A8
    ck = KernelHandle(W8A8, (-1, 4, 2, 32, 4, 192, 1024), {"BLOCK_M": 16}, 0)
    assert ck.kernel == "w8a8" and ck.variant == -1
    assert ck.grid == (4, 2, 32) and ck.cluster == 4 and ck.num_warps == 6
    assert ck.n_regs == 0 and ck.n_spills == 0
    assert ck.metadata.shared == 1024 and ck.metadata.num_warps == 6
    assert ck.hints == {"BLOCK_M": 16}
    assert "w8a8" in repr(ck)


def test_output_buffers_checked_before_launch():
    """A caller-supplied `out` that the kernel would write past the end of is rejected on the
    host: wrong dtype, too few columns or rows, non-positive strides (the C ABI rejects
    non-positive output strides and an accumulator row stride below N as well)."""
    import specq
    from specq import _lib
    a = torch.zeros(4, 128, dtype=torch.int8)
    w = torch.zeros(8, 128, dtype=torch.int8)
    s4, s8 = torch.ones(4), torch.ones(8)
    with pytest.raises(ValueError, match="columns"):
        specq.w8a8_matmul(a, s4, w, s8, out=torch.empty(4, 7, dtype=torch.float16))
    with pytest.raises(ValueError, match="rows"):
        specq.w8a8_matmul(a, s4, w, s8, out=torch.empty(3, 8, dtype=torch.float16))
    with pytest.raises(TypeError):
        specq.w8a8_accumulator(a, w, out=torch.empty(4, 8, dtype=torch.float32))
    with pytest.raises(ValueError, match="columns"):
        specq.w8a8_accumulator(a, w, out=torch.empty(4, 6, dtype=torch.int32))
    with pytest.raises(ValueError, match="entries"):
        specq.w8a8_matmul(a, torch.ones(3), w, s8)
    x = torch.zeros(2, 256, dtype=torch.float16)
    wp = torch.zeros(8, 128, dtype=torch.uint8)
    with pytest.raises(ValueError, match="columns"):
        specq.w4a16_matmul(x, wp, torch.ones(8, 2, dtype=torch.float16), out=torch.empty(2, 4, dtype=torch.float16))
    with pytest.raises(ValueError, match="ceil"):          # 256 / 96 -> 3 scale columns needed
        specq.w4a16_matmul(x, wp, torch.ones(8, 2, dtype=torch.float16), group=96, BLOCK_K=32)
    lib = _lib.load()
    rc = lib.specq_w8a8_acc(16, 128, 16, 128, 16, 7, None, 4, 8, 128, None)           # ldacc < N
    assert rc == _lib.SPECQ_ERR_INVALID_ARG
    rc = lib.specq_w8a8(16, 128, 16, 16, 128, 16, 16, 0, 1, None, 4, 8, 128, None)    # ldo = 0
    assert rc == _lib.SPECQ_ERR_INVALID_ARG
    rc = lib.specq_w4a16(16, 256, 16, 128, 16, 2, 128, 16, 8, -1, None, 2, 8, 256, None)  # ldo_n < 0
    assert rc == _lib.SPECQ_ERR_INVALID_ARG

"""CPU: pin the timed CPU baseline (oracle/cpu_reference.py, the reference's exact PyTorch path
as bench.py times it) to the reference's own outputs in tests/golden/.

W8A8 at these sizes keeps every fp32 partial sum below 2**24, so the port's fp32 matmul is exact
and must match the reference's PyTorch oracle (correctness.py:37) and its Triton kernel bit for
bit.  W4A16 and attention compare within the fp32-summation / fp16-output tolerances stated
beside each check.
"""
import numpy as np
import pytest
import torch

from oracle import cpu_reference as R
from oracle import specq_oracle as O


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


@pytest.mark.parametrize("name", ["w8a8_small", "w8a8_ragged", "w8a8_m1"])
def test_port_w8a8_bit_exact_with_reference(golden, name):
    g = golden(name)
    out = R.w8a8(_t(g["a_q"]), _t(g["sa"]), _t(g["w_q"]), _t(g["sw"])).numpy()
    assert np.array_equal(out.view(np.uint16), g["ref"].astype(np.float16).view(np.uint16))
    assert np.array_equal(out.view(np.uint16), g["out"].view(np.uint16))   # the Triton kernel's output


def test_port_w8a8_plan_rows(golden):
    g = golden("w8a8_plan")
    M = int(g["plan"][0])
    out = R.w8a8(_t(g["a_q"][:M]), _t(g["sa"][:M]), _t(g["w_q"]), _t(g["sw"])).numpy()
    assert np.array_equal(out.view(np.uint16), g["out"][:M].view(np.uint16))


@pytest.mark.parametrize("name", ["w4a16_small", "w4a16_mid"])
def test_port_w4a16_matches_reference(golden, name):
    g = golden(name)
    x, wp, sc = _t(g["x"]), _t(g["wp"]), _t(g["sc"])
    # the reference's own oracle: x.float() @ deq.float().T with its fp32-scale deq (correctness.py:76)
    ref_port = R.w4a16(x, _t(g["deq"])).float().numpy()
    assert O.rel_fro_err(ref_port, g["ref"]) < 1e-3          # fp16 output rounding only
    # the kernel-semantics dequantisation (fp16 scale, one rounding) equals the oracle's, bit for bit
    deq_k = R.dequant_int4(wp, sc).numpy()
    assert np.array_equal(deq_k.view(np.uint16), O.dequant_int4_kernel(g["wp"], g["sc"], 128).view(np.uint16))
    # and with it the port reproduces the reference Triton kernel's output
    out = R.w4a16(x, R.dequant_int4(wp, sc)).numpy()
    assert O.rel_fro_err(out, g["out"]) < 1e-3                 # fp32 summation order differs


@pytest.mark.parametrize("name", ["attn_small", "attn_f32scales"])
def test_port_attention_matches_reference(golden, name):
    g = golden(name)
    ql = int(g["q_len"])
    t = {k: _t(g[k]) for k in ("q", "kc", "vc", "ks", "vs", "bt", "cl")}
    out = R.paged_attention(t["q"], t["kc"], t["vc"], t["ks"], t["vs"], t["bt"], t["cl"], ql).numpy()
    # the reference's paged_attention_ref (kernels.py:289-309): same fp32 formula, fp16 output
    assert O.max_abs_err(out[:, :ql], g["ref"][:, :ql]) <= 2 ** -10
    assert O.max_abs_err(out, g["out_fused"]) < 2e-2          # the Triton kernel, correctness.py:100


def test_port_attention_plan_rows(golden):
    g = golden("attn_plan")
    b_act, ql = int(g["plan"][0]), int(g["plan"][1])
    t = {k: _t(g[k]) for k in ("q", "kc", "vc", "ks", "vs", "bt", "cl")}
    out = R.paged_attention(t["q"][:b_act], t["kc"], t["vc"], t["ks"], t["vs"], t["bt"][:b_act], t["cl"][:b_act],
                            ql).numpy()
    assert O.max_abs_err(out[:, :ql], g["ref"][:, :ql]) <= 2 ** -10


def test_port_catches_a_planted_scale_mistake(golden):
    """A port that forgot the per-channel weight scale is caught by the bit-exact W8A8 check."""
    g = golden("w8a8_small")
    out = R.w8a8(_t(g["a_q"]), _t(g["sa"]), _t(g["w_q"]), torch.ones_like(_t(g["sw"]))).numpy()
    assert not np.array_equal(out.view(np.uint16), g["out"].view(np.uint16))

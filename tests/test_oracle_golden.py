"""CPU: pin the oracle (and the package's reference-API helpers) to the reference's own outputs.

The golden vectors were produced by the reference implementation itself
(tests/golden/make_golden.py): its quantisers, its fixture generator, its exact PyTorch
oracles and its three Triton kernels run by Triton's CPU interpreter.
"""
import numpy as np
import pytest
import torch

from oracle import specq_oracle as O


# ------------------------------------------------------------------------ quantisers
def test_oracle_quantizers_bit_exact(golden):
    g = golden("quant")
    q, s = O.quantize_act_int8(g["x"])
    assert np.array_equal(q, g["a_q"]) and np.array_equal(s, g["sa"])
    q, s = O.quantize_weight_int8(g["w"])
    assert np.array_equal(q, g["w_q"]) and np.array_equal(s, g["sw"])
    wp, sc, deq = O.quantize_weight_int4(g["w4"], 128)
    assert np.array_equal(wp, g["wp"]) and np.array_equal(sc, g["sc"]) and np.array_equal(deq, g["deq"])
    q, s = O.quantize_act_int8(g["x_edge"])          # zero row (1e-8 clamp) and fp16 max
    assert np.array_equal(q, g["e_q"]) and np.array_equal(s, g["e_s"])


def test_oracle_gpu_division_semantics():
    """on_cuda=True restates torch's GPU evaluation of `tensor / scalar` (a multiplication by
    the fp32 reciprocal); on_cuda=False its CPU evaluation (an IEEE division)."""
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((16, 512)) * 0.05).astype(np.float16)
    amax = np.abs(w.astype(np.float32).reshape(16, 4, 128)).max(-1)
    _, sc_gpu, _ = O.quantize_weight_int4(w, 128, on_cuda=True)
    _, sc_cpu, _ = O.quantize_weight_int4(w, 128)
    t = torch.from_numpy(amax)
    assert np.array_equal(sc_gpu, (t * torch.tensor(1.0 / 7.0, dtype=torch.float32)).half().numpy())
    assert np.array_equal(sc_cpu, (t / 7.0).half().numpy())
    _, s_gpu = O.quantize_act_int8(w, on_cuda=True)
    assert np.array_equal(s_gpu, (torch.from_numpy(np.abs(w.astype(np.float32)).max(-1)) *
                                  torch.tensor(1.0 / 127.0, dtype=torch.float32)).numpy())


def test_package_quantizers_bit_exact(golden):
    import specq
    g = golden("quant")
    q, s = specq.quantize_act_int8(torch.from_numpy(g["x"]))
    assert np.array_equal(q.numpy(), g["a_q"]) and np.array_equal(s.numpy(), g["sa"])
    q, s = specq.quantize_weight_int8(torch.from_numpy(g["w"]))
    assert np.array_equal(q.numpy(), g["w_q"]) and np.array_equal(s.numpy(), g["sw"])
    wp, sc, deq = specq.quantize_weight_int4(torch.from_numpy(g["w4"]), 128)
    assert np.array_equal(wp.numpy(), g["wp"]) and np.array_equal(sc.numpy(), g["sc"])
    assert np.array_equal(deq.numpy(), g["deq"])
    q, s = specq.quantize_act_int8(torch.from_numpy(g["x_edge"]))
    assert np.array_equal(q.numpy(), g["e_q"]) and np.array_equal(s.numpy(), g["e_s"])


def test_unpack_roundtrip(golden):
    g = golden("quant")
    q = O.unpack_int4(g["wp"])
    n, k = q.shape
    repacked = ((q[:, : k // 2].astype(np.int16) + 8) | ((q[:, k // 2:].astype(np.int16) + 8) << 4)).astype(np.uint8)
    assert np.array_equal(repacked, g["wp"])
    assert q.min() >= -8 and q.max() <= 7


# ------------------------------------------------------------------------ W8A8
@pytest.mark.parametrize("name", ["w8a8_small", "w8a8_ragged", "w8a8_m1"])
def test_w8a8_oracle_matches_reference_kernel(golden, name):
    g = golden(name)
    out = O.w8a8_ref(g["a_q"], g["sa"], g["w_q"], g["sw"])
    # The reference kernel (int32 accumulate, fp32 epilogue) is bit-identical to the exact oracle.
    assert np.array_equal(out.view(np.uint16), g["out"].view(np.uint16))
    assert O.max_rel_err_plus1(out, g["ref"]) < 2e-3          # correctness.py:38-40


def test_w8a8_oracle_plan_mode(golden):
    g = golden("w8a8_plan")
    M = int(g["plan"][0])
    ref = O.w8a8_ref(g["a_q"][:M], g["sa"][:M], g["w_q"], g["sw"])
    assert np.array_equal(g["out"][:M].view(np.uint16), ref.view(np.uint16))
    assert np.all(g["out"][M:] == np.float16(12345.0))         # correctness.py:57,63


def test_w8a8_acc_exact_beyond_fp32():
    # |acc| > 2**24: fp32 accumulation would round, the oracle's must not.
    a = np.full((2, 4096), 127, np.int8)
    w = np.full((3, 4096), 127, np.int8)
    w[1, ::2] = -127
    acc = O.w8a8_acc(a, w)
    assert acc[0, 0] == 127 * 127 * 4096 and acc[0, 1] == 0


# ------------------------------------------------------------------------ W4A16
@pytest.mark.parametrize("name", ["w4a16_small", "w4a16_mid"])
def test_w4a16_oracle_matches_reference_kernel(golden, name):
    g = golden(name)
    out = O.w4a16_ref(g["x"], g["wp"], g["sc"], 128)
    # same dequantised weights (fp16 scale, one rounding); only fp32 vs fp64 summation differs
    assert O.rel_fro_err(out, g["out"]) < 1e-3
    assert O.max_rel_err_plus1(out, g["out"]) < 2e-3
    assert O.rel_fro_err(g["out"], g["ref"]) < 2e-3           # correctness.py:77-79


def test_w4a16_kernel_dequant_vs_fp32_scale_dequant(golden):
    g = golden("quant")
    deq_k = O.dequant_int4_kernel(g["wp"], g["sc"], 128)
    # the kernel rounds q*fp16(scale); the reference's deq rounds q*fp32(scale): close, not equal
    assert np.abs(deq_k.astype(np.float32) - g["deq"].astype(np.float32)).max() < 2e-3 * np.abs(g["deq"]).max()


def test_w4a16_oracle_plan_mode(golden):
    g = golden("w4a16_plan")
    M = int(g["plan"][0])
    ref = O.w4a16_ref(g["x"][:M], g["wp"], g["sc"], 128)
    assert O.rel_fro_err(g["out"][:M], ref) < 1e-3
    assert np.all(g["out"][M:] == np.float16(12345.0))


# ------------------------------------------------------------------------ attention
@pytest.mark.parametrize("name", ["attn_small", "attn_f32scales"])
def test_attention_oracle_matches_reference(golden, name):
    g = golden(name)
    ql = int(g["q_len"])
    out = O.paged_attention_ref(g["q"], g["kc"], g["vc"], g["ks"], g["vs"], g["bt"], g["cl"], ql)
    assert O.max_abs_err(out, g["ref"]) <= 2 ** -10             # fp64 vs fp32 oracle, fp16 output
    assert O.max_abs_err(out, g["out_fused"]) < 2e-2            # correctness.py:100
    assert O.rel_fro_err(out, g["out_fused"]) < 1e-3
    if "out_tok" in g:
        assert O.rel_fro_err(out, g["out_tok"]) < 1e-3


def test_attention_oracle_plan_mode(golden):
    g = golden("attn_plan")
    b_act, ql = int(g["plan"][0]), int(g["plan"][1])
    out = O.paged_attention_ref(g["q"][:b_act], g["kc"], g["vc"], g["ks"], g["vs"], g["bt"][:b_act],
                                g["cl"][:b_act], ql)
    assert O.max_abs_err(out[:, :ql], g["out"][:b_act, :ql]) < 2e-2
    assert O.max_abs_err(out, g["ref"]) <= 2 ** -10
    assert np.all(g["out"][b_act:] == np.float16(7.0)) and np.all(g["out"][:b_act, ql:] == np.float16(7.0))


def test_make_paged_kv_reproduces_reference_fixture(golden):
    import specq
    for name, (B, ctx, seed) in {"attn_small": (2, [37, 70], 5), "attn_plan": (3, [20, 45, 33], 9)}.items():
        g = golden(name)
        kc, vc, ks, vs, bt, cl = specq.make_paged_kv(B, ctx, 2, 128, device="cpu", seed=seed)
        for got, key in ((kc, "kc"), (vc, "vc"), (ks, "ks"), (vs, "vs"), (bt, "bt"), (cl, "cl")):
            assert np.array_equal(got.numpy().view(np.uint8), g[key].view(np.uint8)), (name, key)


def test_package_attention_ref_matches_reference(golden):
    import specq
    g = golden("attn_small")
    t = {k: torch.from_numpy(g[k]) for k in ("q", "kc", "vc", "ks", "vs", "bt", "cl")}
    out = specq.paged_attention_ref(t["q"], t["kc"], t["vc"], t["ks"], t["vs"], t["bt"], t["cl"], int(g["q_len"]))
    assert O.max_abs_err(out.numpy(), g["ref"]) <= 2 ** -10


# ------------------------------------------------------------------------ planted mistakes
def test_checks_catch_a_planted_packing_mistake(golden):
    """A nibble-order slip in the oracle is caught by the golden comparison."""
    g = golden("w4a16_small")
    wrong = ((g["wp"] >> 4) | (g["wp"] << 4)).astype(np.uint8)   # swap the two halves
    out = O.w4a16_ref(g["x"], wrong, g["sc"], 128)
    assert O.rel_fro_err(out, g["out"]) > 0.1


def test_checks_catch_a_planted_causal_mistake(golden):
    """Shifting the causal window by one token is caught by the golden comparison."""
    g = golden("attn_small")
    ql = int(g["q_len"])
    out = O.paged_attention_ref(g["q"], g["kc"], g["vc"], g["ks"], g["vs"], g["bt"], g["cl"] - 1, ql - 1)
    full = np.zeros_like(g["ref"])
    full[:, : ql - 1] = out[:, : ql - 1]
    assert O.max_abs_err(full[:, : ql - 1], g["ref"][:, 1:ql]) > 1e-2 or O.max_abs_err(full, g["ref"]) > 1e-2


def test_oracle_kv_quant_reproduces_reference_cache(golden):
    """kv_quant_rows (the per-token cache quantiser the stack's KV append restates) gives the
    reference fixture's int8 cache and fp16 scales (make_paged_kv, kernels.py:265-286) from the
    same fp16 draws (CPU division semantics, as the fixture ran)."""
    g = golden("attn_small")
    gen = torch.Generator().manual_seed(5)
    total = (37 + 15) // 16 + (70 + 15) // 16
    torch.randperm(total, generator=gen)
    kf = torch.randn((total, 16, 2, 128), generator=gen).half().numpy()
    vf = torch.randn((total, 16, 2, 128), generator=gen).half().numpy()
    for x, qk, sk in ((kf, "kc", "ks"), (vf, "vc", "vs")):
        q, s = O.kv_quant_rows(x, on_cuda=False)
        assert np.array_equal(q, g[qk]) and np.array_equal(s.view(np.uint16), g[sk].view(np.uint16))


def test_oracle_residual_add_is_one_fp16_rounding():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(4096) * rng.choice([1e-3, 1.0, 300.0], 4096)).astype(np.float16)
    r = (rng.standard_normal(4096) * rng.choice([1e-3, 1.0, 300.0], 4096)).astype(np.float16)
    exact = (x.astype(np.float64) + r.astype(np.float64)).astype(np.float16)
    assert np.array_equal(O.residual_add(x, r).view(np.uint16), exact.view(np.uint16))

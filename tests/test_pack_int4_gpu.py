"""INT4 weight packer on the GPU (the reference's quantize_weight_int4, kernels.py:138-147).

Bit-exact against the oracle evaluated with torch's GPU semantics (the division of the group
maximum by 7 is a multiplication by fp32(1/7) on a CUDA tensor) and against the reference's
torch formula run on the GPU; the W4A16 kernel consumes what it packs."""
import numpy as np
import pytest
import torch

from oracle import specq_oracle as O

pytestmark = pytest.mark.gpu


def _check_vs_oracle(w, group):
    import specq
    wp, sc, deq = specq.pack_int4(w, group)
    ewp, esc, edeq = O.quantize_weight_int4(w.float().cpu().numpy().astype(np.float32), group, on_cuda=True)
    assert np.array_equal(wp.cpu().numpy(), ewp)
    assert np.array_equal(sc.cpu().numpy(), esc)
    assert np.array_equal(deq.cpu().numpy(), edeq)


@pytest.mark.parametrize("N,K,group", [(40, 512, 128), (64, 256, 32), (33, 384, 64), (16, 1024, 256)])
def test_pack_int4_matches_oracle(cuda, N, K, group):
    g = torch.Generator(device="cuda").manual_seed(N * K + group)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    w[0, :group] = 0                                  # an all-zero group: the 1e-8 clamp
    w[1, 3] = 65504.0                                 # fp16 max in a group
    _check_vs_oracle(w, group)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_pack_int4_other_dtypes_and_strides(cuda, dtype):
    g = torch.Generator(device="cuda").manual_seed(3)
    base = torch.randn(24, 768, device="cuda", generator=g).to(dtype)
    w = base[:, :512]                                 # row stride 768 > K
    _check_vs_oracle(w, 128)
    _check_vs_oracle(base[:, 1:513], 128)             # rows not vector-aligned: element loads


def test_pack_int4_equals_reference_formula_on_gpu(cuda):
    """The reference's torch function evaluated on the GPU (config 1 weight shape)."""
    import specq
    g = torch.Generator(device="cuda").manual_seed(11)
    w = (torch.randn(14336, 4096, device="cuda", generator=g) * 0.02).half()
    wp, sc, deq = specq.pack_int4(w, 128)
    rwp, rsc, rdeq = specq.fixtures.quantize_weight_int4(w, 128)
    assert torch.equal(wp, rwp) and torch.equal(sc, rsc) and torch.equal(deq, rdeq)
    # the public drop-in name routes a CUDA tensor to the kernel
    pwp, psc, pdeq = specq.quantize_weight_int4(w, 128)
    assert torch.equal(pwp, wp) and torch.equal(psc, sc) and torch.equal(pdeq, deq)


def test_pack_int4_golden_within_division_semantics(cuda, golden):
    """The reference's own outputs (made on a CPU tensor, IEEE division by 7): identical
    except where the two scale evaluations differ in the last fp32 bit."""
    import specq
    gd = golden("quant")
    wp, sc, deq = specq.pack_int4(torch.from_numpy(gd["w4"]).cuda(), 128)
    same_bytes = float((wp.cpu().numpy() == gd["wp"]).mean())
    assert same_bytes > 0.999
    d = np.abs(sc.cpu().numpy().astype(np.float32) - gd["sc"].astype(np.float32))
    assert float(d.max()) <= float(np.abs(gd["sc"].astype(np.float32)).max()) * 2.0 ** -10


def test_pack_int4_feeds_w4a16(cuda):
    import specq
    g = torch.Generator(device="cuda").manual_seed(5)
    w = (torch.randn(256, 1024, device="cuda", generator=g) * 0.02).half()
    x = torch.randn(8, 1024, device="cuda", generator=g).half()
    wp, sc, deq = specq.pack_int4(w, 128)
    out, _ = specq.w4a16_matmul(x, wp, sc)
    ref = x.float() @ deq.float().T
    rel = (out.float() - ref).norm() / ref.norm()
    assert float(rel) < 1e-3


def test_pack_int4_rejects_bad_shapes(cuda):
    import specq
    w = torch.randn(8, 200, device="cuda").half()     # (K/2) % 128 != 0
    with pytest.raises(ValueError):
        specq.pack_int4(w, 128)
    w = torch.randn(8, 96 * 2, device="cuda").half()
    with pytest.raises((ValueError, RuntimeError)):
        specq.pack_int4(w, 96)                         # group 96: not built

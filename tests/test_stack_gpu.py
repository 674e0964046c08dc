"""The INT8 verification stack under a single plan-buffer graph equals eager execution bit
for bit (residual stream and the KV appended to every layer's cache), for several active
(B, q_len) inside one graph captured at the maximum shape."""
import pytest

pytestmark = pytest.mark.gpu


def test_plan_graph_bit_exact_small_stack(cuda):
    from specq.stack import Stack, plan_vs_eager
    st = Stack(layers=2, hid=1024, ff=2048, heads=8, kv_heads=2, ctx=128, b_max=4, ks=(0, 2, 4), seed=3)
    assert plan_vs_eager(st, [(1, 1), (4, 5), (2, 3), (3, 5)]) == 0.0


def test_stack_run_reports_every_strategy(cuda):
    from specq.stack import run
    res = run(layers=1, steps=12, b_max=4, ks=(0, 2), ctx=128, seed=1)
    for name in ("eager", "maxpad", "plan", "allshapes"):
        assert res[name]["tok_per_s"] > 0
    assert res["plan_vs_eager_max_abs_diff"] == 0.0
    assert res["maxpad"]["waste_pct"] >= 0.0

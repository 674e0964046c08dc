"""Multi-GPU decomposition of the verification step (host side, one process per GPU).

The path partitions into independent units, so ranks need no data-path collective:

  * W8A8 / W4A16 GEMMs are column-parallel: rank r owns a contiguous range of output
    channels -- the matching rows of `w_q` / `wp` and of `sw` / `sc`, and the matching
    columns of `out`.  Activations and their scales are replicated.
  * Paged attention is KV-head-parallel: rank r owns a contiguous range of KV heads, the
    query heads of their GQA groups, and those heads' slices of the KV cache and its scales.
    The block table and the context lengths are replicated.

Only a multi-layer stack needs an all-gather of the column shards (not part of these
kernels).  `shard_plan` gives the ranges; `shard_inputs` cuts a full set of step inputs down
to one rank's share.
"""
from __future__ import annotations


def _split(n: int, world: int, rank: int) -> slice:
    if n % world:
        raise ValueError(f"{n} does not split evenly over {world} ranks")
    per = n // world
    return slice(rank * per, (rank + 1) * per)


def shard_plan(world: int, rank: int, n_w8a8: int, n_w4a16: int, h_kv: int, h: int) -> dict:
    """The output-channel and head ranges rank `rank` of `world` owns."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if h % h_kv:
        raise ValueError(f"H={h} is not a multiple of H_KV={h_kv}")
    kv = _split(h_kv, world, rank)
    g = h // h_kv
    return {"w8a8_cols": _split(n_w8a8, world, rank), "w4a16_cols": _split(n_w4a16, world, rank),
            "kv_heads": kv, "q_heads": slice(kv.start * g, kv.stop * g)}


def shard_inputs(x: dict, plan: dict) -> dict:
    """One rank's share of a step's inputs (keys as produced by the benchmark / tests)."""
    c8, c4, kv, qh = plan["w8a8_cols"], plan["w4a16_cols"], plan["kv_heads"], plan["q_heads"]
    y = dict(x)
    y["w8"], y["sw"] = x["w8"][c8], x["sw"][c8]
    y["wp"], y["sc"] = x["wp"][c4], x["sc"][c4]
    y["kc"], y["vc"] = x["kc"][:, :, kv], x["vc"][:, :, kv]
    y["ks"], y["vs"] = x["ks"][:, :, kv], x["vs"][:, :, kv]
    y["q"] = x["q"][:, :, qh]
    return y

"""Work partition of the decode path over GPUs (one process per GPU).

Everything on the path is per (sequence, layer, kv head): slot pools, read
budgets, top-k selection and the correction are computed inside one kv
head's pages (the reference's vectorized_joint_correction runs per kv head,
attention.py:576), so a partition of the (sequence, kv head) grid needs no
exchange.  Two partitions are used:

* batch: rank r of N owns sequences [r*B/N, (r+1)*B/N) with every kv head
  (Llama-2-7B MHA shape, batch-sharded);
* kv head: rank r owns kv heads [r*H/N, (r+1)*H/N) of every sequence, its
  arena built with num_kv_heads = H/N and its engine given the shard
  (Mistral-7B GQA shape: 8 kv heads, one per GPU).

A rank's decode output covers its own rows (batch) or its own query heads
(kv head); reassemble() puts the ranks' parts back into the model's layout.
"""

from typing import List, Sequence, Tuple


def contiguous_share(total: int, world: int, rank: int) -> Tuple[int, int]:
    """(first, count) of rank's contiguous share of `total` items; the shares
    of all ranks are disjoint, cover every item and differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    q, r = divmod(total, world)
    first = rank * q + min(rank, r)
    return first, q + (1 if rank < r else 0)


def batch_shard(global_batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Sequences [first, first + count) of `rank` under batch sharding."""
    return contiguous_share(global_batch, world, rank)


def kv_head_shard(num_kv_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """(kvh_begin, kvh_count) of `rank` under kv-head sharding; also the
    engine's shard argument is (kvh_begin, num_kv_heads)."""
    return contiguous_share(num_kv_heads, world, rank)


def owner(seq: int, kv_head: int, global_batch: int, num_kv_heads: int, world: int, mode: str) -> int:
    """Rank that holds (seq, kv_head) under `mode` ("batch" or "kv_head")."""
    n, idx = (global_batch, seq) if mode == "batch" else (num_kv_heads, kv_head)
    for r in range(world):
        first, count = contiguous_share(n, world, r)
        if first <= idx < first + count:
            return r
    raise ValueError(f"{idx} outside [0, {n})")


def reassemble_batch(parts: Sequence):
    """Model output [B, Hq, D] from the ranks' batch shares [count_r, Hq, D]
    in rank order."""
    import torch
    return torch.cat(list(parts), dim=0)


def reassemble_kv_heads(parts: Sequence, query_heads_per_kv: int, model_rows: bool = True):
    """Model output [B, Hq, D] from the ranks' kv-head shares in rank order.
    model_rows: each part is the model's rows [B, Hq, D] in which the rank
    wrote only its own query heads (what a sharded engine's attend returns);
    else each part holds the rank's heads alone [B, count_r * QN, D]."""
    import torch
    world = len(parts)
    if not model_rows:
        return torch.cat(list(parts), dim=1)
    Hq = parts[0].shape[1]
    H = Hq // query_heads_per_kv
    out = torch.empty_like(parts[0])
    for r, p in enumerate(parts):
        b, n = kv_head_shard(H, world, r)
        sl = slice(b * query_heads_per_kv, (b + n) * query_heads_per_kv)
        out[:, sl] = p[:, sl]
    return out

"""The N>1 host logic of bench.py on CPU: two gloo ranks (127.0.0.1).

Each rank owns its own batch (weak scaling); the job time is the max over
ranks of the device timings, which every rank receives, and the aggregate
throughput counts every rank's sequences.  The path has no data collective;
this covers the only exchange bench.py makes.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        mine = [10.0 + 5 * rank, 20.0 - 3 * rank, 1.5 + rank]
        got = bench.max_over_ranks(mine, world)
        q.put((rank, got, bench.aggregate_tok_s(world, 32, 10, got[0])))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_gloo_ranks_max_and_aggregate():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=100) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got, tok in res:
        assert got == [15.0, 20.0, 2.5]
        assert tok == pytest.approx(2 * 32 * 10 / 0.015)


def test_single_rank_passthrough():
    import bench
    assert bench.max_over_ranks([1.0, 2.0], 1) == [1.0, 2.0]
    assert bench.aggregate_tok_s(1, 32, 20, 100.0) == pytest.approx(6400.0)


def test_rank_batch_partition():
    """Strong scaling: the global batch splits into contiguous, disjoint
    shares that cover it; weak scaling gives every rank a full batch."""
    import bench
    for world in (1, 2, 4, 8):
        owned = []
        for r in range(world):
            s0, n = bench.rank_batch(32, world, r, "strong")
            assert n == 32 // world
            owned += list(range(s0, s0 + n))
        assert owned == list(range(32))
        assert bench.aggregate_tok_s(world, 32 // world, 10, 100.0) == pytest.approx(3200.0)
    assert bench.rank_batch(32, 4, 2, "weak") == (64, 32)
    with pytest.raises(ValueError):
        bench.rank_batch(32, 3, 0, "strong")


def _partition_worker(rank, world, port, q):
    """Each rank computes a stand-in output for the (sequence, kv head) pairs
    it owns under both partitions; the ranks' parts are gathered and
    reassembled into the model layout."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import importlib
        P = importlib.import_module(
            "care-kv-sparse-residual-correction-for-low-bit-kv-cache-quantization_b200").partition
        B, H, QN, D = 6, 8, 4, 3
        full = torch.arange(B * H * QN * D, dtype=torch.float32).view(B, H * QN, D)

        def out_of(seq, qhead):          # what the owner of (seq, qhead // QN) computes
            return full[seq, qhead]

        # kv-head shards: the rank writes its query heads into model rows
        kb, kn = P.kv_head_shard(H, world, rank)
        mine = torch.zeros_like(full)
        for s in range(B):
            for qh in range(kb * QN, (kb + kn) * QN):
                assert P.owner(s, qh // QN, B, H, world, "kv_head") == rank
                mine[s, qh] = out_of(s, qh)
        parts = [torch.empty_like(full) for _ in range(world)]
        dist.all_gather(parts, mine)
        got_kv = P.reassemble_kv_heads(parts, QN)
        # batch shards: the rank computes every head of its sequences
        sb, sn = P.batch_shard(B, world, rank)
        rows = torch.stack([full[s] for s in range(sb, sb + sn)])
        for s in range(sb, sb + sn):
            assert P.owner(s, 0, B, H, world, "batch") == rank
        sizes = [P.batch_shard(B, world, r)[1] for r in range(world)]
        bparts = [torch.empty(n, H * QN, D) for n in sizes]
        dist.all_gather(bparts, rows)
        got_b = P.reassemble_batch(bparts)
        q.put((rank, bool(torch.equal(got_kv, full)), bool(torch.equal(got_b, full))))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_gloo_ranks_partition_and_reassembly():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_partition_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=100) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == [(0, True, True), (1, True, True)]


def test_contiguous_shares_cover_and_balance():
    import importlib
    P = importlib.import_module("care-kv-sparse-residual-correction-for-low-bit-kv-cache-quantization_b200").partition
    for total in (1, 7, 8, 32):
        for world in (1, 2, 3, 8):
            shares = [P.contiguous_share(total, world, r) for r in range(world)]
            items = [i for b, n in shares for i in range(b, b + n)]
            assert items == list(range(total))
            assert max(n for _, n in shares) - min(n for _, n in shares) <= 1

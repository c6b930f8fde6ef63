"""Request sharding across ranks (host logic; CPU, gloo world_size 2).

The multi-GPU path splits a batch by request with no data-path collective;
these tests check the split (coverage, determinism, balance) and run it as
two gloo ranks, each decoding its shard with the oracle, rank 0 comparing
the gathered shards with the single-process result."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mini_llm_runtime_b200.sharding import decode_cost, imbalance, prefill_cost, shard_requests


def test_every_request_lands_on_exactly_one_rank():
    rng = np.random.default_rng(0)
    costs = rng.integers(128, 4097, size=257).tolist()
    for world in (1, 2, 3, 4, 8):
        shards = shard_requests(costs, world)
        got = sorted(i for s in shards for i in s.requests)
        assert got == list(range(len(costs)))
        assert all(s.requests == sorted(s.requests) for s in shards)
        assert sum(s.cost for s in shards) == sum(costs)


def test_split_is_deterministic_and_balanced():
    rng = np.random.default_rng(1)
    costs = [decode_cost(c) for c in rng.integers(128, 4097, size=512)]
    a = shard_requests(costs, 8)
    b = shard_requests(list(costs), 8)
    assert [s.requests for s in a] == [s.requests for s in b]
    # LPT on 64 uniform requests per rank lands within a fraction of a percent.
    assert imbalance(a) < 1.01
    # Balancing by count alone would be much worse on skewed costs.
    skew = [100_000] * 4 + [1] * 60
    assert imbalance(shard_requests(skew, 4)) < 1.01


def test_edge_cases():
    assert [s.requests for s in shard_requests([], 3)] == [[], [], []]
    assert [s.requests for s in shard_requests([5], 2)] == [[0], []]
    with pytest.raises(ValueError):
        shard_requests([1, 2], 0)
    with pytest.raises(ValueError):
        shard_requests([-1], 2)
    assert prefill_cost(0, 1) == 1
    assert prefill_cost(10, 4) == 4 * 11 + 6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    from oracle import paged_attention_oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # Every rank draws the same global batch and computes the same split.
        rng = np.random.default_rng(7)
        ctx = rng.integers(1, 300, size=12)
        hq, hkv, d, bs = 14, 2, 64, 16
        need = (ctx + bs - 1) // bs
        nb = int(need.sum()) + 4
        perm = rng.permutation(nb)
        tables = np.full((len(ctx), int(need.max())), -1, dtype=np.int64)
        cur = 0
        for i, n in enumerate(need):
            tables[i, :n] = perm[cur:cur + n]
            cur += n
        k = rng.standard_normal((nb, bs, hkv, d), dtype=np.float32)
        v = rng.standard_normal((nb, bs, hkv, d), dtype=np.float32)
        q = rng.standard_normal((len(ctx), hq, d), dtype=np.float32)
        mine = shard_requests([decode_cost(c) for c in ctx], world)[rank].requests
        out = O.decode_batch(q[mine], k, v, tables[mine], ctx[mine], bs) if mine else np.zeros((0, hq, d), np.float32)
        gathered = [None] * world
        dist.all_gather_object(gathered, (mine, out))
        if rank == 0:
            full = np.zeros((len(ctx), hq, d), np.float32)
            seen = []
            for idx, part in gathered:
                full[idx] = part
                seen += idx
            ref = O.decode_batch(q, k, v, tables, ctx, bs)
            ok = sorted(seen) == list(range(len(ctx))) and np.allclose(full, ref, rtol=1e-6, atol=1e-6)
            with open(result_path, "w") as f:
                f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_decode_their_shards(tmp_path):
    port = _free_port()
    path = str(tmp_path / "result")
    mp.start_processes(_rank_main, args=(2, port, path), nprocs=2, join=True, start_method="spawn")
    assert open(path).read() == "ok"


def test_bench_shards_cover_the_global_batch():
    """bench.py's per-rank metadata: every rank's contexts are its shard of
    the same global draw, pools hold exactly the shard's blocks + 10 %, and
    the N = 1 draw is the config-2 workload."""
    import bench

    full, _, _, _ = bench.make_metadata(1000)
    assert len(full) == bench.BATCH
    for world in (2, 4):
        glob = np.random.default_rng(1000).integers(bench.CTX_LO, bench.CTX_HI + 1, size=bench.BATCH * world)
        parts = [bench.make_metadata(1000, world, r) for r in range(world)]
        got = np.sort(np.concatenate([p[0] for p in parts]))
        assert np.array_equal(got, np.sort(glob))
        for ctx, tables, slots, nb in parts:
            need = (ctx + bench.BS - 1) // bench.BS
            used = tables[tables >= 0]
            assert len(np.unique(used)) == need.sum() and used.max() < nb
            pos = ctx - 1
            assert np.array_equal(slots, tables[np.arange(len(ctx)), pos // bench.BS] * bench.BS + pos % bench.BS)

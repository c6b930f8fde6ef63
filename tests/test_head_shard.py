"""KV-head-sharded decode of long sequences (host logic; CPU, gloo ranks).

Each rank keeps its KV heads' slice of the pools and its query heads, decodes
them (the oracle stands in for the CUDA kernel on CPU ranks), and the
all-gather of head outputs must rebuild the unsharded result exactly."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mini_llm_runtime_b200.head_shard import head_slices, shard_pool


def test_head_slices_cover_all_heads_by_group():
    for hq, hkv, world in ((14, 2, 2), (28, 4, 4), (28, 4, 2), (32, 8, 8), (8, 8, 4)):
        qs, ks = [], []
        for r in range(world):
            q, k = head_slices(hq, hkv, world, r)
            qs += list(range(hq))[q]
            ks += list(range(hkv))[k]
            # every query head of the slice reads a KV head of the slice
            group = hq // hkv
            assert all(h // group in range(hkv)[k] for h in range(hq)[q])
        assert qs == list(range(hq)) and ks == list(range(hkv))
    with pytest.raises(ValueError, match="divisible by the world size"):
        head_slices(14, 2, 4, 0)
    with pytest.raises(ValueError):
        head_slices(14, 2, 2, 2)


def test_shard_pool_keeps_only_the_slice():
    pool = torch.arange(2 * 3 * 4 * 4 * 8, dtype=torch.float32).reshape(2, 3, 4, 4, 8)
    part = shard_pool(pool, slice(2, 4))
    assert part.is_contiguous() and part.shape == (2, 3, 4, 2, 8)
    assert torch.equal(part, pool[:, :, :, 2:4])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_decode(q, k, v, tables, lens, bs):
    from oracle import paged_attention_oracle as O

    out = O.decode_batch(q.numpy(), k.numpy(), v.numpy(), tables.numpy(), lens.numpy(), bs)
    return torch.from_numpy(out)


def _rank_main(rank, world, port, hq, hkv, result_path):
    from mini_llm_runtime_b200.head_shard import HeadShardedDecode

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # Every rank draws the same long sequences and full pools.
        g = torch.Generator().manual_seed(11)
        bs, d = 16, 64
        ctx = torch.tensor([700, 1500, 33])
        need = ((ctx + bs - 1) // bs).tolist()
        nb = sum(need) + 3
        perm = torch.randperm(nb, generator=g).tolist()
        tables, cur = [], 0
        for n in need:
            tables.append(perm[cur:cur + n] + [-1] * (max(need) - n))
            cur += n
        tables = torch.tensor(tables)
        k = torch.randn(nb, bs, hkv, d, generator=g)
        v = torch.randn(nb, bs, hkv, d, generator=g)
        q = torch.randn(len(ctx), hq, d, generator=g)
        hs = HeadShardedDecode(hq, hkv, local_decode=_oracle_decode)
        out = hs(hs.local_queries(q), shard_pool(k, hs.kv_slice), shard_pool(v, hs.kv_slice), tables, ctx, bs)
        ref = _oracle_decode(q, k, v, tables, ctx, bs)
        ok = out.shape == ref.shape and torch.allclose(out, ref, rtol=1e-6, atol=1e-6)
        flags = [None] * world
        dist.all_gather_object(flags, bool(ok))
        if rank == 0:
            with open(result_path, "w") as f:
                f.write("ok" if all(flags) else f"mismatch {flags}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("hq,hkv,world", [(14, 2, 2), (28, 4, 4)])
def test_gloo_ranks_rebuild_the_unsharded_decode(tmp_path, hq, hkv, world):
    port = _free_port()
    path = str(tmp_path / "result")
    mp.start_processes(_rank_main, args=(world, port, hq, hkv, path), nprocs=world, join=True, start_method="spawn")
    assert open(path).read() == "ok"

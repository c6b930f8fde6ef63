"""KV-head-sharded decode on 2 GPUs over NCCL: each rank decodes its KV
heads with the CUDA kernels and the all-gather of head outputs must rebuild
the oracle's unsharded result (BF16 tolerance).  Needs two GPUs; skipped with
fewer."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    from datetime import timedelta

    import torch.distributed as dist

    from mini_llm_runtime_b200.head_shard import HeadShardedDecode, shard_pool
    from oracle import paged_attention_oracle as O
    from tests.paged_inputs import make_decode_case

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        case = make_decode_case([4097, 30000, 17], 14, 2, 64, 16, torch.bfloat16, dev, seed=21)
        hs = HeadShardedDecode(14, 2)
        out = hs(hs.local_queries(case["q"]), shard_pool(case["k"], hs.kv_slice), shard_pool(case["v"], hs.kv_slice),
                 case["tables"], case["lens"], 16)
        q, k, v, tables, lens = case["np"]
        ref = O.decode_batch(q, k, v, tables, lens, 16)
        err = (out.float().cpu() - torch.from_numpy(ref)).abs()
        ok = bool(torch.isfinite(out.float()).all()) and bool((err <= 2e-2 + 1e-2 * torch.from_numpy(ref).abs()).all())
        flags = [None] * world
        dist.all_gather_object(flags, ok)
        if rank == 0:
            with open(result_path, "w") as f:
                f.write("ok" if all(flags) else f"mismatch {flags}")
    finally:
        dist.destroy_process_group()


def test_two_gpus_rebuild_the_unsharded_decode(cuda_device, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = str(tmp_path / "result")
    mp.start_processes(_rank_main, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    assert open(path).read() == "ok"

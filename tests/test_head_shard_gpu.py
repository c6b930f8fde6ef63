"""KV-head-sharded decode on 2 GPUs: each rank decodes its KV heads with the
CUDA kernels, and the all-gather of head outputs (fused into the decode's
merge kernel, as a kernel of its own over NVLink peer stores, and over NCCL)
must rebuild the oracle's unsharded result (BF16 tolerance), bit-identically
between the three, call after call and under CUDA-graph replay.  Needs two
GPUs; skipped with fewer."""

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
        q, k, v, tables, lens = case["np"]
        ref = torch.from_numpy(O.decode_batch(q, k, v, tables, lens, 16))
        checks, outs = {}, {}
        for transport, fuse in (("peer", True), ("peer-unfused", False), ("collective", True)):
            hs = HeadShardedDecode(14, 2, transport=transport.split("-")[0], max_batch=4, fuse=fuse)
            ql = hs.local_queries(case["q"])
            kl, vl = shard_pool(case["k"], hs.kv_slice), shard_pool(case["v"], hs.kv_slice)
            for _ in range(3):  # the exchange alternates its two slots call by call
                out = hs(ql, kl, vl, case["tables"], case["lens"], 16)
            torch.cuda.synchronize()
            hs.check()
            err = (out.float().cpu() - ref).abs()
            checks[transport] = bool(torch.isfinite(out.float()).all()) and bool((err <= 2e-2 + 1e-2 * ref.abs()).all())
            outs[transport] = out
            if transport == "peer":
                # Replays of a captured call keep the ranks in step: the call
                # number lives in device memory.
                s = torch.cuda.Stream(dev)
                s.wait_stream(torch.cuda.current_stream())
                out_g = torch.empty_like(out)
                with torch.cuda.stream(s):
                    hs(ql, kl, vl, case["tables"], case["lens"], 16, out=out_g)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=s):
                    hs(ql, kl, vl, case["tables"], case["lens"], 16, out=out_g)
                out_g.zero_()
                for _ in range(3):
                    graph.replay()
                torch.cuda.synchronize()
                hs.check()
                checks["graph"] = torch.equal(out_g, out)
                del graph
            hs.close()
        checks["peer == collective"] = torch.equal(outs["peer"], outs["collective"])
        checks["peer == unfused"] = torch.equal(outs["peer"], outs["peer-unfused"])
        flags = [None] * world
        dist.all_gather_object(flags, checks)
        if rank == 0:
            with open(result_path, "w") as f:
                f.write("ok" if all(all(c.values()) for c in flags) else f"mismatch {flags}")
    finally:
        dist.destroy_process_group()


def test_two_gpus_rebuild_the_unsharded_decode(cuda_device, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = str(tmp_path / "result")
    mp.start_processes(_rank_main, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    assert open(path).read() == "ok"

"""Benchmark of the paged-attention hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: BF16 batched paged decode at
Qwen2.5-0.5B attention geometry — 24 layers, 14 Q / 2 KV heads, head_dim 64,
block_size 16, batch 64 per GPU with context lengths U[128, 4096], seeded
random block tables over a pool of total blocks + 10 %, Q/K/V ~ N(0, 1) in
BF16.  One step = for every layer, the batched KV write of the new token
(PagedKVCache.write_slots) followed by batched paged decode
(paged_attention_decode_batch_parallel) — the reference's per-layer hot path
(model/qwen2.py:608-621).  Per step the KV pools stream ~1.66 GB, far above the
126 MB L2, so no flush is needed between steps.

Multi-GPU: one process per GPU (torchrun).  The global batch is 64 * N
requests drawn once; every rank keeps its shard (longest-first on context
length, so ranks stream equal KV) in its own pool and decodes it with no
communication (weak scaling: ~64 requests per GPU).

The JSON line: ``value`` = whole-job algorithmic KV bytes per second (device
time, inputs resident); ``e2e`` = the same metric through the public API with
the step's inputs copied from pinned host memory and the outputs copied back
inside the timed region; ``roofline`` for the decode kernel; ``cpu_baseline``
= the oracle port on the host cores (rank 0, N=1).

``e2e_per_layer`` = the same metric through the per-layer drop-in call
(24 x paged_decode_with_kv_write per step, each layer's inputs copied from
pinned host memory and its output copied back).

``--impl reference`` times the reference's algorithm on the host CPU (the
oracle port; the reference is PyTorch code with no compiled path to build) on
the same workload: the rank-0 batch of the same metadata draw, 24 layers
(KV write + decode) per step, all host cores.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent

# Workload constants.
LAYERS, HQ, HKV, D, BS, BATCH = 24, 14, 2, 64, 16, 64
CTX_LO, CTX_HI = 128, 4096
METRIC = "paged-decode KV GB/s"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--kernel", choices=sorted(KERNEL_CASES), default=None,
                    help="time one kernel case alone (secondary configs; the small ncu targets)")
    ap.add_argument("--layers", type=int, default=None, help="layers the --kernel case rotates over")
    ap.add_argument("--reps", type=int, default=None, help="graph replays timed by the --kernel case")
    ap.add_argument("--mode", choices=["request-shard", "head-shard", "mixed"], default="request-shard",
                    help="head-shard: config 3 split by KV head over the GPUs, all-gather of head outputs over "
                         "NVLink peer stores (and, for comparison, NCCL); "
                         "mixed: config 5 as one prefill + decode step per layer, sharded by request")
    return ap.parse_args()


def run_env() -> dict:
    """What produced the numbers: source and library hashes (the GPU box has
    no .git), the git HEAD when readable, and the toolchain and device."""
    import hashlib
    import platform

    root = Path(__file__).resolve().parent
    pkg = root / "mini_llm_runtime_b200"
    h = hashlib.sha256()
    for f in sorted([*pkg.glob("*.py"), *(pkg / "csrc").glob("*.cu*"), *(root / "include").glob("*.h")]):
        h.update(f.name.encode())
        h.update(f.read_bytes())
    so = pkg / "libpagedattn.so"
    env = {"source_sha256": h.hexdigest()[:16],
           "library_sha256": hashlib.sha256(so.read_bytes()).hexdigest()[:16] if so.exists() else None,
           "python": platform.python_version(), "torch": torch.__version__, "torch_cuda": torch.version.cuda,
           "nccl": ".".join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else None}
    head = root / ".git" / "HEAD"
    if head.exists():
        ref = head.read_text().strip()
        if ref.startswith("ref: "):
            ref_file = root / ".git" / ref[5:]
            ref = ref_file.read_text().strip() if ref_file.exists() else ref
        env["git_head"] = ref[:12]
    if torch.cuda.is_available():
        env["gpu"] = torch.cuda.get_device_name(0)
        try:
            import pynvml

            pynvml.nvmlInit()
            env["driver"] = pynvml.nvmlSystemGetDriverVersion()
            pynvml.nvmlShutdown()
        except Exception:  # noqa: BLE001 - the record is informational
            pass
    return env


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


FALLBACK_BF16_TFLOPS = 1590.0


def _peak(key: str, fallback: float):
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())[key]), "measured"
        except (KeyError, ValueError):
            pass
    return fallback, "fallback"


def hbm_peak():
    return _peak("hbm_gbs", FALLBACK_HBM_GBS)


def bf16_peak():
    """Burst BF16 peak: the kernel cases are timed alone, a few ms at a time."""
    return _peak("bf16_tflops", FALLBACK_BF16_TFLOPS)


def make_metadata(seed: int, world: int = 1, rank: int = 0):
    """Seeded contexts / block tables / slots for one rank (numpy).

    The global batch is BATCH * world requests; every rank draws the same
    contexts and keeps its request shard (LPT on context length,
    mini_llm_runtime_b200.sharding), with a pool of its shard's blocks + 10 %.
    world = 1 is exactly the config-2 draw."""
    from mini_llm_runtime_b200.sharding import decode_cost, shard_requests

    rng = np.random.default_rng(seed)
    ctx = rng.integers(CTX_LO, CTX_HI + 1, size=BATCH * world).astype(np.int64)
    if world > 1:
        ctx = ctx[shard_requests([decode_cost(c) for c in ctx], world)[rank].requests]
    n = len(ctx)
    need = (ctx + BS - 1) // BS
    nb = int(math.ceil(need.sum() * 1.1))
    perm = rng.permutation(nb)
    width = int(need.max())
    tables = np.full((n, width), -1, dtype=np.int64)
    cur = 0
    for b in range(n):
        tables[b, : need[b]] = perm[cur : cur + need[b]]
        cur += need[b]
    pos = ctx - 1
    slots = tables[np.arange(n), pos // BS] * BS + pos % BS
    return ctx, tables, slots, nb


def algorithmic_bytes(ctx: np.ndarray) -> dict:
    """Bytes the decode step must move per layer (BF16):
    KV reads sum(ctx) * Hkv * D * 2 B * 2 (K and V), Q reads and O writes
    B * Hq * D * 2 B each, block-table reads sum(ceil(ctx/16)) * 8 B, and the
    new-token KV write B * Hkv * D * 2 B * 2."""
    kv = int(ctx.sum()) * HKV * D * 2 * 2
    n = len(ctx)
    qo = 2 * n * HQ * D * 2
    table = int(((ctx + BS - 1) // BS).sum()) * 8
    scatter = n * HKV * D * 2 * 2
    return {"kv": kv, "decode": kv + qo + table, "layer": kv + qo + table + scatter}


class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            self._out = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu_index)],
                stdout=self._out, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._out.close()
        rows = []
        try:
            for line in Path(self.path).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        finally:
            os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def physical_gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# ---------------------------------------------------------------------------
# Single-kernel cases: BASELINE configs 3, 4 and the two halves of config 5,
# and one layer of config 2.  Each case builds `layers` independent layers
# (pools, queries) so consecutive launches stream different memory, captures
# one launch per layer into a CUDA graph and times graph replays.
# ---------------------------------------------------------------------------


def _random_tables(rng, ctx: np.ndarray, bs: int, slack: float = 1.1):
    """Block tables from a random permutation of a pool of total blocks x
    slack, padded with -1 (benchmarks/benchmark_paged_attention.py:449-456)."""
    need = (ctx + bs - 1) // bs
    nb = int(math.ceil(need.sum() * slack))
    perm = rng.permutation(nb)
    tables = np.full((len(ctx), int(need.max())), -1, dtype=np.int64)
    cur = 0
    for b in range(len(ctx)):
        tables[b, : need[b]] = perm[cur : cur + need[b]]
        cur += need[b]
    return tables, nb


def _bf16_randn(shape, device, gen):
    return torch.randn(shape, device=device, generator=gen).to(torch.bfloat16)


FP8_SCALES = (0.0625, 0.0625)  # k_scale, v_scale of the FP8 cases (N(0,1) values, well inside +-448 * scale)


def _decode_case(device, layers, ctx, hq, hkv, d, partition, seed, fp8=False):
    """A decode kernel case: ``fn(l)`` runs layer l; ``inputs`` holds the
    tensors (the parity tests run the oracle on them); ``work`` is the
    algorithmic bytes of one launch.  ``fp8``: the pools hold the e4m3
    quantization of the same N(0, 1) draw (clamp(x / scale) to nearest even)."""
    from mini_llm_runtime_b200 import paged_attention_decode_batch_parallel, paged_attention_decode_split_kv

    rng = np.random.default_rng(seed)
    tables, nb = _random_tables(rng, ctx, BS)
    gen = torch.Generator(device=device).manual_seed(seed)
    k = _bf16_randn((layers, nb, BS, hkv, d), device, gen)
    v = _bf16_randn((layers, nb, BS, hkv, d), device, gen)
    q = _bf16_randn((layers, len(ctx), hq, d), device, gen)
    ks, vs = FP8_SCALES if fp8 else (1.0, 1.0)
    if fp8:
        k = (k.float() / ks).clamp_(-448.0, 448.0).to(torch.float8_e4m3fn)
        v = (v.float() / vs).clamp_(-448.0, 448.0).to(torch.float8_e4m3fn)
    bt, cl = torch.tensor(tables, device=device), torch.tensor(ctx, device=device)
    sc = {"k_scale": ks, "v_scale": vs}
    if partition:
        fn = lambda l: paged_attention_decode_split_kv(q[l], k[l], v[l], bt, cl, BS, partition, **sc)  # noqa: E731
    else:
        fn = lambda l: paged_attention_decode_batch_parallel(q[l], k[l], v[l], bt, cl, BS, **sc)  # noqa: E731
    esize = 1 if fp8 else 2
    work = (int(ctx.sum()) * hkv * d * esize * 2 + 2 * len(ctx) * hq * d * 2
            + int(((ctx + BS - 1) // BS).sum()) * 8)
    inputs = {"kind": "decode", "q": q, "k": k, "v": v, "tables": tables, "ctx": ctx, "block_tables": bt,
              "context_lens": cl, "partition": partition, "k_scale": ks, "v_scale": vs}
    return {"fn": fn, "work": work, "inputs": inputs}


def _prefill_case(device, layers, prefix, chunk, hq, hkv, d, seed):
    from mini_llm_runtime_b200 import paged_attention_prefill_varlen

    rng = np.random.default_rng(seed)
    ctx = prefix + chunk
    tables, nb = _random_tables(rng, ctx, BS)
    gen = torch.Generator(device=device).manual_seed(seed)
    k = _bf16_randn((layers, nb, BS, hkv, d), device, gen)
    v = _bf16_randn((layers, nb, BS, hkv, d), device, gen)
    q = _bf16_randn((layers, int(chunk.sum()), hq, d), device, gen)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(chunk)]), device=device)
    bt, cl = torch.tensor(tables, device=device), torch.tensor(ctx, device=device)
    cmax = int(chunk.max())
    fn = lambda l: paged_attention_prefill_varlen(q[l], cu, cl, bt, k[l], v[l], cmax)  # noqa: E731
    inputs = {"kind": "prefill", "q": q, "k": k, "v": v, "tables": tables, "prefix": prefix, "chunk": chunk,
              "ctx": ctx, "cu_q_lens": cu, "block_tables": bt, "context_lens": cl}
    return {"fn": fn, "work": prefill_flops(prefix, chunk, hq, d), "inputs": inputs}


def prefill_flops(prefix: np.ndarray, chunk: np.ndarray, hq: int, d: int) -> int:
    """Unmasked causal FLOPs: QK^T and PV each cost 2*D per (query, key)
    pair, over the keys at or before each query's absolute position."""
    pairs = sum(int(c) * (int(p) + 1) + int(c) * (int(c) - 1) // 2 for p, c in zip(prefix, chunk))
    return 4 * d * hq * pairs


def _case_config2(device, layers):
    ctx = make_metadata(1000)[0]
    return _decode_case(device, layers, ctx, HQ, HKV, D, 0, 11)


def _case_config2_fp8(device, layers):
    ctx = make_metadata(1000)[0]
    return _decode_case(device, layers, ctx, HQ, HKV, D, 0, 11, fp8=True)


def _case_config3(device, layers):
    ctx = np.full(8, 32768, dtype=np.int64)
    return _decode_case(device, layers, ctx, HQ, HKV, D, 32768 // 16, 13)


def _case_config4(device, layers):
    rng = np.random.default_rng(4)
    prefix = rng.integers(0, 2049, size=16).astype(np.int64)
    return _prefill_case(device, layers, prefix, np.full(16, 512, dtype=np.int64), HQ, HKV, D, 14)


def _case_config5_decode(device, layers):
    ctx = np.random.default_rng(5).integers(256, 8193, size=256).astype(np.int64)
    return _decode_case(device, layers, ctx, 28, 4, 128, 0, 15)


def _case_config5_decode_fp8(device, layers):
    ctx = np.random.default_rng(5).integers(256, 8193, size=256).astype(np.int64)
    return _decode_case(device, layers, ctx, 28, 4, 128, 0, 15, fp8=True)


def _case_config5_prefill(device, layers):
    prefix = np.random.default_rng(6).integers(0, 4097, size=4).astype(np.int64)
    return _prefill_case(device, layers, prefix, np.full(4, 1024, dtype=np.int64), 28, 4, 128, 16)


# name -> (builder, bound, default layers, description)
KERNEL_CASES = {
    "decode-config2": (_case_config2, "hbm", 8,
                       "config2 one layer: bf16 batched decode, B64, 14/2, D64, ctx U[128,4096]"),
    "decode-config2-fp8": (_case_config2_fp8, "hbm", 8,
                           "config2 one layer over an FP8 (e4m3) KV pool: bf16 queries, B64, 14/2, D64, "
                           "ctx U[128,4096]; bytes counted at 1 B per KV element"),
    "split-config3": (_case_config3, "hbm", 4,
                      "config3: bf16 split-KV decode, B8 x 32768, 14/2, D64, 16 partitions of 2048"),
    "prefill-config4": (_case_config4, "tensor", 4,
                        "config4: bf16 causal chunk-prefill, 16 seqs x 512 on prefix U[0,2048], 14/2, D64"),
    "decode-config5": (_case_config5_decode, "hbm", 2,
                       "config5 decode half: bf16 batched decode, B256, 28/4, D128, ctx U[256,8192]"),
    "decode-config5-fp8": (_case_config5_decode_fp8, "hbm", 2,
                           "config5 decode half over an FP8 (e4m3) KV pool: bf16 queries, B256, 28/4, D128, "
                           "ctx U[256,8192]; bytes counted at 1 B per KV element"),
    "prefill-config5": (_case_config5_prefill, "tensor", 4,
                        "config5 prefill half: bf16 chunk-prefill, 4 x 1024 on prefix U[0,4096], 28/4, D128"),
}


def time_kernel_case(name: str, device, layers: int | None = None, reps: int | None = None,
                     warmup: int = 3) -> dict:
    """Device time per launch of one kernel case (CUDA events around graph
    replays on the current stream) and its roofline figures."""
    build, bound, default_layers, desc = KERNEL_CASES[name]
    layers = layers or default_layers
    reps = reps or max(1, 64 // layers)
    case = build(device, layers)
    fn, work = case["fn"], case["work"]
    for l in range(layers):
        fn(l)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for l in range(layers):
            fn(l)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (reps * layers)
    del graph, case, fn
    if bound == "hbm":
        peak, src = hbm_peak()
        achieved, unit = work / (ms * 1e-3) / 1e9, "GB/s"
    else:
        peak, src = bf16_peak()
        achieved, unit = work / (ms * 1e-3) / 1e12, "TFLOP/s"
    return {"case": name, "workload": desc, "bound": bound, "us_per_launch": ms * 1e3,
            "work_per_launch": work, "work_unit": "bytes" if bound == "hbm" else "flops",
            "achieved": achieved, "unit": unit, "peak": peak, "peak_source": src, "frac": achieved / peak,
            "layers": layers, "reps": reps}


def run_kernel_case(args):
    rank, world, local_rank = env_rank()
    torch.cuda.set_device(local_rank)
    r = time_kernel_case(args.kernel, torch.device("cuda", local_rank), args.layers, args.reps, max(args.warmup, 1))
    if rank == 0:
        print(json.dumps(r), flush=True)


# ---------------------------------------------------------------------------
# Reference arm: the reference's algorithm on the host CPU (oracle port)
# ---------------------------------------------------------------------------


def bench_config(world: int, rank0_batch: int) -> dict:
    """The workload both arms report (the driver compares the two)."""
    return {
        "workload": "config2: bf16 batched paged decode (KV write + decode per layer), 24 layers, "
                    "14/2 heads, D64, bs16, global batch 64*N sharded by request (LPT on ctx), "
                    "ctx U[128,4096], pool = blocks*1.1 per rank",
        "global_batch": BATCH * world,
        "parallelism": f"request-sharded dp{world}, no communication",
        "rank0_batch": rank0_batch,
        "l2": "inputs larger than L2 (1.66 GB of KV streamed per step per GPU), no flush",
    }


def cpu_reference_sample(steps: int, warmup: int, layers: int, world: int = 1, rank: int = 0):
    """Time the oracle port of paged_attention_decode_batch_parallel plus the
    write_slots restatement (paged_kv_cache.py:194-249) on the host cores:
    `layers` layers of the GPU arm's rank-0 batch (the same metadata draw) per
    step.  The layers share one FP32 pool (the CPU work per layer does not
    depend on the values)."""
    from oracle import paged_attention_oracle as O

    ctx, tables, slots, nb = make_metadata(1000, world, rank)
    n = len(ctx)
    rng = np.random.default_rng(1001)
    k = rng.standard_normal((1, nb, BS, HKV, D), dtype=np.float32)
    v = rng.standard_normal((1, nb, BS, HKV, D), dtype=np.float32)
    q = O.round_to_bf16(rng.standard_normal((n, HQ, D), dtype=np.float32))
    nk = O.round_to_bf16(rng.standard_normal((n, HKV, D), dtype=np.float32))
    nv = O.round_to_bf16(rng.standard_normal((n, HKV, D), dtype=np.float32))
    threads = os.cpu_count() or 1
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        for _ in range(layers):
            O.write_slots(k, v, slots, nk, nv, 0)
            O.decode_batch_threaded(q, k[0], v[0], tables, ctx, BS, threads)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    step = statistics.median(times)
    kv = algorithmic_bytes(ctx)["kv"] * layers
    return {
        "value": kv / step / 1e9,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": f"{layers} layer(s) of the rank-0 batch ({n} seqs, sum ctx {int(ctx.sum())}) per step, "
                  f"median of {steps} steps, FP32 numpy on BF16-valued inputs, {threads} threads",
        "ms_per_step": step * 1e3,
        "spread": {"min_gbs": kv / max(times) / 1e9, "max_gbs": kv / min(times) / 1e9, "steps": steps},
        "batch": n,
    }


def run_reference(args, rank, world):
    if rank != 0:
        return
    r = cpu_reference_sample(args.steps, args.warmup, LAYERS, world, 0)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": r["value"],
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": r["ms_per_step"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": bench_config(world, r["batch"]),
        "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "spread")},
        "e2e": {"value": r["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "env": run_env(),
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------


def build_rank_workload(rank: int, world: int, device):
    from mini_llm_runtime_b200 import PagedKVCache

    ctx, tables, slots, nb = make_metadata(1000, world, rank)
    n = len(ctx)
    cache = PagedKVCache(LAYERS, nb, BS, HKV, D, dtype=torch.bfloat16, device=device)
    g = torch.Generator(device=device).manual_seed(2000 + rank)
    cache.k_cache.normal_(generator=g)
    cache.v_cache.normal_(generator=g)
    gen = torch.Generator().manual_seed(3000 + rank)
    inputs = {
        "q": torch.randn(LAYERS, n, HQ, D, generator=gen).to(torch.bfloat16),
        "new_k": torch.randn(LAYERS, n, HKV, D, generator=gen).to(torch.bfloat16),
        "new_v": torch.randn(LAYERS, n, HKV, D, generator=gen).to(torch.bfloat16),
        "slot_mapping": torch.tensor(slots),
        "block_tables": torch.tensor(tables),
        "context_lens": torch.tensor(ctx),
    }
    return {"cache": cache, "ctx": ctx, "width": tables.shape[1], "inputs": inputs}


def stage(graph, inputs: dict, device_resident: bool) -> None:
    """Load one step's inputs into a graph's static buffers (device copies
    for the device-resident measurement, pinned host buffers for e2e)."""
    for k, v in inputs.items():
        if device_resident:
            graph._dev_inputs[k].copy_(v)
        else:
            graph.host_inputs[k].copy_(v)


def run_per_layer_e2e(w: dict, device, steps: int, warmup: int, barrier) -> dict:
    """Time `steps` decode steps through the per-layer drop-in call
    (paged_decode_with_kv_write) with host I/O per layer; CUDA events on the
    current stream."""
    from mini_llm_runtime_b200 import paged_decode_with_kv_write

    cache, hin = w["cache"], w["inputs"]
    meta = ("slot_mapping", "block_tables", "context_lens")
    pin = {k: hin[k].pin_memory() for k in meta}
    dev = {k: torch.empty_like(hin[k], device=device) for k in meta}
    n = len(w["ctx"])
    # A layer's q / new_k / new_v packed in one pinned buffer: one H2D copy per layer.
    parts = [hin[k].reshape(LAYERS, -1) for k in ("q", "new_k", "new_v")]
    widths = [t.shape[1] for t in parts]
    pin_l = torch.cat(parts, dim=1).pin_memory()
    dev_l = torch.empty_like(pin_l, device=device)
    shapes = [hin[k].shape[1:] for k in ("q", "new_k", "new_v")]
    views = []
    for layer in range(LAYERS):
        q_, k_, v_ = torch.split(dev_l[layer], widths)
        views.append((pin_l[layer], dev_l[layer], q_.view(shapes[0]), k_.view(shapes[1]), v_.view(shapes[2]),
                      cache.k_cache[layer], cache.v_cache[layer]))
    out_h = torch.empty(LAYERS, n, HQ, D, dtype=torch.bfloat16).pin_memory()
    out_rows = [out_h[layer] for layer in range(LAYERS)]

    def step():
        for k in meta:
            dev[k].copy_(pin[k], non_blocking=True)
        sm, bt, cl = dev["slot_mapping"], dev["block_tables"], dev["context_lens"]
        for layer, (src, dst, q_, k_, v_, kc, vc) in enumerate(views):
            dst.copy_(src, non_blocking=True)
            o = paged_decode_with_kv_write(q_, k_, v_, sm, kc, vc, bt, cl, BS)
            out_rows[layer].copy_(o, non_blocking=True)

    for _ in range(warmup):
        step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    barrier()
    h2d = sum(t.numel() * t.element_size() for t in pin.values()) + pin_l.numel() * pin_l.element_size()
    return {"ms": e0.elapsed_time(e1) / steps, "h2d": h2d, "d2h": out_h.numel() * out_h.element_size()}


def run_head_shard(args, rank, world, local_rank):
    """Config 3 (8 x 32,768 tokens, 14/2 heads) decoded with its KV heads split
    over the ranks: each rank streams its heads' KV from its own pools and one
    all-gather per layer rebuilds [B, Hq, D].  The all-gather runs two ways:
    pa_head_allgather (peer stores over NVLink of self-validating lines, the
    default `transport="peer"`) and NCCL's all_gather_into_tensor.  Layers x
    (decode + all-gather) are captured in one CUDA graph; `value` is the whole
    batch's algorithmic KV bytes per second with the peer all-gather (max over
    ranks)."""
    import torch.distributed as dist

    from mini_llm_runtime_b200 import _lib
    from mini_llm_runtime_b200.head_shard import HeadShardedDecode, head_slices

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29531")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=device)
    _lib.load()
    layers = 4
    ctx = np.full(8, 32768, dtype=np.int64)
    q_sl, kv_sl = head_slices(HQ, HKV, world, rank)
    hq_l, hkv_l = q_sl.stop - q_sl.start, kv_sl.stop - kv_sl.start
    rng = np.random.default_rng(13)
    tables, nb = _random_tables(rng, ctx, BS)
    gen = torch.Generator(device=device).manual_seed(13 + rank)
    k = _bf16_randn((layers, nb, BS, hkv_l, D), device, gen)
    v = _bf16_randn((layers, nb, BS, hkv_l, D), device, gen)
    q = _bf16_randn((layers, len(ctx), hq_l, D), device, gen)
    bt, cl = torch.tensor(tables, device=device), torch.tensor(ctx, device=device)
    out = torch.empty(layers, len(ctx), HQ, D, dtype=torch.bfloat16, device=device)
    part = torch.empty(layers, world, len(ctx), hq_l, D, dtype=torch.bfloat16, device=device)
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream())

    def measure(transport: str, fuse: bool = True) -> dict:
        hs = HeadShardedDecode(HQ, HKV, transport=transport, max_batch=len(ctx), fuse=fuse)

        def body(gather_only=False):
            for l in range(layers):
                if not gather_only:
                    hs(q[l], k[l], v[l], bt, cl, BS, out=out[l])
                elif transport == "peer":
                    hs._peer(q[l], out[l])
                else:
                    dist.all_gather_into_tensor(part[l], q[l].contiguous())

        with torch.cuda.stream(s):
            body()  # the peer transport maps the peers' exchange areas here
            body(True)
        torch.cuda.synchronize()

        def time_graph(gather_only: bool) -> float:
            # A graph holding NCCL calls must be gone before the process group
            # is destroyed, so it lives only inside this function.
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                body(gather_only)
            for _ in range(max(args.warmup, 3)):
                graph.replay()
            dist.barrier(device_ids=[local_rank])
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            del graph
            t = torch.tensor([e0.elapsed_time(e1) / (args.steps * layers)], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        r = {"step": time_graph(False), "gather": time_graph(True)}
        hs.check()
        hs.close()
        return r

    peer = measure("peer")
    unfused = measure("peer", fuse=False)
    coll = measure("collective")
    torch.cuda.synchronize()
    kv = int(ctx.sum()) * HKV * D * 2 * 2
    if rank == 0:
        print(json.dumps({
            "mode": "head-shard", "metric": METRIC, "value": kv / (peer["step"] * 1e-3) / 1e9, "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
            "data": "synthetic", "ms_per_layer": peer["step"],
            "transport": "pa_paged_decode_allgather: the decode's merge kernel stores its output rows into the "
                         "peers' memory over NVLink as lines carrying the call number and polls for theirs",
            "unfused": {"value": kv / (unfused["step"] * 1e-3) / 1e9, "ms_per_layer": unfused["step"],
                        "allgather_ms_per_layer": unfused["gather"],
                        "transport": "decode, then pa_head_allgather (a kernel of its own)"},
            "nccl": {"value": kv / (coll["step"] * 1e-3) / 1e9, "ms_per_layer": coll["step"],
                     "allgather_ms_per_layer": coll["gather"]},
            "config": {"workload": "config3: 8 x 32768 tokens, 14/2 heads, D64, bs16, KV heads split over the "
                                   "GPUs, all-gather of the [B, Hq/N, D] head outputs per layer",
                       "layers_in_graph": layers}}), flush=True)
    dist.barrier(device_ids=[local_rank])
    dist.destroy_process_group()


def run_mixed(args, rank, world, local_rank):
    """BASELINE config 5 as one mixed step: per layer, the prefill chunks'
    KV write (pa_kv_scatter), one batched chunk-prefill (pa_chunk_prefill,
    tcgen05) and one decode with the fused KV write (balanced kernel), 28
    layers at 28/4 heads, D 128, bs 16; random Q/K/V ~ N(0, 1).  Requests are
    sharded over the ranks longest first (decodes by context, chunks by
    causal work).  One CUDA graph per step; the same layers as decode-only
    and prefill-only graphs give the split.  `value` is the whole job's
    decode KV GB/s; time is the max over ranks."""
    from mini_llm_runtime_b200 import PagedKVCache, _lib, paged_attention_prefill_varlen, paged_decode_with_kv_write
    from mini_llm_runtime_b200.sharding import decode_cost, prefill_cost, shard_requests

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29541")
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=device)
    _lib.load()
    L5, HQ5, HKV5, D5 = 28, 28, 4, 128
    ctx_all = np.random.default_rng(5).integers(256, 8193, size=256).astype(np.int64)
    prefix_all = np.random.default_rng(6).integers(0, 4097, size=4).astype(np.int64)
    chunk_all = np.full(4, 1024, dtype=np.int64)
    dec = shard_requests([decode_cost(c) for c in ctx_all], world)[rank].requests
    pre = shard_requests([prefill_cost(p, c) for p, c in zip(prefix_all, chunk_all)], world)[rank].requests
    ctx_d = ctx_all[dec]
    prefix, chunk = prefix_all[pre], chunk_all[pre]
    ctx_p = prefix + chunk
    nd, npf = len(ctx_d), len(pre)
    rng = np.random.default_rng(500 + rank)
    tables, nb = _random_tables(rng, np.concatenate([ctx_d, ctx_p]), BS)
    cache = PagedKVCache(L5, nb, BS, HKV5, D5, dtype=torch.bfloat16, device=device)
    gen = torch.Generator(device=device).manual_seed(600 + rank)
    cache.k_cache.normal_(generator=gen)
    cache.v_cache.normal_(generator=gen)
    bt = torch.tensor(tables, device=device)
    bt_d, bt_p = bt[:nd], bt[nd:]
    cl_d = torch.tensor(ctx_d, device=device)
    cl_p = torch.tensor(ctx_p, device=device)
    pos_d = ctx_d - 1
    slots_d = torch.tensor(tables[np.arange(nd), pos_d // BS] * BS + pos_d % BS, device=device)
    tp = int(chunk.sum())
    seq_p = np.repeat(np.arange(npf), chunk)
    pos_p = (np.arange(tp) - np.concatenate([[0], np.cumsum(chunk)[:-1]])[seq_p] + prefix[seq_p]) if tp else seq_p
    slots_p = torch.tensor(tables[nd + seq_p, pos_p // BS] * BS + pos_p % BS, device=device) if tp else None
    cu_p = torch.tensor(np.concatenate([[0], np.cumsum(chunk)]), device=device)
    q_d = _bf16_randn((L5, nd, HQ5, D5), device, gen)
    nk_d = _bf16_randn((L5, nd, HKV5, D5), device, gen)
    nv_d = _bf16_randn((L5, nd, HKV5, D5), device, gen)
    q_p = _bf16_randn((L5, tp, HQ5, D5), device, gen) if tp else None
    k_p = _bf16_randn((L5, tp, HKV5, D5), device, gen) if tp else None
    v_p = _bf16_randn((L5, tp, HKV5, D5), device, gen) if tp else None
    max_q = int(chunk.max()) if npf else 0

    def body(do_prefill: bool, do_decode: bool):
        for l in range(L5):
            if do_prefill and tp:
                cache.write_slots(slots_p, k_p[l], v_p[l], layer_idx=l, validate=False)
                paged_attention_prefill_varlen(q_p[l], cu_p, cl_p, bt_p, cache.k_cache[l], cache.v_cache[l], max_q)
            if do_decode and nd:
                paged_decode_with_kv_write(q_d[l], nk_d[l], nv_d[l], slots_d, cache.k_cache[l], cache.v_cache[l],
                                           bt_d, cl_d, BS)

    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        body(True, True)
    torch.cuda.synchronize()

    def time_graph(do_prefill: bool, do_decode: bool) -> float:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            body(do_prefill, do_decode)
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        del graph
        t = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device=device)
        if dist is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms = {"step": time_graph(True, True), "decode_only": time_graph(False, True),
          "prefill_only": time_graph(True, False)}
    _lib.check_device_status(device)
    kv_total = int(ctx_all.sum()) * HKV5 * D5 * 2 * 2 * L5  # decode KV bytes per step, all ranks
    flops_total = prefill_flops(prefix_all, chunk_all, HQ5, D5) * L5
    kv_rank = int(ctx_d.sum()) * HKV5 * D5 * 2 * 2 * L5
    flops_rank = prefill_flops(prefix, chunk, HQ5, D5) * L5 if npf else 0
    ideal = torch.tensor([(kv_rank / (hbm_peak()[0] * 1e9) + flops_rank / (bf16_peak()[0] * 1e12)) * 1e3],
                         dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(ideal, op=dist.ReduceOp.MAX)
    if rank == 0:
        step_s = ms["step"] * 1e-3
        print(json.dumps({
            "mode": "mixed", "metric": METRIC, "value": kv_total / step_s / 1e9, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms["step"], "higher_is_better": True,
            "scaling": "strong", "dtype": "bf16", "data": "synthetic",
            "prefill_tflops": flops_total / step_s / 1e12,
            "tok_per_s": (len(ctx_all) + int(chunk_all.sum())) / step_s,
            "ms_decode_only": ms["decode_only"], "ms_prefill_only": ms["prefill_only"],
            "roofline": {"ideal_ms": float(ideal.item()), "frac": float(ideal.item()) / ms["step"],
                         "model": "max over ranks of (decode KV bytes / measured HBM peak + prefill FLOPs / "
                                  "measured BF16 peak), the two in sequence"},
            "config": {"workload": "config5: mixed step, 28 layers x (prefill KV write + chunk-prefill of 4 x 1024 "
                                   "on prefix U[0,4096] + decode with fused KV write of 256 seqs, ctx U[256,8192]), "
                                   "28/4 heads, D128, bs16, requests sharded longest first",
                       "parallelism": f"request-sharded dp{world}, no communication"}}), flush=True)
    if dist is not None:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def main():
    args = parse_args()
    rank, world, local_rank = env_rank()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.kernel:
        run_kernel_case(args)
        return
    if args.mode == "head-shard":
        run_head_shard(args, rank, world, local_rank)
        return
    if args.mode == "mixed":
        run_mixed(args, rank, world, local_rank)
        return

    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    from mini_llm_runtime_b200 import PagedDecodeGraph, _lib

    _lib.load()
    w = build_rank_workload(rank, world, device)
    nbytes = algorithmic_bytes(w["ctx"])
    warmup = max(args.warmup, 3)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    def reduce(x: float, op) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=op)
        return float(t.item())

    batch = len(w["ctx"])
    mk = lambda **kw: PagedDecodeGraph(w["cache"], batch, w["width"], HQ, range(LAYERS), **kw)  # noqa: E731

    # ---- device-resident step: KV write + decode for 24 layers, one graph --
    g_dev = mk(host_io=False)
    stage(g_dev, w["inputs"], device_resident=True)
    g_dev.validate({k: w["inputs"][k] for k in ("context_lens", "block_tables", "slot_mapping")})
    for _ in range(warmup):
        g_dev.run(validate=False)
    # nvidia-smi samples every 100 ms: keep the same step running (untimed)
    # for about a second so the samples see the load the timed region runs
    # under, then time K steps straight after.
    sampler = ClockSampler(physical_gpu_index(local_rank))
    sampler.start()
    soak_end = time.perf_counter() + 1.0
    while time.perf_counter() < soak_end:
        for _ in range(50):
            g_dev.run(validate=False)
        torch.cuda.synchronize()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        g_dev.run(validate=False)
    t1.record()
    barrier()
    clocks = sampler.stop()
    ms_step = reduce(t0.elapsed_time(t1) / args.steps, dist.ReduceOp.MAX if world > 1 else None)

    # ---- decode kernel alone (roofline): 24 decode launches, one graph -----
    g_dec = mk(host_io=False, write_kv=False)
    stage(g_dec, w["inputs"], device_resident=True)
    for _ in range(warmup):
        g_dec.run(validate=False)
    torch.cuda.synchronize()
    d0 = torch.cuda.Event(enable_timing=True)
    d1 = torch.cuda.Event(enable_timing=True)
    d0.record()
    for _ in range(args.steps):
        g_dec.run(validate=False)
    d1.record()
    torch.cuda.synchronize()
    dec_ms = d0.elapsed_time(d1) / (args.steps * LAYERS)

    # ---- end to end: pinned host inputs -> H2D -> step -> D2H, host checks --
    g_e2e = mk(host_io=True)
    stage(g_e2e, w["inputs"], device_resident=False)
    h2d = sum(t.numel() * t.element_size() for t in g_e2e.host_inputs.values())
    d2h = g_e2e.host_output.numel() * g_e2e.host_output.element_size()
    for _ in range(warmup):
        g_e2e.run(validate=True)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        g_e2e.run(validate=True)
    e1.record()
    barrier()
    e2e_ms = reduce(e0.elapsed_time(e1) / args.steps, dist.ReduceOp.MAX if world > 1 else None)

    # ---- end to end per layer: the drop-in call, one layer at a time --------
    # Each layer copies its own q / new_k / new_v from pinned host memory,
    # calls paged_decode_with_kv_write (the fused write_slots + batched decode
    # of Qwen2Attention.forward_decode_batch_with_cache) and copies its output
    # back, all on the current stream; the metadata goes over once per step.
    e2l = run_per_layer_e2e(w, device, args.steps, warmup, barrier)
    e2l_ms = reduce(e2l["ms"], dist.ReduceOp.MAX if world > 1 else None)

    total_kv = reduce(nbytes["kv"] * LAYERS, dist.ReduceOp.SUM if world > 1 else None)
    tokens = reduce(batch, dist.ReduceOp.SUM if world > 1 else None)
    value = total_kv / (ms_step * 1e-3) / 1e9
    e2e_value = total_kv / (e2e_ms * 1e-3) / 1e9

    peak, peak_kind = hbm_peak()
    achieved = nbytes["decode"] / (dec_ms * 1e-3) / 1e9
    traffic = None
    tfile = ROOT / "profiles" / "decode_bf16_config2_traffic.txt"
    if tfile.exists():
        for line in tfile.read_text().splitlines():
            if line.startswith("dram_bytes_per_launch:"):
                traffic = float(line.split(":", 1)[1])

    # ---- secondary configs, one kernel at a time (same GPU, after the step) --
    # With N > 1 every rank times the same case on its own GPU at the same
    # time, and the slowest rank's launch time is reported.
    secondary = {}
    for name in ("split-config3", "prefill-config4", "decode-config5", "prefill-config5", "decode-config2-fp8",
                 "decode-config5-fp8"):
        barrier()
        r = time_kernel_case(name, device)
        entry = {k: r[k] for k in ("workload", "us_per_launch", "achieved", "unit", "frac")}
        if world > 1:
            us = reduce(r["us_per_launch"], dist.ReduceOp.MAX)
            scale = 1e9 if r["bound"] == "hbm" else 1e12
            entry.update(us_per_launch=us, achieved=r["work_per_launch"] / (us * 1e-6) / scale,
                         ranks=world, timing="max over ranks, every rank running the case at once")
            entry["frac"] = entry["achieved"] / r["peak"]
        secondary[name] = entry
        torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = cpu_reference_sample(steps=20, warmup=2, layers=1)
        cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "spread")}

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": warmup,
            "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": bench_config(world, batch),
            "launch": "one CUDA graph per step: 24 x (decode with the fused KV write + combine), "
                      "PA_DECODE_EARLY_INPUTS",
            "tok_per_s": tokens / (ms_step * 1e-3),
            "frac_of_hbm_peak": value / world / peak,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms, "tok_per_s": tokens / (e2e_ms * 1e-3),
                    "path": "PagedDecodeGraph.run(): host metadata checks, pinned H2D, 24x(KV write+decode), D2H"},
            "e2e_per_layer": {"value": total_kv / (e2l_ms * 1e-3) / 1e9, "unit": UNIT,
                              "h2d_bytes_per_step": e2l["h2d"], "d2h_bytes_per_step": e2l["d2h"],
                              "ms_per_step": e2l_ms,
                              "path": "24 x paged_decode_with_kv_write, each with its layer's pinned H2D of "
                                      "q/new_k/new_v (one packed copy) and D2H of its output"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                         "kernel": "decode_flat_kernel<bf16,64>",
                         "bytes_per_launch": nbytes["decode"], "avg_launch_ms": dec_ms},
            "secondary": secondary,
            "gpu_launches": args.steps * g_dev.launches_per_step,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "env": run_env(),
        }
        print(json.dumps(line), flush=True)
    # Graphs go before the process group.
    del g_dev, g_dec, g_e2e
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

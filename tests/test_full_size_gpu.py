"""Parity at the full benched sizes: the inputs of every bench.py kernel case
(one layer, the bench's own seeds) through the CUDA
path, each output row checked against the oracle.

The oracle runs per sequence on that sequence's blocks only (gathered on the
device, copied to the host), so the FP32 host copies stay small even for the
2.4 GB config-5 pools.  Tolerance (north_star, BF16 against FP32 math on the
same BF16 inputs): 2e-2 absolute / 1e-2 relative.
"""

from __future__ import annotations

import concurrent.futures as cf
import os

import numpy as np
import pytest
import torch

import bench
from oracle import paged_attention_oracle as O

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-2, atol=2e-2)
HOST_BATCH = 16  # sequences gathered to the host at a time


def _gather(pool: torch.Tensor, table_row: np.ndarray, need: int, scale: float = 1.0) -> np.ndarray:
    """A sequence's blocks of a pool on the host in FP32 (FP8 pools: the
    dequantized values, element * scale)."""
    idx = torch.as_tensor(np.ascontiguousarray(table_row[:need]), device=pool.device)
    blocks = pool.index_select(0, idx)
    if blocks.dtype == torch.float8_e4m3fn:
        return O.dequantize_e4m3(blocks.view(torch.uint8).cpu().numpy(), scale)
    return blocks.float().cpu().numpy()


def oracle_case(inp: dict) -> np.ndarray:
    """The oracle's result for layer 0 of a bench kernel case."""
    q, k, v = inp["q"][0], inp["k"][0], inp["v"][0]
    bs = k.shape[1]
    tables, ctx = inp["tables"], inp["ctx"]
    q_np = q.float().cpu().numpy()
    out = np.empty(q_np.shape, dtype=np.float32)
    decode = inp["kind"] == "decode"
    if not decode:
        cu = np.concatenate([[0], np.cumsum(inp["chunk"])])
    workers = max(1, min(16, os.cpu_count() or 1))

    def run(b: int, kb: np.ndarray, vb: np.ndarray) -> None:
        need = kb.shape[0]
        table = np.arange(need)
        if decode:
            out[b] = O.decode_single(q_np[b], kb, vb, table, int(ctx[b]), bs)
            return
        prefix, c0 = int(inp["prefix"][b]), int(cu[b])
        step = 256  # query rows per oracle call: rows [i0, i1) see positions <= prefix + i
        for i0 in range(0, int(inp["chunk"][b]), step):
            i1 = min(i0 + step, int(inp["chunk"][b]))
            out[c0 + i0:c0 + i1] = O.prefill_chunk(q_np[c0 + i0:c0 + i1], kb, vb, table, prefix + i0, prefix + i1,
                                                   bs)

    with cf.ThreadPoolExecutor(workers) as ex:
        for b0 in range(0, len(ctx), HOST_BATCH):
            batch = []
            for b in range(b0, min(b0 + HOST_BATCH, len(ctx))):
                need = (int(ctx[b]) + bs - 1) // bs
                batch.append((b, _gather(k, tables[b], need, inp.get("k_scale", 1.0)),
                              _gather(v, tables[b], need, inp.get("v_scale", 1.0))))
            list(ex.map(lambda a: run(*a), batch))
    return out


@pytest.mark.parametrize("name", ["decode-config2", "decode-config2-fp8", "split-config3", "prefill-config4",
                                  "decode-config5", "prefill-config5"])
def test_bench_case_matches_oracle_at_full_size(cuda_device, name):
    build = bench.KERNEL_CASES[name][0]
    case = build(cuda_device, 1)
    out = case["fn"](0)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all(), "NaN/Inf in kernel output"
    expected = oracle_case(case["inputs"])
    np.testing.assert_allclose(got, expected, **TOL)
    del case, out
    torch.cuda.empty_cache()

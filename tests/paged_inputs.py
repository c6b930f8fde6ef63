"""Seeded paged-cache inputs shared by the GPU parity tests.

Follows the reference's input generation (benchmarks/benchmark_paged_attention.py
:437-512): block tables from a seeded randperm over the pool, padded with -1;
Q/K/V ~ N(0, 1) in the test dtype.  Slots that no sequence owns (whole
unused blocks and the tail of each sequence's last block) hold NaN, as in
tests/kernels/test_paged_attention.py:292-297, so any read outside the block
table poisons the output.
"""

from __future__ import annotations

import numpy as np
import torch


def to_f32_numpy(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def make_decode_case(
    ctx: list[int],
    hq: int,
    hkv: int,
    d: int,
    bs: int,
    dtype: torch.dtype,
    device,
    seed: int = 0,
    extra_blocks: int = 3,
    reverse_tables: bool = False,
    poison: bool = True,
):
    g = torch.Generator().manual_seed(seed)
    need = [(c + bs - 1) // bs for c in ctx]
    nb = sum(need) + extra_blocks
    perm = torch.randperm(nb, generator=g).tolist()
    width = max(need)
    tables, cur = [], 0
    for n in need:
        row = perm[cur : cur + n]
        if reverse_tables:
            row = row[::-1]
        cur += n
        tables.append(row + [-1] * (width - n))
    fill = float("nan") if poison else 0.0
    k = torch.full((nb, bs, hkv, d), fill, dtype=torch.float32)
    v = torch.full((nb, bs, hkv, d), fill, dtype=torch.float32)
    for b, c in enumerate(ctx):
        pos = torch.arange(c)
        blk = torch.tensor(tables[b][: need[b]])[pos // bs]
        k[blk, pos % bs] = torch.randn(c, hkv, d, generator=g)
        v[blk, pos % bs] = torch.randn(c, hkv, d, generator=g)
    q = torch.randn(len(ctx), hq, d, generator=g)
    k, v, q = k.to(dtype), v.to(dtype), q.to(dtype)
    return {
        "q": q.to(device),
        "k": k.to(device),
        "v": v.to(device),
        "tables": torch.tensor(tables, dtype=torch.long, device=device),
        "lens": torch.tensor(ctx, dtype=torch.long, device=device),
        "np": (to_f32_numpy(q), to_f32_numpy(k), to_f32_numpy(v), np.array(tables), np.array(ctx)),
        "bs": bs,
    }


def make_prefill_case(
    prefix: list[int],
    chunk: list[int],
    hq: int,
    hkv: int,
    d: int,
    bs: int,
    dtype: torch.dtype,
    device,
    seed: int = 0,
    extra_blocks: int = 3,
):
    """Varlen chunk-prefill batch: sequence s has prefix[s] cached tokens and a
    chunk of chunk[s] new tokens already written into the pools."""
    ctx = [p + c for p, c in zip(prefix, chunk)]
    case = make_decode_case(ctx, hq, hkv, d, bs, dtype, device, seed, extra_blocks)
    g = torch.Generator().manual_seed(seed + 1000)
    total = sum(chunk)
    q = torch.randn(total, hq, d, generator=g).to(dtype)
    cu = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int64)
    case.update(
        q=q.to(device),
        q_np=to_f32_numpy(q),
        cu=torch.tensor(cu, device=device),
        cu_np=cu,
        prefix=prefix,
        chunk=chunk,
        ctx=ctx,
        max_q=max(chunk),
    )
    return case

"""Single-long-sequence decode sharded by KV head across GPUs.

Request sharding (sharding.py) cannot spread a batch of a few very long
sequences: one sequence's KV is the unit of work.  Attention heads are
independent, though, so such a batch can split by KV head instead: rank r of
``g`` ranks keeps only KV heads ``[r * Hkv/g, (r+1) * Hkv/g)`` of every layer's
pool (``[NB, bs, Hkv/g, D]``), gets the query heads of those KV heads' GQA
groups (``[r * Hq/g, (r+1) * Hq/g)``, contiguous because head ``h`` reads KV
head ``h // (Hq/Hkv)``), decodes them with the balanced decode kernel, and one
all-gather of the ``[B, Hq/g, D]`` head outputs rebuilds ``[B, Hq, D]`` on
every rank.  Each rank streams 1/g of the KV bytes; the all-gather moves
``B * Hq * D`` elements (14 KB for 8 sequences of Qwen2.5-0.5B geometry), so
the collective is latency-bound, not bandwidth-bound.

This is the one place a collective sits on the path: NCCL over NVLink
(``torch.distributed``, backend "nccl"); the head outputs arrive through NCCL
into local memory.  The reference runs one process on one device
(runtime/model_runner.py:146-288), so it has no counterpart; the per-rank math
is its paged_attention_decode_batch_parallel
(kernels/reference/paged_attention.py:178-254) on a head slice.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def head_slices(num_q_heads: int, num_kv_heads: int, world_size: int, rank: int) -> tuple[slice, slice]:
    """(query-head slice, KV-head slice) owned by ``rank``."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("rank must lie in [0, world_size)")
    if num_q_heads % num_kv_heads != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if num_kv_heads % world_size != 0:
        raise ValueError(f"num_kv_heads ({num_kv_heads}) must be divisible by the world size ({world_size})")
    kv_per, q_per = num_kv_heads // world_size, num_q_heads // world_size
    return slice(rank * q_per, (rank + 1) * q_per), slice(rank * kv_per, (rank + 1) * kv_per)


def shard_pool(pool: torch.Tensor, kv_slice: slice) -> torch.Tensor:
    """This rank's contiguous copy of a pool ``[..., bs, Hkv, D]`` (one layer
    or all layers): only its KV heads."""
    return pool[..., kv_slice, :].contiguous()


class HeadShardedDecode:
    """Batched paged decode of this rank's KV heads plus the all-gather of the
    head outputs.

    ``local_decode(q_local, k_pool_local, v_pool_local, block_tables,
    context_lens, block_size)`` computes ``[B, Hq/g, D]``; by default it is
    paged_attention_decode_batch_parallel (the CUDA kernels).  Tests on CPU
    ranks pass the oracle instead.  Every rank must call with the same
    metadata (the block tables and context lengths are shared; only the pools
    and query heads are split).
    """

    def __init__(
        self,
        num_q_heads: int,
        num_kv_heads: int,
        group: dist.ProcessGroup | None = None,
        local_decode: Callable | None = None,
    ):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.hq, self.hkv = num_q_heads, num_kv_heads
        self.q_slice, self.kv_slice = head_slices(num_q_heads, num_kv_heads, self.world, self.rank)
        if local_decode is None:
            from .paged_attention import paged_attention_decode_batch_parallel as local_decode
        self.local_decode = local_decode
        self._nccl = dist.get_backend(group) == "nccl"

    def local_queries(self, q: torch.Tensor) -> torch.Tensor:
        """This rank's query heads of a full ``[B, Hq, D]`` query."""
        return q[:, self.q_slice]

    def __call__(
        self,
        q_local: torch.Tensor,
        k_pool_local: torch.Tensor,
        v_pool_local: torch.Tensor,
        block_tables: torch.Tensor,
        context_lens: torch.Tensor,
        block_size: int,
        out: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """[B, Hq/g, D] local queries -> [B, Hq, D] attention output on every rank."""
        b, hq_local, d = q_local.shape
        if hq_local * self.world != self.hq or k_pool_local.shape[2] * self.world != self.hkv:
            raise ValueError("q_local / pools do not hold this rank's share of the heads")
        part = self.local_decode(q_local, k_pool_local, v_pool_local, block_tables, context_lens, block_size)
        gathered = torch.empty((self.world, b, hq_local, d), dtype=part.dtype, device=part.device)
        if self._nccl:
            dist.all_gather_into_tensor(gathered, part.contiguous(), group=self.group)
        else:
            dist.all_gather(list(gathered.unbind(0)), part.contiguous(), group=self.group)
        full = gathered.permute(1, 0, 2, 3).reshape(b, self.hq, d)
        if out is None:
            return full
        out.copy_(full)
        return out

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

This is the one place an exchange between GPUs sits on the path.  By default
(``transport="peer"`` on CUDA ranks) it is fused into the decode
(``pa_paged_decode_allgather``): the decode's merge kernel stores each CTA's
finished output rows straight into every peer's memory over NVLink (CUDA IPC
mappings set up once) as lines that carry the call's number, and polls
(bounded) for the peers' rows.  Where that path is unsupported (or with
``fuse=False``) the decode is followed by ``pa_head_allgather``, the same
exchange as a kernel of its own.  ``transport="collective"`` runs
``torch.distributed`` all-gather instead (NCCL on GPUs, gloo on CPU ranks).  The reference runs one process on one device
(runtime/model_runner.py:146-288), so it has no counterpart; the per-rank math
is its paged_attention_decode_batch_parallel
(kernels/reference/paged_attention.py:178-254) on a head slice.
"""

from __future__ import annotations

import ctypes
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib


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


class PeerHeadGather:
    """All-gather of ``[B, heads_local, D]`` head outputs over NVLink peer
    memory: ``pa_head_allgather`` on this rank's exchange area and its IPC
    mappings of every peer's.  Construction is collective (every rank of
    ``group`` builds one with the same arguments): it exports this rank's
    area, maps every peer's and ends with a barrier.  Calls must follow the
    same sequence on every rank; they may be captured in a CUDA graph."""

    def __init__(self, group: dist.ProcessGroup | None, max_batch: int, heads_local: int, head_dim: int,
                 dtype: torch.dtype, device: torch.device, wait_limit_ns: int = 0,
                 kv_heads_local: int | None = None):
        lib = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.PA_PEER_MAX_RANKS:
            raise ValueError(f"at most {_lib.PA_PEER_MAX_RANKS} ranks share a peer all-gather")
        self.device = torch.device(device)
        self.max_batch, self.heads_local, self.head_dim, self.dtype = max_batch, heads_local, head_dim, dtype
        self.wait_limit_ns = wait_limit_ns
        esize = torch.empty((), dtype=dtype).element_size()
        nbytes = lib.pa_peer_gather_bytes(self.world, max_batch * heads_local * head_dim * esize)
        if nbytes == 0:
            raise ValueError("invalid peer all-gather size")
        if kv_heads_local is not None:
            # Room for the decode with the exchange fused into it as well.
            nbytes = max(nbytes, lib.pa_decode_allgather_bytes(max_batch, kv_heads_local, heads_local, head_dim,
                                                               self.world))
        # Above the caching allocator's 10 MB split limit the area gets a
        # segment (one cudaMalloc) of its own: its IPC handle is distinct from
        # every other area's, and a peer maps it exactly once.
        self.area = torch.zeros(max(nbytes, 12 << 20), dtype=torch.uint8, device=self.device)
        if self.area.data_ptr() % 256:
            raise _lib.PagedAttentionError("exchange area is not 256-byte aligned")
        handle = ctypes.create_string_buffer(_lib.PA_IPC_HANDLE_BYTES)
        offset = ctypes.c_uint64()
        _lib.check(lib.pa_ipc_export(self.area.data_ptr(), handle, ctypes.byref(offset)), "pa_ipc_export")
        torch.cuda.synchronize(self.device)  # zeroed before any peer can write into it
        infos: list = [None] * self.world
        dist.all_gather_object(infos, (handle.raw, offset.value), group=group)
        ptrs, self._bases = [], []
        for r, (h, off) in enumerate(infos):
            if r == self.rank:
                ptrs.append(self.area.data_ptr())
                continue
            ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
            _lib.check(lib.pa_ipc_import(h, off, ctypes.byref(ptr), ctypes.byref(base)), "pa_ipc_import")
            ptrs.append(ptr.value)
            self._bases.append(base.value)
        self._areas = (ctypes.c_void_p * self.world)(*ptrs)
        self._nbytes = nbytes
        self._barrier()  # every area is zeroed and mapped on every rank

    def _barrier(self) -> None:
        if dist.get_backend(self.group) == "nccl":
            dist.barrier(group=self.group, device_ids=[self.device.index])
        else:
            dist.barrier(group=self.group)

    def __call__(self, part: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """part [B, heads_local, D] -> out [B, world * heads_local, D]."""
        b, hl, d = part.shape
        if hl != self.heads_local or d != self.head_dim or b > self.max_batch or part.dtype != self.dtype:
            raise ValueError("part does not match the exchange this all-gather was built for")
        if tuple(out.shape) != (b, hl * self.world, d) or out.dtype != part.dtype:
            raise ValueError("out must be [B, world * heads_local, D] of part's dtype")
        if part.stride(2) != 1 or out.stride(2) != 1:
            raise ValueError("head_dim must be contiguous")
        _lib.check(
            _lib.load().pa_head_allgather(
                part.data_ptr(), part.stride(0), part.stride(1), b, hl, d, _lib.dtype_code(part.dtype), self.rank,
                self.world, self._areas, self._nbytes, out.data_ptr(), out.stride(0), out.stride(1),
                self.wait_limit_ns, _lib.stream_handle(part.device)),
            "pa_head_allgather")
        return out

    def status(self) -> int:
        """0, or PA_DEVICE_TIMEOUT_PEER when a wait for a peer gave up
        (synchronises the device)."""
        return int(self.area[136:140].view(torch.int32).item())

    def check(self) -> None:
        code = self.status()
        if code:
            raise _lib.PagedAttentionError(
                f"peer all-gather: {_lib.load().pa_status_string(code).decode()} (status {code})")

    def close(self) -> None:
        """Unmap the peers' areas (collective: ends with a barrier, after which
        each rank may free its own area)."""
        torch.cuda.synchronize(self.device)
        lib = _lib.load()
        for base in self._bases:
            _lib.check(lib.pa_ipc_close(base), "pa_ipc_close")
        self._bases = []
        self._barrier()


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
        transport: str = "peer",
        max_batch: int = 256,
        fuse: bool = True,
    ):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.hq, self.hkv = num_q_heads, num_kv_heads
        self.q_slice, self.kv_slice = head_slices(num_q_heads, num_kv_heads, self.world, self.rank)
        # With the package's own decode the exchange rides inside it
        # (pa_paged_decode_allgather); a custom local_decode is followed by it.
        self._fusable = fuse and local_decode is None and self.world > 1
        if local_decode is None:
            from .paged_attention import paged_attention_decode_batch_parallel as local_decode
        self.local_decode = local_decode
        self._nccl = dist.get_backend(group) == "nccl"
        if transport not in ("peer", "collective"):
            raise ValueError("transport must be 'peer' or 'collective'")
        # The peer exchange needs CUDA ranks; CPU (gloo) ranks use the collective.
        self.transport = transport if self._nccl else "collective"
        self.max_batch = max_batch
        self._peer: PeerHeadGather | None = None

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
        if self.transport == "peer":
            peer = self._peer
            if peer is None or peer.dtype != q_local.dtype or b > peer.max_batch:
                # Collective set-up: every rank reaches it at the same call
                # (the same metadata on every rank).
                if peer is not None:
                    peer.close()
                peer = self._peer = PeerHeadGather(self.group, max(b, self.max_batch), hq_local, d, q_local.dtype,
                                                   q_local.device, kv_heads_local=k_pool_local.shape[2])
            if out is None:
                out = torch.empty((b, self.hq, d), dtype=q_local.dtype, device=q_local.device)
            if self._fusable:
                from .paged_attention import decode_allgather_launch

                lo = self.rank * hq_local
                st = decode_allgather_launch(q_local, k_pool_local, v_pool_local, block_tables, context_lens,
                                             block_size, out[:, lo:lo + hq_local], self.rank, self.world,
                                             peer._areas, peer._nbytes, peer.wait_limit_ns)
                if st == _lib.PA_OK:
                    return out
                # PA_ERR_UNSUPPORTED (nothing launched, same answer on every
                # rank for the same shapes): decode, then the exchange kernel.
            part = self.local_decode(q_local, k_pool_local, v_pool_local, block_tables, context_lens, block_size)
            return peer(part, out)
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

    def check(self) -> None:
        """Raise PagedAttentionError if a peer wait gave up (synchronises)."""
        if self._peer is not None:
            self._peer.check()

    def close(self) -> None:
        """Release the peer mappings (collective)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None

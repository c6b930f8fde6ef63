"""Qwen2Attention with its paged methods running on this library's kernels.

The reference's attention module (model/qwen2.py:243-767) reaches the paged
hot path through three methods:

* ``forward_decode_with_cache`` (:441-539), one request, one token;
* ``forward_decode_batch_with_cache`` (:542-622), one token per request;
* ``forward_prefill_chunk_with_cache`` (:624-767), one request, a chunk.

Each validates its metadata before touching the cache, projects Q/K/V, applies
RoPE, writes the new K/V rows through ``PagedKVCache.write_slots`` and runs
paged attention, then ``o_proj``.  This module keeps those signatures, the
checks (same order, exception types and messages) and the parameter names
(``qkv_proj.{q,k,v}_proj``, ``o_proj``), so a reference state dict loads
unchanged.  The KV write and the attention run the CUDA kernels of
``libpagedattn.so``.  The projections and RoPE are plain PyTorch: dense GEMMs
and elementwise work outside the paged path.

The reference validates batch metadata with a chain of ``torch.any`` calls,
each a device->host sync.  Here the metadata comes to the host in ONE copy
and is checked with numpy; the conditions and messages are the same.

``forward_prefill_batch_with_cache`` is the batched varlen chunk-prefill over
``ModelBatch``-style metadata (``query_start_loc`` / ``context_lens`` /
``block_tables``, runtime/model_runner.py:14-27).  The reference has no such
method: its runner loops per request.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn

from .paged_attention import (
    paged_attention_decode,
    paged_attention_decode_batch_parallel,
    paged_attention_prefill_chunk_tiled,
    paged_attention_prefill_varlen,
    paged_decode_with_kv_write,
)
from .paged_kv_cache import PagedKVCache


def new_token_blocks_private(context_lens: np.ndarray, block_tables: np.ndarray, block_size: int) -> bool:
    """True when no sequence's context reaches the block that receives
    another sequence's new token.  The fused write + decode patches the new
    rows into the decoding sequence's own staged K/V only, so a block shared
    with another sequence's context must take the unfused write-then-decode
    order instead."""
    need = (context_lens + block_size - 1) // block_size
    width = block_tables.shape[1]
    used = np.arange(width)[None, :] < need[:, None]
    pos = context_lens - 1
    new_blocks = block_tables[np.arange(len(context_lens)), pos // block_size]
    blocks = block_tables[used]
    counts = np.bincount(blocks[blocks >= 0], minlength=int(new_blocks.max()) + 1 if len(new_blocks) else 1)
    return bool(np.all(counts[new_blocks] == 1))


def check_decode_metadata(context_lens: np.ndarray, block_tables: np.ndarray, slot_mapping: np.ndarray,
                          positions: np.ndarray | None, block_size: int, num_blocks: int) -> None:
    """The page-metadata checks of forward_decode_batch_with_cache
    (model/qwen2.py:590-620), in the same order and with the same messages,
    on host arrays.  ``positions`` None skips the position check (callers
    that derive positions from context_lens)."""
    if np.any(context_lens <= 0):
        raise ValueError("context_lens must be greater than 0")
    if positions is not None and np.any(positions != context_lens - 1):
        raise ValueError("decode positions must equal context_lens - 1")
    need = (context_lens + block_size - 1) // block_size
    if np.any(need > block_tables.shape[1]):
        raise ValueError("block_tables have insufficient blocks for context_lens")
    used = np.arange(block_tables.shape[1])[None, :] < need[:, None]
    if np.any(used & ((block_tables < 0) | (block_tables >= num_blocks))):
        raise ValueError("block_tables contain an invalid physical block")
    pos = context_lens - 1
    expected = block_tables[np.arange(len(context_lens)), pos // block_size] * block_size + pos % block_size
    if np.any(slot_mapping != expected):
        raise ValueError("slot_mapping must match block_tables and positions")
    if np.unique(slot_mapping).size != slot_mapping.size:
        raise ValueError("decode requests must use distinct write slots")


class Qwen2RotaryEmbedding(nn.Module):
    """cos/sin tables of rotary position embedding (model/qwen2.py:125-172):
    inv_freq = theta^(-2i/D), angles in FP32, both halves identical."""

    def __init__(self, head_dim: int, theta: float = 1_000_000.0) -> None:
        super().__init__()
        if head_dim <= 0 or head_dim % 2 != 0:
            raise ValueError("head_dim must be a positive even integer")
        if theta <= 0:
            raise ValueError("theta must be greater than 0")
        self.head_dim = head_dim
        self.theta = theta
        exponent = torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim
        self.register_buffer("inv_freq", 1.0 / (theta ** exponent), persistent=False)

    def forward(self, hidden_states: torch.Tensor, position_ids: torch.Tensor):
        if tuple(hidden_states.shape[:-2]) != tuple(position_ids.shape):
            raise ValueError("position_ids shape must match hidden_states dimensions before the head dimensions")
        angles = position_ids.to(hidden_states.device, torch.float32).unsqueeze(-1) * self.inv_freq.to(
            hidden_states.device)
        angles = torch.cat((angles, angles), dim=-1)
        return angles.cos().to(hidden_states.dtype), angles.sin().to(hidden_states.dtype)


def apply_rotary_pos_emb(query: torch.Tensor, key: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """x*cos + rotate_half(x)*sin on [..., heads, D] (model/qwen2.py:175-211),
    rotate_half(x) = cat(-x2, x1) over the two contiguous halves."""

    def rot(x: torch.Tensor) -> torch.Tensor:
        a, b = x.chunk(2, dim=-1)
        return torch.cat((-b, a), dim=-1)

    cos = cos.to(query.dtype).unsqueeze(-2)
    sin = sin.to(query.dtype).unsqueeze(-2)
    return query * cos + rot(query) * sin, key * cos + rot(key) * sin


class Qwen2QKVProjection(nn.Module):
    """q/k/v projections with bias (model/qwen2.py:213-240), reshaped to heads."""

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: int) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.num_attention_heads = num_heads
        self.num_key_value_heads = num_kv_heads
        self.hidden_dim = head_dim
        self.q_proj = nn.Linear(hidden_size, num_heads * head_dim)
        self.v_proj = nn.Linear(hidden_size, num_kv_heads * head_dim)
        self.k_proj = nn.Linear(hidden_size, num_kv_heads * head_dim)

    def forward(self, hidden_states: torch.Tensor):
        if hidden_states.shape[-1] != self.hidden_size:
            raise ValueError("Unexpect input shape")
        lead = hidden_states.shape[:-1]
        q = self.q_proj(hidden_states).reshape(lead + (self.num_attention_heads, self.hidden_dim))
        k = self.k_proj(hidden_states).reshape(lead + (self.num_key_value_heads, self.hidden_dim))
        v = self.v_proj(hidden_states).reshape(lead + (self.num_key_value_heads, self.hidden_dim))
        return q, k, v


def _is_fp8(kv_cache) -> bool:
    return getattr(kv_cache, "is_fp8", False)


def _scales(kv_cache, layer_idx: int) -> dict:
    """The layer's FP8 pool scales as op keywords ({} for 16/32-bit pools and
    for caches without scales, such as the reference's own PagedKVCache)."""
    if not _is_fp8(kv_cache):
        return {}
    ks, vs = kv_cache.layer_scales(layer_idx)
    return {"k_scale": ks, "v_scale": vs}


class Qwen2Attention(nn.Module):
    """Drop-in for the reference's Qwen2Attention paged methods.

    ``config`` is any object with hidden_size, num_attention_heads,
    num_key_value_heads and rope_theta (the reference's TinyQwen2Config, or a
    transformers Qwen2Config); head_dim = hidden_size / num_attention_heads.
    """

    def __init__(self, config) -> None:
        super().__init__()
        self.hidden_size = int(config.hidden_size)
        self.num_attention_heads = int(config.num_attention_heads)
        self.num_key_value_heads = int(config.num_key_value_heads)
        if self.hidden_size % self.num_attention_heads or self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("hidden_size / heads / kv heads must divide evenly")
        self.num_key_value_groups = self.num_attention_heads // self.num_key_value_heads
        self.head_dim = self.hidden_size // self.num_attention_heads
        self.scale = self.head_dim ** -0.5
        self.qkv_proj = Qwen2QKVProjection(self.hidden_size, self.num_attention_heads, self.num_key_value_heads,
                                           self.head_dim)
        self.rotary_embedding = Qwen2RotaryEmbedding(self.head_dim, float(getattr(config, "rope_theta", 1e6)))
        self.o_proj = nn.Linear(self.hidden_size, self.hidden_size, bias=False)

    # -- shared pieces ---------------------------------------------------------
    def project(self, hidden_states: torch.Tensor, position_ids: torch.Tensor):
        """QKV projection + RoPE (model/qwen2.py:604-606): the tensors the
        paged path receives."""
        q, k, v = self.qkv_proj(hidden_states)
        cos, sin = self.rotary_embedding(q, position_ids)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        return q, k, v

    def _check_hidden(self, hidden_states: torch.Tensor, position_ids: torch.Tensor, what: str) -> None:
        if hidden_states.shape[-1] != self.hidden_size:
            raise ValueError(
                "hidden_states last dimension must match hidden_size "
                f"({self.hidden_size}), got {hidden_states.shape[-1]}")
        if position_ids.shape != hidden_states.shape[:2]:
            raise ValueError(
                "position_ids shape must match hidden_states batch and "
                f"{what} dimensions {tuple(hidden_states.shape[:2])}, got {tuple(position_ids.shape)}")

    # -- model/qwen2.py:441-539 ------------------------------------------------
    def forward_decode_with_cache(self, hidden_states, position_ids, kv_cache: PagedKVCache, layer_idx: int,
                                  slot_mapping, block_table: list[int], context_len: int) -> torch.Tensor:
        if hidden_states.ndim != 3:
            raise ValueError(
                f"hidden_states must have shape [1, 1, hidden_size], got {tuple(hidden_states.shape)}")
        if hidden_states.shape[0] != 1:
            raise ValueError(
                f"decode with cache currently supports exactly one request, got batch_size={hidden_states.shape[0]}")
        if hidden_states.shape[1] != 1:
            raise ValueError(f"decode with cache requires exactly one input token, got {hidden_states.shape[1]}")
        self._check_hidden(hidden_states, position_ids, "sequence")
        if slot_mapping.ndim != 1 or slot_mapping.shape[0] != 1:
            raise ValueError(f"slot_mapping must have shape [1] for decode, got {tuple(slot_mapping.shape)}")
        if context_len <= 0:
            raise ValueError("context_len must be greater than 0")
        pos = int(position_ids.reshape(-1)[0])
        if pos != context_len - 1:
            raise ValueError(
                "decode position must equal context_len - 1, "
                f"got position={pos} and context_len={context_len}")
        q, k, v = self.project(hidden_states, position_ids)
        kv_cache.write_slots(slot_mapping=slot_mapping, k=k.squeeze(1), v=v.squeeze(1), layer_idx=layer_idx)
        k_layer, v_layer = kv_cache.get_layer_cache(layer_idx)
        out = paged_attention_decode(q[0, 0], k_layer, v_layer, block_table, context_len, kv_cache.block_size,
                                     **_scales(kv_cache, layer_idx))
        return self.o_proj(out.reshape(1, 1, self.hidden_size))

    # -- model/qwen2.py:542-622 ------------------------------------------------
    def forward_decode_batch_with_cache(self, hidden_states, position_ids, kv_cache: PagedKVCache, layer_idx: int,
                                        slot_mapping, block_tables, context_lens) -> torch.Tensor:
        """Decode one token per request; context lengths include this token."""
        if hidden_states.ndim != 3 or hidden_states.shape[1:] != (1, self.hidden_size):
            raise ValueError("hidden_states must have shape [B, 1, hidden_size]")
        batch = hidden_states.shape[0]
        if batch == 0:
            raise ValueError("decode batch must not be empty")
        if position_ids.shape != (batch, 1):
            raise ValueError("position_ids must have shape [B, 1]")
        if slot_mapping.shape != (batch,):
            raise ValueError("slot_mapping must have shape [B]")
        if context_lens.shape != (batch,):
            raise ValueError("context_lens must have shape [B]")
        if block_tables.ndim != 2 or block_tables.shape[0] != batch:
            raise ValueError("block_tables must have shape [B, max_num_blocks]")
        for name, t in (("position_ids", position_ids), ("slot_mapping", slot_mapping),
                        ("context_lens", context_lens), ("block_tables", block_tables)):
            if t.dtype != torch.long:
                raise ValueError(f"{name} must use torch.long dtype")
            if t.device != hidden_states.device:
                raise ValueError(f"{name} must be on the hidden_states device")
        if kv_cache.k_cache.device != hidden_states.device:
            raise ValueError("KV cache must be on the hidden_states device")
        if kv_cache.dtype != hidden_states.dtype and not _is_fp8(kv_cache):
            raise ValueError("KV cache dtype must match hidden_states dtype")
        # One device->host copy of all metadata, then the reference's checks.
        w = block_tables.shape[1]
        host = torch.cat([position_ids[:, 0], slot_mapping, context_lens, block_tables.reshape(-1)]).cpu().numpy()
        check_decode_metadata(host[2 * batch:3 * batch], host[3 * batch:].reshape(batch, w), host[batch:2 * batch],
                              host[:batch], kv_cache.block_size, kv_cache.num_blocks)
        fused = new_token_blocks_private(host[2 * batch:3 * batch], host[3 * batch:].reshape(batch, w),
                                         kv_cache.block_size)
        return self.decode_batch_planned(hidden_states, position_ids, kv_cache, layer_idx, slot_mapping,
                                         block_tables, context_lens, fused)

    def decode_batch_planned(self, hidden_states, position_ids, kv_cache: PagedKVCache, layer_idx: int,
                             slot_mapping, block_tables, context_lens, fused: bool) -> torch.Tensor:
        """The compute of forward_decode_batch_with_cache on metadata the
        caller has already checked (once per scheduler step, for every
        layer): no device->host copy.  ``fused`` (new_token_blocks_private of
        the step's metadata) selects the one-launch KV write + decode."""
        batch = hidden_states.shape[0]
        k_layer, v_layer = kv_cache.get_layer_cache(layer_idx)
        q, k, v = self.project(hidden_states, position_ids)
        if fused:
            out = paged_decode_with_kv_write(q.squeeze(1), k.squeeze(1), v.squeeze(1), slot_mapping, k_layer,
                                             v_layer, block_tables, context_lens, kv_cache.block_size,
                                             **_scales(kv_cache, layer_idx))
        else:
            kv_cache.write_slots(slot_mapping=slot_mapping, k=k.squeeze(1), v=v.squeeze(1), layer_idx=layer_idx,
                                 validate=False)
            out = paged_attention_decode_batch_parallel(q.squeeze(1), k_layer, v_layer, block_tables, context_lens,
                                                        kv_cache.block_size, **_scales(kv_cache, layer_idx))
        return self.o_proj(out.reshape(batch, 1, self.hidden_size))

    # -- model/qwen2.py:624-767 ------------------------------------------------
    def forward_prefill_chunk_with_cache(self, hidden_states, position_ids, kv_cache: PagedKVCache, layer_idx: int,
                                         slot_mapping, block_table: list[int], prefix_len: int, context_len: int,
                                         tile_size: int) -> torch.Tensor:
        if hidden_states.ndim != 3:
            raise ValueError(
                f"hidden_states must have shape [1, chunk_len, hidden_size], got {tuple(hidden_states.shape)}")
        if hidden_states.shape[0] != 1:
            raise ValueError(
                f"chunk prefill currently supports exactly one request, got batch_size={hidden_states.shape[0]}")
        chunk = hidden_states.shape[1]
        if chunk == 0:
            raise ValueError("chunk_len must be greater than 0")
        self._check_hidden(hidden_states, position_ids, "chunk")
        if position_ids.dtype not in (torch.int32, torch.int64):
            raise TypeError("position_ids must use an integer dtype")
        if slot_mapping.ndim != 1 or slot_mapping.shape[0] != chunk:
            raise ValueError(f"slot_mapping must have shape [chunk_len], got {tuple(slot_mapping.shape)}")
        if prefix_len < 0:
            raise ValueError("prefix_len cannot be negative")
        if context_len != prefix_len + chunk:
            raise ValueError(
                "context_len must equal prefix_len + chunk_len, "
                f"got prefix_len={prefix_len}, chunk_len={chunk}, and context_len={context_len}")
        if tile_size <= 0:
            raise ValueError("tile_size must be greater than 0")
        bs = kv_cache.block_size
        # One copy of positions and slots to the host for the contiguity and slot checks.
        host = torch.cat([position_ids.reshape(-1).long(), slot_mapping.long()]).cpu().numpy()
        if not np.array_equal(host[:chunk], np.arange(prefix_len, context_len)):
            raise ValueError(
                "position_ids must contain the contiguous global positions from prefix_len through context_len - 1")
        need = (context_len + bs - 1) // bs
        if len(block_table) < need:
            raise ValueError("block_table does not contain enough blocks for context_len")
        used = np.asarray(list(block_table[:need]), dtype=np.int64)
        if np.any((used < 0) | (used >= kv_cache.num_blocks)):
            raise ValueError("block_table contains an out-of-range physical block")
        pos = np.arange(prefix_len, context_len)
        if not np.array_equal(host[chunk:], used[pos // bs] * bs + pos % bs):
            raise ValueError("slot_mapping does not match block_table for the chunk positions")
        q, k, v = self.project(hidden_states, position_ids)
        kv_cache.write_slots(slot_mapping=slot_mapping, k=k.squeeze(0), v=v.squeeze(0), layer_idx=layer_idx)
        k_layer, v_layer = kv_cache.get_layer_cache(layer_idx)
        out = paged_attention_prefill_chunk_tiled(q.squeeze(0), k_layer, v_layer, block_table, prefix_len,
                                                  context_len, bs, tile_size, **_scales(kv_cache, layer_idx))
        return self.o_proj(out.reshape(1, chunk, self.hidden_size))

    # -- batched varlen chunk-prefill (no reference counterpart) --------------
    def forward_prefill_batch_with_cache(self, hidden_states, position_ids, kv_cache: PagedKVCache, layer_idx: int,
                                         slot_mapping, query_start_loc, block_tables, context_lens) -> torch.Tensor:
        """Chunks of several requests packed as hidden_states [1, T, H]:
        request s owns rows [query_start_loc[s], query_start_loc[s+1]) at
        positions context_lens[s] - chunk_s ... context_lens[s] - 1."""
        if hidden_states.ndim != 3 or hidden_states.shape[0] != 1:
            raise ValueError("hidden_states must have shape [1, total_tokens, hidden_size]")
        self._check_hidden(hidden_states, position_ids, "token")
        total = hidden_states.shape[1]
        nseq = context_lens.shape[0]
        if query_start_loc.shape != (nseq + 1,) or block_tables.ndim != 2 or block_tables.shape[0] != nseq:
            raise ValueError("query_start_loc must be [num_seqs + 1] and block_tables [num_seqs, max_num_blocks]")
        if slot_mapping.shape != (total,):
            raise ValueError("slot_mapping must have shape [total_tokens]")
        bs = kv_cache.block_size
        w = block_tables.shape[1]
        host = torch.cat([query_start_loc.long(), context_lens.long(), position_ids.reshape(-1).long(),
                          slot_mapping.long(), block_tables.reshape(-1).long()]).cpu().numpy()
        cu = host[:nseq + 1]
        lens = host[nseq + 1:2 * nseq + 1]
        pos = host[2 * nseq + 1:2 * nseq + 1 + total]
        slots = host[2 * nseq + 1 + total:2 * nseq + 1 + 2 * total]
        tables = host[2 * nseq + 1 + 2 * total:].reshape(nseq, w)
        chunks = np.diff(cu)
        if cu[0] != 0 or cu[-1] != total or np.any(chunks < 0):
            raise ValueError("query_start_loc must rise from 0 to total_tokens")
        if np.any(lens < chunks):
            raise ValueError("context_lens must cover each request's chunk")
        need = (lens + bs - 1) // bs
        if np.any(need > w):
            raise ValueError("block_tables have insufficient blocks for context_lens")
        used = np.arange(w)[None, :] < need[:, None]
        if np.any(used & ((tables < 0) | (tables >= kv_cache.num_blocks))):
            raise ValueError("block_tables contain an invalid physical block")
        seq = np.repeat(np.arange(nseq), chunks)
        expect_pos = np.arange(total) - cu[seq] + (lens - chunks)[seq]
        if np.any(pos != expect_pos):
            raise ValueError("position_ids must be each request's contiguous chunk positions")
        if np.any(slots != tables[seq, expect_pos // bs] * bs + expect_pos % bs):
            raise ValueError("slot_mapping must match block_tables and positions")
        if np.unique(slots).size != total:
            raise ValueError("slot_mapping must contain distinct slots")
        return self.prefill_batch_planned(hidden_states, position_ids, kv_cache, layer_idx, slot_mapping,
                                          query_start_loc, block_tables, context_lens,
                                          int(chunks.max()) if nseq else 0)

    def prefill_batch_planned(self, hidden_states, position_ids, kv_cache: PagedKVCache, layer_idx: int,
                              slot_mapping, query_start_loc, block_tables, context_lens, max_q: int) -> torch.Tensor:
        """The compute of forward_prefill_batch_with_cache on metadata the
        caller has already checked: no device->host copy.  ``max_q`` is the
        longest chunk."""
        total = hidden_states.shape[1]
        k_layer, v_layer = kv_cache.get_layer_cache(layer_idx)
        q, k, v = self.project(hidden_states, position_ids)
        kv_cache.write_slots(slot_mapping=slot_mapping, k=k.squeeze(0), v=v.squeeze(0), layer_idx=layer_idx,
                             validate=False)
        out = paged_attention_prefill_varlen(q.squeeze(0), query_start_loc, context_lens, block_tables, k_layer,
                                             v_layer, max_q, **_scales(kv_cache, layer_idx))
        return self.o_proj(out.reshape(1, total, self.hidden_size))

"""Paged-attention ops with the reference's Python signatures, on sm_100a CUDA.

Drop-in for ``mini_llm_runtime.kernels.reference.paged_attention``: the same
function names, arguments, output shapes/dtypes and ``ValueError`` messages,
but every call launches a hand-written kernel from libpagedattn.so through its
C ABI.  Inputs must be CUDA tensors; there is no CPU fallback.

Differences from the reference that callers can observe:
* no host synchronisation (the reference calls ``seq_lens.max().item()``,
  paged_attention.py:222);
* slots past a sequence's context length are never read (the reference's
  padded gather reads block 0 / tail slots and multiplies them by 0, so a NaN
  there poisons its output — paged_attention.py:232-235, :253);
* BF16/F16 inputs keep scores and probabilities in FP32 inside the kernel
  (the reference rounds scores and probabilities to the input dtype,
  paged_attention.py:247-253), so results are closer to the FP32 reference.
* the pools may be FP8 (torch.float8_e4m3fn, see PagedKVCache): pass the
  layer's ``k_scale`` / ``v_scale`` keywords; q and the output keep q.dtype.
"""

from __future__ import annotations

import math

import torch

from . import _lib

__all__ = [
    "paged_decode_with_kv_write",
    "paged_attention_decode",
    "paged_attention_decode_batch_parallel",
    "paged_attention_decode_split_kv",
    "paged_attention_prefill_chunk_tiled",
    "paged_attention_prefill_varlen",
    "paged_attention_accumulator_cuda",
]


def _check_caches(k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
    # paged_attention.py:17-24 / :189-196
    if k_cache.ndim != 4 or v_cache.ndim != 4:
        raise ValueError("k_cache and v_cache must have shape [num_blocks, block_size, Hkv, D]")
    if k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache must have the same shape")


def _pool_ok(k_cache: torch.Tensor, v_cache: torch.Tensor, dtype: torch.dtype) -> None:
    fp8 = k_cache.dtype == _lib.FP8_DTYPE and v_cache.dtype == _lib.FP8_DTYPE
    if not fp8 and (k_cache.dtype != dtype or v_cache.dtype != dtype):
        raise TypeError("q, k_cache and v_cache must share one dtype (or the pools are FP8)")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("k_cache and v_cache must be contiguous [num_blocks, block_size, Hkv, D] views")


def _as_long(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    if isinstance(t, torch.Tensor) and t.dtype is torch.long and t.device == device:
        return t
    t = torch.as_tensor(t, device=device)
    if t.dtype != torch.long:
        t = t.long()
    return t


def _decode_launch(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    out: torch.Tensor,
    partition_tokens: int,
    scale: float | None = None,
    k_scale: float = 1.0,
    v_scale: float = 1.0,
) -> torch.Tensor:
    dev = _lib.require_cuda(q, k_cache, v_cache, block_tables, seq_lens, out, what="paged decode")
    lib = _lib.load()
    b, hq, d = q.shape
    nb, bs, hkv, _ = k_cache.shape
    if q.stride(2) != 1 or out.stride(2) != 1:
        q = q.contiguous()
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    seq_lens = seq_lens.contiguous()
    code = _lib.dtype_code(q.dtype)
    width = block_tables.shape[1]
    ws_bytes = _lib.decode_workspace_bytes(b, hkv, hq, d, bs, width, partition_tokens, code)
    if ws_bytes == 0:
        raise ValueError("invalid decode arguments")
    ws = _lib.decode_workspace(dev, ws_bytes, b, hq)
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    with _lib.device_guard(dev):
        if k_cache.dtype == _lib.FP8_DTYPE:
            st = lib.pa_paged_decode_fp8(
                q.data_ptr(), q.stride(0), q.stride(1), None, None, None,
                k_cache.data_ptr(), v_cache.data_ptr(), nb, bs, hkv, d,
                block_tables.data_ptr(), block_tables.stride(0), width, seq_lens.data_ptr(),
                out.data_ptr(), out.stride(0), out.stride(1), b, hq, float(scale), code, float(k_scale),
                float(v_scale), int(partition_tokens), 0, ws.data_ptr(), ws.numel(), _lib.stream_handle(dev),
            )
        else:
            st = lib.pa_paged_decode(
                q.data_ptr(), q.stride(0), q.stride(1),
                k_cache.data_ptr(), v_cache.data_ptr(), nb, bs, hkv, d,
                block_tables.data_ptr(), block_tables.stride(0), width, seq_lens.data_ptr(),
                out.data_ptr(), out.stride(0), out.stride(1), b, hq, float(scale), code,
                int(partition_tokens), ws.data_ptr(), ws.numel(), _lib.stream_handle(dev),
            )
    _lib.check(st, "pa_paged_decode")
    _lib.after_launch(dev)
    return out


def paged_decode_with_kv_write(
    q: torch.Tensor,
    new_k: torch.Tensor,
    new_v: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    block_size: int,
    scale: float | None = None,
    *,
    k_scale: float = 1.0,
    v_scale: float = 1.0,
) -> torch.Tensor:
    """The decode step of Qwen2Attention.forward_decode_batch_with_cache
    (model/qwen2.py:608-621) in one fused launch: write the new token's K/V
    [B, Hkv, D] to ``slot_mapping`` of the layer pools, then decode
    q [B, Hq, D] over ``seq_lens`` tokens (which include the new one).

    Same results, bit for bit, as ``PagedKVCache.write_slots`` followed by
    ``paged_attention_decode_batch_parallel``.  ``slot_mapping[b]`` must be
    the slot of position ``seq_lens[b] - 1`` in ``block_tables[b]`` (what
    the reference's decode checks enforce) and no other sequence may read it;
    the caller validates, as ``Qwen2Attention`` and ``PagedDecodeGraph`` do.
    """
    if q.ndim != 3 or new_k.ndim != 3 or new_k.shape != new_v.shape:
        raise ValueError("q must be [B, Hq, D] and new_k / new_v [B, Hkv, D]")
    _check_caches(k_cache, v_cache)
    b, hq, d = q.shape
    nb, bs, hkv, dk = k_cache.shape
    if tuple(new_k.shape) != (b, hkv, dk) or d != dk:
        raise ValueError("new_k / new_v must have shape [B, Hkv, D] matching the cache")
    if hq % hkv != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if block_size != bs:
        raise ValueError("block_size does not match KV cache layout")
    if slot_mapping.shape != (b,) or block_tables.ndim != 2 or block_tables.shape[0] != b or seq_lens.shape != (b,):
        raise ValueError("slot_mapping / seq_lens must be [B] and block_tables [B, max_num_blocks]")
    dev = _lib.require_cuda(q, new_k, new_v, slot_mapping, k_cache, v_cache, block_tables, seq_lens,
                            what="paged_decode_with_kv_write")
    _pool_ok(k_cache, v_cache, q.dtype)
    fp8 = k_cache.dtype == _lib.FP8_DTYPE
    if new_k.dtype != q.dtype or new_v.dtype != q.dtype or (not fp8 and new_k.dtype != k_cache.dtype):
        raise TypeError("new_k / new_v must have the dtype of q (and of the KV cache unless it is FP8)")
    lib = _lib.load()
    new_k, new_v = new_k.contiguous(), new_v.contiguous()
    slots = _as_long(slot_mapping, dev).contiguous()
    block_tables = _as_long(block_tables, dev)
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    seq_lens = _as_long(seq_lens, dev).contiguous()
    if q.stride(2) != 1:
        q = q.contiguous()
    out = torch.empty((b, hq, d), dtype=q.dtype, device=dev)
    code = _lib.dtype_code(q.dtype)
    width = block_tables.shape[1]
    ws_bytes = _lib.decode_workspace_bytes(b, hkv, hq, d, bs, width, 0, code)
    if ws_bytes == 0:
        raise ValueError("invalid decode arguments")
    ws = _lib.decode_workspace(dev, ws_bytes, b, hq)
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    with _lib.device_guard(dev):
        if fp8:
            st = lib.pa_paged_decode_fp8(
                q.data_ptr(), q.stride(0), q.stride(1), new_k.data_ptr(), new_v.data_ptr(), slots.data_ptr(),
                k_cache.data_ptr(), v_cache.data_ptr(), nb, bs, hkv, d, block_tables.data_ptr(),
                block_tables.stride(0), width, seq_lens.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1), b,
                hq, float(scale), code, float(k_scale), float(v_scale), 0, 0, ws.data_ptr(), ws.numel(),
                _lib.stream_handle(dev),
            )
        else:
            st = lib.pa_paged_decode_write(
                q.data_ptr(), q.stride(0), q.stride(1), new_k.data_ptr(), new_v.data_ptr(), slots.data_ptr(),
                k_cache.data_ptr(), v_cache.data_ptr(), nb, bs, hkv, d, block_tables.data_ptr(),
                block_tables.stride(0), width, seq_lens.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1), b,
                hq, float(scale), code, ws.data_ptr(), ws.numel(), _lib.stream_handle(dev),
            )
    _lib.check(st, "pa_paged_decode_write")
    _lib.after_launch(dev)
    return out


def paged_attention_decode_batch_parallel(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    block_size: int,
    *,
    k_scale: float = 1.0,
    v_scale: float = 1.0,
) -> torch.Tensor:
    """Batched single-token decode: q [B, Hq, D] -> [B, Hq, D] (q.dtype).

    Same contract as the reference (kernels/reference/paged_attention.py:178-254):
    ``block_tables`` [B, W] (padded with -1), ``seq_lens`` [B] including the
    token being decoded, one layer's pools [num_blocks, block_size, Hkv, D].
    """
    if q.ndim != 3:
        raise ValueError("q must have shape [B, Hq, D]")
    _check_caches(k_cache, v_cache)
    num_query_heads, num_kv_heads, head_dim = q.shape[1], k_cache.shape[2], q.shape[-1]
    if head_dim != k_cache.shape[-1]:
        raise ValueError("q and KV cache must have the same head_dim")
    if num_query_heads % num_kv_heads != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if len(block_tables) != q.shape[0]:
        raise ValueError("block_tables length must match batch size of q")
    if len(seq_lens) != q.shape[0]:
        raise ValueError("seq_lens length must match batch size of q")
    if block_size != k_cache.shape[1]:
        raise ValueError("block_size does not match KV cache layout")
    _lib.require_cuda(q, k_cache, v_cache, what="paged_attention_decode_batch_parallel")
    _pool_ok(k_cache, v_cache, q.dtype)
    block_tables = _as_long(block_tables, q.device)
    seq_lens = _as_long(seq_lens, q.device)
    if block_tables.ndim != 2:
        raise ValueError("block_tables must have shape [B, max_num_blocks]")
    out = torch.empty_like(q, memory_format=torch.contiguous_format)
    return _decode_launch(q, k_cache, v_cache, block_tables, seq_lens, out, 0, k_scale=k_scale, v_scale=v_scale)


def decode_allgather_launch(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    block_size: int,
    out_local: torch.Tensor,
    rank: int,
    world: int,
    areas,
    area_bytes: int,
    wait_limit_ns: int = 0,
) -> int:
    """Batched decode of this rank's heads with the all-gather of head outputs
    fused into it (pa_paged_decode_allgather); KV-head-sharded decode.

    ``out_local`` is this rank's head slice ``[:, rank*Hq:(rank+1)*Hq]`` of the
    ``[B, world*Hq, D]`` output of all ranks; ``areas`` the ctypes array of every
    rank's exchange area.  Returns 0, or PA_ERR_UNSUPPORTED (nothing launched)
    when the call must take the unfused path; other errors raise.  The same
    checks as paged_attention_decode_batch_parallel run first."""
    if q.ndim != 3:
        raise ValueError("q must have shape [B, Hq, D]")
    _check_caches(k_cache, v_cache)
    num_query_heads, num_kv_heads, head_dim = q.shape[1], k_cache.shape[2], q.shape[-1]
    if head_dim != k_cache.shape[-1]:
        raise ValueError("q and KV cache must have the same head_dim")
    if num_query_heads % num_kv_heads != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if len(block_tables) != q.shape[0] or len(seq_lens) != q.shape[0]:
        raise ValueError("block_tables and seq_lens must match the batch size of q")
    if block_size != k_cache.shape[1]:
        raise ValueError("block_size does not match KV cache layout")
    dev = _lib.require_cuda(q, k_cache, v_cache, out_local, what="paged decode with head all-gather")
    if k_cache.dtype == _lib.FP8_DTYPE:
        return _lib.PA_ERR_UNSUPPORTED
    _pool_ok(k_cache, v_cache, q.dtype)
    block_tables = _as_long(block_tables, dev)
    seq_lens = _as_long(seq_lens, dev).contiguous()
    if block_tables.ndim != 2:
        raise ValueError("block_tables must have shape [B, max_num_blocks]")
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    if q.stride(2) != 1:
        q = q.contiguous()
    if tuple(out_local.shape) != tuple(q.shape) or out_local.dtype != q.dtype or out_local.stride(2) != 1:
        raise ValueError("out_local must be this rank's [B, Hq, D] slice of the gathered output")
    lib = _lib.load()
    b, hq, d = q.shape
    nb, bs, hkv, _ = k_cache.shape
    code = _lib.dtype_code(q.dtype)
    width = block_tables.shape[1]
    ws_bytes = _lib.decode_workspace_bytes(b, hkv, hq, d, bs, width, 0, code)
    if ws_bytes == 0:
        raise ValueError("invalid decode arguments")
    ws = _lib.decode_workspace(dev, ws_bytes, b, hq)
    with _lib.device_guard(dev):
        st = lib.pa_paged_decode_allgather(
            q.data_ptr(), q.stride(0), q.stride(1), None, None, None,
            k_cache.data_ptr(), v_cache.data_ptr(), nb, bs, hkv, d,
            block_tables.data_ptr(), block_tables.stride(0), width, seq_lens.data_ptr(),
            out_local.data_ptr(), out_local.stride(0), out_local.stride(1), b, hq, 1.0 / math.sqrt(d), code, 0,
            rank, world, areas, area_bytes, wait_limit_ns, ws.data_ptr(), ws.numel(), _lib.stream_handle(dev),
        )
    if st == _lib.PA_ERR_UNSUPPORTED:
        return st
    _lib.check(st, "pa_paged_decode_allgather")
    _lib.after_launch(dev)
    return st


def paged_attention_decode_split_kv(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    block_size: int,
    partition_size: int = 512,
    *,
    k_scale: float = 1.0,
    v_scale: float = 1.0,
) -> torch.Tensor:
    """Split-KV decode with an LSE merge, batched.

    The context of each sequence is cut into ``partition_size``-token
    partitions (rounded up to a multiple of 16); each partition's
    (max, sum, acc) partial is merged by log-sum-exp — the math of the
    reference's Triton split-KV pair (kernels/triton/paged_attention.py:24-213,
    stage 1 :528-700, merge :1530-1618), here for a whole batch in one launch.
    Accepts q [Hq, D] with a single block table / length like the Triton
    function, or q [B, Hq, D] with [B, W] tables and [B] lengths.
    """
    if partition_size <= 0:
        raise ValueError("partition_size must be greater than 0")
    single = q.ndim == 2
    if single:
        if isinstance(seq_lens, int) and seq_lens <= 0:
            raise ValueError("seq_len must be greater than 0")
        bt = torch.as_tensor(block_tables, dtype=torch.long, device=q.device).reshape(1, -1)
        sl = torch.as_tensor([int(seq_lens)] if isinstance(seq_lens, int) else seq_lens,
                             dtype=torch.long, device=q.device).reshape(1)
        q3 = q.unsqueeze(0)
    else:
        bt, sl, q3 = block_tables, seq_lens, q
    if q3.ndim != 3:
        raise ValueError("q must have shape [Hq, D] or [B, Hq, D]")
    _check_caches(k_cache, v_cache)
    if q3.shape[-1] != k_cache.shape[-1]:
        raise ValueError("q and KV cache must have the same head_dim")
    if q3.shape[1] % k_cache.shape[2] != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if block_size != k_cache.shape[1]:
        raise ValueError("block_size does not match KV cache layout")
    if len(bt) != q3.shape[0] or len(sl) != q3.shape[0]:
        raise ValueError("block_tables and seq_lens must match the batch size of q")
    _lib.require_cuda(q3, k_cache, v_cache, what="paged_attention_decode_split_kv")
    _pool_ok(k_cache, v_cache, q3.dtype)
    bt = _as_long(bt, q3.device)
    sl = _as_long(sl, q3.device)
    out = torch.empty_like(q3, memory_format=torch.contiguous_format)
    _decode_launch(q3, k_cache, v_cache, bt, sl, out, int(partition_size), k_scale=k_scale, v_scale=v_scale)
    return out[0] if single else out


def paged_attention_decode(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: list[int],
    seq_len: int,
    block_size: int,
    *,
    k_scale: float = 1.0,
    v_scale: float = 1.0,
) -> torch.Tensor:
    """Single-sequence decode: q [Hq, D] -> [Hq, D].

    Same contract and checks as the reference
    (kernels/reference/paged_attention.py:6-105); runs the batched kernel with
    B = 1.
    """
    if q.ndim != 2:
        raise ValueError("q must have shape [Hq, D]")
    _check_caches(k_cache, v_cache)
    num_query_heads, num_kv_heads, head_dim = q.shape[0], k_cache.shape[2], q.shape[-1]
    if head_dim != k_cache.shape[-1]:
        raise ValueError("q and KV cache must have the same head_dim")
    if num_query_heads % num_kv_heads != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if seq_len <= 0:
        raise ValueError("seq_len must be greater than 0")
    required_blocks = (seq_len + block_size - 1) // block_size
    if len(block_table) < required_blocks:
        raise ValueError("block_table does not contain enough blocks for seq_len")
    if block_size != k_cache.shape[1]:
        raise ValueError("block_size does not match KV cache layout")
    _lib.require_cuda(q, k_cache, v_cache, what="paged_attention_decode")
    _pool_ok(k_cache, v_cache, q.dtype)
    bt = torch.as_tensor(list(block_table)[:required_blocks], dtype=torch.long).to(q.device, non_blocking=True)
    sl = torch.tensor([seq_len], dtype=torch.long).to(q.device, non_blocking=True)
    q3 = q.unsqueeze(0)
    out = torch.empty_like(q3, memory_format=torch.contiguous_format)
    _decode_launch(q3, k_cache, v_cache, bt.reshape(1, -1), sl, out, 0, k_scale=k_scale, v_scale=v_scale)
    return out[0]


def _prefill_launch(
    q: torch.Tensor,
    cu_q_lens: torch.Tensor,
    context_lens: torch.Tensor,
    block_tables: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    max_q_len: int,
    scale: float | None = None,
    k_scale: float = 1.0,
    v_scale: float = 1.0,
) -> torch.Tensor:
    dev = _lib.require_cuda(q, cu_q_lens, context_lens, block_tables, k_cache, v_cache, what="chunk prefill")
    lib = _lib.load()
    total_q, hq, d = q.shape
    nb, bs, hkv, _ = k_cache.shape
    if q.stride(2) != 1:
        q = q.contiguous()
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    out = torch.empty((total_q, hq, d), dtype=q.dtype, device=q.device)
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    cu_q_lens, context_lens = cu_q_lens.contiguous(), context_lens.contiguous()
    with _lib.device_guard(dev):
        if k_cache.dtype == _lib.FP8_DTYPE:
            st = lib.pa_chunk_prefill_fp8(
                q.data_ptr(), q.stride(0), q.stride(1), cu_q_lens.data_ptr(), context_lens.data_ptr(),
                block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1], k_cache.data_ptr(),
                v_cache.data_ptr(), nb, bs, hkv, d, out.data_ptr(), out.stride(0), out.stride(1),
                cu_q_lens.shape[0] - 1, total_q, int(max_q_len), hq, float(scale), _lib.dtype_code(q.dtype),
                float(k_scale), float(v_scale), _lib.stream_handle(dev),
            )
        else:
            st = lib.pa_chunk_prefill(
                q.data_ptr(), q.stride(0), q.stride(1), cu_q_lens.data_ptr(), context_lens.data_ptr(),
                block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1], k_cache.data_ptr(),
                v_cache.data_ptr(), nb, bs, hkv, d, out.data_ptr(), out.stride(0), out.stride(1),
                cu_q_lens.shape[0] - 1, total_q, int(max_q_len), hq, float(scale), _lib.dtype_code(q.dtype),
                _lib.status_word(dev).data_ptr(), _lib.stream_handle(dev),
            )
    _lib.check(st, "pa_chunk_prefill")
    _lib.after_launch(dev)
    return out


def paged_attention_prefill_chunk_tiled(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: list[int] | torch.Tensor,
    prefix_len: int,
    context_len: int,
    block_size: int,
    tile_size: int,
    *,
    k_scale: float = 1.0,
    v_scale: float = 1.0,
) -> torch.Tensor:
    """Causal chunk-prefill for one request: q [C, Hq, D] -> [C, Hq, D].

    Same contract and checks as the reference
    (kernels/reference/paged_attention.py:346-434).  ``tile_size`` is
    validated like the reference; the kernel picks its own KV tiling (the
    result does not depend on it beyond FP32 rounding).
    """
    if tile_size <= 0:
        raise ValueError("tile_size must be greater than 0")
    if context_len != prefix_len + q.shape[0]:
        raise ValueError("context_len must equal prefix_len + q.shape[0]")
    if q.shape[1] % k_cache.shape[2] != 0:
        raise ValueError("q_num_heads must be divisible by kv_num_heads")
    _check_caches(k_cache, v_cache)
    if block_size != k_cache.shape[1]:
        raise ValueError("block_size does not match KV cache layout")
    _lib.require_cuda(q, k_cache, v_cache, what="paged_attention_prefill_chunk_tiled")
    _pool_ok(k_cache, v_cache, q.dtype)
    dev = q.device
    if isinstance(block_table, torch.Tensor):
        bt = block_table.to(device=dev, dtype=torch.long).reshape(1, -1)
    else:
        bt = torch.tensor(list(block_table), dtype=torch.long).to(dev, non_blocking=True).reshape(1, -1)
    if bt.shape[1] * block_size < context_len:
        raise ValueError("block_table does not contain enough blocks for context_len")
    meta = torch.tensor([0, q.shape[0], context_len], dtype=torch.long).to(dev, non_blocking=True)
    return _prefill_launch(q, meta[:2], meta[2:], bt, k_cache, v_cache, q.shape[0], k_scale=k_scale, v_scale=v_scale)


def paged_attention_prefill_varlen(
    q: torch.Tensor,
    cu_q_lens: torch.Tensor,
    context_lens: torch.Tensor,
    block_tables: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    max_q_len: int,
    scale: float | None = None,
    *,
    k_scale: float = 1.0,
    v_scale: float = 1.0,
) -> torch.Tensor:
    """Batched causal chunk-prefill over packed queries (ModelBatch layout).

    q [T, Hq, D] packs the chunks of all sequences; sequence s owns rows
    [cu_q_lens[s], cu_q_lens[s+1]) (``ModelBatch.query_start_loc``,
    runtime/model_runner.py:14-27) and sees ``context_lens[s]`` cached tokens
    including its chunk, through ``block_tables[s]``.  Query i of a chunk
    attends to positions <= context_len - chunk_len + i.  ``max_q_len`` is an
    upper bound of the chunk lengths.
    """
    if q.ndim != 3:
        raise ValueError("q must have shape [T, Hq, D]")
    _check_caches(k_cache, v_cache)
    if q.shape[-1] != k_cache.shape[-1]:
        raise ValueError("q and KV cache must have the same head_dim")
    if q.shape[1] % k_cache.shape[2] != 0:
        raise ValueError("q_num_heads must be divisible by kv_num_heads")
    if cu_q_lens.ndim != 1 or context_lens.ndim != 1 or cu_q_lens.shape[0] != context_lens.shape[0] + 1:
        raise ValueError("cu_q_lens must have shape [num_seqs + 1] and context_lens [num_seqs]")
    if block_tables.ndim != 2 or block_tables.shape[0] != context_lens.shape[0]:
        raise ValueError("block_tables must have shape [num_seqs, max_num_blocks]")
    _lib.require_cuda(q, k_cache, v_cache, what="paged_attention_prefill_varlen")
    _pool_ok(k_cache, v_cache, q.dtype)
    return _prefill_launch(
        q, _as_long(cu_q_lens, q.device), _as_long(context_lens, q.device), _as_long(block_tables, q.device),
        k_cache, v_cache, max_q_len, scale, k_scale, v_scale,
    )


def paged_attention_accumulator_cuda(p: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Batched ``sum_n p[n] * v[n, d]`` for N=64, D=256 (FP32).

    Same checks and result as the reference's extension
    (kernels/cuda/accumulator.py:21-37).
    """
    if not p.is_cuda or not v.is_cuda:
        raise ValueError("p and v must be CUDA tensors")
    if p.dtype != torch.float32 or v.dtype != torch.float32:
        raise TypeError("p and v must have dtype torch.float32")
    if p.ndim != 2 or p.shape[1] != 64:
        raise ValueError("p must have shape [batch, 64]")
    if v.ndim != 3 or v.shape[1:] != (64, 256):
        raise ValueError("v must have shape [batch, 64, 256]")
    if p.shape[0] != v.shape[0]:
        raise ValueError("p and v must have the same batch dimension")
    dev = _lib.require_cuda(p, v, what="paged_attention_accumulator_cuda")
    p = p.contiguous()
    v = v.contiguous()
    out = torch.empty((p.shape[0], 256), dtype=torch.float32, device=p.device)
    with _lib.device_guard(dev):
        st = _lib.load().pa_accumulate_pv(p.data_ptr(), v.data_ptr(), out.data_ptr(), p.shape[0],
                                          _lib.stream_handle(dev))
    _lib.check(st, "pa_accumulate_pv")
    return out

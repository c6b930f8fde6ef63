"""CPU oracle for the paged-attention hot path — TEST INFRASTRUCTURE ONLY.

This module is a numpy restatement of mini-llm-runtime's PyTorch reference
path.  It is the checker the parity tests compare the CUDA kernels against,
and the timed CPU baseline of ``bench.py --impl reference``.  Nothing in the
product package imports it; the product path has no CPU fallback.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference itself
(imported from its source tree) on seeded inputs and stores inputs/outputs as
``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks every function
here against those vectors (bit-exact for the scatter, 1e-6 for FP32 math).

Every function cites the reference code it restates
(paths inside src/mini_llm_runtime/).
"""

from __future__ import annotations

import math

import numpy as np

# ---------------------------------------------------------------------------
# bfloat16 / float16 rounding (integer arithmetic, round-to-nearest-even)
# ---------------------------------------------------------------------------


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (uint16), round-to-nearest-even.

    Same rounding as ``tensor.to(torch.bfloat16)`` (c10 round_to_nearest_even)
    for finite values; NaN maps to the quiet NaN 0x7fc0 as c10 does on the CPU.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    rounded = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = np.uint16(0x7FC0)
    return rounded


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns (uint16) -> float32 (exact)."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 values rounded to the nearest bfloat16, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def round_to_f16(x: np.ndarray) -> np.ndarray:
    """float32 values rounded to the nearest float16 (numpy RNE), as float32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


# ---------------------------------------------------------------------------
# FP8 (e4m3, "fn": no infinities, max finite 448) KV-pool elements
# ---------------------------------------------------------------------------

E4M3_MAX = 448.0


def f32_to_e4m3_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> e4m3fn bit patterns (uint8): saturate to +-448, round to
    nearest even; every NaN -> 0x7f.  For non-NaN inputs the same bytes as
    ``torch.clamp(x, -448, 448).to(torch.float8_e4m3fn)`` (c10's
    round-to-nearest-even cast; the clamp because torch's plain cast maps
    overflow to NaN).  NaN signs are not kept: GPU arithmetic on a NaN (the
    division by the scale) returns the canonical positive NaN.  The reference
    has no FP8 pool; this is the storage format the FP8 PagedKVCache defines."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    sign = (np.signbit(x).astype(np.uint8)) << 7
    a = np.minimum(np.abs(x), np.float32(E4M3_MAX)).astype(np.float32)
    u = a.view(np.uint32).astype(np.int64)
    exp = (u >> 23) - 127
    out = np.zeros(x.shape, dtype=np.int64)
    normal = exp >= -6
    # Normal range: keep 3 mantissa bits, round to nearest even on the 20 dropped.
    lsb = (u >> 20) & 1
    r = (u + 0x7FFFF + lsb) >> 20  # (exponent << 3 | mantissa), float32 bias
    out = np.where(normal, r - ((127 - 7) << 3), out)
    # Subnormal range: multiples of 2^-9, nearest even (np.rint is RNE).
    sub = np.rint(np.nan_to_num(a.astype(np.float64)) * 512.0).astype(np.int64)
    out = np.where(normal, out, sub)
    out = out.astype(np.uint8) | sign
    nan = np.isnan(x)
    if nan.any():
        out = out.copy()
        out[nan] = 0x7F
    return out


def e4m3_bits_to_f32(b: np.ndarray) -> np.ndarray:
    """e4m3fn bit patterns -> float32 (exact)."""
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * 2.0 ** (e - 7.0))
    val = np.where((e == 0xF) & (m == 0x7), np.nan, val)
    return (s * val).astype(np.float32)


def quantize_e4m3(x: np.ndarray, scale: float) -> np.ndarray:
    """Stored FP8 byte of each element: e4m3(x / scale), the division in FP32."""
    return f32_to_e4m3_bits(np.asarray(x, dtype=np.float32) / np.float32(scale))


def dequantize_e4m3(bits: np.ndarray, scale: float) -> np.ndarray:
    """What attention reads from an FP8 pool: element * scale (FP32)."""
    return e4m3_bits_to_f32(bits) * np.float32(scale)


# ---------------------------------------------------------------------------
# KV-cache write
# ---------------------------------------------------------------------------


def write_slots(
    k_pool: np.ndarray,
    v_pool: np.ndarray,
    slot_mapping: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    layer_idx: int,
) -> None:
    """In-place scatter of k/v rows into flat slots of one layer.

    Restates PagedKVCache.write_slots (runtime/paged_kv_cache.py:194-249):
    pools are [L, NB, bs, Hkv, D]; layer ``layer_idx`` is flattened to
    [NB*bs, Hkv, D] (:243-244) and row t goes to slot slot_mapping[t] after a
    cast to the pool dtype (:245-249).  The pools here are float32 arrays that
    hold values of the pool dtype; callers round the source beforehand with
    :func:`round_to_bf16` / :func:`round_to_f16` to emulate a BF16/F16 pool.
    Validation (range / distinctness, :228-239) is the caller's job.
    """
    L, NB, bs, H, D = k_pool.shape
    flat_k = k_pool.reshape(L, NB * bs, H, D)
    flat_v = v_pool.reshape(L, NB * bs, H, D)
    idx = np.asarray(slot_mapping, dtype=np.int64)
    flat_k[layer_idx, idx] = k
    flat_v[layer_idx, idx] = v


# ---------------------------------------------------------------------------
# Decode
# ---------------------------------------------------------------------------


def _softmax_lastdim(scores: np.ndarray) -> np.ndarray:
    # torch.softmax(dim=-1, dtype=float32): exp(x - max) / sum
    m = np.max(scores, axis=-1, keepdims=True)
    e = np.exp(scores - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def decode_single(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    block_table,
    seq_len: int,
    block_size: int,
    dtype=np.float32,
) -> np.ndarray:
    """One sequence, one query token: q [Hq, D] -> [Hq, D].

    Restates paged_attention_decode (kernels/reference/paged_attention.py:6-105):
    per-position block lookup (:70-80), GQA by repeating KV heads (:89-91),
    scores = q k^T * 1/sqrt(D) (:64, :95), FP32 softmax (:97-101), probs @ v.
    """
    hq, d = q.shape
    hkv = k_cache.shape[2]
    group = hq // hkv
    pos = np.arange(seq_len)
    blocks = np.asarray(block_table, dtype=np.int64)[pos // block_size]
    k = k_cache[blocks, pos % block_size].astype(dtype)  # [S, Hkv, D]
    v = v_cache[blocks, pos % block_size].astype(dtype)
    k = np.repeat(k.transpose(1, 0, 2), group, axis=0)  # [Hq, S, D]
    v = np.repeat(v.transpose(1, 0, 2), group, axis=0)
    scale = dtype(1.0 / math.sqrt(d))
    scores = np.einsum("hd,hsd->hs", q.astype(dtype), k) * scale
    probs = _softmax_lastdim(scores.astype(np.float64 if dtype == np.float64 else np.float32)).astype(dtype)
    return np.einsum("hs,hsd->hd", probs, v)


def decode_batch(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    block_tables: np.ndarray,
    seq_lens: np.ndarray,
    block_size: int,
    dtype=np.float32,
) -> np.ndarray:
    """Batched decode: q [B, Hq, D] -> [B, Hq, D].

    Restates paged_attention_decode_batch_parallel
    (kernels/reference/paged_attention.py:178-254): positions past a
    sequence's length are masked to -inf (:230-232, :249) so padded (-1)
    table entries are never used; the result per sequence equals
    :func:`decode_single` (paged_attention_decode_batch_reference, :109-176).
    """
    out = np.empty(q.shape, dtype=dtype)
    for b in range(q.shape[0]):
        out[b] = decode_single(q[b], k_cache, v_cache, block_tables[b], int(seq_lens[b]), block_size, dtype)
    return out


def decode_batch_vectorized(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    block_tables: np.ndarray,
    seq_lens: np.ndarray,
    block_size: int,
) -> np.ndarray:
    """Same result as :func:`decode_batch`, with the reference's padded
    gather (paged_attention.py:222-254): one [B, maxS] gather, a -inf mask for
    padded positions, one batched softmax.  Used as the timed CPU baseline.
    """
    b, hq, d = q.shape
    hkv = k_cache.shape[2]
    group = hq // hkv
    seq_lens = np.asarray(seq_lens, dtype=np.int64)
    max_s = int(seq_lens.max())
    pos = np.arange(max_s)
    valid = pos[None, :] < seq_lens[:, None]
    phys = np.where(valid, np.asarray(block_tables)[:, pos // block_size], 0)
    off = pos % block_size
    k = k_cache[phys, off[None, :]].astype(np.float32)  # [B, S, Hkv, D]
    v = v_cache[phys, off[None, :]].astype(np.float32)
    qg = q.astype(np.float32).reshape(b, hkv, group, d)
    scores = np.einsum("bhgd,bshd->bhgs", qg, k) * np.float32(1.0 / math.sqrt(d))
    scores = np.where(valid[:, None, None, :], scores, -np.inf)
    probs = _softmax_lastdim(scores).astype(np.float32)
    out = np.einsum("bhgs,bshd->bhgd", probs, v)
    return out.reshape(b, hq, d)


def decode_split_kv(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    block_tables: np.ndarray,
    seq_lens: np.ndarray,
    block_size: int,
    partition_size: int,
) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """Split-KV decode with a log-sum-exp merge.

    Restates the Triton split-KV pair (kernels/triton/paged_attention.py):
    stage 1 (:528-700) gives each partition of ``partition_size`` tokens its
    running max m_p, sum l_p = sum exp(s - m_p) and acc_p = sum exp(s - m_p) v;
    the merge (:1530-1618) computes m* = max_p m_p,
    l* = sum_p exp(m_p - m*) l_p and out = sum_p exp(m_p - m*) acc_p / l*.
    Returns (out [B, Hq, D], m [B, Hq, P], l [B, Hq, P], acc [B, Hq, P, D])
    with P = max partitions; unused partitions have m = -inf, l = 0.
    """
    b, hq, d = q.shape
    hkv = k_cache.shape[2]
    group = hq // hkv
    scale = 1.0 / math.sqrt(d)
    max_p = int(-(-int(np.max(seq_lens)) // partition_size))
    m = np.full((b, hq, max_p), -np.inf, dtype=np.float64)
    l = np.zeros((b, hq, max_p), dtype=np.float64)
    acc = np.zeros((b, hq, max_p, d), dtype=np.float64)
    out = np.zeros((b, hq, d), dtype=np.float64)
    for i in range(b):
        s_len = int(seq_lens[i])
        pos = np.arange(s_len)
        blocks = np.asarray(block_tables[i], dtype=np.int64)[pos // block_size]
        k = k_cache[blocks, pos % block_size].astype(np.float64)
        v = v_cache[blocks, pos % block_size].astype(np.float64)
        for h in range(hq):
            kh = k[:, h // group]
            vh = v[:, h // group]
            s = (kh @ q[i, h].astype(np.float64)) * scale
            for p in range(-(-s_len // partition_size)):
                sp = s[p * partition_size : (p + 1) * partition_size]
                m[i, h, p] = sp.max()
                e = np.exp(sp - m[i, h, p])
                l[i, h, p] = e.sum()
                acc[i, h, p] = e @ vh[p * partition_size : (p + 1) * partition_size]
            ms = m[i, h].max()
            w = np.exp(m[i, h] - ms)
            out[i, h] = (w[:, None] * acc[i, h]).sum(0) / (w * l[i, h]).sum()
    return out, m, l, acc


# ---------------------------------------------------------------------------
# Chunk prefill
# ---------------------------------------------------------------------------


def prefill_chunk(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    block_table,
    prefix_len: int,
    context_len: int,
    block_size: int,
    dtype=np.float32,
) -> np.ndarray:
    """Causal chunk attention over a paged prefix: q [C, Hq, D] -> [C, Hq, D].

    Restates paged_attention_prefill_chunk_tiled_reference
    (kernels/reference/paged_attention.py:282-343): gather all context_len
    slots through the block table (:307-321), repeat KV heads for GQA
    (:322-323), scores / sqrt(D) (:326-328), mask pos_k > prefix + i to -inf
    (:329-337), FP32 softmax (:338-342), probs @ values.
    """
    c, hq, d = q.shape
    if context_len != prefix_len + c:
        raise ValueError("context_len must equal prefix_len + q.shape[0]")
    hkv = k_cache.shape[2]
    group = hq // hkv
    pos = np.arange(context_len)
    slots = np.asarray(block_table, dtype=np.int64)[pos // block_size] * block_size + pos % block_size
    flat_k = k_cache.reshape(-1, hkv, d)
    flat_v = v_cache.reshape(-1, hkv, d)
    keys = np.repeat(flat_k[slots].transpose(1, 0, 2).astype(dtype), group, axis=0)  # [Hq, S, D]
    values = np.repeat(flat_v[slots].transpose(1, 0, 2).astype(dtype), group, axis=0)
    query = q.transpose(1, 0, 2).astype(dtype)  # [Hq, C, D]
    scores = np.einsum("hcd,hsd->hcs", query, keys) / dtype(math.sqrt(d))
    qpos = prefix_len + np.arange(c)
    causal = pos[None, :] <= qpos[:, None]
    scores = np.where(causal[None], scores, -np.inf)
    probs = _softmax_lastdim(scores.astype(np.float64 if dtype == np.float64 else np.float32)).astype(dtype)
    # Masked positions carry probability exactly 0; keep NaN-poisoned unused
    # slots (never selected by the table) out of the product anyway.
    return np.einsum("hcs,hsd->hcd", probs, values).transpose(1, 0, 2)


def prefill_chunk_tiled(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    block_table,
    prefix_len: int,
    context_len: int,
    block_size: int,
    tile_size: int,
) -> np.ndarray:
    """Same result as :func:`prefill_chunk` by tiled online softmax.

    Restates paged_attention_prefill_chunk_tiled
    (kernels/reference/paged_attention.py:346-434): for each KV tile of
    ``tile_size`` positions (:398), tile max, rescale of the running sum and
    accumulator by exp(old_max - new_max) (:419-431), final acc / sum (:433).
    """
    if tile_size <= 0:
        raise ValueError("tile_size must be greater than 0")
    c, hq, d = q.shape
    if context_len != prefix_len + c:
        raise ValueError("context_len must equal prefix_len + q.shape[0]")
    hkv = k_cache.shape[2]
    group = hq // hkv
    flat_k = k_cache.reshape(-1, hkv, d)
    flat_v = v_cache.reshape(-1, hkv, d)
    table = np.asarray(block_table, dtype=np.int64)
    query = q.transpose(1, 0, 2).astype(np.float32)
    qpos = prefix_len + np.arange(c)
    acc = np.zeros((hq, c, d), dtype=np.float32)
    mx = np.full((hq, c, 1), -np.inf, dtype=np.float32)
    sm = np.zeros((hq, c, 1), dtype=np.float32)
    for t0 in range(0, context_len, tile_size):
        pos = np.arange(t0, min(t0 + tile_size, context_len))
        slots = table[pos // block_size] * block_size + pos % block_size
        keys = np.repeat(flat_k[slots].transpose(1, 0, 2).astype(np.float32), group, axis=0)
        values = np.repeat(flat_v[slots].transpose(1, 0, 2).astype(np.float32), group, axis=0)
        scores = np.einsum("hcd,hsd->hcs", query, keys) / np.float32(math.sqrt(d))
        scores = np.where((pos[None, :] <= qpos[:, None])[None], scores, -np.inf).astype(np.float32)
        tile_max = scores.max(-1, keepdims=True)
        new_max = np.maximum(mx, tile_max)
        with np.errstate(invalid="ignore"):
            old_scale = np.where(np.isneginf(new_max), 0.0, np.exp(mx - new_max)).astype(np.float32)
            w = np.where(np.isneginf(new_max), 0.0, np.exp(scores - new_max)).astype(np.float32)
        sm = sm * old_scale + w.sum(-1, keepdims=True)
        acc = acc * old_scale + np.einsum("hcs,hsd->hcd", w, values)
        mx = new_max
    return (acc / sm).transpose(1, 0, 2)


# ---------------------------------------------------------------------------
# P.V accumulator
# ---------------------------------------------------------------------------


def accumulate_pv(p: np.ndarray, v: np.ndarray) -> np.ndarray:
    """out[b, d] = sum_n p[b, n] v[b, n, d] — the expected value of
    tests/kernels/test_accumulator_cuda.py:25 for paged_attention_accumulator_cuda
    (kernels/cuda/paged_attention_accumulator.cu:15-68)."""
    return np.einsum("bn,bnd->bd", p.astype(np.float64), v.astype(np.float64)).astype(np.float32)


# ---------------------------------------------------------------------------
# Timed CPU baseline
# ---------------------------------------------------------------------------


def decode_batch_threaded(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    block_tables: np.ndarray,
    seq_lens: np.ndarray,
    block_size: int,
    threads: int,
) -> np.ndarray:
    """:func:`decode_batch` (FP32) spread over ``threads`` host threads, one
    sequence per task, with BLAS matmuls per KV head; the CPU baseline timed by
    ``bench.py --impl reference``.  Numerically the same restatement of
    paged_attention_decode_batch_parallel (paged_attention.py:178-254)."""
    import concurrent.futures as cf

    b, hq, d = q.shape
    hkv = k_cache.shape[2]
    group = hq // hkv
    scale = np.float32(1.0 / math.sqrt(d))
    out = np.empty((b, hq, d), dtype=np.float32)

    def one(i: int) -> None:
        s = int(seq_lens[i])
        pos = np.arange(s)
        blocks = np.asarray(block_tables[i], dtype=np.int64)[pos // block_size]
        k = k_cache[blocks, pos % block_size].astype(np.float32)  # [S, Hkv, D]
        v = v_cache[blocks, pos % block_size].astype(np.float32)
        for h in range(hkv):
            qg = q[i, h * group : (h + 1) * group].astype(np.float32)  # [G, D]
            sc = (qg @ k[:, h].T) * scale  # [G, S]
            p = _softmax_lastdim(sc).astype(np.float32)
            out[i, h * group : (h + 1) * group] = p @ v[:, h]

    with cf.ThreadPoolExecutor(max_workers=max(1, threads)) as ex:
        list(ex.map(one, range(b)))
    return out

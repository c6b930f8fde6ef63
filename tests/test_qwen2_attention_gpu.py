"""Qwen2Attention's paged methods on the GPU (model/qwen2.py:441-767 call
sites): the batched decode equals request-by-request decode
(tests/model/test_qwen2_batch_decode.py:33-71), the KV rows land in the
mapped slots and nowhere else, and the attention output matches the oracle
within the north-star tolerances (FP32: 1e-5 relative; BF16: 2e-2 absolute /
1e-2 relative against FP32 math on the same inputs)."""

import copy
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.nn as nn

from mini_llm_runtime_b200 import PagedKVCache, Qwen2Attention
from oracle import paged_attention_oracle as O

pytestmark = pytest.mark.gpu

TINY = SimpleNamespace(hidden_size=64, num_attention_heads=4, num_key_value_heads=2, rope_theta=1e6)
QWEN05 = SimpleNamespace(hidden_size=896, num_attention_heads=14, num_key_value_heads=2, rope_theta=1e6)
TOL = {torch.float32: dict(rtol=1e-5, atol=1e-5), torch.bfloat16: dict(rtol=1e-2, atol=2e-2)}


def np32(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("num_kv_heads", [1, 2, 4])
@pytest.mark.parametrize("batch_size", [1, 2])
def test_batch_decode_matches_single_requests(cuda_device, num_kv_heads, batch_size):
    torch.manual_seed(42)
    cfg = SimpleNamespace(**{**vars(TINY), "num_key_value_heads": num_kv_heads})
    attention = Qwen2Attention(cfg).to(cuda_device)
    cache = PagedKVCache(2, 6, 2, num_kv_heads, 16, dtype=torch.float32, device=cuda_device)
    cache.k_cache.normal_()
    cache.v_cache.normal_()
    inputs = dict(
        hidden_states=torch.randn(2, 1, 64, device=cuda_device)[:batch_size],
        position_ids=torch.tensor([[2], [4]], device=cuda_device)[:batch_size],
        layer_idx=1,
        slot_mapping=torch.tensor([0, 8], device=cuda_device)[:batch_size],
        block_tables=torch.tensor([[2, 0, -1], [1, 3, 4]], device=cuda_device)[:batch_size],
        context_lens=torch.tensor([3, 5], device=cuda_device)[:batch_size],
    )
    ref_cache = copy.deepcopy(cache)
    old_k, old_v = cache.k_cache.clone(), cache.v_cache.clone()
    with torch.no_grad():
        expected = torch.cat([
            attention.forward_decode_with_cache(
                inputs["hidden_states"][i:i + 1], inputs["position_ids"][i:i + 1], ref_cache, 1,
                inputs["slot_mapping"][i:i + 1], inputs["block_tables"][i].tolist(),
                int(inputs["context_lens"][i]))
            for i in range(batch_size)
        ])
        actual = attention.forward_decode_batch_with_cache(kv_cache=cache, **inputs)
    assert actual.shape == inputs["hidden_states"].shape
    torch.testing.assert_close(actual, expected, rtol=1e-5, atol=1e-6)
    # Batched and one-row projections may round differently (cuBLAS picks
    # another kernel per M): close, as in the reference's own test.
    torch.testing.assert_close(cache.k_cache, ref_cache.k_cache)
    torch.testing.assert_close(cache.v_cache, ref_cache.v_cache)
    unchanged = torch.ones(cache.k_cache.shape[:3], dtype=torch.bool, device=cuda_device)
    s = inputs["slot_mapping"]
    unchanged[1, s // 2, s % 2] = False
    assert torch.equal(cache.k_cache[unchanged], old_k[unchanged])
    assert torch.equal(cache.v_cache[unchanged], old_v[unchanged])


def _decode_batch_setup(device, dtype, ctx, seed):
    torch.manual_seed(seed)
    attention = Qwen2Attention(QWEN05).to(device=device, dtype=dtype)
    attention.o_proj = nn.Identity()  # compare the attention output itself
    bs = 16
    need = [(c + bs - 1) // bs for c in ctx]
    nb = sum(need) + 5
    cache = PagedKVCache(2, nb, bs, 2, 64, dtype=dtype, device=device)
    cache.k_cache.normal_()
    cache.v_cache.normal_()
    perm = torch.randperm(nb).tolist()
    width = max(need)
    tables, cur = [], 0
    for n in need:
        tables.append(perm[cur:cur + n] + [-1] * (width - n))
        cur += n
    tables = torch.tensor(tables, device=device)
    lens = torch.tensor(ctx, device=device)
    pos = lens - 1
    slots = tables[torch.arange(len(ctx), device=device), pos // bs] * bs + pos % bs
    hidden = torch.randn(len(ctx), 1, 896, device=device).to(dtype)
    return attention, cache, hidden, pos[:, None], slots, tables, lens


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_batch_decode_matches_oracle_at_qwen05_geometry(cuda_device, dtype):
    ctx = [1, 15, 16, 17, 100, 255, 256, 999]
    attention, cache, hidden, pos, slots, tables, lens = _decode_batch_setup(cuda_device, dtype, ctx, 3)
    with torch.no_grad():
        q, k, v = attention.project(hidden, pos)
        out = attention.forward_decode_batch_with_cache(hidden, pos, cache, 1, slots, tables, lens)
    torch.cuda.synchronize()
    bs = cache.block_size
    s = slots.cpu()
    assert torch.equal(cache.k_cache[1].reshape(-1, 2, 64)[s.to(cuda_device)], k[:, 0])
    assert torch.equal(cache.v_cache[1].reshape(-1, 2, 64)[s.to(cuda_device)], v[:, 0])
    expect = O.decode_batch(np32(q[:, 0]), np32(cache.k_cache[1]), np32(cache.v_cache[1]), tables.cpu().numpy(),
                            np.array(ctx), bs)
    torch.testing.assert_close(out[:, 0].float().cpu().reshape(expect.shape), torch.from_numpy(expect), **TOL[dtype])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("prefix,chunk", [(0, 1), (0, 130), (37, 77), (300, 200)])
def test_chunk_prefill_matches_oracle(cuda_device, dtype, prefix, chunk):
    torch.manual_seed(5)
    attention = Qwen2Attention(QWEN05).to(device=cuda_device, dtype=dtype)
    attention.o_proj = nn.Identity()
    bs = 16
    ctx = prefix + chunk
    nb = (ctx + bs - 1) // bs + 4
    cache = PagedKVCache(1, nb, bs, 2, 64, dtype=dtype, device=cuda_device)
    cache.k_cache.normal_()
    cache.v_cache.normal_()
    table = torch.randperm(nb)[: (ctx + bs - 1) // bs].tolist()
    p = torch.arange(prefix, ctx)
    slots = torch.tensor([table[i // bs] * bs + i % bs for i in p.tolist()], device=cuda_device)
    hidden = torch.randn(1, chunk, 896, device=cuda_device).to(dtype)
    pos = p[None].to(cuda_device)
    with torch.no_grad():
        q, k, v = attention.project(hidden, pos)
        out = attention.forward_prefill_chunk_with_cache(hidden, pos, cache, 0, slots, table, prefix, ctx, 64)
    torch.cuda.synchronize()
    assert torch.equal(cache.k_cache[0].reshape(-1, 2, 64)[slots], k[0])
    expect = O.prefill_chunk(np32(q[0]), np32(cache.k_cache[0]), np32(cache.v_cache[0]), table, prefix, ctx, bs)
    torch.testing.assert_close(out[0].float().cpu().reshape(expect.shape), torch.from_numpy(expect), **TOL[dtype])


def test_batched_prefill_equals_request_by_request(cuda_device):
    """forward_prefill_batch_with_cache over packed chunks == one
    forward_prefill_chunk_with_cache call per request (same cache state)."""
    torch.manual_seed(9)
    dtype = torch.bfloat16
    attention = Qwen2Attention(QWEN05).to(device=cuda_device, dtype=dtype)
    bs = 16
    prefix, chunk = [0, 40, 129, 500], [33, 64, 1, 200]
    ctx = [a + b for a, b in zip(prefix, chunk)]
    need = [(c + bs - 1) // bs for c in ctx]
    nb = sum(need) + 3
    cache = PagedKVCache(1, nb, bs, 2, 64, dtype=dtype, device=cuda_device)
    cache.k_cache.normal_()
    cache.v_cache.normal_()
    perm = torch.randperm(nb).tolist()
    tables, cur = [], 0
    for n in need:
        tables.append(perm[cur:cur + n])
        cur += n
    ref_cache = copy.deepcopy(cache)
    hidden = torch.randn(1, sum(chunk), 896, device=cuda_device).to(dtype)
    positions, slots = [], []
    for s in range(4):
        for i in range(prefix[s], ctx[s]):
            positions.append(i)
            slots.append(tables[s][i // bs] * bs + i % bs)
    pos = torch.tensor([positions], device=cuda_device)
    slots = torch.tensor(slots, device=cuda_device)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(chunk)]), device=cuda_device)
    width = max(need)
    bt = torch.tensor([t + [-1] * (width - len(t)) for t in tables], device=cuda_device)
    with torch.no_grad():
        out = attention.forward_prefill_batch_with_cache(hidden, pos, cache, 0, slots, cu,
                                                         bt, torch.tensor(ctx, device=cuda_device))
        parts = []
        for s in range(4):
            a, b = int(cu[s]), int(cu[s + 1])
            parts.append(attention.forward_prefill_chunk_with_cache(
                hidden[:, a:b], pos[:, a:b], ref_cache, 0, slots[a:b], tables[s], prefix[s], ctx[s], 32))
    torch.testing.assert_close(out, torch.cat(parts, dim=1), rtol=0, atol=0)
    assert torch.equal(cache.k_cache, ref_cache.k_cache)
    assert torch.equal(cache.v_cache, ref_cache.v_cache)

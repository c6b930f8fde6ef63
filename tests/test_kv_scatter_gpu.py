"""Batched KV-cache write on the GPU: bit-exact against the reference's golden
pools and against torch's own GPU ``index_copy_`` (the reference's
implementation, runtime/paged_kv_cache.py:243-249)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from mini_llm_runtime_b200 import PagedKVCache

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def reference_write(cache_k, cache_v, slots, k, v, layer):
    """The reference's write_slots body on GPU tensors."""
    lk = cache_k[layer].flatten(0, 1)
    lv = cache_v[layer].flatten(0, 1)
    idx = slots.to(torch.long)
    lk.index_copy_(0, idx, k.to(lk.dtype))
    lv.index_copy_(0, idx, v.to(lv.dtype))


def bits(t):
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


@pytest.mark.parametrize("name,dtype", [("f32", torch.float32), ("f16", torch.float16), ("bf16", torch.bfloat16)])
def test_golden_write_slots(cuda_device, name, dtype):
    g = np.load(GOLDEN / "write_slots.npz")

    def pool(key):
        a = g[key]
        t = torch.tensor(a.view(np.int16) if a.dtype == np.uint16 else a)
        return (t.view(dtype) if a.dtype == np.uint16 else t).to(cuda_device)

    cache = PagedKVCache(2, 3, 4, 2, 8, dtype=dtype, device=cuda_device)
    cache.k_cache.copy_(pool(f"{name}_before_k"))
    cache.v_cache.copy_(pool(f"{name}_before_v"))
    # The reference test's source is a non-contiguous FP32 view.
    k = torch.tensor(g[f"{name}_k"]).to(cuda_device).transpose(1, 2).contiguous().transpose(1, 2)
    v = torch.tensor(g[f"{name}_v"]).to(cuda_device).transpose(1, 2).contiguous().transpose(1, 2)
    assert not k.is_contiguous()
    cache.write_slots(torch.tensor(g["slots"], dtype=torch.int32, device=cuda_device), k, v, layer_idx=1)
    assert torch.equal(bits(cache.k_cache), bits(pool(f"{name}_after_k")))
    assert torch.equal(bits(cache.v_cache), bits(pool(f"{name}_after_v")))


@pytest.mark.parametrize("pool_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("src_dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("slots", [[], [11], [11, 0, 7, 4, 2]])
@pytest.mark.parametrize("idx_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("contiguous", [True, False])
def test_write_matches_index_copy(cuda_device, pool_dtype, src_dtype, slots, idx_dtype, contiguous):
    torch.manual_seed(42)
    cache = PagedKVCache(2, 3, 4, 2, 8, dtype=pool_dtype, device=cuda_device)
    cache.k_cache.normal_()
    cache.v_cache.normal_()
    ek, ev = cache.k_cache.clone(), cache.v_cache.clone()
    idx = torch.tensor(slots, dtype=idx_dtype, device=cuda_device)
    if contiguous:
        k = torch.randn(len(slots), 2, 8, device=cuda_device).to(src_dtype)
    else:
        k = torch.randn(len(slots), 8, 2, device=cuda_device).to(src_dtype).transpose(1, 2)
    v = torch.randn_like(k)
    reference_write(ek, ev, idx, k, v, 1)
    cache.write_slots(idx, k, v, layer_idx=1)
    assert torch.equal(bits(cache.k_cache), bits(ek))
    assert torch.equal(bits(cache.v_cache), bits(ev))
    # Rewriting the same slots later is allowed.
    reference_write(ek, ev, idx, k + 1, v + 1, 1)
    cache.write_slots(idx, k + 1, v + 1, layer_idx=1)
    assert torch.equal(bits(cache.k_cache), bits(ek))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("hkv,d", [(2, 64), (4, 128), (1, 40)])
def test_write_large_shuffled_batch(cuda_device, dtype, hkv, d):
    """Chunk-prefill sized write (16 x 512 tokens) to a
    shuffled slot set; every untouched slot keeps its bits."""
    torch.manual_seed(0)
    nb, bs = 700, 16
    cache = PagedKVCache(3, nb, bs, hkv, d, dtype=dtype, device=cuda_device)
    cache.k_cache.normal_()
    cache.v_cache.normal_()
    ek, ev = cache.k_cache.clone(), cache.v_cache.clone()
    t = 16 * 512
    slots = torch.randperm(nb * bs, device=cuda_device)[:t]
    k = torch.randn(t, hkv, d, device=cuda_device).to(dtype)
    v = torch.randn(t, hkv, d, device=cuda_device).to(dtype)
    reference_write(ek, ev, slots, k, v, 2)
    cache.write_slots(slots, k, v, layer_idx=2)
    assert torch.equal(bits(cache.k_cache), bits(ek))
    assert torch.equal(bits(cache.v_cache), bits(ev))


def test_nan_and_inf_sources_round_like_torch(cuda_device):
    cache = PagedKVCache(1, 2, 4, 1, 8, dtype=torch.bfloat16, device=cuda_device)
    cache.k_cache.zero_()
    cache.v_cache.zero_()
    src = torch.tensor([[float("nan"), float("inf"), -float("inf"), 3.0e38, 1e-40, -0.0, 1.00390625, 1.01171875]],
                       device=cuda_device).reshape(1, 1, 8)
    ek, ev = cache.k_cache.clone(), cache.v_cache.clone()
    idx = torch.tensor([5], device=cuda_device)
    reference_write(ek, ev, idx, src, src, 0)
    cache.write_slots(idx, src, src, 0)
    assert torch.equal(bits(cache.k_cache), bits(ek))


@pytest.mark.parametrize("slots,error,message", [
    ([0, 0], ValueError, "distinct"),
    ([0, -1], IndexError, "out-of-range"),
    ([0, 12], IndexError, "out-of-range"),
])
def test_invalid_slots_leave_cache_untouched(cuda_device, slots, error, message):
    cache = PagedKVCache(2, 3, 4, 2, 8, dtype=torch.float32, device=cuda_device)
    cache.k_cache.fill_(17)
    cache.v_cache.fill_(23)
    with pytest.raises(error, match=message):
        cache.write_slots(torch.tensor(slots, device=cuda_device), torch.randn(2, 2, 8, device=cuda_device),
                          torch.randn(2, 2, 8, device=cuda_device), layer_idx=1)
    assert torch.all(cache.k_cache == 17) and torch.all(cache.v_cache == 23)

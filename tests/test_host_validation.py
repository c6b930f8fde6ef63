"""Host-side checks mirror the reference's exceptions and run before any device
work (CPU only).  Valid calls on CPU tensors must fail loudly: the product path
has no CPU fallback."""

import pytest
import torch

from mini_llm_runtime_b200 import (
    PagedKVCache,
    paged_attention_decode,
    paged_attention_decode_batch_parallel,
    paged_attention_decode_split_kv,
    paged_attention_prefill_chunk_tiled,
    paged_attention_prefill_varlen,
)
from mini_llm_runtime_b200._lib import PagedAttentionError


# tests/runtime/test_write_slots_batch.py:39-55 of the reference
@pytest.mark.parametrize(
    "slots,error,message",
    [
        ([0, 0], ValueError, "distinct"),
        ([0, -1], IndexError, "out-of-range"),
        ([0, 12], IndexError, "out-of-range"),
        ([0.0, 1.0], TypeError, "integer"),
    ],
)
def test_invalid_slot_write_does_not_modify_cache(slots, error, message):
    cache = PagedKVCache(2, 3, 4, 2, 8, dtype=torch.float32, device="cpu")
    cache.k_cache.fill_(17)
    cache.v_cache.fill_(23)
    with pytest.raises(error, match=message):
        cache.write_slots(torch.tensor(slots), torch.randn(2, 2, 8), torch.randn(2, 2, 8), layer_idx=1)
    assert torch.all(cache.k_cache == 17)
    assert torch.all(cache.v_cache == 23)


@pytest.mark.parametrize(
    "kwargs,error,message",
    [
        (dict(layer_idx=2), IndexError, "layer_idx"),
        (dict(k=torch.randn(2, 8)), ValueError, r"\[T, H_kv, D\]"),
        (dict(k=torch.randn(2, 3, 8), v=torch.randn(2, 3, 8)), ValueError, r"\[T, 2, 8\]"),
        (dict(v=torch.randn(3, 2, 8)), ValueError, "same shape"),
        (dict(slot_mapping=torch.tensor([[0, 1]])), ValueError, r"shape \[T\]"),
        (dict(slot_mapping=torch.tensor([0, 1, 2])), ValueError, "length must match"),
    ],
)
def test_write_slots_shape_errors(kwargs, error, message):
    cache = PagedKVCache(2, 3, 4, 2, 8, dtype=torch.float32, device="cpu")
    cache.k_cache.zero_()
    args = dict(slot_mapping=torch.tensor([0, 1]), k=torch.randn(2, 2, 8), v=torch.randn(2, 2, 8), layer_idx=1)
    args.update(kwargs)
    with pytest.raises(error, match=message):
        cache.write_slots(**args)
    assert torch.all(cache.k_cache == 0)


def test_valid_write_on_cpu_fails_loudly_without_touching_cache():
    cache = PagedKVCache(2, 3, 4, 2, 8, dtype=torch.float32, device="cpu")
    cache.k_cache.fill_(5)
    with pytest.raises(PagedAttentionError, match="CUDA"):
        cache.write_slots(torch.tensor([3, 1]), torch.randn(2, 2, 8), torch.randn(2, 2, 8), layer_idx=0)
    assert torch.all(cache.k_cache == 5)


def test_empty_write_is_allowed():
    cache = PagedKVCache(1, 3, 4, 2, 8, dtype=torch.float32, device="cpu")
    cache.write_slots(torch.tensor([], dtype=torch.long), torch.randn(0, 2, 8), torch.randn(0, 2, 8))


def test_allocator_matches_reference_behaviour():
    cache = PagedKVCache(1, 4, 2, 1, 8, dtype=torch.float32, device="cpu")
    cache.add_sequence(0)
    with pytest.raises(KeyError):
        cache.add_sequence(0)
    assert cache.reserve_tokens(0, 3)
    assert cache.block_tables[0] == [0, 1]  # LIFO list hands out block 0 first
    cache.add_sequence(1)
    assert cache.reserve_tokens(1, 4)
    assert cache.block_tables[1] == [2, 3]
    assert not cache.reserve_tokens(1, 5)
    cache.free_sequence(0)
    assert cache.free_blocks[-2:] == [0, 1]
    with pytest.raises(KeyError):
        cache.free_sequence(0)
    with pytest.raises(ValueError, match="negative"):
        cache.reserve_tokens(1, -1)
    with pytest.raises(IndexError):
        cache.get_layer_cache(1)


def _decode_inputs():
    q = torch.randn(2, 4, 8)
    k = torch.randn(5, 2, 2, 8)
    v = torch.randn_like(k)
    return q, k, v, torch.tensor([[2, 0, -1], [1, 3, 4]]), torch.tensor([3, 5])


@pytest.mark.parametrize(
    "mutate,message",
    [
        (lambda a: a.__setitem__(0, torch.randn(4, 8)), r"q must have shape \[B, Hq, D\]"),
        (lambda a: a.__setitem__(1, torch.randn(5, 2, 8)), "k_cache and v_cache must have shape"),
        (lambda a: a.__setitem__(2, torch.randn(5, 2, 2, 4)), "same shape"),
        (lambda a: a.__setitem__(0, torch.randn(2, 4, 4)), "same head_dim"),
        (lambda a: a.__setitem__(0, torch.randn(2, 3, 8)), "divisible"),
        (lambda a: a.__setitem__(3, torch.tensor([[2, 0, -1]])), "block_tables length"),
        (lambda a: a.__setitem__(4, torch.tensor([3])), "seq_lens length"),
    ],
)
def test_decode_batch_validation_messages(mutate, message):
    args = list(_decode_inputs())
    mutate(args)
    with pytest.raises(ValueError, match=message):
        paged_attention_decode_batch_parallel(*args, block_size=2)


def test_decode_batch_on_cpu_fails_loudly():
    with pytest.raises(PagedAttentionError, match="CUDA"):
        paged_attention_decode_batch_parallel(*_decode_inputs(), block_size=2)


def test_single_decode_validation_messages():
    q, k, v, _, _ = _decode_inputs()
    with pytest.raises(ValueError, match="seq_len must be greater than 0"):
        paged_attention_decode(q[0], k, v, [2, 0], 0, 2)
    with pytest.raises(ValueError, match="enough blocks"):
        paged_attention_decode(q[0], k, v, [2], 3, 2)
    with pytest.raises(ValueError, match="block_size does not match"):
        paged_attention_decode(q[0], k, v, [2, 0, 1], 3, 1)
    with pytest.raises(PagedAttentionError):
        paged_attention_decode(q[0], k, v, [2, 0], 3, 2)


def test_split_kv_validation():
    q, k, v, bt, sl = _decode_inputs()
    with pytest.raises(ValueError, match="partition_size"):
        paged_attention_decode_split_kv(q, k, v, bt, sl, 2, partition_size=0)
    with pytest.raises(ValueError, match="seq_len must be greater than 0"):
        paged_attention_decode_split_kv(q[0], k, v, [2, 0], 0, 2, partition_size=16)


def test_prefill_validation_messages():
    q = torch.randn(4, 4, 8)
    k = torch.randn(4, 3, 2, 8)
    v = torch.randn_like(k)
    with pytest.raises(ValueError, match="tile_size must be greater than 0"):
        paged_attention_prefill_chunk_tiled(q, k, v, [2, 0, 3], 5, 9, 3, 0)
    with pytest.raises(ValueError, match="context_len must equal prefix_len"):
        paged_attention_prefill_chunk_tiled(q, k, v, [2, 0, 3], 5, 8, 3, 4)
    with pytest.raises(ValueError, match="divisible"):
        paged_attention_prefill_chunk_tiled(torch.randn(4, 3, 8), k, v, [2, 0, 3], 5, 9, 3, 4)
    with pytest.raises(PagedAttentionError, match="CUDA"):
        paged_attention_prefill_chunk_tiled(q, k, v, [2, 0, 3], 5, 9, 3, 4)
    with pytest.raises(ValueError, match="cu_q_lens"):
        paged_attention_prefill_varlen(q, torch.tensor([0, 4]), torch.tensor([9, 9]), torch.zeros(2, 3), k, v, 4)

"""Host-side behaviour of the Qwen2Attention drop-in (no GPU): metadata is
rejected with the reference's exception types and messages before the cache
is touched (tests/model/test_qwen2_batch_decode.py:74-94 and the chunk-prefill
checks of model/qwen2.py:636-725), and the module's parameter names match the
reference's so its state dict loads unchanged."""

from types import SimpleNamespace

import pytest
import torch

from mini_llm_runtime_b200 import PagedKVCache, Qwen2Attention

CONFIG = SimpleNamespace(hidden_size=64, num_attention_heads=4, num_key_value_heads=2, rope_theta=1_000_000.0)


def decode_case():
    torch.manual_seed(42)
    attention = Qwen2Attention(CONFIG)
    cache = PagedKVCache(2, 6, 2, 2, 16, dtype=torch.float32)
    cache.k_cache.normal_()
    cache.v_cache.normal_()
    inputs = dict(
        hidden_states=torch.randn(2, 1, 64),
        position_ids=torch.tensor([[2], [4]]),
        layer_idx=1,
        slot_mapping=torch.tensor([0, 8]),
        block_tables=torch.tensor([[2, 0, -1], [1, 3, 4]]),
        context_lens=torch.tensor([3, 5]),
    )
    return attention, cache, inputs


@pytest.mark.parametrize(
    "field,value,message",
    [
        ("hidden_states", torch.zeros(2, 2, 64), "hidden_states must have shape"),
        ("position_ids", torch.tensor([[1], [4]]), "decode positions"),
        ("context_lens", torch.tensor([0, 5]), "greater than 0"),
        ("block_tables", torch.tensor([[2, 0], [1, 3]]), "insufficient blocks"),
        ("block_tables", torch.tensor([[2, -1, -1], [1, 3, 4]]), "invalid physical block"),
        ("block_tables", torch.tensor([[2, 6, -1], [1, 3, 4]]), "invalid physical block"),
        ("slot_mapping", torch.tensor([1, 8]), "slot_mapping must match"),
        ("context_lens", torch.tensor([3.0, 5.0]), "torch.long dtype"),
        ("slot_mapping", torch.tensor([0, 8], dtype=torch.int32), "torch.long dtype"),
        ("position_ids", torch.tensor([2, 4]), r"position_ids must have shape \[B, 1\]"),
    ],
)
def test_batch_decode_rejects_metadata_before_cache_write(field, value, message):
    attention, cache, inputs = decode_case()
    old_k, old_v = cache.k_cache.clone(), cache.v_cache.clone()
    inputs[field] = value
    with pytest.raises(ValueError, match=message):
        attention.forward_decode_batch_with_cache(kv_cache=cache, **inputs)
    assert torch.equal(cache.k_cache, old_k)
    assert torch.equal(cache.v_cache, old_v)


def test_batch_decode_rejects_shared_write_slot():
    attention, cache, inputs = decode_case()
    # Both requests map their position 2 to block 1, offset 0: slot 2.
    inputs.update(block_tables=torch.tensor([[2, 1, -1], [3, 1, -1]]), position_ids=torch.tensor([[2], [2]]),
                  context_lens=torch.tensor([3, 3]), slot_mapping=torch.tensor([2, 2]))
    with pytest.raises(ValueError, match="distinct write slots"):
        attention.forward_decode_batch_with_cache(kv_cache=cache, **inputs)


def test_batch_decode_rejects_empty_batch_and_dtype_mismatch():
    attention, cache, inputs = decode_case()
    empty = {k: (v[:0] if isinstance(v, torch.Tensor) else v) for k, v in inputs.items()}
    with pytest.raises(ValueError, match="must not be empty"):
        attention.forward_decode_batch_with_cache(kv_cache=cache, **empty)
    inputs["hidden_states"] = inputs["hidden_states"].double()
    with pytest.raises(ValueError, match="KV cache dtype must match"):
        attention.forward_decode_batch_with_cache(kv_cache=cache, **inputs)


def prefill_case():
    attention = Qwen2Attention(CONFIG)
    cache = PagedKVCache(1, 8, 2, 2, 16, dtype=torch.float32)
    cache.k_cache.normal_()
    cache.v_cache.normal_()
    table = [5, 1, 6, 2]
    prefix, chunk = 3, 4
    pos = torch.arange(prefix, prefix + chunk)
    slots = torch.tensor([table[p // 2] * 2 + p % 2 for p in pos.tolist()])
    inputs = dict(hidden_states=torch.randn(1, chunk, 64), position_ids=pos[None], layer_idx=0,
                  slot_mapping=slots, block_table=table, prefix_len=prefix, context_len=prefix + chunk, tile_size=2)
    return attention, cache, inputs


@pytest.mark.parametrize(
    "field,value,error,message",
    [
        ("position_ids", torch.tensor([[3, 4, 5, 7]]), ValueError, "contiguous global positions"),
        ("position_ids", torch.tensor([[3.0, 4.0, 5.0, 6.0]]), TypeError, "integer dtype"),
        ("context_len", 8, ValueError, "context_len must equal prefix_len"),
        ("prefix_len", -1, ValueError, "cannot be negative"),
        ("tile_size", 0, ValueError, "tile_size must be greater than 0"),
        ("block_table", [5, 1, 6], ValueError, "enough blocks"),
        ("block_table", [5, 1, 6, 8], ValueError, "out-of-range physical block"),
        ("slot_mapping", torch.tensor([3, 10, 11, 12]), ValueError, "slot_mapping does not match"),
        ("slot_mapping", torch.tensor([3, 10, 11]), ValueError, r"shape \[chunk_len\]"),
        ("hidden_states", torch.randn(2, 4, 64), ValueError, "exactly one request"),
    ],
)
def test_chunk_prefill_rejects_metadata_before_cache_write(field, value, error, message):
    attention, cache, inputs = prefill_case()
    old_k, old_v = cache.k_cache.clone(), cache.v_cache.clone()
    inputs[field] = value
    with pytest.raises(error, match=message):
        attention.forward_prefill_chunk_with_cache(kv_cache=cache, **inputs)
    assert torch.equal(cache.k_cache, old_k)
    assert torch.equal(cache.v_cache, old_v)


def test_single_decode_rejects_wrong_position():
    attention, cache, inputs = decode_case()
    with pytest.raises(ValueError, match="decode position must equal context_len - 1"):
        attention.forward_decode_with_cache(inputs["hidden_states"][:1], torch.tensor([[1]]), cache, 1,
                                            torch.tensor([0]), [2, 0], 3)
    with pytest.raises(ValueError, match="exactly one input token"):
        attention.forward_decode_with_cache(torch.zeros(1, 2, 64), torch.tensor([[1, 2]]), cache, 1,
                                            torch.tensor([0]), [2, 0], 3)


def test_parameter_names_match_reference_layout():
    names = set(Qwen2Attention(CONFIG).state_dict())
    assert names == {
        "qkv_proj.q_proj.weight", "qkv_proj.q_proj.bias", "qkv_proj.k_proj.weight", "qkv_proj.k_proj.bias",
        "qkv_proj.v_proj.weight", "qkv_proj.v_proj.bias", "o_proj.weight",
    }


def test_rope_rotates_pairs_of_halves():
    """RoPE at position p rotates (x_i, x_{i+D/2}) by p * theta^(-2i/D)."""
    attention = Qwen2Attention(CONFIG)
    x = torch.randn(1, 3, 4, 16)
    pos = torch.tensor([[0, 1, 7]])
    cos, sin = attention.rotary_embedding(x, pos)
    from mini_llm_runtime_b200.qwen2_attention import apply_rotary_pos_emb

    q, _ = apply_rotary_pos_emb(x, x, cos, sin)
    inv = 1.0 / (1e6 ** (torch.arange(0, 16, 2, dtype=torch.float32) / 16))
    ang = pos[0, :, None].float() * inv  # [3, 8]
    a, b = x[..., :8], x[..., 8:]
    c, s = ang.cos()[None, :, None], ang.sin()[None, :, None]
    torch.testing.assert_close(q[..., :8], a * c - b * s)
    torch.testing.assert_close(q[..., 8:], b * c + a * s)
    torch.testing.assert_close(q[:, 0], x[:, 0])

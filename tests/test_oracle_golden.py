"""Pin the numpy oracle to the reference: every oracle function reproduces the
golden vectors that tests/golden/make_golden.py recorded from the reference's
own PyTorch code (CPU only)."""

from pathlib import Path

import numpy as np
import pytest

from oracle import paged_attention_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return np.load(GOLDEN / f"{name}.npz")


def test_decode_config1_matches_reference():
    g = load("decode_config1")
    bs = int(g["block_size"])
    # Rebuild the pre-write pool and replay the new-token write.
    k_pool = g["k_pool"].copy()
    v_pool = g["v_pool"].copy()
    flat_k = k_pool.reshape(1, -1, *k_pool.shape[3:])
    flat_v = v_pool.reshape(1, -1, *v_pool.shape[3:])
    flat_k[0, g["slot_mapping"]] = g["old_k_at_slots"]
    flat_v[0, g["slot_mapping"]] = g["old_v_at_slots"]
    O.write_slots(k_pool, v_pool, g["slot_mapping"], g["new_k"], g["new_v"], 0)
    np.testing.assert_array_equal(k_pool, g["k_pool"])
    np.testing.assert_array_equal(v_pool, g["v_pool"])
    out = O.decode_batch(g["q"], k_pool[0], v_pool[0], g["block_tables"], g["context_lens"], bs)
    np.testing.assert_allclose(out, g["out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(out, g["out_request_reference"], rtol=1e-5, atol=1e-6)
    vec = O.decode_batch_vectorized(g["q"], k_pool[0], v_pool[0], g["block_tables"], g["context_lens"], bs)
    np.testing.assert_allclose(vec, g["out"], rtol=1e-5, atol=1e-6)


def test_decode_small_cases_match_reference():
    g = load("decode_small")
    bs = int(g["block_size"])
    for i in range(int(g["num_cases"])):
        out = O.decode_batch(g[f"c{i}_q"], g[f"c{i}_k"], g[f"c{i}_v"], g[f"c{i}_tables"], g[f"c{i}_lens"], bs)
        np.testing.assert_allclose(out, g[f"c{i}_out"], rtol=1e-5, atol=1e-6)


def test_decode_bf16_inputs_match_fp32_reference():
    g = load("decode_bf16")
    k = O.bf16_bits_to_f32(g["k_pool_bits"])
    v = O.bf16_bits_to_f32(g["v_pool_bits"])
    q = O.bf16_bits_to_f32(g["q_bits"])
    out = O.decode_batch(q, k, v, g["block_tables"], g["context_lens"], int(g["block_size"]))
    np.testing.assert_allclose(out, g["out_fp32_reference"], rtol=1e-5, atol=1e-6)
    # The reference's own BF16 path (bf16 scores and probabilities) is within
    # the BF16 tolerance of the FP32 reference the kernels are held to.
    ref_bf16 = O.bf16_bits_to_f32(g["out_bf16_reference_bits"])
    np.testing.assert_allclose(ref_bf16, g["out_fp32_reference"], rtol=1e-2, atol=2e-2)


def test_split_kv_merge_equals_decode():
    g = load("decode_config1")
    bs = int(g["block_size"])
    kp, vp = g["k_pool"][0], g["v_pool"][0]
    for part in (16, 48, 100, 256):
        out, m, l, acc = O.decode_split_kv(g["q"], kp, vp, g["block_tables"], g["context_lens"], bs, part)
        np.testing.assert_allclose(out, g["out"], rtol=1e-5, atol=1e-6)
        # Unused partitions carry the merge identity (m=-inf, l=0).
        lens = g["context_lens"]
        for b in range(len(lens)):
            used = -(-int(lens[b]) // part)
            assert np.all(np.isneginf(m[b, :, used:])) and np.all(l[b, :, used:] == 0)


def test_prefill_small_grid_matches_reference():
    g = load("prefill_small")
    for i in range(int(g["num_cases"])):
        prefix, ctx, bs, tile = (int(x) for x in g[f"c{i}_meta"])
        args = (g[f"c{i}_q"], g[f"c{i}_k"], g[f"c{i}_v"], g[f"c{i}_table"], prefix, ctx, bs)
        dense = O.prefill_chunk(*args)
        tiled = O.prefill_chunk_tiled(*args, tile)
        assert np.isfinite(dense).all()
        np.testing.assert_allclose(dense, g[f"c{i}_out"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(tiled, g[f"c{i}_out"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(dense, g[f"c{i}_out_dense"], rtol=1e-5, atol=1e-6)


def test_prefill_medium_matches_reference():
    g = load("prefill_medium")
    prefix, ctx, bs = (int(x) for x in g["meta"])
    out = O.prefill_chunk(g["q"], g["k"], g["v"], g["table"], prefix, ctx, bs)
    np.testing.assert_allclose(out, g["out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(out, g["out_dense"], rtol=1e-5, atol=1e-6)
    tiled = O.prefill_chunk_tiled(g["q"], g["k"], g["v"], g["table"], prefix, ctx, bs, 16)
    np.testing.assert_allclose(tiled, g["out"], rtol=1e-5, atol=1e-6)
    qb, kb, vb = (O.bf16_bits_to_f32(g[n]) for n in ("q_bits", "k_bits", "v_bits"))
    outb = O.prefill_chunk(qb, kb, vb, g["table"], prefix, ctx, bs)
    np.testing.assert_allclose(outb, g["out_bf16_inputs_fp32_reference"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", ["f32", "f16", "bf16"])
def test_write_slots_bitwise(name):
    g = load("write_slots")
    before_k, before_v = g[f"{name}_before_k"], g[f"{name}_before_v"]
    after_k, after_v = g[f"{name}_after_k"], g[f"{name}_after_v"]
    if name == "f32":
        k_pool, v_pool = before_k.copy(), before_v.copy()
        O.write_slots(k_pool, v_pool, g["slots"], g[f"{name}_k"], g[f"{name}_v"], 1)
        np.testing.assert_array_equal(k_pool, after_k)
        np.testing.assert_array_equal(v_pool, after_v)
        return
    if name == "bf16":
        to_f32, rnd = O.bf16_bits_to_f32, O.round_to_bf16
    else:
        to_f32 = lambda b: np.asarray(b, dtype=np.uint16).view(np.float16).astype(np.float32)  # noqa: E731
        rnd = O.round_to_f16
    k_pool, v_pool = to_f32(before_k), to_f32(before_v)
    O.write_slots(k_pool, v_pool, g["slots"], rnd(g[f"{name}_k"]), rnd(g[f"{name}_v"]), 1)
    np.testing.assert_array_equal(k_pool, to_f32(after_k))
    np.testing.assert_array_equal(v_pool, to_f32(after_v))
    if name == "bf16":
        np.testing.assert_array_equal(O.f32_to_bf16_bits(k_pool), after_k)


def test_accumulator_matches_reference_expectation():
    g = load("accumulator")
    np.testing.assert_allclose(O.accumulate_pv(g["p"], g["v"]), g["out"], rtol=2e-5, atol=2e-5)


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.0 + 2**-8, 1.0 + 3 * 2**-8, -2.5, 3.0e38, 1e-40], dtype=np.float32)
    bits = O.f32_to_bf16_bits(x)
    # 1 + 2^-8 is a tie -> even (1.0); 1 + 3*2^-8 is a tie -> even (1 + 2^-6).
    np.testing.assert_array_equal(O.bf16_bits_to_f32(bits[:3]), np.array([1.0, 1.0, 1.0 + 2**-6], np.float32))
    assert O.bf16_bits_to_f32(bits[3:4])[0] == -2.5

"""Decode parity on the GPU: the CUDA kernels (through the C ABI) against the
oracle and the reference's golden vectors.

Tolerances (north_star): FP32 within 1e-5 relative (atol 1e-6); BF16/F16
within 2e-2 absolute / 1e-2 relative of the FP32 reference run on the
up-cast inputs."""

from pathlib import Path

import numpy as np
import pytest
import torch

from mini_llm_runtime_b200 import (
    PagedKVCache,
    paged_attention_decode,
    paged_attention_decode_batch_parallel,
    paged_attention_decode_split_kv,
)
from oracle import paged_attention_oracle as O
from tests.paged_inputs import make_decode_case

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = {
    torch.float32: dict(rtol=1e-5, atol=1e-6),
    torch.bfloat16: dict(rtol=1e-2, atol=2e-2),
    torch.float16: dict(rtol=1e-2, atol=2e-2),
}


def check(actual: torch.Tensor, expected: np.ndarray, dtype):
    a = actual.float().cpu().numpy()
    assert np.isfinite(a).all(), "NaN/Inf in kernel output"
    np.testing.assert_allclose(a, expected, **TOL[dtype])


def oracle_decode(case):
    q, k, v, tables, lens = case["np"]
    return O.decode_batch(q, k, v, tables, lens, case["bs"])


def test_golden_config1_fp32(cuda_device):
    """Config 1 end to end: write the new tokens through write_slots, then
    decode; both match the reference's recorded outputs."""
    g = np.load(GOLDEN / "decode_config1.npz")
    bs = int(g["block_size"])
    k_pool = torch.tensor(g["k_pool"])
    v_pool = torch.tensor(g["v_pool"])
    slots = torch.tensor(g["slot_mapping"])
    k_pool.flatten(1, 2)[0, slots] = torch.tensor(g["old_k_at_slots"])
    v_pool.flatten(1, 2)[0, slots] = torch.tensor(g["old_v_at_slots"])
    cache = PagedKVCache(1, k_pool.shape[1], bs, 2, 64, dtype=torch.float32, device=cuda_device)
    cache.k_cache.copy_(k_pool)
    cache.v_cache.copy_(v_pool)
    cache.write_slots(slots.to(cuda_device), torch.tensor(g["new_k"]).to(cuda_device),
                      torch.tensor(g["new_v"]).to(cuda_device), layer_idx=0)
    assert torch.equal(cache.k_cache.cpu(), torch.tensor(g["k_pool"]))
    assert torch.equal(cache.v_cache.cpu(), torch.tensor(g["v_pool"]))
    kc, vc = cache.get_layer_cache(0)
    out = paged_attention_decode_batch_parallel(
        torch.tensor(g["q"]).to(cuda_device), kc, vc, torch.tensor(g["block_tables"]).to(cuda_device),
        torch.tensor(g["context_lens"]).to(cuda_device), bs)
    check(out, g["out"], torch.float32)


def test_golden_small_cases(cuda_device):
    g = np.load(GOLDEN / "decode_small.npz")
    for i in range(int(g["num_cases"])):
        t = lambda n: torch.tensor(g[f"c{i}_{n}"]).to(cuda_device)  # noqa: E731
        out = paged_attention_decode_batch_parallel(t("q"), t("k"), t("v"), t("tables"), t("lens"), 2)
        check(out, g[f"c{i}_out"], torch.float32)


def test_golden_bf16_against_fp32_reference(cuda_device):
    g = np.load(GOLDEN / "decode_bf16.npz")

    def bf(name):
        return torch.tensor(g[name].view(np.int16)).view(torch.bfloat16).to(cuda_device)

    out = paged_attention_decode_batch_parallel(
        bf("q_bits"), bf("k_pool_bits"), bf("v_pool_bits"), torch.tensor(g["block_tables"]).to(cuda_device),
        torch.tensor(g["context_lens"]).to(cuda_device), int(g["block_size"]))
    assert out.dtype == torch.bfloat16
    check(out, g["out_fp32_reference"], torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv", [(14, 2), (4, 4), (8, 1), (28, 4), (32, 8), (40, 2)],
                         ids=["gqa7", "mha", "mqa", "gqa7x4", "gqa4", "gqa20"])
@pytest.mark.parametrize("d", [64, 128])
def test_decode_geometries(cuda_device, dtype, hq, hkv, d):
    ctx = [1, 15, 16, 17, 63, 64, 65, 127, 128, 255, 513, 700]
    case = make_decode_case(ctx, hq, hkv, d, 16, dtype, cuda_device, seed=hq * 7 + d)
    out = paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16)
    check(out, oracle_decode(case), dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("d", [8, 16, 40, 80, 96, 160])
def test_decode_odd_head_dims(cuda_device, dtype, d):
    """Head dims outside the tensor-core set (Triton test grid,
    tests/kernels/test_paged_attention_triton.py:418-427)."""
    case = make_decode_case([1, 33, 129, 600], 8, 2, d, 16, dtype, cuda_device, seed=d)
    out = paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16)
    check(out, oracle_decode(case), dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("bs", [2, 3, 8, 32, 64])
def test_decode_block_sizes(cuda_device, dtype, bs):
    case = make_decode_case([1, 5, 31, 64, 200], 14, 2, 64, bs, dtype, cuda_device, seed=bs, reverse_tables=True)
    out = paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], bs)
    check(out, oracle_decode(case), dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("seq_len", list(range(1, 66)))
def test_decode_tile_boundaries(cuda_device, dtype, seq_len):
    """Every length 1..65 (test_paged_attention_triton.py:406-415)."""
    case = make_decode_case([seq_len, 65 - seq_len + 1], 14, 2, 64, 16, dtype, cuda_device, seed=seq_len)
    out = paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16)
    check(out, oracle_decode(case), dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("partition", [16, 64, 128, 512, 2048])
def test_split_kv_partitions(cuda_device, dtype, partition):
    """Split-KV at partition edges (seq lens 513 / 529 / 600 / 4096 / 4097)."""
    case = make_decode_case([513, 529, 600, 4096, 4097, 1], 14, 2, 64, 16, dtype, cuda_device, seed=partition)
    out = paged_attention_decode_split_kv(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16,
                                          partition_size=partition)
    check(out, oracle_decode(case), dtype)
    # Tickets reset: a second call on the same workspace gives the same result.
    out2 = paged_attention_decode_split_kv(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16,
                                           partition_size=partition)
    assert torch.equal(out, out2)


def test_split_kv_single_sequence_signature(cuda_device):
    """The Triton-style single-sequence call (q [Hq, D], list table, int len)."""
    case = make_decode_case([3000], 32, 8, 128, 16, torch.float16, cuda_device, seed=5, reverse_tables=True)
    table = case["tables"][0].tolist()
    out = paged_attention_decode_split_kv(case["q"][0], case["k"], case["v"], table, 3000, 16, partition_size=128)
    check(out, oracle_decode(case)[0], torch.float16)


def test_single_decode_api(cuda_device):
    case = make_decode_case([37], 14, 2, 64, 16, torch.float32, cuda_device, seed=9)
    table = case["tables"][0].tolist()
    out = paged_attention_decode(case["q"][0], case["k"], case["v"], table, 37, 16)
    check(out, oracle_decode(case)[0], torch.float32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_config2_full_size(cuda_device, dtype):
    """BASELINE config 2 geometry at full size (one layer): B=64, contexts
    U[128, 4096], 14/2 heads, D=64, bs=16, pool = total blocks + 10%."""
    rng = np.random.default_rng(0)
    ctx = rng.integers(128, 4097, size=64).tolist()
    need = sum((c + 15) // 16 for c in ctx)
    case = make_decode_case(ctx, 14, 2, 64, 16, dtype, cuda_device, seed=2, extra_blocks=need // 10)
    out = paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16)
    check(out, oracle_decode(case), dtype)


def test_config3_long_context_split(cuda_device):
    """BASELINE config 3 shape at reduced batch: 32768-token contexts split
    into 16 partitions of 2048, LSE-merged."""
    case = make_decode_case([32768, 32768], 14, 2, 64, 16, torch.bfloat16, cuda_device, seed=3, extra_blocks=10)
    out = paged_attention_decode_split_kv(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16,
                                          partition_size=2048)
    check(out, oracle_decode(case), torch.bfloat16)


def test_decode_is_deterministic_and_does_not_write_pools(cuda_device):
    case = make_decode_case([100, 2000, 5], 14, 2, 64, 16, torch.bfloat16, cuda_device, seed=11)
    k0, v0 = case["k"].clone(), case["v"].clone()
    a = paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16)
    b = paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16)
    assert torch.equal(a, b)
    assert torch.equal(k0.view(torch.int16), case["k"].view(torch.int16))
    assert torch.equal(v0.view(torch.int16), case["v"].view(torch.int16))


def test_workspace_reuse_across_batch_sizes(cuda_device):
    """Calls with growing batch on one stream share the cached workspace; the
    ticket range of the larger call must not see the smaller call's partials."""
    for i, ctx in enumerate([[700, 3000], [4000] * 16, [100, 5000, 33], [2500] * 64]):
        case = make_decode_case(ctx, 14, 2, 64, 16, torch.bfloat16, cuda_device, seed=50 + i)
        for part in (0, 256):
            out = paged_attention_decode_split_kv(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16,
                                                  partition_size=part) if part else \
                paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16)
            check(out, oracle_decode(case), torch.bfloat16)


def test_tiny_batches_leave_ctas_idle(cuda_device):
    """Fewer KV sub-blocks than CTAs: most CTAs get an empty range and one
    sequence spans many single-sub-block CTAs."""
    for ctx in ([1], [160], [16 * 40 + 3], [5, 7, 300]):
        case = make_decode_case(ctx, 8, 1, 128, 16, torch.float16, cuda_device, seed=len(ctx) + ctx[0])
        out = paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16)
        check(out, oracle_decode(case), torch.float16)


@pytest.mark.parametrize("layers", [3, 9])
def test_decode_graph_step_matches_eager(cuda_device, layers):
    """PagedDecodeGraph (CUDA graph of KV write + decode per layer, with
    pinned host I/O copied in layer chunks that overlap the kernels) gives
    the same cache and outputs as eager calls, step after step."""
    from mini_llm_runtime_b200 import PagedDecodeGraph

    torch.manual_seed(3)
    ctx = [37, 600, 1025, 64]
    hq, hkv, d, bs = 14, 2, 64, 16
    need = [(c + bs - 1) // bs for c in ctx]
    nb = sum(need) + 5
    perm = torch.randperm(nb).tolist()
    tables, cur = [], 0
    for n in need:
        tables.append(perm[cur:cur + n] + [-1] * (max(need) - n))
        cur += n
    cache = PagedKVCache(layers, nb, bs, hkv, d, dtype=torch.bfloat16, device=cuda_device)
    cache.k_cache.normal_()
    cache.v_cache.normal_()
    ref = PagedKVCache(layers, nb, bs, hkv, d, dtype=torch.bfloat16, device=cuda_device)
    ref.k_cache.copy_(cache.k_cache)
    ref.v_cache.copy_(cache.v_cache)
    g = PagedDecodeGraph(cache, batch=len(ctx), max_blocks=max(need), num_q_heads=hq, layers=range(layers))
    hi = g.host_inputs
    hi["q"].copy_(torch.randn(hi["q"].shape).to(torch.bfloat16))
    hi["new_k"].copy_(torch.randn(hi["new_k"].shape).to(torch.bfloat16))
    hi["new_v"].copy_(torch.randn(hi["new_v"].shape).to(torch.bfloat16))
    hi["block_tables"].copy_(torch.tensor(tables))
    hi["context_lens"].copy_(torch.tensor(ctx))
    hi["slot_mapping"].copy_(torch.tensor([tables[b][(c - 1) // bs] * bs + (c - 1) % bs for b, c in enumerate(ctx)]))
    for step in range(2):
        if step:
            hi["q"].copy_(torch.randn(hi["q"].shape).to(torch.bfloat16))
            hi["new_k"].copy_(torch.randn(hi["new_k"].shape).to(torch.bfloat16))
        g.run()
        g.synchronize()
        dv = {k: v.to(cuda_device) for k, v in hi.items()}
        for layer in range(layers):
            ref.write_slots(dv["slot_mapping"], dv["new_k"][layer], dv["new_v"][layer], layer)
            exp = paged_attention_decode_batch_parallel(dv["q"][layer], ref.k_cache[layer], ref.v_cache[layer],
                                                        dv["block_tables"], dv["context_lens"], bs)
            assert torch.equal(g.host_output[layer], exp.cpu())
        assert torch.equal(cache.k_cache.view(torch.int16), ref.k_cache.view(torch.int16))
    with pytest.raises(ValueError, match="slot_mapping must match"):
        hi["slot_mapping"][0] += 1
        g.run()


@pytest.mark.parametrize(
    "dtype,d,hq,hkv,bs",
    [
        (torch.bfloat16, 64, 14, 2, 16),   # config-2 geometry: fused into the balanced kernel
        (torch.float16, 128, 28, 4, 16),   # config-5 geometry: fused
        (torch.bfloat16, 64, 8, 1, 32),    # MQA, two boxes per block: fused
        (torch.bfloat16, 128, 36, 2, 16),  # group of 18: two head tiles, both patch, tile 0 writes
        (torch.float32, 64, 14, 2, 16),    # FP32: scatter + CUDA-core decode
        (torch.bfloat16, 64, 14, 2, 8),    # block size 8: scatter + CUDA-core decode
    ],
)
def test_fused_kv_write_matches_scatter_then_decode(cuda_device, dtype, d, hq, hkv, bs):
    """pa_paged_decode_write == write_slots then decode, bit for bit, for the
    output and for both pools; the new token lands in every block position
    (first / middle / last row of a sub-block and of a block)."""
    from mini_llm_runtime_b200 import paged_decode_with_kv_write

    ctx = [1, 15, 16, 17, 31, 33, 300, 1025, 4096]
    case = make_decode_case(ctx, hq, hkv, d, bs, dtype, cuda_device, seed=d + hq + bs)
    g = torch.Generator().manual_seed(99)
    new_k = torch.randn(len(ctx), hkv, d, generator=g).to(dtype).to(cuda_device)
    new_v = torch.randn(len(ctx), hkv, d, generator=g).to(dtype).to(cuda_device)
    tables, lens = case["tables"], case["lens"]
    pos = lens - 1
    slots = tables[torch.arange(len(ctx), device=cuda_device), pos // bs] * bs + pos % bs
    k1, v1 = case["k"].clone(), case["v"].clone()
    k2, v2 = case["k"].clone(), case["v"].clone()
    out = paged_decode_with_kv_write(case["q"], new_k, new_v, slots, k1, v1, tables, lens, bs)
    k2.view(-1, hkv, d)[slots] = new_k
    v2.view(-1, hkv, d)[slots] = new_v
    ref = paged_attention_decode_batch_parallel(case["q"], k2, v2, tables, lens, bs)
    torch.cuda.synchronize()
    bits = torch.int32 if dtype == torch.float32 else torch.int16
    assert torch.equal(out.view(bits), ref.view(bits))
    assert torch.equal(k1.view(bits), k2.view(bits))
    assert torch.equal(v1.view(bits), v2.view(bits))
    # And it is the attention over the written cache (oracle, FP32 math).
    q_np, _, _, tab_np, ctx_np = case["np"]
    exp = O.decode_batch(q_np, k2.float().cpu().numpy(), v2.float().cpu().numpy(), tab_np, ctx_np, bs)
    check(out, exp, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv,d", [(14, 2, 64), (28, 4, 128), (40, 2, 64)], ids=["gqa7", "gqa7x4", "gqa20"])
def test_decode_batches_above_the_balanced_limit(cuda_device, dtype, hq, hkv, d):
    """More than 1024 sequences: one CTA per (sequence, head tile,
    partition) with a last-ticket merge instead of the balanced kernel."""
    rng = np.random.default_rng(hq * 3 + d)
    ctx = rng.integers(1, 160, size=1100).tolist()
    ctx[7], ctx[1000] = 1500, 16
    case = make_decode_case(ctx, hq, hkv, d, 16, dtype, cuda_device, seed=hq + d)
    out = paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16)
    check(out, oracle_decode(case), dtype)
    split = paged_attention_decode_split_kv(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16,
                                            partition_size=256)
    check(split, oracle_decode(case), dtype)

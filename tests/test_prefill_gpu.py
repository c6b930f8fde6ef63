"""Chunk-prefill parity on the GPU against the oracle and the reference's
golden vectors (FP32 1e-5 relative; BF16 2e-2 abs / 1e-2 rel vs FP32)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from mini_llm_runtime_b200 import (
    PagedKVCache,
    paged_attention_prefill_chunk_tiled,
    paged_attention_prefill_varlen,
)
from oracle import paged_attention_oracle as O
from tests.paged_inputs import make_prefill_case

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = {
    torch.float32: dict(rtol=1e-5, atol=1e-6),
    torch.bfloat16: dict(rtol=1e-2, atol=2e-2),
    torch.float16: dict(rtol=1e-2, atol=2e-2),
}


def check(actual, expected, dtype):
    a = actual.float().cpu().numpy()
    assert np.isfinite(a).all(), "NaN/Inf in kernel output"
    np.testing.assert_allclose(a, expected, **TOL[dtype])


def oracle_prefill(case):
    _, k, v, tables, _ = case["np"]
    outs = []
    for s, (p, c) in enumerate(zip(case["prefix"], case["chunk"])):
        q = case["q_np"][case["cu_np"][s] : case["cu_np"][s + 1]]
        outs.append(O.prefill_chunk(q, k, v, tables[s], p, p + c, case["bs"]))
    return np.concatenate(outs, 0)


def test_golden_small_grid(cuda_device):
    """tests/kernels/test_paged_attention.py:249-351 cases (bs 3, NaN pools)."""
    g = np.load(GOLDEN / "prefill_small.npz")
    for i in range(int(g["num_cases"])):
        prefix, ctx, bs, tile = (int(x) for x in g[f"c{i}_meta"])
        t = lambda n: torch.tensor(g[f"c{i}_{n}"]).to(cuda_device)  # noqa: E731
        out = paged_attention_prefill_chunk_tiled(t("q"), t("k"), t("v"), g[f"c{i}_table"].tolist(), prefix, ctx,
                                                  bs, tile)
        assert out.shape == t("q").shape and out.dtype == torch.float32
        check(out, g[f"c{i}_out"], torch.float32)


def test_golden_medium(cuda_device):
    g = np.load(GOLDEN / "prefill_medium.npz")
    prefix, ctx, bs = (int(x) for x in g["meta"])
    t = lambda n: torch.tensor(g[n]).to(cuda_device)  # noqa: E731
    out = paged_attention_prefill_chunk_tiled(t("q"), t("k"), t("v"), torch.tensor(g["table"]), prefix, ctx, bs, 16)
    check(out, g["out"], torch.float32)

    def bf(name):
        return torch.tensor(g[name].view(np.int16)).view(torch.bfloat16).to(cuda_device)

    outb = paged_attention_prefill_chunk_tiled(bf("q_bits"), bf("k_bits"), bf("v_bits"), g["table"].tolist(),
                                               prefix, ctx, bs, 16)
    check(outb, g["out_bf16_inputs_fp32_reference"], torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv", [(14, 2), (4, 4), (8, 1)], ids=["gqa7", "mha", "mqa"])
@pytest.mark.parametrize("d", [64, 128])
def test_varlen_batch(cuda_device, dtype, hq, hkv, d):
    prefix = [0, 5, 16, 200, 37, 0]
    chunk = [1, 17, 128, 130, 64, 300]
    case = make_prefill_case(prefix, chunk, hq, hkv, d, 16, dtype, cuda_device, seed=hq + d)
    out = paged_attention_prefill_varlen(case["q"], case["cu"], case["lens"], case["tables"], case["k"], case["v"],
                                         case["max_q"])
    check(out, oracle_prefill(case), dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("d,bs", [(8, 16), (40, 16), (64, 3), (64, 8), (96, 32), (64, 64)])
def test_odd_shapes(cuda_device, dtype, d, bs):
    case = make_prefill_case([0, 9, 50], [7, 33, 65], 8, 2, d, bs, dtype, cuda_device, seed=d * bs)
    out = paged_attention_prefill_varlen(case["q"], case["cu"], case["lens"], case["tables"], case["k"], case["v"],
                                         case["max_q"])
    check(out, oracle_prefill(case), dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_config4_geometry(cuda_device, dtype):
    """BASELINE config 4 at reduced batch: prefix U[0, 2048], 512-token chunks,
    14/2 heads, D 64, bs 16, new K/V scattered through the slot mapping first."""
    rng = np.random.default_rng(4)
    nseq = 4
    prefix = rng.integers(0, 2049, size=nseq).tolist()
    chunk = [512] * nseq
    case = make_prefill_case(prefix, chunk, 14, 2, 64, 16, dtype, cuda_device, seed=4)
    # Rewrite the chunks' K/V through write_slots to exercise the whole path.
    k_pool, v_pool = case["k"], case["v"]
    nb = k_pool.shape[0]
    cache = PagedKVCache(1, nb, 16, 2, 64, dtype=dtype, device=cuda_device)
    cache.k_cache[0].copy_(k_pool)
    cache.v_cache[0].copy_(v_pool)
    g = torch.Generator().manual_seed(44)
    slots, ks, vs = [], [], []
    for s in range(nseq):
        tbl = case["tables"][s].tolist()
        for pos in range(prefix[s], prefix[s] + chunk[s]):
            slots.append(tbl[pos // 16] * 16 + pos % 16)
    new_k = torch.randn(len(slots), 2, 64, generator=g).to(dtype)
    new_v = torch.randn(len(slots), 2, 64, generator=g).to(dtype)
    cache.write_slots(torch.tensor(slots, device=cuda_device), new_k.to(cuda_device), new_v.to(cuda_device), 0)
    kc, vc = cache.get_layer_cache(0)
    out = paged_attention_prefill_varlen(case["q"], case["cu"], case["lens"], case["tables"], kc, vc, 512)
    k_np = kc.float().cpu().numpy()
    v_np = vc.float().cpu().numpy()
    exp = []
    for s in range(nseq):
        q = case["q_np"][case["cu_np"][s] : case["cu_np"][s + 1]]
        exp.append(O.prefill_chunk(q, k_np, v_np, case["np"][3][s], prefix[s], prefix[s] + 512, 16))
    check(out, np.concatenate(exp, 0), dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv,d", [(14, 2, 64), (28, 4, 128), (8, 8, 64), (16, 1, 128)])
def test_many_items_per_cta(cuda_device, dtype, hq, hkv, d):
    """More work items than SMs, so each persistent CTA runs several items
    back to back (Q buffers and O accumulators recycled across items), with
    ragged chunks, empty-prefix and long-prefix sequences mixed."""
    rng = np.random.default_rng(hq * d + hkv)
    nseq = 40
    prefix = rng.integers(0, 700, size=nseq).tolist()
    chunk = rng.integers(1, 300, size=nseq).tolist()
    prefix[0], chunk[0] = 0, 299
    prefix[1], chunk[1] = 2900, 260
    case = make_prefill_case(prefix, chunk, hq, hkv, d, 16, dtype, cuda_device, seed=hq + 3 * d)
    out = paged_attention_prefill_varlen(case["q"], case["cu"], case["lens"], case["tables"], case["k"], case["v"],
                                         case["max_q"])
    check(out, oracle_prefill(case), dtype)
    # Same call again: the kernel keeps no state between launches.
    out2 = paged_attention_prefill_varlen(case["q"], case["cu"], case["lens"], case["tables"], case["k"], case["v"],
                                          case["max_q"])
    assert torch.equal(out, out2)


def test_prefill_block_size_32(cuda_device):
    """Blocks of 32 tokens: two 16-token TMA boxes per table entry."""
    case = make_prefill_case([0, 100, 31], [64, 90, 1], 14, 2, 64, 32, torch.bfloat16, cuda_device, seed=3)
    out = paged_attention_prefill_varlen(case["q"], case["cu"], case["lens"], case["tables"], case["k"], case["v"],
                                         case["max_q"])
    check(out, oracle_prefill(case), torch.bfloat16)


@pytest.mark.parametrize("layout", ["units", "levels"])
def test_schedule_past_the_order_table(cuda_device, layout):
    """Work past the kernel's longest-first order table (more than 512
    sequences, or a chunk whose KV range spans 512 or more 128-key tiles)
    keeps the query-position order; results are unchanged."""
    if layout == "units":
        rng = np.random.default_rng(21)
        nseq = 2100  # 1 query head per KV head: 256 positions per unit, one unit per sequence
        prefix = rng.integers(0, 40, size=nseq).tolist()
        chunk = rng.integers(1, 4, size=nseq).tolist()
        case = make_prefill_case(prefix, chunk, 8, 8, 64, 16, torch.bfloat16, cuda_device, seed=21, extra_blocks=1)
    else:
        # 8 sequences (the order table's minimum), one spanning 516 key tiles
        case = make_prefill_case([66000, 3, 17, 100, 0, 250, 64, 9], [5, 40, 33, 1, 90, 7, 64, 2], 8, 1, 64, 16,
                                 torch.bfloat16, cuda_device, seed=22)
    out = paged_attention_prefill_varlen(case["q"], case["cu"], case["lens"], case["tables"], case["k"], case["v"],
                                         case["max_q"])
    check(out, oracle_prefill(case), torch.bfloat16)


def test_static_schedule_without_control_block(cuda_device):
    """control = NULL: the kernel hands out items statically; same result as
    the dynamic schedule."""
    import ctypes

    from mini_llm_runtime_b200 import _lib

    case = make_prefill_case([0, 300, 1000] * 20, [200, 77, 5] * 20, 14, 2, 64, 16, torch.bfloat16, cuda_device,
                             seed=12)
    ref = paged_attention_prefill_varlen(case["q"], case["cu"], case["lens"], case["tables"], case["k"], case["v"],
                                         case["max_q"])
    q, out = case["q"], torch.empty_like(case["q"])
    bt = case["tables"]
    nb, bs, hkv, d = case["k"].shape
    st = _lib.load().pa_chunk_prefill(
        q.data_ptr(), q.stride(0), q.stride(1), case["cu"].data_ptr(), case["lens"].data_ptr(), bt.data_ptr(),
        bt.stride(0), bt.shape[1], case["k"].data_ptr(), case["v"].data_ptr(), nb, bs, hkv, d, out.data_ptr(),
        out.stride(0), out.stride(1), len(case["chunk"]), q.shape[0], case["max_q"], q.shape[1], d ** -0.5,
        _lib.dtype_code(q.dtype), None, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.PA_OK
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    # The shared control block was left rewound by the dynamic launches.
    assert _lib.status_word(cuda_device).tolist() == [0, 0, 0, 0]

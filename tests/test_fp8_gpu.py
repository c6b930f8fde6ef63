"""FP8 (e4m3) KV-cache pools on the GPU.

* The quantizing write (PagedKVCache.write_slots into an FP8 pool, the fused
  decode write) stores exactly the oracle's bytes: clamp(x / scale) rounded
  to nearest even.
* Decode and chunk-prefill over FP8 pools match the oracle run on the
  dequantized pools (element * scale, FP32) within the BF16 tolerance
  (2e-2 absolute / 1e-2 relative): the kernels' only extra rounding is the
  f16 probabilities of the FP8 MMA path, finer than BF16's.
"""

import numpy as np
import pytest
import torch

from mini_llm_runtime_b200 import (
    PagedDecodeGraph,
    PagedKVCache,
    paged_attention_decode_batch_parallel,
    paged_attention_prefill_varlen,
    paged_decode_with_kv_write,
)
from oracle import paged_attention_oracle as O
from tests.paged_inputs import make_decode_case, make_prefill_case

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-2, atol=2e-2)
FP8 = torch.float8_e4m3fn


def to_fp8(x32: np.ndarray, scale: float, device) -> torch.Tensor:
    """Oracle-quantized FP8 pool on the device."""
    return torch.from_numpy(O.quantize_e4m3(x32, scale)).view(FP8).to(device)


def fp8_case(case, ks, vs, device):
    """Replace a case's pools by FP8 quantizations; returns the dequantized
    pools the oracle sees."""
    q, k, v, tables, lens = case["np"]
    case["k"], case["v"] = to_fp8(k, ks, device), to_fp8(v, vs, device)
    kd = O.dequantize_e4m3(O.quantize_e4m3(k, ks), ks)
    vd = O.dequantize_e4m3(O.quantize_e4m3(v, vs), vs)
    return kd, vd


@pytest.mark.parametrize("src", [torch.bfloat16, torch.float32, torch.float16])
def test_fp8_write_slots_stores_the_oracle_bytes(cuda_device, src):
    g = torch.Generator().manual_seed(1)
    ks, vs = [0.05, 0.5], [0.07, 2.0]
    cache = PagedKVCache(2, 10, 16, 2, 64, dtype=FP8, device=cuda_device, k_scale=ks, v_scale=vs)
    cache.k_cache.view(torch.uint8).fill_(0x11)
    cache.v_cache.view(torch.uint8).fill_(0x22)
    k = (torch.randn(7, 2, 64, generator=g) * 20).to(src)
    v = (torch.randn(7, 2, 64, generator=g) * 20).to(src)
    k[0, 0, :4] = torch.tensor([1e5, -1e5, float("nan"), 0.0]).to(src)
    slots = torch.tensor([3, 17, 40, 41, 100, 159, 5])
    for layer in (0, 1):
        cache.write_slots(slots.to(cuda_device), k.to(cuda_device), v.to(cuda_device), layer)
        kf = cache.k_cache[layer].view(torch.uint8).reshape(-1, 2, 64).cpu().numpy()
        vf = cache.v_cache[layer].view(torch.uint8).reshape(-1, 2, 64).cpu().numpy()
        assert np.array_equal(kf[slots.numpy()], O.quantize_e4m3(k.float().numpy(), ks[layer]))
        assert np.array_equal(vf[slots.numpy()], O.quantize_e4m3(v.float().numpy(), vs[layer]))
        untouched = np.setdiff1d(np.arange(160), slots.numpy())
        assert (kf[untouched] == 0x11).all() and (vf[untouched] == 0x22).all()


@pytest.mark.parametrize("hq,hkv,d,bs,qdt", [
    (14, 2, 64, 16, torch.bfloat16),   # config-2 geometry: balanced kernel, two KV heads per warp
    (28, 4, 128, 16, torch.bfloat16),  # config-5 geometry
    (8, 1, 64, 32, torch.float16),     # MQA: one KV head per warp
    (36, 2, 128, 16, torch.bfloat16),  # group of 18: two head tiles
    (8, 2, 80, 16, torch.bfloat16),    # odd head_dim: CUDA-core kernel
    (14, 2, 64, 8, torch.float32),     # FP32 queries, block size 8: CUDA-core kernel
])
def test_fp8_decode_matches_oracle_on_dequantized_pools(cuda_device, hq, hkv, d, bs, qdt):
    ctx = [1, 15, 16, 17, 129, 700, 2049, 33]
    case = make_decode_case(ctx, hq, hkv, d, bs, qdt, cuda_device, seed=hq + d + bs)
    ks, vs = 0.037, 0.11
    kd, vd = fp8_case(case, ks, vs, cuda_device)
    out = paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], bs,
                                                k_scale=ks, v_scale=vs)
    assert out.dtype == qdt
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    q, _, _, tables, lens = case["np"]
    np.testing.assert_allclose(got, O.decode_batch(q, kd, vd, tables, lens, bs), **TOL)


def test_fp8_fused_write_equals_write_then_decode(cuda_device):
    hq, hkv, d, bs = 14, 2, 64, 16
    ctx = [40, 999, 16, 2500]
    case = make_decode_case(ctx, hq, hkv, d, bs, torch.bfloat16, cuda_device, seed=31, poison=False)
    ks, vs = 0.05, 0.09
    fp8_case(case, ks, vs, cuda_device)
    g = torch.Generator().manual_seed(5)
    nk = torch.randn(len(ctx), hkv, d, generator=g).to(torch.bfloat16).to(cuda_device)
    nv = torch.randn(len(ctx), hkv, d, generator=g).to(torch.bfloat16).to(cuda_device)
    tab = case["tables"].cpu().numpy()
    slots = torch.tensor([tab[b][(c - 1) // bs] * bs + (c - 1) % bs for b, c in enumerate(ctx)], device=cuda_device)
    k1, v1 = case["k"].clone(), case["v"].clone()
    out_fused = paged_decode_with_kv_write(case["q"], nk, nv, slots, k1, v1, case["tables"], case["lens"], bs,
                                           k_scale=ks, v_scale=vs)
    cache = PagedKVCache(1, case["k"].shape[0], bs, hkv, d, dtype=FP8, device=cuda_device, k_scale=ks, v_scale=vs)
    cache.k_cache[0].copy_(case["k"])
    cache.v_cache[0].copy_(case["v"])
    cache.write_slots(slots, nk, nv, 0)
    out_ref = paged_attention_decode_batch_parallel(case["q"], cache.k_cache[0], cache.v_cache[0], case["tables"],
                                                    case["lens"], bs, k_scale=ks, v_scale=vs)
    assert torch.equal(k1.view(torch.uint8), cache.k_cache[0].view(torch.uint8))
    assert torch.equal(v1.view(torch.uint8), cache.v_cache[0].view(torch.uint8))
    assert torch.equal(out_fused, out_ref)


@pytest.mark.parametrize("d", [64, 128])
def test_fp8_prefill_matches_oracle(cuda_device, d):
    prefix, chunk = [0, 100, 1000], [64, 200, 33]
    case = make_prefill_case(prefix, chunk, 14, 2, d, 16, torch.bfloat16, cuda_device, seed=d)
    ks, vs = 0.06, 0.08
    kd, vd = fp8_case(case, ks, vs, cuda_device)
    out = paged_attention_prefill_varlen(case["q"], case["cu"], case["lens"], case["tables"], case["k"], case["v"],
                                         case["max_q"], k_scale=ks, v_scale=vs)
    got = out.float().cpu().numpy()
    tables = case["np"][3]
    for s, (p, c) in enumerate(zip(prefix, chunk)):
        c0 = int(case["cu_np"][s])
        exp = O.prefill_chunk(case["q_np"][c0:c0 + c], kd, vd, tables[s], p, p + c, 16)
        np.testing.assert_allclose(got[c0:c0 + c], exp, **TOL)


def test_fp8_decode_graph_matches_eager(cuda_device):
    hq, hkv, d, bs, layers = 14, 2, 64, 16, 3
    ctx = [37, 600, 1025, 64]
    need = [(c + bs - 1) // bs for c in ctx]
    nb = sum(need) + 5
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(2)).tolist()
    tables, cur = [], 0
    for n in need:
        tables.append(perm[cur:cur + n] + [-1] * (max(need) - n))
        cur += n
    ks, vs = [0.04, 0.05, 0.06], [0.07, 0.08, 0.09]
    cache = PagedKVCache(layers, nb, bs, hkv, d, dtype=FP8, device=cuda_device, k_scale=ks, v_scale=vs)
    src = torch.randn(2, layers, nb, bs, hkv, d) * 0.2
    cache.k_cache.copy_(src[0].to(FP8))
    cache.v_cache.copy_(src[1].to(FP8))
    ref_k, ref_v = cache.k_cache.clone(), cache.v_cache.clone()
    g = PagedDecodeGraph(cache, batch=len(ctx), max_blocks=max(need), num_q_heads=hq, layers=range(layers))
    hi = g.host_inputs
    hi["q"].copy_(torch.randn(hi["q"].shape).to(torch.bfloat16))
    hi["new_k"].copy_(torch.randn(hi["new_k"].shape).to(torch.bfloat16))
    hi["new_v"].copy_(torch.randn(hi["new_v"].shape).to(torch.bfloat16))
    hi["block_tables"].copy_(torch.tensor(tables))
    hi["context_lens"].copy_(torch.tensor(ctx))
    hi["slot_mapping"].copy_(torch.tensor([tables[b][(c - 1) // bs] * bs + (c - 1) % bs for b, c in enumerate(ctx)]))
    g.run()
    g.synchronize()
    ref = PagedKVCache(layers, nb, bs, hkv, d, dtype=FP8, device=cuda_device, k_scale=ks, v_scale=vs)
    ref.k_cache.copy_(ref_k)
    ref.v_cache.copy_(ref_v)
    dv = {k: v.to(cuda_device) for k, v in hi.items()}
    for layer in range(layers):
        ref.write_slots(dv["slot_mapping"], dv["new_k"][layer], dv["new_v"][layer], layer)
        exp = paged_attention_decode_batch_parallel(dv["q"][layer], ref.k_cache[layer], ref.v_cache[layer],
                                                    dv["block_tables"], dv["context_lens"], bs,
                                                    k_scale=ks[layer], v_scale=vs[layer])
        assert torch.equal(g.host_output[layer], exp.cpu())
    assert torch.equal(cache.k_cache.view(torch.uint8), ref.k_cache.view(torch.uint8))

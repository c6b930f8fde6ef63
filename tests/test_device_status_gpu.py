"""Device-side failure reporting, tested without a GPU fault.

Every wait inside the kernels is bounded: when it runs out the kernel writes
PA_DEVICE_TIMEOUT_* into a status word and returns.  pa_selftest_wait_timeout
runs that path on an mbarrier nothing arrives on (a short limit, no fault, no
hang); these tests check that the status reaches the host through every
reporting route: the raw word, check_device_status() for the ops' workspaces
and control blocks, PagedDecodeGraph.synchronize(), and the allocation-free
decode's status query.  Afterwards the same workspaces must serve a normal
call again."""

import ctypes

import numpy as np
import pytest
import torch

from mini_llm_runtime_b200 import (
    PagedAttentionError,
    PagedDecodeGraph,
    PagedKVCache,
    _lib,
    check_device_status,
    device_status,
    paged_attention_decode_batch_parallel,
    paged_attention_prefill_varlen,
)
from oracle import paged_attention_oracle as O
from tests.paged_inputs import make_decode_case, make_prefill_case

pytestmark = pytest.mark.gpu
LIMIT_NS = 20_000_000  # 20 ms


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _time_out_into(word: torch.Tensor) -> None:
    """Make one bounded wait run out and record its status in `word` (int32)."""
    assert word.dtype == torch.int32 and word.is_cuda
    assert _lib.load().pa_selftest_wait_timeout(word.data_ptr(), LIMIT_NS, _stream()) == _lib.PA_OK


def test_bounded_wait_runs_out_and_reports(cuda_device):
    word = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _time_out_into(word)
    torch.cuda.synchronize()
    assert int(word.item()) == _lib.PA_DEVICE_TIMEOUT_TMA
    # The first recorded status is kept.
    word.fill_(_lib.PA_DEVICE_TIMEOUT_MMA)
    _time_out_into(word)
    torch.cuda.synchronize()
    assert int(word.item()) == _lib.PA_DEVICE_TIMEOUT_MMA
    # The context is still usable.
    assert torch.arange(4, device=cuda_device).sum().item() == 6


def test_selftest_rejects_bad_limits(cuda_device):
    word = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    lib = _lib.load()
    assert lib.pa_selftest_wait_timeout(word.data_ptr(), 10, _stream()) == _lib.PA_ERR_INVALID
    assert lib.pa_selftest_wait_timeout(word.data_ptr(), 10**10, _stream()) == _lib.PA_ERR_INVALID
    assert lib.pa_selftest_wait_timeout(None, LIMIT_NS, _stream()) == _lib.PA_ERR_INVALID


def test_ops_raise_after_a_device_timeout_and_recover(cuda_device):
    case = make_decode_case([100, 700, 33], 14, 2, 64, 16, torch.bfloat16, cuda_device, seed=4)
    args = (case["q"], case["k"], case["v"], case["tables"], case["lens"], 16)
    first = paged_attention_decode_batch_parallel(*args)
    check_device_status(cuda_device)  # clean
    # Record a timeout in the workspace status word that call used.
    key = (cuda_device.index, torch.cuda.current_stream().cuda_stream)
    ws = _lib._workspaces[key].tensor
    _time_out_into(ws[:4].view(torch.int32))
    assert device_status(cuda_device), "the recorded status is visible"
    with pytest.raises(PagedAttentionError, match="TMA"):
        check_device_status(cuda_device)
    assert device_status(cuda_device) == []  # re-zeroed before raising
    again = paged_attention_decode_batch_parallel(*args)
    assert torch.equal(first, again)


def test_prefill_control_block_is_per_stream_and_reports(cuda_device):
    case = make_prefill_case([40, 300], [16, 100], 14, 2, 64, 16, torch.bfloat16, cuda_device, seed=6)
    args = (case["q"], case["cu"], case["lens"], case["tables"], case["k"], case["v"], case["max_q"])
    out_main = paged_attention_prefill_varlen(*args)
    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        out_side = paged_attention_prefill_varlen(*args)
        block_side = _lib.status_word(cuda_device)
    torch.cuda.synchronize()
    block_main = _lib.status_word(cuda_device)
    assert block_main.data_ptr() != block_side.data_ptr()
    assert torch.equal(out_main, out_side)
    _time_out_into(block_side[:1])
    torch.cuda.synchronize()
    with pytest.raises(PagedAttentionError, match="prefill control block"):
        check_device_status(cuda_device)
    assert int(block_side[0].item()) == 0


def test_decode_graph_synchronize_reports_and_recovers(cuda_device):
    hq, hkv, d, bs = 14, 2, 64, 16
    ctx = [50, 333]
    need = [(c + bs - 1) // bs for c in ctx]
    nb = sum(need) + 2
    tables = [list(range(need[0])), list(range(need[0], need[0] + need[1]))]
    width = max(need)
    cache = PagedKVCache(1, nb, bs, hkv, d, dtype=torch.bfloat16, device=cuda_device)
    cache.k_cache.normal_()
    cache.v_cache.normal_()
    g = PagedDecodeGraph(cache, batch=2, max_blocks=width, num_q_heads=hq, layers=[0], write_kv=False)
    hi = g.host_inputs
    hi["q"].copy_(torch.randn(hi["q"].shape).to(torch.bfloat16))
    hi["block_tables"].copy_(torch.tensor([t + [-1] * (width - len(t)) for t in tables]))
    hi["context_lens"].copy_(torch.tensor(ctx))
    hi["slot_mapping"].copy_(torch.tensor([tables[b][(c - 1) // bs] * bs + (c - 1) % bs for b, c in enumerate(ctx)]))
    g.run()
    g.synchronize()
    ok = g.host_output.clone()
    _time_out_into(g.workspace[:4].view(torch.int32))
    with pytest.raises(PagedAttentionError, match="TMA"):
        g.synchronize()
    g.run()
    g.synchronize()  # workspace re-zeroed: the next step is clean
    assert torch.equal(g.host_output, ok)


def test_decode_graph_inputs_refilled_after_wait(cuda_device):
    """Inputs refilled after wait_inputs_consumed() are the ones the next
    replay uses (no mix of two steps)."""
    hq, hkv, d, bs = 14, 2, 64, 16
    ctx = [64, 1000, 17]
    need = [(c + bs - 1) // bs for c in ctx]
    width = max(need)
    case = make_decode_case(ctx, hq, hkv, d, bs, torch.bfloat16, cuda_device, seed=9, poison=False)
    cache = PagedKVCache(2, case["k"].shape[0], bs, hkv, d, dtype=torch.bfloat16, device=cuda_device)
    for layer in range(2):
        cache.k_cache[layer].copy_(case["k"])
        cache.v_cache[layer].copy_(case["v"])
    g = PagedDecodeGraph(cache, batch=3, max_blocks=width, num_q_heads=hq, layers=[0, 1], write_kv=False)
    hi = g.host_inputs
    hi["block_tables"].copy_(case["tables"].cpu())
    hi["context_lens"].copy_(case["lens"].cpu())
    tab = case["tables"].cpu().numpy()
    hi["slot_mapping"].copy_(torch.tensor([tab[b][(c - 1) // bs] * bs + (c - 1) % bs for b, c in enumerate(ctx)]))
    k_np, v_np = case["np"][1], case["np"][2]
    for step in range(3):
        g.wait_inputs_consumed()
        q = torch.randn(hi["q"].shape).to(torch.bfloat16)
        hi["q"].copy_(q)
        g.run()
        g.synchronize()
        for layer in range(2):
            exp = O.decode_batch(q[layer].float().numpy(), k_np, v_np, tab, np.array(ctx), bs)
            np.testing.assert_allclose(g.host_output[layer].float().numpy(), exp, rtol=1e-2, atol=2e-2)


def test_noalloc_status_query_reports_the_scratch_word(cuda_device):
    """pa_decode_noalloc_status reads the built-in scratch's status word: 0
    after a normal call (the call clears it first)."""
    from tests.test_zz_no_alloc import noalloc_decode

    case = make_decode_case([300, 5], 14, 2, 64, 16, torch.bfloat16, cuda_device, seed=12)
    st, _ = noalloc_decode(case, torch.bfloat16)
    assert st == _lib.PA_OK
    status = ctypes.c_int(-1)
    assert _lib.load().pa_decode_noalloc_status(ctypes.byref(status), _stream()) == _lib.PA_OK
    torch.cuda.synchronize()
    assert status.value == 0
    assert _lib.load().pa_decode_noalloc_status(None, _stream()) == _lib.PA_ERR_INVALID

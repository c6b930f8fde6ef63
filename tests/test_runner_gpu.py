"""The runner on the GPU against the reference's own runner
(tests/golden/runner_steps.npz: the reference's TinyQwen2ForCausalLM through
its build_model_batch and execute_model_batch, three scheduler steps).

* build_model_batch on the device reproduces the reference's ModelBatch
  tensors bit for bit.
* execute_model_batch replays the steps (same pending tokens) with this
  package's Qwen2Attention swapped into the reference's module tree: FP32
  logits within 1e-4 of the reference's, the same greedy tokens, the written
  KV rows within 1e-5; BF16 (tensor-core prefill, balanced decode) within
  5e-2 of the FP32 reference logits.
"""

import numpy as np
import pytest
import torch

from mini_llm_runtime_b200 import PagedKVCache
from mini_llm_runtime_b200.runner import build_model_batch, execute_model_batch, swap_attention
from tests.test_runner_host import FIELDS, M, replay_outputs
from tests.tiny_qwen2 import CausalLM, WeightsOnlyAttention, make_config

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("debug", [False, True])
def test_device_builder_matches_the_reference_model_batches(cuda_device, monkeypatch, debug):
    monkeypatch.setenv("MINI_LLM_RUNTIME_DEBUG_CHECKS", "1" if debug else "0")
    steps, _ = replay_outputs()
    for out, want, _, _ in steps:
        b = build_model_batch(out, M.BLOCK_SIZE, cuda_device)
        for k in FIELDS:
            got = getattr(b, k)
            assert got.is_cuda and got.dtype == torch.long
            assert np.array_equal(got.cpu().numpy(), want[k]), k


def _model(dtype, device):
    model = CausalLM(make_config(M.CONFIG), WeightsOnlyAttention)
    model.load_state_dict(M.weights(), strict=True)
    swap_attention(model)
    return model.to(device=device, dtype=dtype).eval()


def _replay(dtype, device):
    steps, g = replay_outputs()
    model = _model(dtype, device)
    d = M.CONFIG["hidden_size"] // M.CONFIG["num_attention_heads"]
    cache = PagedKVCache(M.CONFIG["num_hidden_layers"], M.NUM_BLOCKS, M.BLOCK_SIZE, M.CONFIG["num_key_value_heads"], d,
                         dtype=dtype, device=device)
    logits = []
    with torch.no_grad():
        for out, _, want, _ in steps:
            batch = build_model_batch(out, M.BLOCK_SIZE, device)
            logits.append((execute_model_batch(model, batch, cache).float().cpu().numpy(), want))
    return logits, cache, g


def test_fp32_replay_matches_the_reference_runner(cuda_device):
    logits, cache, g = _replay(torch.float32, cuda_device)
    for s, (got, want) in enumerate(logits):
        assert got.shape == want.shape
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
        qsl = g[f"s{s}_query_start_loc"]
        assert [int(got[qsl[i + 1] - 1].argmax()) for i in range(len(qsl) - 1)] == g[f"s{s}_sampled"].tolist()
    slots = torch.from_numpy(g["written_slots"]).to(cuda_device)
    for pool, name in ((cache.k_cache, "k_written"), (cache.v_cache, "v_written")):
        np.testing.assert_allclose(pool.flatten(1, 2)[:, slots].cpu().numpy(), g[name], rtol=1e-5, atol=1e-5)


def test_bf16_replay_matches_the_reference_runner(cuda_device):
    logits, _, _ = _replay(torch.bfloat16, cuda_device)
    for got, want in logits:
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, want, rtol=5e-2, atol=5e-2)


def test_interleaved_phases_take_the_indexed_rows(cuda_device):
    """Decode and prefill requests interleaved in the packed order (the
    reference keeps that order, model_runner.py:250): the same logits as the
    grouped order, row for row."""
    steps, _ = replay_outputs()
    model = _model(torch.float32, cuda_device)
    d = M.CONFIG["hidden_size"] // M.CONFIG["num_attention_heads"]

    def run(order):
        cache = PagedKVCache(M.CONFIG["num_hidden_layers"], M.NUM_BLOCKS, M.BLOCK_SIZE,
                             M.CONFIG["num_key_value_heads"], d, dtype=torch.float32, device=cuda_device)
        with torch.no_grad():
            execute_model_batch(model, build_model_batch(steps[0][0], M.BLOCK_SIZE, cuda_device), cache)
            b = build_model_batch(steps[1][0], M.BLOCK_SIZE, cuda_device)
            if order is not None:
                b = _reorder(b, order)
            return execute_model_batch(model, b, cache), b

    base, b0 = run(None)
    perm = [1, 0, 3, 2]  # decode A, prefill D, decode C, decode B
    mixed, b1 = run(perm)
    qsl0 = b0.query_start_loc.tolist()
    qsl1 = b1.query_start_loc.tolist()
    for new, old in enumerate(perm):
        torch.testing.assert_close(mixed[qsl1[new]:qsl1[new + 1]], base[qsl0[old]:qsl0[old + 1]], rtol=1e-5,
                                   atol=1e-5)


def _reorder(b, order):
    from mini_llm_runtime_b200.runner import BatchHostMeta, ModelBatch

    h = b.host
    qsl = h.query_start_loc
    rows = np.concatenate([np.arange(qsl[i], qsl[i + 1]) for i in order])
    r = torch.from_numpy(rows).to(b.input_token_ids.device)
    counts = np.diff(qsl)[order]
    nq = np.concatenate([[0], np.cumsum(counts)])
    o = torch.tensor(order, device=b.input_token_ids.device)
    host = BatchHostMeta(nq, h.context_lens[order], h.block_tables[order])
    return ModelBatch([b.request_ids[i] for i in order], b.input_token_ids[r], b.positions[r],
                      torch.from_numpy(nq).to(r.device), [b.request_phases[i] for i in order], b.context_lens[o],
                      b.block_tables[o], b.slot_mapping[r], host)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_step_graph_replays_the_model_decode_step(cuda_device, dtype):
    """The fixture's third step (decodes only) as one CUDA graph of the whole
    model (DecodeStepGraph): its logits match the eager execute_model_batch
    (FP32 within 1e-5, BF16 within 1e-2) and the reference runner's (FP32
    within 1e-4), it writes the same KV rows, and replaying the same step
    again gives the same logits bit for bit."""
    from mini_llm_runtime_b200 import DecodeStepGraph

    steps, _ = replay_outputs()
    model = _model(dtype, cuda_device)
    d = M.CONFIG["hidden_size"] // M.CONFIG["num_attention_heads"]

    def cache_after_two_steps():
        cache = PagedKVCache(M.CONFIG["num_hidden_layers"], M.NUM_BLOCKS, M.BLOCK_SIZE,
                             M.CONFIG["num_key_value_heads"], d, dtype=dtype, device=cuda_device)
        cache.k_cache.zero_()  # the pools start uninitialised; zeroed, they compare whole
        cache.v_cache.zero_()
        for out, _, _, _ in steps[:2]:
            execute_model_batch(model, build_model_batch(out, M.BLOCK_SIZE, cuda_device), cache)
        return cache

    out3, _, want3, _ = steps[2]
    with torch.no_grad():
        eager_cache = cache_after_two_steps()
        eager = execute_model_batch(model, build_model_batch(out3, M.BLOCK_SIZE, cuda_device), eager_cache).clone()
        cache = cache_after_two_steps()
        batch = build_model_batch(out3, M.BLOCK_SIZE, cuda_device)
        g = DecodeStepGraph(model, cache, len(batch.request_ids), batch.block_tables.shape[1] + 3)
        first = g.run(batch).clone()
        again = g.run(build_model_batch(out3, M.BLOCK_SIZE, cuda_device)).clone()
        torch.cuda.synchronize()
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    torch.testing.assert_close(first, eager, rtol=tol, atol=tol)
    assert torch.equal(first, again)
    torch.testing.assert_close(cache.k_cache, eager_cache.k_cache, rtol=tol, atol=tol)
    torch.testing.assert_close(cache.v_cache, eager_cache.v_cache, rtol=tol, atol=tol)
    if dtype == torch.float32:
        np.testing.assert_allclose(first.float().cpu().numpy(), want3, rtol=1e-4, atol=1e-4)

"""Runner host logic on CPU: build_model_batch against the reference's own
ModelBatch tensors (tests/golden/runner_steps.npz), its error messages, the
attention swap, and execute_model_batch's checks (all made before any
kernel runs)."""

import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from mini_llm_runtime_b200 import PagedKVCache, Qwen2Attention
from mini_llm_runtime_b200.runner import ModelBatch, RequestStatus, build_model_batch, execute_model_batch, swap_attention
from tests.tiny_qwen2 import CausalLM, WeightsOnlyAttention, make_config

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import runner_model as M  # noqa: E402

FIELDS = ("input_token_ids", "positions", "query_start_loc", "context_lens", "block_tables", "slot_mapping")


def replay_outputs():
    """The fixture's scheduler outputs, as duck-typed requests: each step's
    prefill/decode lists with the pending tokens the reference sampled."""
    g = np.load(GOLDEN / "runner_steps.npz")
    prompts, tables = M.prompts(), M.block_tables()
    state = {rid: SimpleNamespace(request_id=rid, prompt_token_ids=prompts[rid], block_table=list(tables[rid]),
                                  num_computed_tokens=0, output_token_ids=[]) for rid in M.PROMPT_LENS}
    steps = []
    for s, (pre, dec) in enumerate(M.STEPS):
        sched = {rid: len(prompts[rid]) - state[rid].num_computed_tokens for rid in pre}
        sched.update({rid: 1 for rid in dec})
        reqs = {}
        for rid in pre + dec:
            r = state[rid]
            reqs[rid] = SimpleNamespace(request_id=rid, prompt_token_ids=r.prompt_token_ids,
                                        block_table=list(r.block_table), num_computed_tokens=r.num_computed_tokens,
                                        pending_token_id=r.output_token_ids[-1] if r.output_token_ids else None)
        out = SimpleNamespace(prefill_requests=[reqs[r] for r in pre], decode_requests=[reqs[r] for r in dec],
                              num_scheduled_tokens=sched)
        steps.append((out, {k: g[f"s{s}_{k}"] for k in FIELDS}, g[f"s{s}_logits"], g[f"s{s}_request_ids"]))
        for i, rid in enumerate(g[f"s{s}_request_ids"]):
            state[str(rid)].num_computed_tokens += sched[str(rid)]
            state[str(rid)].output_token_ids.append(int(g[f"s{s}_sampled"][i]))
    return steps, g


def test_cpu_builder_matches_the_reference_model_batches():
    steps, _ = replay_outputs()
    for out, want, _, rids in steps:
        b = build_model_batch(out, M.BLOCK_SIZE, "cpu")
        assert b.request_ids == [str(r) for r in rids]
        for k in FIELDS:
            got = getattr(b, k)
            assert got.dtype == torch.long and np.array_equal(got.numpy(), want[k]), k
        assert np.array_equal(b.host.query_start_loc, want["query_start_loc"])
        assert np.array_equal(b.host.context_lens, want["context_lens"])
        assert np.array_equal(b.host.block_tables, want["block_tables"])


def _req(rid, prompt, table, computed=0, pending=None):
    return SimpleNamespace(request_id=rid, prompt_token_ids=prompt, block_table=table, num_computed_tokens=computed,
                           pending_token_id=pending)


def test_builder_errors_match_the_reference_messages():
    out = SimpleNamespace(prefill_requests=[_req("a", [1, 2, 3], [0])], decode_requests=[],
                          num_scheduled_tokens={"a": 3})
    with pytest.raises(ValueError, match="block_size must be greater than 0"):
        build_model_batch(out, 0)
    out.num_scheduled_tokens = {"a": 5}
    with pytest.raises(ValueError, match="Request a expected 5 prefill tokens, got 3"):
        build_model_batch(out, 4)
    out.num_scheduled_tokens = {"a": 3}
    with pytest.raises(ValueError, match="Request a has no KV cache block for position 2"):
        build_model_batch(out, 2)
    dec = SimpleNamespace(prefill_requests=[], decode_requests=[_req("d", [1], [0], 1, 7)],
                          num_scheduled_tokens={"d": 2})
    with pytest.raises(ValueError, match="Decode currently supports exactly one token per request"):
        build_model_batch(dec, 4)
    dec.num_scheduled_tokens = {"d": 1}
    dec.decode_requests[0].pending_token_id = None
    with pytest.raises(ValueError, match="Decode request d has no pending token"):
        build_model_batch(dec, 4)
    empty = build_model_batch(SimpleNamespace(prefill_requests=[], decode_requests=[], num_scheduled_tokens={}), 4)
    assert empty.block_tables.shape == (0, 0) and empty.query_start_loc.tolist() == [0]


def test_swap_attention_carries_the_reference_weights():
    cfg = make_config(M.CONFIG)
    model = CausalLM(cfg, WeightsOnlyAttention)
    model.load_state_dict(M.weights(), strict=True)
    before = {k: v.clone() for k, v in model.state_dict().items()}
    swap_attention(model)
    assert all(isinstance(layer.self_attn, Qwen2Attention) for layer in model.model.layers)
    after = model.state_dict()
    assert before.keys() == after.keys()
    assert all(torch.equal(before[k], after[k]) for k in before)


def _batch(phases, qsl, ctx, tables, tokens=None):
    t = int(qsl[-1])
    return ModelBatch(request_ids=[f"r{i}" for i in range(len(phases))],
                      input_token_ids=torch.zeros(t, dtype=torch.long) if tokens is None else tokens,
                      positions=torch.zeros(t, dtype=torch.long), query_start_loc=torch.tensor(qsl),
                      request_phases=phases, context_lens=torch.tensor(ctx), block_tables=torch.tensor(tables),
                      slot_mapping=torch.zeros(t, dtype=torch.long))


def test_execute_checks_run_before_any_kernel():
    cfg = make_config(M.CONFIG)
    model = CausalLM(cfg, Qwen2Attention)
    cache = PagedKVCache(2, 8, 16, 1, 64, dtype=torch.float32, device="cpu")
    P, D = RequestStatus.PREFILLING, RequestStatus.DECODING
    with pytest.raises(ValueError, match="Cannot execute an empty ModelBatch"):
        execute_model_batch(model, _batch([], [0], [], np.zeros((0, 1), np.int64)), cache)
    with pytest.raises(ValueError, match="query_start_loc must be strictly increasing"):
        execute_model_batch(model, _batch([P, P], [0, 2, 2], [2, 1], [[0], [1]]), cache)
    with pytest.raises(ValueError, match="Request r1 block_table contains an invalid physical block"):
        execute_model_batch(model, _batch([P, P], [0, 2, 3], [2, 1], [[0], [8]]), cache)
    with pytest.raises(ValueError, match="Request r0 block_table has insufficient blocks"):
        execute_model_batch(model, _batch([P], [0, 2], [17], [[0]]), cache)
    with pytest.raises(ValueError, match="Decode requires exactly one token per request"):
        execute_model_batch(model, _batch([D], [0, 2], [2], [[0]]), cache)
    with pytest.raises(ValueError, match="Unsupported request phase"):
        execute_model_batch(model, _batch([RequestStatus.WAITING], [0, 1], [1], [[0]]), cache)
    bad = _batch([P], [0, 1], [1], [[0]])
    bad.positions = bad.positions.int()
    with pytest.raises(ValueError, match="positions must use torch.long dtype"):
        execute_model_batch(model, bad, cache)
    weights_only = CausalLM(cfg, WeightsOnlyAttention)
    with pytest.raises(TypeError, match="swap_attention"):
        execute_model_batch(weights_only, _batch([P], [0, 1], [1], [[0]]), cache)

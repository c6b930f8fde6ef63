"""Scheduler-step runner on the paged kernels: ModelBatch built on the device,
one batched chunk-prefill per layer for every prefill request of the step.

Mirrors runtime/model_runner.py of the reference:

* ``ModelBatch`` (:13-27): the same fields, plus ``host``, the per-request
  metadata the builder already holds on the host (query starts, context
  lengths, padded block tables), so the runner never reads it back.
* ``build_model_batch`` (:37-143): the same checks, order and messages.  The
  per-token work (positions, KV slots; a Python loop per token in the
  reference, :56-66) and the padded tables run on the GPU in one kernel
  (``pa_build_batch_metadata``) after ONE host->device copy of per-request
  numbers, block tables and token ids.
* ``execute_model_batch`` (:146-272): the same checks and messages, made on
  host arrays (``batch.host``, or one device->host copy of the metadata for a
  batch built elsewhere) instead of an ``.item()`` / ``torch.any`` per check.
  The reference runs each prefill request through the whole model on its own
  (:261-272, ``forward_prefill_with_cache``); here every layer runs all of
  the step's prefill tokens at once through ``pa_chunk_prefill``
  (Qwen2Attention.prefill_batch_planned) and all decode tokens through the
  balanced decode (decode_batch_planned), with the per-token modules (RMSNorm,
  MLP, embeddings, lm_head) applied to the packed [T, hidden] rows.

Chunk semantics: a prefill request's attention covers its cached prefix plus
its chunk (context_lens = num_computed_tokens + scheduled tokens), which is
what the reference's forward_prefill_chunk_with_cache computes.  For a whole
prompt (num_computed_tokens = 0) that equals the reference runner's dense
per-request prefill; for a prompt split across steps the reference runner's
dense path attends the chunk alone.

The model is any module tree with the reference's names
(``model.embed_tokens``, ``model.layers[i].{input_layernorm, self_attn,
post_attention_layernorm, mlp}``, ``model.norm``, ``lm_head``) whose attention
modules are this package's ``Qwen2Attention``: ``swap_attention`` replaces the
reference's modules in place, carrying their weights over.
"""

from __future__ import annotations

import enum
import os
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .paged_kv_cache import PagedKVCache
from .qwen2_attention import Qwen2Attention, new_token_blocks_private


class RequestStatus(enum.Enum):
    """Request phases as the reference names them (runtime/request.py:5-10).
    Phases are compared by value, so the reference's own enum works too."""

    WAITING = "WAITING"
    PREFILLING = "PREFILLING"
    DECODING = "DECODING"
    FINISHED = "FINISHED"


def _phase(p) -> str:
    return getattr(p, "value", p)


def debug_checks_enabled() -> bool:
    """MINI_LLM_RUNTIME_DEBUG_CHECKS=1: read back and compare what the device
    built (one extra sync per step)."""
    return os.environ.get("MINI_LLM_RUNTIME_DEBUG_CHECKS", "0") not in ("", "0", "false", "False")


@dataclass
class BatchHostMeta:
    """Per-request metadata of a ModelBatch, on the host."""

    query_start_loc: np.ndarray  # [R + 1] int64
    context_lens: np.ndarray  # [R] int64
    block_tables: np.ndarray  # [R, W] int64, -1 padded


@dataclass
class ModelBatch:
    """Flattened model inputs of one scheduler step (model_runner.py:13-27)."""

    request_ids: list[str]
    input_token_ids: torch.Tensor
    positions: torch.Tensor
    query_start_loc: torch.Tensor
    request_phases: list
    context_lens: torch.Tensor
    block_tables: torch.Tensor
    slot_mapping: torch.Tensor
    host: BatchHostMeta | None = None


def build_model_batch(scheduler_output, block_size: int, device: torch.device | str = "cpu") -> ModelBatch:
    """ModelBatch of one scheduler step (model_runner.py:37-143).

    Host work is per request (the checks, token gathering); positions, slots
    and padded tables are built by one kernel on a CUDA device.  A CPU device
    gets the same tensors assembled with numpy."""
    if block_size <= 0:
        raise ValueError("block_size must be greater than 0")
    request_ids: list[str] = []
    phases: list = []
    starts: list[int] = []
    counts: list[int] = []
    tables: list[list[int]] = []
    tokens: list[int] = []

    def check_slots(request, first: int, n: int) -> None:
        # append_slots (:56-66) raises at the first position without a block.
        have = len(request.block_table) * block_size
        if first + n > have:
            raise ValueError(
                f"Request {request.request_id} has no KV cache block for position {max(first, have)}")

    for request in scheduler_output.prefill_requests:
        phases.append(RequestStatus.PREFILLING)
        n = scheduler_output.num_scheduled_tokens[request.request_id]
        start = request.num_computed_tokens
        toks = request.prompt_token_ids[start:start + n]
        if len(toks) != n:
            raise ValueError(f"Request {request.request_id} expected {n} prefill tokens, got {len(toks)}")
        request_ids.append(request.request_id)
        tokens.extend(toks)
        starts.append(start)
        counts.append(n)
        tables.append(list(request.block_table))
        check_slots(request, start, n)
    for request in scheduler_output.decode_requests:
        phases.append(RequestStatus.DECODING)
        n = scheduler_output.num_scheduled_tokens[request.request_id]
        if n != 1:
            raise ValueError("Decode currently supports exactly one token per request")
        pending = request.pending_token_id
        if pending is None:
            raise ValueError(f"Decode request {request.request_id} has no pending token")
        request_ids.append(request.request_id)
        tokens.append(pending)
        starts.append(request.num_computed_tokens)
        counts.append(1)
        tables.append(list(request.block_table))
        check_slots(request, request.num_computed_tokens, 1)

    dev = torch.device(device)
    R, T = len(request_ids), len(tokens)
    W = max((len(t) for t in tables), default=0)
    start_h = np.asarray(starts, dtype=np.int64)
    count_h = np.asarray(counts, dtype=np.int64)
    tlen_h = np.asarray([len(t) for t in tables], dtype=np.int64)
    toff_h = np.concatenate([[0], np.cumsum(tlen_h)[:-1]]).astype(np.int64) if R else np.zeros(0, np.int64)
    flat_h = np.asarray([b for t in tables for b in t], dtype=np.int64)
    tok_h = np.asarray(tokens, dtype=np.int64)
    qsl_h = np.concatenate([[0], np.cumsum(count_h)]).astype(np.int64)
    ctx_h = start_h + count_h
    bt_h = np.full((R, W), -1, dtype=np.int64)
    for i, t in enumerate(tables):
        bt_h[i, :len(t)] = t
    host = BatchHostMeta(qsl_h, ctx_h, bt_h)

    if dev.type != "cuda":
        pos_h = np.concatenate([np.arange(s, s + n) for s, n in zip(starts, counts)]) if T else np.zeros(0, np.int64)
        seq = np.repeat(np.arange(R), count_h)
        slot_h = bt_h[seq, pos_h // block_size] * block_size + pos_h % block_size if T else np.zeros(0, np.int64)

        def cpu(a):
            return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int64)).to(dev)

        return ModelBatch(request_ids, cpu(tok_h), cpu(pos_h), cpu(qsl_h), phases, cpu(ctx_h),
                          cpu(bt_h) if R else torch.empty((0, 0), dtype=torch.long, device=dev), cpu(slot_h), host)

    lib = _lib.load()
    packed_h = np.concatenate([start_h, count_h, toff_h, tlen_h, flat_h, tok_h])
    packed = torch.from_numpy(packed_h).pin_memory().to(dev, non_blocking=True)
    out = torch.empty(R + 1 + R + R * W + 3 * T, dtype=torch.long, device=dev)
    qsl = out[:R + 1]
    ctx = out[R + 1:2 * R + 1]
    bt = out[2 * R + 1:2 * R + 1 + R * W].view(R, W)
    pos, slots, toks = out[2 * R + 1 + R * W:].view(3, T).unbind(0)
    if R == 0:
        qsl.zero_()
    status = torch.zeros(1, dtype=torch.int32, device=dev) if debug_checks_enabled() else None
    rc = lib.pa_build_batch_metadata(packed.data_ptr(), R, int(flat_h.size), T, block_size, W, qsl.data_ptr(),
                                     pos.data_ptr(), ctx.data_ptr(), bt.data_ptr(), slots.data_ptr(),
                                     toks.data_ptr(), None if status is None else status.data_ptr(),
                                     _lib.stream_handle(dev))
    _lib.check(rc, "pa_build_batch_metadata")
    batch = ModelBatch(request_ids, toks, pos, qsl, phases, ctx,
                       bt if R else torch.empty((0, 0), dtype=torch.long, device=dev), slots, host)
    if status is not None:
        _verify_device_batch(batch, status, block_size)
    return batch


def _verify_device_batch(batch: ModelBatch, status: torch.Tensor, block_size: int) -> None:
    """Debug check: the device-built tensors agree with the host metadata."""
    word = int(status.item())
    h = batch.host
    if word != 0:
        raise _lib.PagedAttentionError(f"pa_build_batch_metadata recorded status {word}")
    if not (np.array_equal(batch.query_start_loc.cpu().numpy(), h.query_start_loc)
            and np.array_equal(batch.context_lens.cpu().numpy(), h.context_lens)
            and np.array_equal(batch.block_tables.cpu().numpy().reshape(h.block_tables.shape), h.block_tables)):
        raise _lib.PagedAttentionError("device-built ModelBatch disagrees with its host metadata")


def swap_attention(model, config=None):
    """Replace every decoder layer's ``self_attn`` by this package's
    Qwen2Attention carrying the same weights (the reference's parameter names
    ``qkv_proj.{q,k,v}_proj`` / ``o_proj`` load unchanged).  Returns the model."""
    inner = model.model
    cfg = config if config is not None else inner.config
    for layer in inner.layers:
        old = layer.self_attn
        if isinstance(old, Qwen2Attention):
            continue
        ref = next(old.parameters())
        new = Qwen2Attention(cfg).to(device=ref.device, dtype=ref.dtype)
        new.load_state_dict(old.state_dict(), strict=True)
        layer.self_attn = new
    return model


def _host_meta(batch: ModelBatch) -> BatchHostMeta:
    """batch.host, or one device->host copy of a batch built elsewhere."""
    if batch.host is not None:
        return batch.host
    r = batch.context_lens.numel()
    w = batch.block_tables.shape[1]
    flat = torch.cat([batch.query_start_loc.reshape(-1), batch.context_lens.reshape(-1),
                      batch.block_tables.reshape(-1)]).cpu().numpy()
    return BatchHostMeta(flat[:r + 1], flat[r + 1:2 * r + 1], flat[2 * r + 1:].reshape(r, w))


def execute_model_batch(model, batch: ModelBatch, kv_cache: PagedKVCache) -> torch.Tensor:
    """Packed logits [T, vocab] of one scheduler step (model_runner.py:146-272),
    in the packed token order, with one batched chunk-prefill and one batched
    decode per layer."""
    h, prefill_idx, decode_idx = _check_step(model, batch, kv_cache)
    return _run_step(model, batch, kv_cache, _StepPlan(batch, h, prefill_idx, decode_idx, kv_cache.block_size))


def _check_step(model, batch: ModelBatch, kv_cache: PagedKVCache):
    """The reference's checks of one step (model_runner.py:146-244), on the
    host metadata: (host metadata, prefill request indices, decode request
    indices)."""
    if len(batch.request_phases) != len(batch.request_ids):
        raise ValueError("request_phases length must match request_ids")
    if not batch.request_ids:
        raise ValueError("Cannot execute an empty ModelBatch")
    if batch.input_token_ids.ndim != 1:
        raise ValueError("input_token_ids must be one-dimensional")
    if batch.positions.ndim != 1:
        raise ValueError("positions must be one-dimensional")
    if batch.slot_mapping.ndim != 1:
        raise ValueError("slot_mapping must be one-dimensional")
    total = batch.input_token_ids.numel()
    if batch.positions.numel() != total:
        raise ValueError("positions length must match input_token_ids")
    if batch.slot_mapping.numel() != total:
        raise ValueError("slot_mapping length must match input_token_ids")
    if batch.context_lens.ndim != 1:
        raise ValueError("context_lens must be one-dimensional")
    if batch.context_lens.numel() != len(batch.request_ids):
        raise ValueError("context_lens length must match request_ids")
    if batch.block_tables.ndim != 2:
        raise ValueError("block_tables must be two-dimensional")
    if batch.block_tables.shape[0] != len(batch.request_ids):
        raise ValueError("block_tables rows must match request_ids")
    index_tensors = {
        "input_token_ids": batch.input_token_ids,
        "positions": batch.positions,
        "query_start_loc": batch.query_start_loc,
        "context_lens": batch.context_lens,
        "block_tables": batch.block_tables,
        "slot_mapping": batch.slot_mapping,
    }
    for name, t in index_tensors.items():
        if t.dtype is not torch.long:
            raise ValueError(f"{name} must use torch.long dtype")
    device = batch.input_token_ids.device
    for name, t in index_tensors.items():
        if t.device != device:
            raise ValueError(f"{name} must be on the same device as input_token_ids")
    param = next(model.parameters())
    if device != param.device:
        raise ValueError("ModelBatch and model must be on the same device")
    if kv_cache.device != param.device:
        raise ValueError("KV cache and model must be on the same device")
    if kv_cache.dtype != param.dtype and not kv_cache.is_fp8:
        raise ValueError("KV cache dtype must match model dtype")
    if batch.query_start_loc.ndim != 1:
        raise ValueError("query_start_loc must be one-dimensional")
    if batch.query_start_loc.numel() != len(batch.request_ids) + 1:
        raise ValueError("query_start_loc must contain one more entry than request_ids")

    h = _host_meta(batch)
    qsl, lens, tables = h.query_start_loc, h.context_lens, h.block_tables
    if int(qsl[0]) != 0:
        raise ValueError("query_start_loc must start at 0")
    if np.any(qsl[1:] <= qsl[:-1]):
        raise ValueError("query_start_loc must be strictly increasing")
    if int(qsl[-1]) != total:
        raise ValueError("query_start_loc must end at the packed token count")
    bs = kv_cache.block_size
    for i, rid in enumerate(batch.request_ids):
        if lens[i] <= 0:
            raise ValueError(f"Request {rid} context_len must be greater than 0")
        need = (int(lens[i]) + bs - 1) // bs
        if tables.shape[1] < need:
            raise ValueError(f"Request {rid} block_table has insufficient blocks")
        used = tables[i, :need]
        if np.any(used < 0) or np.any(used >= kv_cache.num_blocks):
            raise ValueError(f"Request {rid} block_table contains an invalid physical block")
    prefill_idx, decode_idx = [], []
    for i, phase in enumerate(batch.request_phases):
        p = _phase(phase)
        if p == "DECODING":
            if qsl[i + 1] - qsl[i] != 1:
                raise ValueError("Decode requires exactly one token per request")
            decode_idx.append(i)
        elif p == "PREFILLING":
            prefill_idx.append(i)
        else:
            raise ValueError(f"Unsupported request phase {phase} for request {batch.request_ids[i]}")
    inner = model.model
    for layer in inner.layers:
        if not isinstance(layer.self_attn, Qwen2Attention):
            raise TypeError("the model's attention modules must be mini_llm_runtime_b200.Qwen2Attention "
                            "(call swap_attention(model) first)")
    if not isinstance(kv_cache, PagedKVCache):
        raise TypeError("kv_cache must be a mini_llm_runtime_b200.PagedKVCache")
    return h, prefill_idx, decode_idx


def _run_step(model, batch: ModelBatch, kv_cache: PagedKVCache, plan: "_StepPlan") -> torch.Tensor:
    """The device work of a checked step: no host synchronisation, so it can
    be captured in a CUDA graph."""
    inner = model.model
    hidden = inner.embed_tokens(batch.input_token_ids)  # [T, hidden]
    for layer_idx, layer in enumerate(inner.layers):
        residual = hidden
        normed = layer.input_layernorm(hidden)
        attn = torch.empty_like(normed)
        if plan.prefill:
            x = plan.take(normed, plan.p_rows)
            out = layer.self_attn.prefill_batch_planned(
                x.unsqueeze(0), plan.p_pos.unsqueeze(0), kv_cache, layer_idx, plan.p_slots, plan.p_qsl,
                plan.p_tables, plan.p_lens, plan.p_max_q)
            plan.put(attn, plan.p_rows, out.squeeze(0))
        if plan.decode:
            x = plan.take(normed, plan.d_rows)
            out = layer.self_attn.decode_batch_planned(
                x.unsqueeze(1), plan.d_pos.unsqueeze(1), kv_cache, layer_idx, plan.d_slots, plan.d_tables,
                plan.d_lens, plan.d_fused)
            plan.put(attn, plan.d_rows, out.squeeze(1))
        hidden = residual + attn
        residual = hidden
        hidden = residual + layer.mlp(layer.post_attention_layernorm(hidden))
    return model.lm_head(inner.norm(hidden))


class DecodeStepGraph:
    """A whole decode step of the model in one CUDA graph: the embedding,
    every layer's norms, projections, RoPE, KV write with paged decode, MLP,
    then the final norm and LM head.  That is the reference's per-layer
    decode loop (model/qwen2.py:1147-1156, run per step by
    model_runner.py:146-288) replayed with one launch.

    Built for ``num_requests`` decode requests with block tables of up to
    ``table_width`` blocks.  ``run(batch)`` checks the step on the host as
    ``execute_model_batch`` does, copies the batch's device tensors into the
    graph's inputs and replays.  It returns the graph's logits
    ``[num_requests, vocab]``, which the next run overwrites.

    The first run captures the graph; its batch fixes whether the new tokens'
    KV write is fused into the decode.  A later batch that needs the other
    choice (a new token in a block shared with another sequence) runs
    eagerly instead.  Capture runs the step once eagerly first: it writes the
    same KV rows the replay writes, so the step's effect is unchanged.
    """

    def __init__(self, model, kv_cache: PagedKVCache, num_requests: int, table_width: int):
        if num_requests <= 0 or table_width <= 0:
            raise ValueError("num_requests and table_width must be positive")
        self.model, self.kv_cache = model, kv_cache
        self.num_requests, self.table_width = num_requests, table_width
        dev = next(model.parameters()).device
        if dev.type != "cuda":
            raise ValueError("DecodeStepGraph needs a model on a CUDA device")
        z = lambda: torch.zeros(num_requests, dtype=torch.long, device=dev)  # noqa: E731
        self.tokens, self.positions, self.slots, self.lens = z(), z(), z(), z()
        self.tables = torch.full((num_requests, table_width), -1, dtype=torch.long, device=dev)
        self.qsl = torch.arange(num_requests + 1, dtype=torch.long, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.logits: torch.Tensor | None = None
        self._fused: bool | None = None
        self._stream = torch.cuda.Stream(dev)

    def run(self, batch: ModelBatch) -> torch.Tensor:
        h, prefill_idx, decode_idx = _check_step(self.model, batch, self.kv_cache)
        if prefill_idx or len(decode_idx) != self.num_requests:
            raise ValueError(f"DecodeStepGraph runs steps of exactly {self.num_requests} decode requests")
        w = batch.block_tables.shape[1]
        if w > self.table_width:
            raise ValueError(f"block_tables wider than the graph's {self.table_width} blocks")
        bs = self.kv_cache.block_size
        fused = new_token_blocks_private(h.context_lens, h.block_tables, bs)
        if self.graph is not None and fused != self._fused:
            return execute_model_batch(self.model, batch, self.kv_cache)
        self.tokens.copy_(batch.input_token_ids)
        self.positions.copy_(batch.positions)
        self.slots.copy_(batch.slot_mapping)
        self.lens.copy_(batch.context_lens)
        self.tables.fill_(-1)
        self.tables[:, :w].copy_(batch.block_tables)
        if self.graph is None:
            self._capture(h, fused)
        self.graph.replay()
        return self.logits

    def _capture(self, h: BatchHostMeta, fused: bool) -> None:
        n = self.num_requests
        tables = np.full((n, self.table_width), -1, dtype=np.int64)
        tables[:, :h.block_tables.shape[1]] = h.block_tables
        host = BatchHostMeta(np.arange(n + 1, dtype=np.int64), h.context_lens.copy(), tables)
        static = ModelBatch([f"decode{i}" for i in range(n)], self.tokens, self.positions, self.qsl,
                            [RequestStatus.DECODING] * n, self.lens, self.tables, self.slots, host)
        plan = _StepPlan(static, host, [], list(range(n)), self.kv_cache.block_size)
        cur = torch.cuda.current_stream(self.tokens.device)
        self._stream.wait_stream(cur)  # the staged inputs
        with torch.cuda.stream(self._stream):
            # Eager run first: the op workspaces of this stream exist before
            # capture, and library kernels are loaded.
            _run_step(self.model, static, self.kv_cache, plan)
        self._stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self._stream):
            self.logits = _run_step(self.model, static, self.kv_cache, plan)
        cur.wait_stream(self._stream)
        self.graph, self._fused = graph, fused


class _StepPlan:
    """Token rows and metadata slices of the step's prefill and decode
    requests, made once per step (every layer reuses them)."""

    def __init__(self, batch: ModelBatch, h: BatchHostMeta, prefill_idx: list[int], decode_idx: list[int],
                 block_size: int):
        dev = batch.input_token_ids.device
        qsl = h.query_start_loc
        self.prefill, self.decode = bool(prefill_idx), bool(decode_idx)

        def rows_of(idx):
            # A contiguous run of requests owns a contiguous run of rows: a slice.
            if idx == list(range(idx[0], idx[-1] + 1)):
                return slice(int(qsl[idx[0]]), int(qsl[idx[-1] + 1]))
            r = np.concatenate([np.arange(qsl[i], qsl[i + 1]) for i in idx])
            return torch.from_numpy(r).to(dev, non_blocking=True)

        def req_index(idx):
            if idx == list(range(idx[0], idx[-1] + 1)):
                return slice(idx[0], idx[-1] + 1)
            return torch.tensor(idx, dtype=torch.long).to(dev, non_blocking=True)

        if self.prefill:
            self.p_rows = rows_of(prefill_idx)
            ri = req_index(prefill_idx)
            self.p_pos = self.take(batch.positions, self.p_rows)
            self.p_slots = self.take(batch.slot_mapping, self.p_rows)
            self.p_lens = batch.context_lens[ri]
            self.p_tables = batch.block_tables[ri]
            chunks = np.asarray([qsl[i + 1] - qsl[i] for i in prefill_idx], dtype=np.int64)
            self.p_qsl = torch.from_numpy(np.concatenate([[0], np.cumsum(chunks)])).to(dev, non_blocking=True)
            self.p_max_q = int(chunks.max())
        if self.decode:
            self.d_rows = rows_of(decode_idx)
            ri = req_index(decode_idx)
            self.d_pos = self.take(batch.positions, self.d_rows)
            self.d_slots = self.take(batch.slot_mapping, self.d_rows)
            self.d_lens = batch.context_lens[ri]
            self.d_tables = batch.block_tables[ri]
            self.d_fused = new_token_blocks_private(h.context_lens[decode_idx], h.block_tables[decode_idx],
                                                    block_size)

    @staticmethod
    def take(t: torch.Tensor, rows):
        return t[rows] if isinstance(rows, slice) else t.index_select(0, rows)

    @staticmethod
    def put(dst: torch.Tensor, rows, src: torch.Tensor) -> None:
        if isinstance(rows, slice):
            dst[rows] = src
        else:
            dst.index_copy_(0, rows, src)

"""CUDA-graph capture of a whole decode step of the attention hot path.

A decode step of the reference runs, for every layer, the KV write of the new
token followed by batched paged decode (model/qwen2.py:608-621, the per-layer
loop at :1147-1156).  With one Python/ctypes round trip per launch that is
~50 host launches per step — more host time than the kernels need on a B200.
``PagedDecodeGraph`` captures the step once (static device buffers, the
decode workspace and the tensor maps baked into the graph) and replays it
with a single launch, optionally including the host->device copy of the
step's inputs from pinned staging buffers and the device->host copy of the
outputs.

Typical use::

    g = PagedDecodeGraph(cache, batch=64, max_blocks=256, layers=range(24))
    inp = g.host_inputs          # pinned: q, new_k, new_v, slot_mapping, block_tables, context_lens
    ... fill inp ...
    g.run()                      # validate metadata on the host, replay
    g.synchronize(); out = g.host_output   # [layers, B, Hq, D]

``host_inputs`` is read by copies inside the replay, after ``run()`` has
returned: refill it for the next step only after ``synchronize()`` or
``wait_inputs_consumed()``, or the replay in flight may copy a mix of two
steps.  ``synchronize()`` also raises ``PagedAttentionError`` when a kernel of
the step recorded a device-side failure (a bounded wait that gave up).

The metadata checks are the ones Qwen2Attention.forward_decode_batch_with_cache
runs before touching the cache (model/qwen2.py:553-602), done on the pinned
host copies, so a step never needs a device->host sync.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import _lib
from .paged_kv_cache import PagedKVCache
from .qwen2_attention import check_decode_metadata, new_token_blocks_private


class PagedDecodeGraph:
    COPY_CHUNK_LAYERS = 4  # layers per host<->device copy chunk (host I/O mode)
    # The first chunk's inputs and the last chunk's outputs cannot overlap
    # any kernel of the step, so those two chunks carry one layer each.
    EDGE_CHUNK_LAYERS = 1

    @classmethod
    def copy_chunks(cls, num_layers: int) -> list[tuple[int, int]]:
        """[first, last) layer ranges of the step's copy chunks."""
        edge, mid = cls.EDGE_CHUNK_LAYERS, cls.COPY_CHUNK_LAYERS
        if num_layers <= 2 * edge:
            return [(a, min(a + edge, num_layers)) for a in range(0, num_layers, edge)]
        chunks = [(0, edge)]
        a = edge
        while a < num_layers - edge:
            b = min(a + mid, num_layers - edge)
            chunks.append((a, b))
            a = b
        chunks.append((num_layers - edge, num_layers))
        return chunks

    def __init__(
        self,
        cache: PagedKVCache,
        batch: int,
        max_blocks: int,
        num_q_heads: int,
        layers=None,
        host_io: bool = True,
        partition_tokens: int = 0,
        scale: float | None = None,
        write_kv: bool = True,
        fuse_write: bool = True,
        early_inputs: bool = True,
        query_dtype: torch.dtype | None = None,
    ):
        dev = _lib.require_cuda(cache.k_cache, what="PagedDecodeGraph")
        if cache.dtype not in (torch.float16, torch.bfloat16, torch.float32, _lib.FP8_DTYPE):
            raise TypeError("unsupported cache dtype")
        # q / new_k / new_v / outputs: the cache dtype, or BF16 over FP8 pools.
        qdt = query_dtype or (torch.bfloat16 if cache.dtype == _lib.FP8_DTYPE else cache.dtype)
        if cache.dtype != _lib.FP8_DTYPE and qdt != cache.dtype:
            raise TypeError("query_dtype must be the cache dtype unless the pools are FP8")
        if num_q_heads % cache.num_kv_heads != 0:
            raise ValueError("num_query_heads must be divisible by num_kv_heads")
        self.cache = cache
        self.device = dev
        self.batch = batch
        self.width = max_blocks
        self.hq = num_q_heads
        self.layers = list(range(cache.num_layers) if layers is None else layers)
        self.host_io = host_io
        self.write_kv = write_kv
        # The KV write rides in the decode kernel (pa_paged_decode_write)
        # unless the split-KV path is asked for.
        self.fuse_write = fuse_write and partition_tokens == 0
        # Inside the graph a layer's decode follows the previous layer's
        # decode (or the input copy), which writes no metadata and no pool
        # row of this layer: its kernel may start on them before that one
        # ends (PA_DECODE_EARLY_INPUTS).  Its queries are inputs of the step,
        # copied before the replay or by a copy the layer's kernel is fully
        # ordered after, so they may be read that early too
        # (PA_DECODE_EARLY_QUERY).
        self._flags = (_lib.PA_DECODE_EARLY_INPUTS | _lib.PA_DECODE_EARLY_QUERY) if early_inputs else 0
        self.scale = (1.0 / math.sqrt(cache.head_dim)) if scale is None else float(scale)
        L, B, H, D, HKV = len(self.layers), batch, num_q_heads, cache.head_dim, cache.num_kv_heads
        dt = qdt
        # All of a step's inputs live in one byte buffer, the same layout on
        # the device and (pinned) on the host: the metadata, then one record
        # per layer [q | new_k | new_v], each 256-byte aligned.  A copy chunk
        # is then one contiguous range, and the first one carries the
        # metadata as well: one copy before the first layer can start.
        es = torch.empty(0, dtype=dt).element_size()
        align = lambda n: (n + 255) // 256 * 256  # noqa: E731
        q_bytes, kv_bytes = B * H * D * es, B * HKV * D * es
        self._meta_bytes = align(8 * (2 * B + B * max_blocks))
        self._rec_bytes = align(q_bytes + 2 * kv_bytes)
        total = self._meta_bytes + L * self._rec_bytes
        self._stage_dev = torch.zeros(total, dtype=torch.uint8, device=dev)
        self._dev_inputs = self._stage_views(self._stage_dev, L, B, H, HKV, D, max_blocks, dt)
        self._dev_inputs["context_lens"].fill_(1)
        self.q, self.new_k, self.new_v = (self._dev_inputs[k] for k in ("q", "new_k", "new_v"))
        self.slot_mapping, self.block_tables, self.context_lens = (
            self._dev_inputs[k] for k in ("slot_mapping", "block_tables", "context_lens"))
        self.out = torch.zeros(L, B, H, D, dtype=dt, device=dev)
        self._stage_host = torch.zeros(total, dtype=torch.uint8).pin_memory()
        self.host_inputs = self._stage_views(self._stage_host, L, B, H, HKV, D, max_blocks, dt)
        self.host_output = torch.zeros(self.out.shape, dtype=dt).pin_memory() if host_io else None

        lib = _lib.load()
        self._lib = lib
        self._code = _lib.dtype_code(dt)
        self.partition_tokens = partition_tokens
        ws_bytes = lib.pa_decode_workspace_bytes(B, HKV, H, D, cache.block_size, max_blocks, partition_tokens,
                                                 self._code)
        if ws_bytes == 0:
            raise ValueError("invalid decode arguments")
        # Private, zeroed once; every replay leaves the tickets at zero.
        self.workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        self.graph = None
        self._replayed = None  # event after the last replay (its copies included)
        self._stream = torch.cuda.Stream(dev)
        self._h2d = torch.cuda.Stream(dev)
        self._d2h = torch.cuda.Stream(dev)
        self._capture()

    def _stage_views(self, buf: torch.Tensor, L: int, B: int, H: int, HKV: int, D: int, W: int,
                     dt: torch.dtype) -> dict:
        """The named inputs as views of a staging buffer (layout in __init__)."""
        i64 = buf.view(torch.int64)
        el = buf.view(dt)
        es = el.element_size()
        rec, meta = self._rec_bytes // es, self._meta_bytes // es
        q_el, kv_el = B * H * D, B * HKV * D
        return {
            "slot_mapping": i64[0:B],
            "context_lens": i64[B:2 * B],
            "block_tables": i64[2 * B:2 * B + B * W].view(B, W),
            "q": torch.as_strided(el, (L, B, H, D), (rec, H * D, D, 1), meta),
            "new_k": torch.as_strided(el, (L, B, HKV, D), (rec, HKV * D, D, 1), meta + q_el),
            "new_v": torch.as_strided(el, (L, B, HKV, D), (rec, HKV * D, D, 1), meta + q_el + kv_el),
        }

    # -- step body --------------------------------------------------------------
    def _body(self, stream: int, warm: bool = False) -> None:
        """Enqueue one step.  ``warm`` = eager first pass before capture: no
        copies and no KV writes (it must not modify the cache), decode only.

        With host I/O the per-layer inputs travel in chunks (``copy_chunks``:
        one layer first and last, ``COPY_CHUNK_LAYERS`` between): the
        metadata and the first chunk on the step's stream, the others on a
        side stream while the first layers run, and each chunk's outputs go
        back on another side stream as soon as its layers finish, so the copy
        engines work under the kernels."""
        lib, c = self._lib, self.cache
        B, H, D, HKV, bs = self.batch, self.hq, c.head_dim, c.num_kv_heads, c.block_size
        io = self.host_io and not warm
        main = torch.cuda.current_stream(self.device)
        chunks = self.copy_chunks(len(self.layers))
        last_of_chunk = {b - 1: a for a, b in chunks}
        ready = {}
        if io:
            meta, rec = self._meta_bytes, self._rec_bytes
            for ci, (a, b) in enumerate(chunks):
                lo, hi = (0 if ci == 0 else meta + a * rec), meta + b * rec
                with torch.cuda.stream(main if ci == 0 else self._h2d):
                    self._stage_dev[lo:hi].copy_(self._stage_host[lo:hi], non_blocking=True)
                    if ci == 0:
                        self._h2d.wait_stream(main)
                    else:
                        ev = torch.cuda.Event()
                        ev.record(self._h2d)
                        ready[a] = ev
            self._d2h.wait_stream(main)
        num_slots = c.num_blocks * bs
        for i, layer in enumerate(self.layers):
            if i in ready:
                main.wait_event(ready[i])
            nk, nv, q, o = self.new_k[i], self.new_v[i], self.q[i], self.out[i]
            kp, vp = c.k_cache[layer], c.v_cache[layer]
            write = self.write_kv and not warm
            fused = write and self.fuse_write
            fp8 = c.is_fp8
            ks, vs = c.layer_scales(layer)
            if write and not fused:
                if fp8:
                    st = lib.pa_kv_scatter_fp8(
                        nk.data_ptr(), nk.stride(0), nk.stride(1), nk.stride(2), nv.data_ptr(), nv.stride(0),
                        nv.stride(1), nv.stride(2), self._code, self.slot_mapping.data_ptr(), 1, B, kp.data_ptr(),
                        vp.data_ptr(), num_slots, HKV, D, ks, vs, stream)
                else:
                    st = lib.pa_kv_scatter(
                        nk.data_ptr(), nk.stride(0), nk.stride(1), nk.stride(2), nv.data_ptr(), nv.stride(0),
                        nv.stride(1), nv.stride(2), self._code, self.slot_mapping.data_ptr(), 1, B, kp.data_ptr(),
                        vp.data_ptr(), num_slots, HKV, D, self._code, stream)
                _lib.check(st, "pa_kv_scatter")
            # After a separate scatter the decode reads pool rows that kernel
            # just wrote, so it waits before touching anything.
            flags = self._flags if (fused or not write) else 0
            args = (q.data_ptr(), q.stride(0), q.stride(1), nk.data_ptr() if fused else None,
                    nv.data_ptr() if fused else None, self.slot_mapping.data_ptr() if fused else None,
                    kp.data_ptr(), vp.data_ptr(), c.num_blocks, bs, HKV, D, self.block_tables.data_ptr(),
                    self.block_tables.stride(0), self.width, self.context_lens.data_ptr(), o.data_ptr(), o.stride(0),
                    o.stride(1), B, H, self.scale, self._code)
            tail = (0 if fused else self.partition_tokens, flags, self.workspace.data_ptr(), self.workspace.numel(),
                    stream)
            if fp8:
                st = lib.pa_paged_decode_fp8(*args, ks, vs, *tail)
            else:
                st = lib.pa_paged_decode_ex(*args, *tail)
            _lib.check(st, "pa_paged_decode_ex")
            if io and i in last_of_chunk:
                a = last_of_chunk[i]
                done = torch.cuda.Event()
                done.record(main)
                self._d2h.wait_event(done)
                with torch.cuda.stream(self._d2h):
                    self.host_output[a:i + 1].copy_(self.out[a:i + 1], non_blocking=True)
        if io:
            main.wait_stream(self._d2h)

    def _capture(self) -> None:
        # One eager decode-only pass on a side stream (first-use kernel
        # attributes; length-1 contexts over block 0, nothing written to the
        # cache), then capture.
        s = self._stream
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self._body(s.cuda_stream, warm=True)
        s.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self._body(s.cuda_stream)
        s.synchronize()

    # -- host-side metadata checks (model/qwen2.py:580-602, paged_kv_cache.py:228-239)
    def validate(self, inputs: dict | None = None) -> None:
        src = self.host_inputs if inputs is None else inputs
        lens, tables = src["context_lens"].numpy(), src["block_tables"].numpy()
        check_decode_metadata(lens, tables, src["slot_mapping"].numpy(), None, self.cache.block_size,
                              self.cache.num_blocks)
        if self.write_kv and self.fuse_write and not new_token_blocks_private(lens, tables, self.cache.block_size):
            raise ValueError("fused KV write needs each new token's block private to its sequence "
                             "(build the graph with fuse_write=False for shared blocks)")

    def run(self, validate: bool = True) -> None:
        """Validate the staged metadata on the host and replay the step on the
        current stream (asynchronous)."""
        if validate:
            self.validate(self.host_inputs if self.host_io else {
                k: v.cpu() for k, v in self._dev_inputs.items() if k in ("context_lens", "block_tables", "slot_mapping")})
        cur = torch.cuda.current_stream(self.device)
        self._stream.wait_stream(cur)
        with torch.cuda.stream(self._stream):
            self.graph.replay()
            self._replayed = torch.cuda.Event()
            self._replayed.record(self._stream)
        cur.wait_stream(self._stream)

    def wait_inputs_consumed(self) -> None:
        """Block the host until the last replay has copied ``host_inputs`` to
        the device (it waits for the whole replay), so the next step's inputs
        can be written."""
        if self._replayed is not None:
            self._replayed.synchronize()

    def synchronize(self) -> None:
        """Wait for the step, then raise ``PagedAttentionError`` if one of its
        kernels recorded a device-side failure in the step's workspace (the
        workspace is re-zeroed first, so later steps start clean)."""
        torch.cuda.current_stream(self.device).synchronize()
        code = int(self.workspace[:4].view(torch.int32)[0].item())
        if code != 0:
            self.workspace.zero_()
            msg = self._lib.pa_status_string(code).decode()
            raise _lib.PagedAttentionError(f"PagedDecodeGraph step: {msg} (status {code})")

    @property
    def launches_per_step(self) -> int:
        """Kernels of this library launched per replay: per layer the decode
        (main + combine kernel on the balanced path, one kernel otherwise)
        and, when the write is not fused into it, the KV scatter."""
        c = self.cache
        balanced = (self.out.dtype in (torch.bfloat16, torch.float16) and c.head_dim in (64, 128)
                    and c.block_size % 16 == 0 and c.block_size <= 256 and self.batch <= 1024)
        per_layer = 2 if balanced else 1
        if self.write_kv and not (self.fuse_write and balanced):
            per_layer += 1
        return per_layer * len(self.layers)

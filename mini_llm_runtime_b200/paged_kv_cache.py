"""Paged K/V pools with the reference's interface and a CUDA batched write.

Mirror of ``mini_llm_runtime.runtime.paged_kv_cache.PagedKVCache``
(runtime/paged_kv_cache.py:6-259): same constructor, pool layout
``[num_layers, num_blocks, block_size, num_kv_heads, head_dim]`` (contiguous,
slot = block * block_size + offset), LIFO free list, per-sequence block
tables and the same exceptions.  The block allocator is host bookkeeping and
stays Python; ``write_slots`` — the batched KV-cache write on the hot path —
launches the scatter kernel of libpagedattn.so.

``dtype=torch.float8_e4m3fn`` stores the pools in FP8 (half the bytes decode
streams; the reference has no FP8 pool): each layer has a K and a V scale
(``k_scale`` / ``v_scale``: one float or one per layer), a stored element is
``clamp(x / scale, -448, 448)`` rounded to nearest even, and the attention
ops read it back as ``element * scale`` (pass ``*cache.layer_scales(l)``).
"""

from __future__ import annotations

import torch

from . import _lib


class PagedKVCache:
    def __init__(
        self,
        num_layers: int,
        num_blocks: int,
        block_size: int,
        num_kv_heads: int,
        head_dim: int,
        dtype: torch.dtype = torch.float16,
        device: torch.device | str = "cpu",
        k_scale: float | list[float] = 1.0,
        v_scale: float | list[float] = 1.0,
    ):
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = torch.device(device)
        self.k_scales = self._per_layer(k_scale, num_layers, "k_scale")
        self.v_scales = self._per_layer(v_scale, num_layers, "v_scale")
        if dtype != _lib.FP8_DTYPE and (any(s != 1.0 for s in self.k_scales) or any(s != 1.0 for s in self.v_scales)):
            raise ValueError("k_scale / v_scale apply to FP8 pools only")
        shape = (num_layers, num_blocks, block_size, num_kv_heads, head_dim)
        self.k_cache = torch.empty(shape, dtype=dtype, device=device)
        self.v_cache = torch.empty_like(self.k_cache)
        # LIFO free list: block 0 is handed out first (paged_kv_cache.py:37, :49-53).
        self.free_blocks = list(range(num_blocks - 1, -1, -1))
        self.block_tables: dict[int, list[int]] = {}
        self.seq_lens: dict[int, int] = {}

    @staticmethod
    def _per_layer(scale, num_layers: int, name: str) -> list[float]:
        vals = [float(scale)] * num_layers if isinstance(scale, (int, float)) else [float(s) for s in scale]
        if len(vals) != num_layers:
            raise ValueError(f"{name} must be one float or one per layer")
        if not all(s > 0 and s != float("inf") for s in vals):
            raise ValueError(f"{name} must be positive and finite")
        return vals

    @property
    def is_fp8(self) -> bool:
        return self.dtype == _lib.FP8_DTYPE

    def layer_scales(self, layer_idx: int) -> tuple[float, float]:
        """(k_scale, v_scale) of a layer (1.0 for 16/32-bit pools)."""
        return self.k_scales[layer_idx], self.v_scales[layer_idx]

    # -- host-side allocator (paged_kv_cache.py:42-192) ---------------------
    def add_sequence(self, seq_id) -> None:
        if seq_id in self.block_tables:
            raise KeyError(f"Sequence {seq_id} is already exists")
        self.block_tables[seq_id] = []
        self.seq_lens[seq_id] = 0

    def _allocate_block(self) -> int:
        if not self.free_blocks:
            raise RuntimeError("KV cache out of physical blocks")
        return self.free_blocks.pop()

    def free_sequence(self, seq_id: int) -> None:
        if seq_id not in self.block_tables:
            raise KeyError(f"Unknown sequence {seq_id}")
        blocks = self.block_tables[seq_id]
        self.free_blocks.extend(blocks)
        blocks.clear()
        del self.block_tables[seq_id]
        del self.seq_lens[seq_id]

    def _check_capacity(self, seq_id: int, num_new_tokens: int) -> bool:
        final_len = self.seq_lens[seq_id] + num_new_tokens
        need = (final_len + self.block_size - 1) // self.block_size - len(self.block_tables[seq_id])
        return len(self.free_blocks) >= need

    def reserve_tokens(self, seq_id: int, total_num_tokens: int) -> bool:
        if total_num_tokens < 0:
            raise ValueError("total_num_tokens cannot be negative")
        need = (total_num_tokens + self.block_size - 1) // self.block_size - len(self.block_tables[seq_id])
        need = max(need, 0)
        if len(self.free_blocks) >= need:
            self.block_tables[seq_id].extend(self._allocate_block() for _ in range(need))
            return True
        return False

    def append_tokens(self, seq_id: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append [T, Hkv, D] tokens to layer 0 of a sequence (paged_kv_cache.py:64-88),
        as one batched write instead of T single-token copies."""
        if k.ndim != 3 or v.ndim != 3:
            raise ValueError("Expected K/V shape [T, H_kv, D]")
        if k.shape != v.shape:
            raise ValueError("K and V must have the same shape")
        if tuple(k.shape[1:]) != (self.num_kv_heads, self.head_dim):
            raise ValueError(f"Expected K/V shape [T, {self.num_kv_heads}, {self.head_dim}]")
        if seq_id not in self.block_tables:
            raise KeyError(f"Unknow sequence {seq_id}")
        t = k.shape[0]
        if not self._check_capacity(seq_id, t):
            raise RuntimeError("out of memory")
        start = self.seq_lens[seq_id]
        self.reserve_tokens(seq_id, start + t)
        table = self.block_tables[seq_id]
        slots = [table[p // self.block_size] * self.block_size + p % self.block_size for p in range(start, start + t)]
        slot_t = torch.tensor(slots, dtype=torch.long).to(self.device)
        self.write_slots(slot_t, k.to(self.device), v.to(self.device), layer_idx=0)
        self.seq_lens[seq_id] = start + t

    def append(self, seq_id: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append one token ([Hkv, D]) to layer 0 (paged_kv_cache.py:146-176)."""
        if seq_id not in self.block_tables:
            raise KeyError(f"Unknow sequence {seq_id}")
        expected = (self.num_kv_heads, self.head_dim)
        if tuple(k.shape) != expected:
            raise ValueError(f"Expected k shape {expected}, got {tuple(k.shape)}")
        if tuple(v.shape) != expected:
            raise ValueError(f"Expected v shape {expected}, got {tuple(v.shape)}")
        self.append_tokens(seq_id, k.unsqueeze(0), v.unsqueeze(0))

    def get_sequence(self, seq_id):
        """Layer-0 K/V of a sequence in logical order (paged_kv_cache.py:121-143)."""
        n = self.seq_lens[seq_id]
        table = torch.tensor(self.block_tables[seq_id], dtype=torch.long, device=self.device)
        pos = torch.arange(n, device=self.device)
        blocks = table[pos // self.block_size]
        return self.k_cache[0, blocks, pos % self.block_size].clone(), self.v_cache[0, blocks, pos % self.block_size].clone()

    def get_layer_cache(self, layer_idx: int = 0):
        if layer_idx < 0 or layer_idx >= self.num_layers:
            raise IndexError("Unexpect layer_idx")
        return self.k_cache[layer_idx], self.v_cache[layer_idx]

    # -- hot path: batched KV write -------------------------------------------
    def validate_slots(self, slot_mapping: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layer_idx: int) -> None:
        """All checks of PagedKVCache.write_slots (paged_kv_cache.py:206-239),
        same order, exception types and messages.  One device->host read for
        the range and distinctness checks together (the reference does three)."""
        if layer_idx < 0 or layer_idx >= self.num_layers:
            raise IndexError("Unexpected layer_idx")
        if k.ndim != 3 or v.ndim != 3:
            raise ValueError("Expected K/V shape [T, H_kv, D]")
        if k.shape != v.shape:
            raise ValueError("K and V must have the same shape")
        if tuple(k.shape[1:]) != (self.num_kv_heads, self.head_dim):
            raise ValueError(f"Expected K/V shape [T, {self.num_kv_heads}, {self.head_dim}]")
        if slot_mapping.ndim != 1:
            raise ValueError("Expected slot_mapping shape [T]")
        if slot_mapping.shape[0] != k.shape[0]:
            raise ValueError("slot_mapping length must match the number of K/V tokens")
        if slot_mapping.dtype not in (torch.int32, torch.int64):
            raise TypeError("slot_mapping must use an integer index dtype")
        dev = self.k_cache.device
        if slot_mapping.device != dev or k.device != dev or v.device != dev:
            raise ValueError("slot_mapping and K/V must be on the KV cache device")
        n = slot_mapping.numel()
        if n == 0:
            return
        num_slots = self.num_blocks * self.block_size
        s = slot_mapping.long()
        bad_range = (s < 0).any() | (s >= num_slots).any()
        srt = torch.sort(s).values
        dup = (srt[1:] == srt[:-1]).any() if n > 1 else torch.zeros((), dtype=torch.bool, device=s.device)
        bad_range, dup = torch.stack([bad_range, dup]).tolist()
        if bad_range:
            raise IndexError("slot_mapping contains an out-of-range slot")
        if dup:
            raise ValueError("slot_mapping must contain distinct slots")

    def write_slots(
        self,
        slot_mapping: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        layer_idx: int = 0,
        *,
        validate: bool = True,
    ) -> None:
        """Write [T, Hkv, D] K/V to distinct flat slots in one layer.

        Empty writes are allowed; duplicate or out-of-range slots raise before
        the cache is touched; the source dtype is converted like ``copy_``.
        ``validate=False`` skips the checks (and their device->host read) for
        callers that already validated this step's slot mapping — the kernel
        still never writes outside the pool.
        """
        if validate:
            self.validate_slots(slot_mapping, k, v, layer_idx)
        if slot_mapping.numel() == 0:
            return
        dev = _lib.require_cuda(self.k_cache, slot_mapping, k, v, what="PagedKVCache.write_slots")
        lib = _lib.load()
        if self.is_fp8:
            # Quantized in FP32: x / scale, saturated to +-448, nearest even.
            if k.dtype != v.dtype:
                k, v = k.float(), v.float()
            layer_k, layer_v = self.k_cache[layer_idx], self.v_cache[layer_idx]
            slot_mapping = slot_mapping.contiguous()
            ks, vs = self.layer_scales(layer_idx)
            with _lib.device_guard(dev):
                st = lib.pa_kv_scatter_fp8(
                    k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
                    v.data_ptr(), v.stride(0), v.stride(1), v.stride(2), _lib.dtype_code(k.dtype),
                    slot_mapping.data_ptr(), int(slot_mapping.dtype == torch.int64), slot_mapping.numel(),
                    layer_k.data_ptr(), layer_v.data_ptr(), self.num_blocks * self.block_size,
                    self.num_kv_heads, self.head_dim, ks, vs, _lib.stream_handle(dev),
                )
            _lib.check(st, "pa_kv_scatter_fp8")
            return
        if k.dtype != v.dtype:
            # Mixed sources: convert each exactly like the reference's `.to` (:246-247).
            k, v = k.to(self.dtype), v.to(self.dtype)
        layer_k = self.k_cache[layer_idx]
        layer_v = self.v_cache[layer_idx]
        if not slot_mapping.is_contiguous():
            slot_mapping = slot_mapping.contiguous()
        with _lib.device_guard(dev):
            st = lib.pa_kv_scatter(
                k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
                v.data_ptr(), v.stride(0), v.stride(1), v.stride(2), _lib.dtype_code(k.dtype),
                slot_mapping.data_ptr(), int(slot_mapping.dtype == torch.int64), slot_mapping.numel(),
                layer_k.data_ptr(), layer_v.data_ptr(), self.num_blocks * self.block_size,
                self.num_kv_heads, self.head_dim, _lib.dtype_code(self.dtype), _lib.stream_handle(dev),
            )
        _lib.check(st, "pa_kv_scatter")

"""B200-native (sm_100a) paged-attention hot path for mini-llm-runtime.

Drop-in replacements for the reference's paged-attention ops and
``PagedKVCache.write_slots``, the attention module's paged methods, and the
runner's step (ModelBatch built on the device, batched chunk-prefill); every
op runs a hand-written CUDA kernel from ``libpagedattn.so`` through its C ABI
(include/pagedattn.h).
"""

from .paged_attention import (
    paged_attention_accumulator_cuda,
    paged_attention_decode,
    paged_attention_decode_batch_parallel,
    paged_attention_decode_split_kv,
    paged_attention_prefill_chunk_tiled,
    paged_attention_prefill_varlen,
    paged_decode_with_kv_write,
)
from ._lib import PagedAttentionError, check_device_status, device_status, reset_device_status
from .decode_graph import PagedDecodeGraph
from .paged_kv_cache import PagedKVCache
from .qwen2_attention import Qwen2Attention
from .runner import DecodeStepGraph, ModelBatch, build_model_batch, execute_model_batch, swap_attention

__all__ = [
    "DecodeStepGraph",
    "ModelBatch",
    "PagedAttentionError",
    "PagedDecodeGraph",
    "PagedKVCache",
    "Qwen2Attention",
    "build_model_batch",
    "check_device_status",
    "device_status",
    "execute_model_batch",
    "paged_attention_accumulator_cuda",
    "paged_attention_decode",
    "paged_attention_decode_batch_parallel",
    "paged_attention_decode_split_kv",
    "paged_attention_prefill_chunk_tiled",
    "paged_attention_prefill_varlen",
    "paged_decode_with_kv_write",
    "reset_device_status",
    "swap_attention",
]

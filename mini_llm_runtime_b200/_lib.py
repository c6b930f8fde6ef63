"""ctypes binding of libpagedattn.so (the C ABI declared in include/pagedattn.h).

The library is built in-tree by ``python -m mini_llm_runtime_b200.build``.
Loading fails loudly when it is missing: there is no CPU or PyTorch fallback
for any op in this package.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libpagedattn.so"

PA_OK = 0
PA_ERR_INVALID = -1
PA_ERR_UNSUPPORTED = -2
PA_ERR_CUDA = -3
PA_ERR_WORKSPACE = -4
PA_ERR_CAPACITY = -5
PA_DECODE_EARLY_INPUTS = 1
PA_DECODE_EARLY_QUERY = 2
PA_DEVICE_TIMEOUT_TMA = 101
PA_DEVICE_TIMEOUT_MMA = 102
PA_DEVICE_TIMEOUT_PEER = 103
PA_PEER_MAX_RANKS = 8
PA_IPC_HANDLE_BYTES = 64

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3, torch.float8_e4m3fn: 4}
PA_DTYPE_FP8_E4M3 = 4
FP8_DTYPE = torch.float8_e4m3fn

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_size = ctypes.c_size_t

# name -> (restype, argtypes); must match include/pagedattn.h
SIGNATURES: dict[str, tuple] = {
    "pa_status_string": (ctypes.c_char_p, [_i32]),
    "pa_abi_version": (_i32, []),
    "pa_kv_scatter": (
        _i32,
        [_c_void_p, _i64, _i64, _i64, _c_void_p, _i64, _i64, _i64, _i32, _c_void_p, _i32, _i64,
         _c_void_p, _c_void_p, _i64, _i32, _i32, _i32, _c_void_p],
    ),
    "pa_decode_workspace_bytes": (_size, [_i32, _i32, _i32, _i32, _i32, _i64, _i32, _i32]),
    "pa_paged_decode": (
        _i32,
        [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64, _i32, _i32, _i32, _c_void_p, _i64, _i64,
         _c_void_p, _c_void_p, _i64, _i64, _i32, _i32, _f32, _i32, _i32, _c_void_p, _size, _c_void_p],
    ),
    "pa_paged_decode_write": (
        _i32,
        [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _i32,
         _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64, _i64, _i32, _i32, _f32, _i32, _c_void_p, _size,
         _c_void_p],
    ),
    "pa_paged_decode_ex": (
        _i32,
        [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _i32,
         _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64, _i64, _i32, _i32, _f32, _i32, _i32, _i32, _c_void_p,
         _size, _c_void_p],
    ),
    "pa_paged_decode_noalloc": (
        _i32,
        [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64, _i32, _i32, _i32, _c_void_p, _i64, _i64,
         _c_void_p, _c_void_p, _i64, _i64, _i32, _i32, _f32, _i32, _i32, _c_void_p],
    ),
    "pa_chunk_prefill": (
        _i32,
        [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64,
         _i32, _i32, _i32, _c_void_p, _i64, _i64, _i32, _i64, _i32, _i32, _f32, _i32, _c_void_p, _c_void_p],
    ),
    "pa_accumulate_pv": (_i32, [_c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p]),
    "pa_build_batch_metadata": (
        _i32,
        [_c_void_p, _i32, _i64, _i64, _i32, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
         _c_void_p, _c_void_p],
    ),
    "pa_decode_noalloc_status": (_i32, [_c_void_p, _c_void_p]),
    "pa_kv_scatter_fp8": (
        _i32,
        [_c_void_p, _i64, _i64, _i64, _c_void_p, _i64, _i64, _i64, _i32, _c_void_p, _i32, _i64,
         _c_void_p, _c_void_p, _i64, _i32, _i32, _f32, _f32, _c_void_p],
    ),
    "pa_paged_decode_fp8": (
        _i32,
        [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _i32,
         _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64, _i64, _i32, _i32, _f32, _i32, _f32, _f32, _i32, _i32,
         _c_void_p, _size, _c_void_p],
    ),
    "pa_chunk_prefill_fp8": (
        _i32,
        [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64,
         _i32, _i32, _i32, _c_void_p, _i64, _i64, _i32, _i64, _i32, _i32, _f32, _i32, _f32, _f32, _c_void_p],
    ),
    "pa_selftest_wait_timeout": (_i32, [_c_void_p, _i64, _c_void_p]),
    "pa_peer_gather_bytes": (_size, [_i32, _i64]),
    "pa_ipc_export": (_i32, [_c_void_p, _c_void_p, ctypes.POINTER(ctypes.c_uint64)]),
    "pa_ipc_import": (_i32, [_c_void_p, ctypes.c_uint64, ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p)]),
    "pa_ipc_close": (_i32, [_c_void_p]),
    "pa_decode_allgather_bytes": (_size, [_i32, _i32, _i32, _i32, _i32]),
    "pa_paged_decode_allgather": (
        _i32,
        [_c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _i32,
         _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i64, _i64, _i32, _i32, _f32, _i32, _i32, _i32, _i32,
         ctypes.POINTER(_c_void_p), _i64, _i64, _c_void_p, _size, _c_void_p],
    ),
    "pa_head_allgather": (
        _i32,
        [_c_void_p, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, ctypes.POINTER(_c_void_p), _i64, _c_void_p,
         _i64, _i64, _i64, _c_void_p],
    ),
}

_lib = None
_lock = threading.Lock()


class PagedAttentionError(RuntimeError):
    """A libpagedattn entry point returned a non-zero status."""


def load() -> ctypes.CDLL:
    """Load libpagedattn.so once and attach the ctypes signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise PagedAttentionError(
                    f"{LIB_PATH} is missing; build it with `python -m mini_llm_runtime_b200.build` "
                    "(there is no CPU fallback)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status != PA_OK:
        msg = load().pa_status_string(status).decode()
        raise PagedAttentionError(f"{what} failed: {msg} (status {status})")


def require_cuda(*tensors: torch.Tensor, what: str) -> torch.device:
    """The product path runs only on CUDA tensors; anything else is an error."""
    dev = None
    for t in tensors:
        if not t.is_cuda:
            raise PagedAttentionError(
                f"{what} requires CUDA tensors (got a tensor on {t.device}); "
                "this package has no CPU fallback"
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise PagedAttentionError(f"{what}: all tensors must be on one device")
    return dev


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device) -> int:
    """The current stream of `device` as a raw cudaStream_t (an op's launch
    stream), without building a torch.cuda.Stream object."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(idx).cuda_stream


def device_guard(device: torch.device):
    """torch.cuda.device(device), entered only when it is not already the
    current device (the common case costs one query, not a switch and back)."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


_ws_size_cache: dict[tuple, int] = {}


def decode_workspace_bytes(batch: int, hkv: int, hq: int, d: int, bs: int, width: int, partition: int,
                           code: int) -> int:
    """pa_decode_workspace_bytes, memoised (a pure function of its arguments)."""
    key = (batch, hkv, hq, d, bs, width, partition, code)
    n = _ws_size_cache.get(key)
    if n is None:
        n = load().pa_decode_workspace_bytes(*key)
        if len(_ws_size_cache) > 4096:
            _ws_size_cache.clear()
        _ws_size_cache[key] = n
    return n


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}") from None


# ---------------------------------------------------------------------------
# Decode workspace: one zero-initialised buffer per (device, stream), grown on
# demand.  Layout (csrc/attn_generic.cuh): a 256-byte status word, then the
# split tickets int32[B * Hq], then the FP32 partials from
# 256 + align256(4 * B * Hq).  Tickets must read zero when a call starts; the
# kernels reset every ticket they use, but a later call with a larger B * Hq
# reaches into bytes an earlier call filled with partials, so those bytes are
# re-zeroed first.  Calls on one stream are ordered, so they never overlap.
# ---------------------------------------------------------------------------
_workspaces: dict[tuple[int, int], "_Workspace"] = {}
_control_blocks: dict[tuple[int, int], torch.Tensor] = {}

# With MINI_LLM_RUNTIME_B200_SYNC_CHECK=1 every op synchronises after its
# launch and raises on a device-side status (a debugging aid: it costs a host
# round trip per op).
SYNC_CHECK = os.environ.get("MINI_LLM_RUNTIME_B200_SYNC_CHECK", "0") not in ("", "0")


class _Workspace:
    def __init__(self, device: torch.device, nbytes: int):
        self.tensor = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        self.clean_end = self.tensor.numel()  # bytes [256, clean_end) hold zeros


def _align256(x: int) -> int:
    return (x + 255) & ~255


PREFILL_CONTROL_INTS = 4  # PA_PREFILL_CONTROL_INTS


def _dev_index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def status_word(device: torch.device) -> torch.Tensor:
    """Control block of pa_chunk_prefill for the current stream of `device`
    (int32[4], zeroed once): [0] is the status the kernels set when a
    bounded wait gives up, [1..2] the self-rewinding work-claim counters.
    One block per (device, stream), so calls that share it are ordered on
    that stream and calls on different streams never share counters."""
    key = (_dev_index(device), stream_handle(device))
    t = _control_blocks.get(key)
    if t is None:
        t = torch.zeros(PREFILL_CONTROL_INTS, dtype=torch.int32, device=device)
        _control_blocks[key] = t
    return t


def device_status(device: torch.device | None = None) -> list[tuple[str, int]]:
    """(what, code) for every non-zero device status word this package owns on
    `device` (all devices when None): the decode workspaces' status words and
    the prefill control blocks.  Synchronises the device (one D2H read)."""
    words = []
    for (idx, st), ws in _workspaces.items():
        if device is None or idx == _dev_index(device):
            words.append((f"decode workspace (device {idx}, stream {st:#x})", ws.tensor[:4].view(torch.int32)[:1]))
    for (idx, st), cb in _control_blocks.items():
        if device is None or idx == _dev_index(device):
            words.append((f"prefill control block (device {idx}, stream {st:#x})", cb[:1]))
    if not words:
        return []
    codes = torch.cat([w.to("cpu", non_blocking=False) for _, w in words]).tolist()
    return [(what, c) for (what, _), c in zip(words, codes) if c != 0]


def reset_device_status(device: torch.device | None = None) -> None:
    """Re-zero every status word, ticket and work counter this package owns
    on `device` (all devices when None): after a device-side timeout those
    may hold values a normal call never leaves behind."""
    for (idx, _), ws in _workspaces.items():
        if device is None or idx == _dev_index(device):
            ws.tensor.zero_()
            ws.clean_end = ws.tensor.numel()
    for (idx, _), cb in _control_blocks.items():
        if device is None or idx == _dev_index(device):
            cb.zero_()


def check_device_status(device: torch.device | None = None) -> None:
    """Raise PagedAttentionError if a kernel of this package recorded a
    device-side failure (a bounded wait that gave up; its outputs are then
    garbage).  The words are re-zeroed before raising, so the next call starts
    clean.  Synchronises the device."""
    bad = device_status(device)
    if bad:
        reset_device_status(device)
        msg = "; ".join(f"{what}: {load().pa_status_string(code).decode()} (status {code})" for what, code in bad)
        raise PagedAttentionError(f"device-side failure: {msg}")


def after_launch(device: torch.device) -> None:
    """Debug hook run after every launch (MINI_LLM_RUNTIME_B200_SYNC_CHECK)."""
    if SYNC_CHECK:
        check_device_status(device)


def prepare_workspace(ws: "_Workspace", batch: int, num_q_heads: int) -> None:
    """Make the ticket range of a (batch, Hq) call read zero (see the
    zeroing rule at pa_decode_workspace_bytes in include/pagedattn.h)."""
    ticket_end = 256 + 4 * batch * num_q_heads
    if ticket_end > ws.clean_end:
        ws.tensor[256:ticket_end].zero_()
        ws.clean_end = ticket_end
    else:
        # This call's partials start at the next 256-byte boundary.
        ws.clean_end = min(ws.clean_end, 256 + _align256(4 * batch * num_q_heads))


def decode_workspace(device: torch.device, nbytes: int, batch: int, num_q_heads: int) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, stream_handle(device))
    ws = _workspaces.get(key)
    if ws is None or ws.tensor.numel() < nbytes:
        ws = _Workspace(device, nbytes)  # zeroed on the current stream
        _workspaces[key] = ws
    prepare_workspace(ws, batch, num_q_heads)
    return ws.tensor

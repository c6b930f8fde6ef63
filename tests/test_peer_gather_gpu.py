"""pa_head_allgather on one GPU, through the C ABI: the one-rank exchange
copies the slice into the output call after call, and a wait for a peer's
lines that nothing stores gives up after its limit with PA_DEVICE_TIMEOUT_PEER
in the area's status word, without a fault or a hang (the two-GPU exchange is
in test_head_shard_gpu.py)."""

import ctypes

import pytest
import torch

from mini_llm_runtime_b200 import _lib

pytestmark = pytest.mark.gpu


def _call(lib, part, out, areas, nbytes, rank, world, limit_ns=0):
    arr = (ctypes.c_void_p * world)(*[a.data_ptr() for a in areas])
    b, hl, d = part.shape
    return lib.pa_head_allgather(part.data_ptr(), part.stride(0), part.stride(1), b, hl, d,
                                 _lib.dtype_code(part.dtype), rank, world, arr, nbytes, out.data_ptr(),
                                 out.stride(0), out.stride(1), limit_ns,
                                 torch.cuda.current_stream().cuda_stream)


def test_one_rank_copies_every_call(cuda_device):
    lib = _lib.load()
    b, hl, d = 8, 7, 64
    nbytes = lib.pa_peer_gather_bytes(1, b * hl * d * 2)
    area = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)
    for i in range(3):
        part = torch.randn(b, hl, d, device=cuda_device).to(torch.bfloat16)
        out = torch.full((b, hl, d), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        assert _call(lib, part, out, [area], nbytes, 0, 1) == 0
        torch.cuda.synchronize()
        assert torch.equal(out, part)
        words = area[128:140].view(torch.int32).tolist()
        assert words == [0, i + 1, 0]  # arrivals rewound, calls counted, status clear


def test_strided_part_and_output(cuda_device):
    lib = _lib.load()
    b, hl, d = 5, 3, 128
    nbytes = lib.pa_peer_gather_bytes(1, b * hl * d * 4)
    area = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)
    big = torch.randn(b, 2 * hl, d, device=cuda_device)
    part = big[:, 1::2]  # head stride 2 * d
    out_big = torch.zeros(b, hl + 2, d, device=cuda_device)
    out = out_big[:, 1:1 + hl]
    assert _call(lib, part, out, [area], nbytes, 0, 1) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, part)
    assert torch.count_nonzero(out_big[:, 0]) == 0 and torch.count_nonzero(out_big[:, -1]) == 0


def test_missing_peer_times_out_with_status(cuda_device):
    # Two ranks, both pointing at this GPU's own area: the kernel stores "rank
    # 0"'s lines and polls for "rank 1"'s, which nothing stores.
    lib = _lib.load()
    b, hl, d = 4, 7, 64
    nbytes = lib.pa_peer_gather_bytes(2, b * hl * d * 2)
    area = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)
    part = torch.randn(b, hl, d, device=cuda_device).to(torch.bfloat16)
    out = torch.zeros(b, 2 * hl, d, device=cuda_device, dtype=torch.bfloat16)
    assert _call(lib, part, out, [area, area], nbytes, 0, 2, limit_ns=20_000_000) == 0
    torch.cuda.synchronize()
    assert area[136:140].view(torch.int32).item() == _lib.PA_DEVICE_TIMEOUT_PEER
    assert torch.equal(out[:, :hl], part)  # this rank's heads landed; the peer's did not
    assert torch.count_nonzero(out[:, hl:]) == 0
    # Re-zeroed, the area serves normal calls again.
    area.zero_()
    one = torch.zeros(b, hl, d, device=cuda_device, dtype=torch.bfloat16)
    assert _call(lib, part, one, [area], lib.pa_peer_gather_bytes(1, b * hl * d * 2), 0, 1) == 0
    torch.cuda.synchronize()
    assert torch.equal(one, part)
    assert area[136:140].view(torch.int32).item() == 0


def test_call_numbers_skip_zero_at_the_wrap(cuda_device):
    """The 32-bit call counter goes from 0xffffffff to 2, never to 0. The
    area's lines start zeroed, so a call numbered 0 would take a missing
    peer's never-written lines for arrived ones."""
    lib = _lib.load()
    b, hl, d = 4, 7, 64
    part = torch.randn(b, hl, d, device=cuda_device).to(torch.bfloat16)
    one_bytes = lib.pa_peer_gather_bytes(1, b * hl * d * 2)
    area = torch.zeros(one_bytes, dtype=torch.uint8, device=cuda_device)
    area[132:136].view(torch.int32).fill_(-2)  # last call 0xfffffffe
    for expect in (-1, 2):  # 0xffffffff, then 2
        out = torch.zeros(b, hl, d, device=cuda_device, dtype=torch.bfloat16)
        assert _call(lib, part, out, [area], one_bytes, 0, 1) == 0
        torch.cuda.synchronize()
        assert torch.equal(out, part)
        assert area[128:140].view(torch.int32).tolist() == [0, expect, 0]
    # "Rank 0 of 2" whose peer area is its own, at the wrap: the peer's lines
    # were never written and must not read as arrived.
    two_bytes = lib.pa_peer_gather_bytes(2, b * hl * d * 2)
    area2 = torch.zeros(two_bytes, dtype=torch.uint8, device=cuda_device)
    area2[132:136].view(torch.int32).fill_(-1)  # last call 0xffffffff
    out = torch.zeros(b, 2 * hl, d, device=cuda_device, dtype=torch.bfloat16)
    assert _call(lib, part, out, [area2, area2], two_bytes, 0, 2, limit_ns=20_000_000) == 0
    torch.cuda.synchronize()
    assert area2[136:140].view(torch.int32).item() == _lib.PA_DEVICE_TIMEOUT_PEER
    assert area2[132:136].view(torch.int32).item() == 2
    assert torch.equal(out[:, :hl], part)
    assert torch.count_nonzero(out[:, hl:]) == 0


def test_fused_decode_exchange_with_a_missing_peer(cuda_device):
    """pa_paged_decode_allgather for "rank 0 of 2" whose peer area is its own:
    this rank's heads equal the plain decode bit for bit, the peer's heads
    never arrive, and the wait ends with PA_DEVICE_TIMEOUT_PEER in the area
    and in the decode workspace, without a fault or a hang."""
    from mini_llm_runtime_b200 import paged_attention_decode_batch_parallel
    from mini_llm_runtime_b200.paged_attention import decode_allgather_launch
    from tests.paged_inputs import make_decode_case

    lib = _lib.load()
    case = make_decode_case([700, 33, 4100], 7, 1, 64, 16, torch.bfloat16, cuda_device, seed=5)
    b, hl, d = case["q"].shape
    nbytes = lib.pa_decode_allgather_bytes(b, 1, hl, d, 2)
    area = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)
    areas = (ctypes.c_void_p * 2)(area.data_ptr(), area.data_ptr())
    out = torch.zeros(b, 2 * hl, d, device=cuda_device, dtype=torch.bfloat16)
    try:
        st = decode_allgather_launch(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16,
                                     out[:, :hl], 0, 2, areas, nbytes, 20_000_000)
        assert st == 0
        torch.cuda.synchronize()
        assert area[136:140].view(torch.int32).item() == _lib.PA_DEVICE_TIMEOUT_PEER
        assert any(code == _lib.PA_DEVICE_TIMEOUT_PEER for _, code in _lib.device_status(cuda_device))
        ref = paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16)
        torch.cuda.synchronize()
        assert torch.equal(out[:, :hl], ref)
        assert torch.count_nonzero(out[:, hl:]) == 0
    finally:
        _lib.reset_device_status(cuda_device)

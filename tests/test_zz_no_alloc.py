"""pa_paged_decode_noalloc: the decode entry point for callers that cannot
allocate device memory (their runtime owns every device byte, or they sit
behind an FFI with no device allocator).  It must give the same results as
pa_paged_decode with a caller-owned workspace, call after call, although its
scratch lives in one fixed array inside the library.

Kept in its own file that pytest collects last, so a failure here cannot stop
an -x run before the other tests ran."""

import ctypes

import numpy as np
import pytest
import torch

from mini_llm_runtime_b200 import _lib, paged_attention_decode_batch_parallel
from tests.paged_inputs import make_decode_case

pytestmark = pytest.mark.gpu

def noalloc_decode(case, dtype, partition_tokens=0):
    """Call the allocation-free entry point straight through the C ABI."""
    lib = _lib.load()
    q, k, v, bt, cl = case["q"], case["k"], case["v"], case["tables"], case["lens"]
    b, hq, d = q.shape
    nb, bs, hkv, _ = k.shape
    out = torch.empty_like(q)
    st = lib.pa_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), v.data_ptr(), nb, bs, hkv, d,
        bt.data_ptr(), bt.stride(0), bt.shape[1], cl.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
        b, hq, float(d ** -0.5), _lib.dtype_code(dtype), partition_tokens,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return st, out


@pytest.mark.parametrize("dtype,partition", [(torch.bfloat16, 0), (torch.bfloat16, 512), (torch.float32, 0)])
def test_noalloc_matches_workspace_entry_point_twice(cuda_device, dtype, partition):
    rng = np.random.default_rng(7)
    ctx = rng.integers(128, 4097, size=64).tolist()
    need = sum((c + 15) // 16 for c in ctx)
    case = make_decode_case(ctx, 14, 2, 64, 16, dtype, cuda_device, seed=77, extra_blocks=need // 10)
    if partition:
        from mini_llm_runtime_b200 import paged_attention_decode_split_kv

        ref = paged_attention_decode_split_kv(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16,
                                              partition_size=partition)
    else:
        ref = paged_attention_decode_batch_parallel(case["q"], case["k"], case["v"], case["tables"], case["lens"], 16)
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        st, out = noalloc_decode(case, dtype, partition)
        assert st == _lib.PA_OK, _lib.load().pa_status_string(st)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        # Same kernels on the same inputs: the results must agree bit for bit.
        assert torch.equal(out, ref)
        status = ctypes.c_int(-1)
        assert _lib.load().pa_decode_noalloc_status(ctypes.byref(status),
                                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
        torch.cuda.synchronize()
        assert status.value == 0


def test_noalloc_rejects_requests_beyond_its_scratch(cuda_device):
    """A request whose scratch exceeds the fixed array fails with
    PA_ERR_CAPACITY before anything is launched."""
    lib = _lib.load()
    # 4096 sequences x 256 query heads x 64 partitions needs far more than 16 MiB.
    need = lib.pa_decode_workspace_bytes(4096, 8, 256, 128, 16, 4096, 1024, 2)
    assert need > 16 << 20
    dummy = torch.zeros(16, dtype=torch.int64, device=cuda_device)
    p = dummy.data_ptr()
    st = lib.pa_paged_decode_noalloc(p, 0, 0, p, p, 1, 16, 8, 128, p, 0, 4096, p, p, 0, 0, 4096, 256, 1.0, 2, 1024,
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.PA_ERR_CAPACITY

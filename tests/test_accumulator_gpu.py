"""P.V accumulator parity (tests/kernels/test_accumulator_cuda.py:9-27 of the
reference: batch {1, 7, 1024}, rtol/atol 2e-5)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from mini_llm_runtime_b200 import paged_attention_accumulator_cuda

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("batch", [1, 7, 1024])
def test_accumulator_matches_sum(cuda_device, batch):
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    p = torch.randn(batch, 64, device="cuda", generator=g)
    v = torch.randn(batch, 64, 256, device="cuda", generator=g)
    actual = paged_attention_accumulator_cuda(p, v)
    expected = torch.sum(p[:, :, None] * v, dim=1)
    torch.testing.assert_close(actual, expected, rtol=2e-5, atol=2e-5)


def test_accumulator_golden(cuda_device):
    gd = np.load(GOLDEN / "accumulator.npz")
    out = paged_attention_accumulator_cuda(torch.tensor(gd["p"]).cuda(), torch.tensor(gd["v"]).cuda())
    np.testing.assert_allclose(out.cpu().numpy(), gd["out"], rtol=2e-5, atol=2e-5)


def test_accumulator_checks():
    with pytest.raises(ValueError, match="CUDA"):
        paged_attention_accumulator_cuda(torch.randn(2, 64), torch.randn(2, 64, 256))

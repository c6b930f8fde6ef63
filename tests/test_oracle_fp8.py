"""The oracle's FP8 (e4m3fn) encoder against torch's own float8 cast: the
stored byte of a pool element is clamp(x / scale, -448, 448) cast to
torch.float8_e4m3fn (round to nearest even), bit for bit, over every
float32 neighbourhood that matters (subnormals, rounding ties, the
saturation edge, NaN, signed zero) and random values."""

import numpy as np
import torch

from oracle import paged_attention_oracle as O


def torch_bits(x: np.ndarray) -> np.ndarray:
    """torch's bytes, every NaN as 0x7f (the pools' contract: NaN signs are
    not kept)."""
    t = torch.clamp(torch.from_numpy(x), -448.0, 448.0).to(torch.float8_e4m3fn)
    b = t.view(torch.uint8).numpy().copy()
    b[np.isnan(x)] = 0x7F
    return b


def test_every_e4m3_value_round_trips():
    bits = np.arange(256, dtype=np.uint8)
    vals = O.e4m3_bits_to_f32(bits)
    ref = torch.from_numpy(bits).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(vals), np.isnan(ref))
    ok = ~np.isnan(vals)
    assert np.array_equal(vals[ok], ref[ok])
    assert np.array_equal(O.f32_to_e4m3_bits(vals[ok]), bits[ok])


def test_encoder_matches_torch_on_edges_and_random_values():
    rng = np.random.default_rng(0)
    grid = O.e4m3_bits_to_f32(np.arange(256, dtype=np.uint8))
    grid = grid[np.isfinite(grid)]
    srt = np.sort(grid)
    ties = ((srt[:-1].astype(np.float64) + srt[1:]) / 2).astype(np.float32)  # exact midpoints: round-to-even cases
    near = np.concatenate([np.nextafter(ties, np.float32(np.inf)), np.nextafter(ties, np.float32(-np.inf))])
    edges = np.array([0.0, -0.0, 448.0, 449.0, 460.0, 464.0, 480.0, 1e6, -1e6, 2.0 ** -10, 2.0 ** -9, 3 * 2.0 ** -10,
                      2.0 ** -6, np.nan, -np.nan, 1e-30], dtype=np.float32)
    rand = np.concatenate([rng.standard_normal(100_000), rng.standard_normal(20_000) * 300,
                           rng.standard_normal(20_000) * 1e-2]).astype(np.float32)
    for x in (ties, near, edges, rand):
        assert np.array_equal(O.f32_to_e4m3_bits(x), torch_bits(x))


def test_quantize_divides_in_fp32():
    x = np.random.default_rng(1).standard_normal(1000).astype(np.float32)
    for scale in (1.0, 0.037, 3.5):
        q = O.quantize_e4m3(x, scale)
        assert np.array_equal(q, torch_bits(x / np.float32(scale)))
        back = O.dequantize_e4m3(q, scale)
        assert np.all(np.abs(back - np.clip(x, -448 * scale, 448 * scale)) <= np.abs(x) * 2.0 ** -3 + scale * 2.0 ** -10)

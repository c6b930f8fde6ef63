"""The C-ABI library loads on a CPU-only host, exports every entry point the
header declares, and rejects bad arguments on the host (no GPU work)."""

import ctypes
import re
from pathlib import Path

import pytest

from mini_llm_runtime_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = "\n".join(p.read_text() for p in sorted((ROOT / "include").glob("*.h")))
    return sorted(set(re.findall(r"PA_API\s+[\w\s\*]+?\b(pa_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("pa_kv_scatter", "pa_paged_decode", "pa_chunk_prefill", "pa_accumulate_pv"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_signatures_cover_header():
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.pa_abi_version() >= 1
    assert lib.pa_status_string(0) == b"ok"
    assert b"invalid" in lib.pa_status_string(-1)
    assert lib.pa_status_string(12345) == b"unknown status"


def test_workspace_bytes():
    lib = _lib.load()
    # Balanced kernel (BF16, D 64): status + tickets + per-CTA partials.
    a = lib.pa_decode_workspace_bytes(64, 2, 14, 64, 16, 256, 0, 2)
    assert a >= 256 + 64 * 14 * 4
    # Explicit partitions (config 3: 16 partitions of 2048 tokens).
    b = lib.pa_decode_workspace_bytes(8, 2, 14, 64, 16, 2048, 2048, 2)
    assert b >= 256 + 8 * 14 * 16 * (64 + 2) * 4
    # FP32 uses the CUDA-core kernel (partitions in multiples of 256 tokens).
    c = lib.pa_decode_workspace_bytes(8, 2, 14, 64, 16, 2048, 2048, 0)
    assert c >= 256 + 8 * 14 * 16 * (64 + 2) * 4
    assert lib.pa_decode_workspace_bytes(0, 2, 14, 64, 16, 256, 0, 2) == 0
    assert lib.pa_decode_workspace_bytes(4, 3, 14, 64, 16, 10, 0, 2) == 0  # Hq % Hkv != 0


@pytest.mark.parametrize(
    "call",
    [
        lambda L: L.pa_paged_decode(None, 0, 0, None, None, 1, 16, 2, 64, None, 0, 1, None, None, 0, 0,
                                    -1, 14, 1.0, 2, 0, None, 0, None),
        lambda L: L.pa_paged_decode(None, 0, 0, None, None, 1, 16, 3, 64, None, 0, 1, None, None, 0, 0,
                                    4, 14, 1.0, 2, 0, None, 0, None),
        lambda L: L.pa_paged_decode(None, 0, 0, None, None, 1, 16, 2, 64, None, 0, 1, None, None, 0, 0,
                                    4, 14, 1.0, 2, 0, None, 0, None),
        lambda L: L.pa_kv_scatter(None, 0, 0, 0, None, 0, 0, 0, 0, None, 1, 4, None, None, 64, 2, 64, 0, None),
        lambda L: L.pa_chunk_prefill(None, 0, 0, None, None, None, 0, 1, None, None, 1, 16, 2, 64, None, 0, 0,
                                     1, 4, 4, 14, 1.0, 2, None, None),
        lambda L: L.pa_accumulate_pv(None, None, None, 3, None),
    ],
)
def test_bad_arguments_rejected_on_host(call):
    assert call(_lib.load()) == _lib.PA_ERR_INVALID


def test_decode_flags_match_header_and_unknown_bits_are_rejected():
    text = (ROOT / "include" / "pagedattn.h").read_text()
    defined = {m[0]: int(m[1]) for m in re.findall(r"#define\s+(PA_DECODE_\w+)\s+(\d+)", text)}
    assert defined == {"PA_DECODE_EARLY_INPUTS": _lib.PA_DECODE_EARLY_INPUTS,
                       "PA_DECODE_EARLY_QUERY": _lib.PA_DECODE_EARLY_QUERY}
    lib = _lib.load()
    fake = ctypes.c_void_p(4096)

    def call(flags):
        return lib.pa_paged_decode_ex(fake, 448, 64, None, None, None, fake, fake, 100, 16, 1, 64, fake, 8, 8, fake,
                                      fake, 896, 64, 8, 7, 0.125, 2, 0, flags, fake, 1 << 20, None)

    assert call(4) == _lib.PA_ERR_INVALID
    assert call(_lib.PA_DECODE_EARLY_INPUTS | 4) == _lib.PA_ERR_INVALID


def test_zero_sized_calls_are_noops():
    lib = _lib.load()
    assert lib.pa_kv_scatter(None, 0, 0, 0, None, 0, 0, 0, 0, None, 1, 0, None, None, 64, 2, 64, 0, None) == 0
    assert lib.pa_accumulate_pv(None, None, None, 0, None) == 0
    assert lib.pa_paged_decode(None, 0, 0, None, None, 1, 16, 2, 64, None, 0, 1, None, None, 0, 0,
                               0, 14, 1.0, 2, 0, None, 0, None) == 0


def test_unsupported_dtype():
    lib = _lib.load()
    # F64 pools are not supported by the scatter (the reference pools are
    # F32/F16/BF16).
    fake = ctypes.c_void_p(16)
    assert lib.pa_kv_scatter(fake, 0, 0, 0, fake, 0, 0, 0, 0, fake, 1, 4, fake, fake, 64, 2, 64, 3, None) == \
        _lib.PA_ERR_UNSUPPORTED


def test_peer_gather_sizes_and_host_checks():
    lib = _lib.load()
    # Header + 2 slots x world x lines (32 bytes of lines per 16 data bytes).
    assert lib.pa_peer_gather_bytes(2, 7168) == 256 + 2 * 2 * 2 * 7168
    assert lib.pa_peer_gather_bytes(1, 10) == 256 + 2 * 2 * 16
    assert lib.pa_peer_gather_bytes(0, 64) == 0
    assert lib.pa_peer_gather_bytes(_lib.PA_PEER_MAX_RANKS + 1, 64) == 0
    fake = ctypes.c_void_p(4096)
    areas = (ctypes.c_void_p * 2)(4096, 8192)
    ok = dict(p_s0=7 * 64, p_s1=64, batch=8, hl=7, d=64, dt=2, rank=0, world=2, nbytes=1 << 20, o_s0=14 * 64,
              o_s1=64, limit=0)

    def call(**kw):
        a = {**ok, **kw}
        return lib.pa_head_allgather(fake, a["p_s0"], a["p_s1"], a["batch"], a["hl"], a["d"], a["dt"], a["rank"],
                                     a["world"], areas, a["nbytes"], fake, a["o_s0"], a["o_s1"], a["limit"], None)

    assert call(rank=2) == _lib.PA_ERR_INVALID              # rank outside the world
    assert call(world=0) == _lib.PA_ERR_INVALID
    assert call(d=4) == _lib.PA_ERR_INVALID                 # a head row of 8 bytes is not 16-byte vectors
    assert call(o_s1=60) == _lib.PA_ERR_INVALID             # unaligned stride
    assert call(limit=-1) == _lib.PA_ERR_INVALID
    assert call(nbytes=256) == _lib.PA_ERR_CAPACITY         # area too small for two slots
    assert lib.pa_ipc_export(None, None, None) == _lib.PA_ERR_INVALID
    assert lib.pa_ipc_close(None) == _lib.PA_ERR_INVALID


def test_decode_allgather_sizes_and_host_checks():
    lib = _lib.load()
    # Config 3 split over 2 ranks: B 8, one KV head and 7 query heads per rank,
    # one segment per sequence, 16 rows x 8 column groups x 32 bytes of lines.
    assert lib.pa_decode_allgather_bytes(8, 1, 7, 64, 2) == 256 + 2 * 2 * 8 * 16 * 8 * 32
    # Two KV heads per segment (group of 7 <= 8): Hkv / 2 segments per sequence.
    assert lib.pa_decode_allgather_bytes(4, 2, 14, 128, 4) == 256 + 2 * 4 * 4 * 16 * 16 * 32
    assert lib.pa_decode_allgather_bytes(0, 1, 7, 64, 2) == 0
    assert lib.pa_decode_allgather_bytes(8, 1, 7, 64, 1) == 256 + 2 * 8 * 16 * 8 * 32
    assert lib.pa_decode_allgather_bytes(8, 2, 7, 64, 2) == 0  # Hq % Hkv != 0
    fake = ctypes.c_void_p(4096)
    areas = (ctypes.c_void_p * 2)(4096, 8192)

    def call(rank=0, world=2, limit=0, flags=0, arr=areas):
        return lib.pa_paged_decode_allgather(fake, 448, 64, None, None, None, fake, fake, 100, 16, 1, 64, fake, 8,
                                             8, fake, fake, 896, 64, 8, 7, 0.125, 2, flags, rank, world, arr,
                                             1 << 20, limit, fake, 1 << 20, None)

    assert call(world=1) == _lib.PA_ERR_INVALID            # a one-rank exchange has no peer
    assert call(rank=2) == _lib.PA_ERR_INVALID
    assert call(limit=-5) == _lib.PA_ERR_INVALID
    assert call(flags=8) == _lib.PA_ERR_INVALID
    assert call(arr=(ctypes.c_void_p * 2)(4096, 8200)) == _lib.PA_ERR_INVALID  # areas must be 256-byte aligned

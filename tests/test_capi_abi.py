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


def test_workspace_size_grows_with_splits():
    lib = _lib.load()
    a = lib.pa_decode_workspace_size(64, 14, 64, 1)
    b = lib.pa_decode_workspace_size(64, 14, 64, 16)
    assert 0 < a < b
    assert b >= 64 * 14 * 16 * (64 + 2) * 4
    assert lib.pa_decode_workspace_size(0, 14, 64, 1) == 0


def test_num_splits_honours_partition_size():
    lib = _lib.load()
    # Config 3: 32768-token contexts, 16 partitions of 2048 tokens.
    assert lib.pa_decode_num_splits(8, 2, 14, 64, 16, 2048, 2048, 2) == 16
    assert lib.pa_decode_num_splits(8, 2, 14, 64, 16, 2048, 4096, 2) == 8
    # FP32 goes to the CUDA-core kernel (partitions in multiples of 256).
    assert lib.pa_decode_num_splits(8, 2, 14, 64, 16, 2048, 2048, 0) == 16
    assert lib.pa_decode_num_splits(4, 3, 14, 64, 16, 10, 0, 2) < 0  # Hq % Hkv != 0


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
                                     1, 4, 4, 14, 1.0, 2, None),
        lambda L: L.pa_accumulate_pv(None, None, None, 3, None),
    ],
)
def test_bad_arguments_rejected_on_host(call):
    assert call(_lib.load()) == _lib.PA_ERR_INVALID


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

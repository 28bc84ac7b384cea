"""The C-ABI library loads and exports every entry point include/*.h
declares; host-side argument checks need no GPU."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from adapterslotsplusplus_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(wp_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 25
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_the_header():
    assert declared_symbols() == set(_lib.SIGNATURES)


def test_rank_supported_table():
    lib = _lib.load()
    for r in (8, 16, 32, 64):
        assert lib.wp_rank_supported(r) == 1
    for r in (4, 24, 48, 128):  # tests/unit/test_rank_variants.py:97-103
        assert lib.wp_rank_supported(r) == 0


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_create_fails_loudly_without_a_device():
    lib = _lib.load()
    h = ctypes.c_void_p()
    rc = lib.wp_create(None, ctypes.byref(h))
    assert rc == _lib.WP_ERR_CUDA
    assert b"no CUDA device" in lib.wp_last_error(None)
    from adapterslotsplusplus_b200 import WarpPipeEngine

    with pytest.raises(RuntimeError):
        WarpPipeEngine()


def test_null_handle_calls_return_errors():
    lib = _lib.load()
    assert lib.wp_evict_adapter(None, 1) == _lib.WP_ERR_INVALID
    assert lib.wp_prefetch_adapter(None, 1) == -1
    assert lib.wp_is_prefetch_ready(None, 1) == 0
    assert lib.wp_build_seg_bounds(None, None, _lib.WP_DTYPE_I64, 4, None) == _lib.WP_ERR_INVALID
    assert lib.wp_tp_unique_id_bytes() == 128

"""Device segmenter (wp_build_seg_bounds) vs the oracle and vs the
reference's own kernel: tables must be bit-exact."""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine
from oracle.seg import seg_bounds
from tests.golden.cases import ADD_LORA_CASES, zipf_ids

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
REF_LIB = ROOT / "oracle" / "_ref" / "libwpref.so"


@pytest.fixture(scope="module")
def engine(cuda):
    return WarpPipeEngine(WarpPipeConfig(max_tokens=16384))


def _check(engine, idx, dtype=torch.int64):
    t = torch.as_tensor(np.asarray(idx), dtype=dtype).cuda()
    assert engine.build_seg_bounds(t)
    got = engine.read_seg_table("live")
    want = [tuple(r) for r in seg_bounds(np.asarray(idx)).tolist()]
    assert got == want


@pytest.mark.parametrize("name", sorted(ADD_LORA_CASES))
def test_reference_index_patterns(engine, name):
    _check(engine, ADD_LORA_CASES[name])


def test_empty_and_single(engine):
    _check(engine, [])
    _check(engine, [7])
    _check(engine, [-1])


@pytest.mark.parametrize("dtype", [torch.int64, torch.int32])
def test_random_patterns_all_sizes(engine, dtype):
    rng = np.random.default_rng(1)
    for T in [1, 2, 31, 32, 33, 255, 256, 257, 1023, 1024, 1025, 4096, 5000, 16384]:
        for kind in range(4):
            if kind == 0:
                idx = rng.integers(-1, 5, T)
            elif kind == 1:
                idx = np.sort(rng.integers(-1, 600, T))
            elif kind == 2:
                idx = np.repeat(rng.integers(-1, 9, T // 100 + 1), 100)[:T]
            else:
                idx = zipf_ids(64, T, seed=T)
            _check(engine, idx, dtype)


def test_one_long_run(engine):
    _check(engine, [3] * 16384)


def test_over_capacity_returns_false(cuda):
    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=512))
    assert eng.build_seg_bounds(torch.zeros(512, dtype=torch.int64, device="cuda"))
    assert not eng.build_seg_bounds(torch.zeros(513, dtype=torch.int64, device="cuda"))


def test_other_int_dtypes_are_cast(engine):
    idx = torch.tensor([1, 1, -1, 2], dtype=torch.int16, device="cuda")
    assert engine.build_seg_bounds(idx)
    assert engine.read_seg_table("live") == [(1, 0, 2), (2, 3, 1)]


@pytest.mark.skipif(not REF_LIB.exists(), reason="oracle/_ref/libwpref.so not built")
def test_bit_exact_with_reference_kernel(engine):
    """Same index vectors through the reference's build_seg_bounds_kernel
    (compiled from its own source into oracle/_ref) and through ours."""
    ref = ctypes.CDLL(str(REF_LIB))
    rng = np.random.default_rng(7)
    cases = [np.asarray(v) for v in ADD_LORA_CASES.values()]
    for T in (1, 16, 64, 100, 200, 255, 256):
        cases += [rng.integers(-1, 6, T), np.sort(rng.integers(-1, 40, T)), zipf_ids(64, T, seed=T),
                  np.repeat(rng.integers(-1, 4, T // 50 + 1), 50)[:T]]
    out = (ctypes.c_int32 * (3 * 256))()
    num = ctypes.c_int32()
    for idx in cases:
        d = torch.as_tensor(idx, dtype=torch.int64).cuda()
        torch.cuda.synchronize()
        assert ref.ref_seg_bounds(ctypes.c_void_p(d.data_ptr()), ctypes.c_int(len(idx)), out, ctypes.byref(num)) == 0
        ref_table = [(out[3 * i], out[3 * i + 1], out[3 * i + 2]) for i in range(num.value)]
        assert engine.build_seg_bounds(d)
        assert engine.read_seg_table("live") == ref_table

"""The allocation-free segmenter, wp_build_seg_bounds_noalloc, through the C ABI.

It exists for callers that may not allocate device memory (code living in
another framework's pre-planned memory, where cudaMalloc would synchronise the
device and bypass that framework's allocator). The test compares it with the
handle-based wp_build_seg_bounds on two calls in a row, and checks that sizes
beyond its fixed scratch are rejected. Integer output: the bound is
bit-exactness. The file name makes pytest collect it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine, _lib
from tests.golden.cases import zipf_ids

pytestmark = pytest.mark.gpu


def _noalloc_table(lib, idx: torch.Tensor):
    T = idx.numel()
    table = torch.full((max(T, 1), 3), -7, dtype=torch.int32, device=idx.device)
    num = torch.full((1,), -1, dtype=torch.int32, device=idx.device)
    code = _lib.WP_DTYPE_I64 if idx.dtype == torch.int64 else _lib.WP_DTYPE_I32
    rc = lib.wp_build_seg_bounds_noalloc(idx.data_ptr(), code, T, table.data_ptr(), num.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.wp_last_error(None)
    torch.cuda.synchronize()
    n = int(num.item())
    return [tuple(int(v) for v in row) for row in table[:n].cpu().tolist()]


def test_noalloc_matches_handle_path_on_two_calls(cuda):
    lib = _lib.load()
    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=8192))
    rng = np.random.default_rng(11)
    cases = [zipf_ids(64, 256, seed=1), rng.integers(-1, 7, 5000)]  # two different calls back to back
    for ids in cases:
        for dtype in (torch.int64, torch.int32):
            idx = torch.as_tensor(ids, dtype=dtype, device="cuda")
            got = _noalloc_table(lib, idx)
            assert eng.build_seg_bounds(idx)
            assert got == eng.read_seg_table("live")


def test_noalloc_rejects_oversized_input(cuda):
    lib = _lib.load()
    cap = lib.wp_seg_bounds_noalloc_max_tokens()
    assert cap == 65536
    idx = torch.zeros(cap + 1, dtype=torch.int64, device="cuda")
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    rc = lib.wp_build_seg_bounds_noalloc(idx.data_ptr(), _lib.WP_DTYPE_I64, cap + 1, out.data_ptr(), out.data_ptr(),
                                         None)
    assert rc == _lib.WP_ERR_CAPACITY
    assert b"65536" in lib.wp_last_error(None)

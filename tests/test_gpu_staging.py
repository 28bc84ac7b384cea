"""Staging slots and the pinned-host adapter store.

Ports tests/unit/test_staging_buffer.py:39-92 of the reference (acquire ->
ready, exhaustion at the pool size, release -> reuse of the same slot,
idempotent double prefetch) and adds the host-store path: adapters
registered from CPU tensors reach the kernels through slots, staged on the
prefetch stream, with LRU reuse of on-demand slots."""

import time

import pytest
import torch

from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine
from oracle import apply as oa

pytestmark = pytest.mark.gpu
RANK, D, O = 32, 4096, 4096
WP_MAX_STAGING = 8  # csrc/bridge/warp_pipe_metadata.h:11


def make_engine(k, slots=WP_MAX_STAGING):
    eng = WarpPipeEngine(WarpPipeConfig(num_staging_slots=slots, max_tokens=4096))
    a = torch.randn(k, RANK, D, device="cuda", dtype=torch.float16) * 0.02
    b = torch.randn(k, O, RANK, device="cuda", dtype=torch.float16) * 0.02
    for i in range(k):
        eng.register_adapter(i, a[i].contiguous(), b[i].contiguous(), 0.5)
    return eng, a, b


def wait_ready(eng, adapter_id, timeout_s=5.0):
    deadline = time.time() + timeout_s
    while time.time() < deadline:
        if eng.is_prefetch_ready(adapter_id):
            return True
        time.sleep(0.001)
    return False


def test_acquire_and_ready(cuda):
    eng, _, _ = make_engine(1)
    assert not eng.is_prefetch_ready(0)
    assert eng.prefetch_adapter(0) >= 0
    assert wait_ready(eng, 0)


def test_pool_exhaustion_is_safe(cuda):
    eng, _, _ = make_engine(WP_MAX_STAGING + 2)
    slots = [eng.prefetch_adapter(i) for i in range(WP_MAX_STAGING + 2)]
    assert sum(s >= 0 for s in slots) == WP_MAX_STAGING
    assert sum(s == -1 for s in slots) == 2
    for i in range(WP_MAX_STAGING):
        assert wait_ready(eng, i)
    for i in range(WP_MAX_STAGING, WP_MAX_STAGING + 2):
        assert not eng.is_prefetch_ready(i)


def test_release_and_reacquire(cuda):
    eng, _, _ = make_engine(2)
    s0 = eng.prefetch_adapter(0)
    assert wait_ready(eng, 0)
    eng.release_prefetch(0)
    assert not eng.is_prefetch_ready(0)
    assert eng.prefetch_adapter(1) == s0
    assert wait_ready(eng, 1)


def test_idempotent_double_prefetch(cuda):
    eng, _, _ = make_engine(1)
    assert eng.prefetch_adapter(0) == eng.prefetch_adapter(0)
    assert wait_ready(eng, 0)


def test_unknown_ids_are_safe(cuda):
    eng, _, _ = make_engine(1)
    assert eng.prefetch_adapter(999) == -1
    assert not eng.is_prefetch_ready(999)
    eng.release_prefetch(999)
    eng.evict_adapter(999)


def test_ready_slot_is_used_and_correct(cuda):
    eng, a, b = make_engine(4)
    for i in range(4):
        eng.prefetch_adapter(i)
        assert wait_ready(eng, i)
    # overwrite the original tensors: a kernel that reads the slot still gets the staged copy
    a_saved, b_saved = a.clone(), b.clone()
    offs = [0, 5, 12, 40, 41]
    eng.build_segments([0, 1, 2, 3], offs)
    a.zero_()
    b.zero_()
    X = (torch.randn(41, D) * 0.1).half()
    Y0 = (torch.randn(41, O) * 0.1).half()
    Y = Y0.cuda()
    eng.expand(eng.shrink(X.cuda(), D, RANK, 41), Y, O, RANK)
    torch.cuda.synchronize()
    table = [(i, offs[i], offs[i + 1] - offs[i]) for i in range(4)]
    _, Y_ref = oa.apply_segments(Y0, X, table, lambda i: a_saved[i].cpu(), lambda i: b_saved[i].cpu(), lambda i: 0.5)
    err = float((Y.float().cpu() - Y_ref).abs().max())
    assert err <= 5e-3 * float(Y_ref.pow(2).mean().sqrt())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_host_store_adapters_stage_on_demand(cuda, dtype):
    """6 host-resident adapters, 4 slots: tables that need different subsets
    reuse on-demand slots least-recently-used first."""
    eng = WarpPipeEngine(WarpPipeConfig(num_staging_slots=4, max_tokens=4096, slot_bytes=2 * RANK * 4096 * 2))
    g = torch.Generator().manual_seed(4)
    A = (torch.randn(6, RANK, D, generator=g) * 0.02).to(dtype)
    B = (torch.randn(6, O, RANK, generator=g) * 0.02).to(dtype)
    for i in range(6):
        eng.register_adapter(i, A[i].contiguous(), B[i].contiguous(), 0.5)
    for subset in ([0, 1, 2], [3, 4, 5], [5, 0, 2, 3], [1, 4]):
        offs = [0]
        for _ in subset:
            offs.append(offs[-1] + 9)
        T = offs[-1]
        eng.build_segments(subset, offs)
        X = (torch.randn(T, D, generator=g) * 0.1).to(dtype)
        Y0 = (torch.randn(T, O, generator=g) * 0.1).to(dtype)
        Y = Y0.cuda()
        eng.expand(eng.shrink(X.cuda(), D, RANK, T), Y, O, RANK)
        torch.cuda.synchronize()
        table = [(a, offs[k], offs[k + 1] - offs[k]) for k, a in enumerate(subset)]
        _, Y_ref = oa.apply_segments(Y0, X, table, lambda i: A[i], lambda i: B[i], lambda i: 0.5)
        err = float((Y.float().cpu() - Y_ref).abs().max())
        assert err <= oa.tolerance(dtype) * float(Y_ref.pow(2).mean().sqrt()), subset
    n, used = eng.slot_stats()
    assert n == 4 and used == 4


def test_host_store_capacity_error(cuda):
    eng = WarpPipeEngine(WarpPipeConfig(num_staging_slots=2, max_tokens=1024, slot_bytes=2 * RANK * 4096 * 2))
    A = torch.zeros(3, RANK, D, dtype=torch.float16)
    B = torch.zeros(3, O, RANK, dtype=torch.float16)
    for i in range(3):
        eng.register_adapter(i, A[i].contiguous(), B[i].contiguous(), 0.5)
    with pytest.raises(RuntimeError):
        eng.build_segments([0, 1, 2], [0, 1, 2, 3])  # three host adapters, two slots

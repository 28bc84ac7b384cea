"""Adapter pool (wp_pool_*): the live apply over a pinned-host adapter store
with paging into GPU slots, against the CPU oracle. Covers the reference's
staging semantics (prefetch_adapter / is_prefetch_ready / release_prefetch,
csrc/memory/staging_buffer.h:62-93, tests/unit/test_staging_buffer.py:39-92)
on the live path: cold misses, eviction of least recently used slots,
prefetch while a step runs, churn over many steps, and replay of a captured
CUDA graph while the slots' contents change."""

import random

import pytest
import torch

from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine
from adapterslotsplusplus_b200.pool import AdapterPool
from oracle import apply as oa

pytestmark = pytest.mark.gpu
DIMS = [(256, 256), (256, 512), (512, 256)]
RANK = 16
N_ADAPTERS = 12
DT = torch.bfloat16


@pytest.fixture(scope="module")
def world(cuda):
    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=1024))
    pool = AdapterPool(eng, num_slots=4, dims=DIMS, rank=RANK, dtype=DT, max_adapters=64)
    g = torch.Generator().manual_seed(4)
    weights = {}
    for a in range(N_ADAPTERS):
        w = [((torch.randn(RANK, d, generator=g) * 0.02).to(DT), (torch.randn(o, RANK, generator=g) * 0.02).to(DT))
             for d, o in DIMS]
        weights[a] = w
        pool.register_host(a, pool.pack(w))
    yield eng, pool, weights
    pool.close()


def stacks(weights, p):
    A = torch.stack([weights[a][p][0] for a in range(N_ADAPTERS)]).unsqueeze(1)
    B = torch.stack([weights[a][p][1] for a in range(N_ADAPTERS)]).unsqueeze(1)
    return A, B


def run_step(eng, pool, weights, ids, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.tensor(sorted(ids), dtype=torch.int64)
    misses = pool.prepare(idx.tolist())
    assert pool.build_seg_bounds(idx.cuda())
    outs = []
    for p, (d, o) in enumerate(DIMS):
        x = (torch.randn(len(ids), d, generator=g) * 0.1).to(DT)
        y = (torch.randn(len(ids), o, generator=g) * 0.1).to(DT)
        yd = y.cuda()
        pool.add_lora(p, yd, x.cuda(), 0.5)
        A, B = stacks(weights, p)
        outs.append((yd, oa.add_lora_grouped(y, x, A, B, 0.5, idx)))
    torch.cuda.synchronize()
    for yd, ref in outs:
        rms = float(ref.pow(2).mean().sqrt())
        assert float((yd.float().cpu() - ref).abs().max()) <= oa.tolerance(DT) * rms
    return misses


def test_cold_then_warm(world):
    eng, pool, weights = world
    ids = [0] * 5 + [3] * 40 + [-1] * 2 + [7] * 9
    assert run_step(eng, pool, weights, ids, 1) == 3
    assert run_step(eng, pool, weights, ids, 2) == 0  # resident now
    assert eng.device_error(clear=True) == 0


def test_churn_with_eviction(world):
    eng, pool, weights = world
    rng = random.Random(0)
    before = pool.stats()["copies"]
    for step in range(25):
        active = rng.sample(range(N_ADAPTERS), rng.randint(1, 4))
        ids = [a for a in active for _ in range(rng.randint(1, 40))]
        run_step(eng, pool, weights, ids, 100 + step)
    assert pool.stats()["copies"] > before  # adapters were paged in and out
    assert pool.stats()["resident"] <= 4
    assert eng.device_error(clear=True) == 0


def test_prefetch_semantics(world):
    eng, pool, weights = world
    run_step(eng, pool, weights, [1] * 8, 7)
    assert pool.prefetch(999) == -1  # unknown id
    slots = [pool.prefetch(a) for a in (8, 9, 10)]
    assert all(s >= 0 for s in slots) and len(set(slots)) == 3
    assert pool.prefetch(8) == slots[0]  # re-prefetch returns the same slot
    torch.cuda.synchronize()
    assert all(pool.is_prefetch_ready(a) for a in (8, 9, 10))
    # prefetched adapters are hits; slot 4 holds adapter 1 or is free
    assert run_step(eng, pool, weights, [8] * 3 + [9] * 3 + [10] * 3, 8) == 0
    # three pinned slots and the step's one: no slot left for a fourth prefetch
    assert pool.prefetch(11) in (-1, *range(4))
    for a in (8, 9, 10):
        pool.release_prefetch(a)
    pool.release_prefetch(12345)  # unknown: no-op
    assert run_step(eng, pool, weights, [2] * 4 + [5] * 4 + [6] * 4 + [11] * 4, 9) >= 3
    pool.release_prefetch(11)


def test_prefetch_overlaps_running_step(world):
    """A prefetch issued while a step's kernels are still queued copies on the
    pool's stream into a slot that step does not read; the step's results
    are unaffected."""
    eng, pool, weights = world
    ids = [0] * 30 + [1] * 30
    pool.prepare(ids)
    assert pool.build_seg_bounds(torch.tensor(ids, device="cuda"))
    g = torch.Generator().manual_seed(11)
    x = (torch.randn(len(ids), 256, generator=g) * 0.1).to(DT)
    y = (torch.randn(len(ids), 256, generator=g) * 0.1).to(DT)
    ys = [y.cuda() for _ in range(20)]
    for yd in ys:  # a long step
        pool.add_lora(0, yd, x.cuda(), 0.5)
    s = pool.prefetch(5)
    assert s >= 0
    torch.cuda.synchronize()
    A, B = stacks(weights, 0)
    ref = oa.add_lora_grouped(y, x, A, B, 0.5, torch.tensor(ids))
    rms = float(ref.pow(2).mean().sqrt())
    for yd in ys:
        assert float((yd.float().cpu() - ref).abs().max()) <= oa.tolerance(DT) * rms
    assert pool.is_prefetch_ready(5)
    pool.release_prefetch(5)


def test_graph_replay_with_paging(world):
    """The step's apply calls captured once; every replay follows prepare +
    build_seg_bounds (outside the graph) with a different active set."""
    eng, pool, weights = world
    T = 48
    g = torch.Generator().manual_seed(12)
    xs = [(torch.randn(T, d, generator=g) * 0.1).to(DT).cuda() for d, _ in DIMS]
    y0 = [(torch.randn(T, o, generator=g) * 0.1).to(DT) for _, o in DIMS]
    ys = [y.cuda() for y in y0]
    idx_buf = torch.zeros(T, dtype=torch.int64, device="cuda")
    ids = [4] * T
    pool.prepare(ids)
    idx_buf.copy_(torch.tensor(ids))
    pool.build_seg_bounds(idx_buf)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for p in range(len(DIMS)):
            pool.add_lora(p, ys[p], xs[p], 0.5)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for p in range(len(DIMS)):
            pool.add_lora(p, ys[p], xs[p], 0.5)
    rng = random.Random(3)
    for step in range(6):
        active = rng.sample(range(N_ADAPTERS), 3)
        ids = sorted(active[i % 3] for i in range(T))
        pool.prepare(ids)
        idx_buf.copy_(torch.tensor(ids))
        pool.build_seg_bounds(idx_buf)
        for p in range(len(DIMS)):
            ys[p].copy_(y0[p].cuda())
        graph.replay()
        torch.cuda.synchronize()
        for p in range(len(DIMS)):
            A, B = stacks(weights, p)
            ref = oa.add_lora_grouped(y0[p], xs[p].cpu(), A, B, 0.5, torch.tensor(ids))
            rms = float(ref.pow(2).mean().sqrt())
            assert float((ys[p].float().cpu() - ref).abs().max()) <= oa.tolerance(DT) * rms, (step, p)
    assert eng.device_error(clear=True) == 0


def test_pool_errors(world):
    eng, pool, _ = world
    with pytest.raises(RuntimeError):
        pool.prepare([40])  # not registered
    with pytest.raises(RuntimeError):
        pool.register_host(1, torch.zeros(pool.slot_bytes, dtype=torch.uint8))  # not pinned
    with pytest.raises(RuntimeError):
        pool.prepare([0, 1, 2, 3, 5])  # five adapters, four slots

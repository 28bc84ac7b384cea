"""Tensor-parallel sharding logic on CPU: two gloo ranks shard the weights
and activations with adapterslotsplusplus_b200.tp's helpers, run their share
of the apply with the oracle, exchange what the GPU path exchanges (the fp32
[T, r] shrink partials of row-parallel layers, summed by an all-reduce) and
must reproduce the unsharded result. No GPU: this checks the host-side
decomposition that TensorParallelApply drives with NCCL."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from adapterslotsplusplus_b200 import tp
from oracle import apply as oa

WORLD = 2
T, D, O, R, L = 24, 64, 96, 16, 5
IDX = [0, 0, 3, 3, 3, -1, 1, 1, 4, 4, 4, 4, 2, -1, -1, 0, 0, 0, 1, 2, 3, 4, 4, 4]


def _inputs():
    g = torch.Generator().manual_seed(7)
    wa = (torch.randn(L, 1, R, D, generator=g) * 0.05).bfloat16()
    wb = (torch.randn(L, 1, O, R, generator=g) * 0.05).bfloat16()
    x = (torch.randn(T, D, generator=g) * 0.2).bfloat16()
    y = (torch.randn(T, O, generator=g) * 0.2).bfloat16()
    return wa, wb, x, y


def _worker(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        wa, wb, x, y = _inputs()
        idx = torch.tensor(IDX)
        scale = 0.75
        # column-parallel: full x and A, this rank's output columns of B and y
        wb_c = tp.shard_column(wb, rank, WORLD)
        y_c = tp.shard_column_output(y, rank, WORLD)
        col = oa.add_lora_grouped(y_c, x, wa, wb_c, scale, idx)
        # row-parallel: this rank's d slice of x and A -> partial H, summed over ranks
        x_r = tp.shard_row_input(x, rank, WORLD)
        wa_r = tp.shard_row(wa, rank, WORLD)
        H = torch.zeros(T, R)
        for a_id in sorted(set(i for i in IDX if i >= 0)):
            rows = (idx == a_id).nonzero().reshape(-1)
            H[rows] = oa.reference_bgmv_shrink(x_r[rows], wa_r[a_id, 0], scale)
        dist.all_reduce(H, op=dist.ReduceOp.SUM)
        row = y.float().clone()
        for a_id in sorted(set(i for i in IDX if i >= 0)):
            rows = (idx == a_id).nonzero().reshape(-1)
            row[rows] = oa.reference_bgmv_expand(H[rows], wb[a_id, 0], y[rows])
        q.put((rank, col, row))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_helpers_split_evenly():
    wa, wb, x, y = _inputs()
    parts = [tp.shard_column(wb, r, WORLD) for r in range(WORLD)]
    assert torch.equal(torch.cat(parts, dim=-2), wb)
    parts = [tp.shard_row(wa, r, WORLD) for r in range(WORLD)]
    assert torch.equal(torch.cat(parts, dim=-1), wa)
    assert all(p.is_contiguous() for p in parts)
    with pytest.raises(ValueError):
        tp.shard_row(wa[..., :D - 1], 0, WORLD)


def test_two_rank_decomposition_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got.sort(key=lambda t: t[0])
    wa, wb, x, y = _inputs()
    full = oa.add_lora_grouped(y, x, wa, wb, 0.75, torch.tensor(IDX))
    # column-parallel: the ranks' column blocks concatenate to the full result
    col = torch.cat([c for _, c, _ in got], dim=1)
    assert torch.allclose(col, full, rtol=0, atol=1e-5)
    # row-parallel: every rank ends with the full result (d-split partials summed)
    for _, _, row in got:
        assert torch.allclose(row, full, rtol=0, atol=1e-4)

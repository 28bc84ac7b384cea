"""Fused live calls with few segments run the clustered decode kernel on
clusters of 4 (each segment's shrink and expand spread over four CTAs):
results against the CPU oracle (same bound as the other apply tests),
the cluster size actually launched, graph replay, and the switch back to
clusters of 2 when the segments outnumber the clusters of 4."""

import pytest
import torch

from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine
from oracle import apply as oa

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng(cuda):
    return WarpPipeEngine(WarpPipeConfig(max_tokens=8192, kernel="cluster"))


def check(y, ref, dtype, what):
    y = y.float().cpu()
    ref = ref.float().cpu()
    rms = float(ref.pow(2).mean().sqrt())
    err = float((y - ref).abs().max())
    assert err <= oa.tolerance(dtype) * rms, f"{what}: {err:.3e} > {oa.tolerance(dtype) * rms:.3e}"


def runs(lengths, ids):
    out = []
    for n, a in zip(lengths, ids):
        out += [a] * n
    return out


def inputs(idx, dtype, d, o, rank, n_adapters, seed):
    g = torch.Generator().manual_seed(seed)
    T = len(idx)
    wa = (torch.randn(n_adapters, 1, rank, d, generator=g) * 0.02).to(dtype)
    wb = (torch.randn(n_adapters, 1, o, rank, generator=g) * 0.02).to(dtype)
    x = (torch.randn(T, d, generator=g) * 0.1).to(dtype)
    y = (torch.randn(T, o, generator=g) * 0.1).to(dtype)
    return wa, wb, x, y


def settle(eng, idx):
    """Segment table for idx, with its segment count landed on the host (the
    kernel choice reads it without a sync)."""
    assert eng.build_seg_bounds(torch.tensor(idx, dtype=torch.int64).cuda())
    torch.cuda.synchronize()


CASES = [
    # (run lengths, d, o, rank): 1, 8 and 16 segments; 32-token pieces and small runs
    ([256], 4096, 4096, 32),
    ([32] * 8, 4096, 11008, 32),
    ([40, 3, 1, 17, 64, 9, 2, 30], 11008, 4096, 32),
    ([5, 1, 7, 2, 33, 12, 1, 1, 4, 8, 16, 2, 3, 1, 6, 20], 4096, 4096, 16),
    ([64, 16, 8, 1], 4096, 4096, 8),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_few_segments_on_clusters_of_4(eng, dtype, case):
    lengths, d, o, rank = CASES[case]
    n_adapters = len(lengths)
    idx = runs(lengths, list(range(n_adapters)))
    wa, wb, x, y = inputs(idx, dtype, d, o, rank, n_adapters, seed=case)
    ref = oa.add_lora_grouped(y, x, wa, wb, 16.0 / rank, torch.tensor(idx))
    settle(eng, idx)
    yd = y.cuda()
    assert eng.add_lora_packed(yd, x.cuda(), wa.cuda(), wb.cuda(), 16.0 / rank)
    torch.cuda.synchronize()
    assert eng.last_apply_cluster() == 4
    assert eng.device_error(clear=True) == 0
    check(yd, ref, dtype, f"case {case}")


def test_graph_replay_on_clusters_of_4(eng):
    dtype, d, o, rank = torch.bfloat16, 4096, 11008, 32
    idx = runs([32, 32, 7, 1, 50], [3, 0, 2, 1, 4])
    wa, wb, x, y = inputs(idx, dtype, d, o, rank, 5, seed=11)
    ref = oa.add_lora_grouped(y, x, wa, wb, 0.5, torch.tensor(idx))
    settle(eng, idx)
    yd = y.cuda()
    y0 = yd.clone()
    xd, wad, wbd = x.cuda(), wa.cuda(), wb.cuda()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        assert eng.add_lora_packed(yd, xd, wad, wbd, 0.5)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        assert eng.add_lora_packed(yd, xd, wad, wbd, 0.5)
    assert eng.last_apply_cluster() == 4
    for _ in range(3):
        yd.copy_(y0)
        g.replay()
    torch.cuda.synchronize()
    check(yd, ref, dtype, "graph replay")


def test_many_segments_stay_on_pairs(eng):
    dtype, d, o, rank = torch.bfloat16, 4096, 4096, 32
    lengths = [1] * 100  # 100 segments: more than the clusters of 4
    idx = runs(lengths, [i % 64 for i in range(100)])
    wa, wb, x, y = inputs(idx, dtype, d, o, rank, 64, seed=5)
    ref = oa.add_lora_grouped(y, x, wa, wb, 0.5, torch.tensor(idx))
    settle(eng, idx)
    yd = y.cuda()
    assert eng.add_lora_packed(yd, x.cuda(), wa.cuda(), wb.cuda(), 0.5)
    torch.cuda.synchronize()
    assert eng.last_apply_cluster() == 2
    check(yd, ref, dtype, "100 segments")

"""Programmatic-dependent-launch prefetch of the apply kernel: with
prefetch_weights (weights and table read before the previous kernel has
finished) and prefetch_inputs (x loaded and the whole shrink run before it;
only y waits), a chain of calls gives results bit-identical to strict stream
order, eagerly and replayed from a CUDA graph. A call whose x the previous
kernel wrote is fenced with note_input_write (engine.add_lora_packed does it
when its reshape had to copy x). The reference has no dependent launch; the
arithmetic is the same kernel's either way."""

import pytest
import torch

from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine
from tests.golden.cases import zipf_ids

pytestmark = pytest.mark.gpu

SHAPES = [(4096, 4096), (4096, 11008), (11008, 4096), (1024, 768)]


def _calls(dev, T, r=32, n_adapters=16, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    out = []
    for d, o in SHAPES:
        wa = torch.randn(n_adapters, 1, r, d, device=dev, dtype=torch.bfloat16, generator=g) * 0.02
        wb = torch.randn(n_adapters, 1, o, r, device=dev, dtype=torch.bfloat16, generator=g) * 0.02
        x = torch.randn(T, d, device=dev, dtype=torch.bfloat16, generator=g) * 0.1
        y0 = torch.randn(T, o, device=dev, dtype=torch.bfloat16, generator=g) * 0.1
        out.append((x, y0, wa, wb))
    return out


def _run(eng, calls, ids, graph):
    ys = [y0.clone() for _, y0, _, _ in calls]
    assert eng.build_seg_bounds(ids)

    def step():
        for (x, _, wa, wb), y in zip(calls, ys):
            eng.add_lora_packed(y, x, wa, wb, 0.5)

    if not graph:
        step()
    else:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        for y, (_, y0, _, _) in zip(ys, calls):
            y.copy_(y0)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            step()
        for y, (_, y0, _, _) in zip(ys, calls):
            y.copy_(y0)
        gr.replay()
    torch.cuda.synchronize()
    assert eng.device_error(clear=True) == 0
    return ys


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("resident,T", [(64, 256), (1, 256), (512, 256), (8, 1)])
def test_prefetch_matches_strict_order(cuda, graph, resident, T):
    dev = torch.device("cuda", 0)
    calls = _calls(dev, T, n_adapters=max(resident, 1))
    ids = torch.as_tensor(zipf_ids(resident, T, seed=3), device=dev)
    strict = WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=False))
    pre = WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=True, prefetch_inputs=True))
    want = _run(strict, calls, ids, graph)
    got = _run(pre, calls, ids, graph)
    for w, g_ in zip(want, got):
        assert torch.equal(w, g_)


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("rank", [8, 16, 32, 64])
@pytest.mark.parametrize("resident,T", [(64, 4096), (512, 256), (4, 64)])
def test_prefetch_ranks_and_segments_per_cluster(cuda, graph, rank, resident, T):
    """Every rank (stage rings of 3 to 8 stages) with one and with several
    segments per cluster: the prefetched first stages, the shrink run before
    the dependency and the expand stages after it share one ring."""
    dev = torch.device("cuda", 0)
    calls = _calls(dev, T, r=rank, n_adapters=max(resident, 1), seed=rank)
    ids = torch.as_tensor(zipf_ids(resident, T, seed=11), device=dev)
    strict = WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=False))
    pre = WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=True, prefetch_inputs=True))
    want = _run(strict, calls, ids, graph)
    got = _run(pre, calls, ids, graph)
    for w, g_ in zip(want, got):
        assert torch.equal(w, g_)


def test_input_written_by_previous_kernel(cuda):
    """x of the second call is the first call's output: note_input_write
    keeps the second call's x loads behind the first call."""
    dev = torch.device("cuda", 0)
    T, d, r = 256, 4096, 32
    g = torch.Generator(device=dev).manual_seed(5)
    wa = torch.randn(16, 1, r, d, device=dev, dtype=torch.bfloat16, generator=g) * 0.02
    wb = torch.randn(16, 1, d, r, device=dev, dtype=torch.bfloat16, generator=g) * 0.02
    x = torch.randn(T, d, device=dev, dtype=torch.bfloat16, generator=g) * 0.1
    ids = torch.as_tensor(zipf_ids(16, T, seed=4), device=dev)

    def chain(eng, note):
        y1 = (torch.randn(T, d, device=dev, dtype=torch.bfloat16, generator=torch.Generator(device=dev).manual_seed(6))
              * 0.1)
        y2 = torch.zeros(T, d, device=dev, dtype=torch.bfloat16)
        torch.cuda.synchronize()
        assert eng.build_seg_bounds(ids)
        eng.add_lora_packed(y1, x, wa, wb, 4.0)  # writes y1
        if note:
            eng.note_input_write()
        eng.add_lora_packed(y2, y1, wa, wb, 4.0)  # reads y1 as its x
        torch.cuda.synchronize()
        assert eng.device_error(clear=True) == 0
        return y2

    want = chain(WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=False)), False)
    got = chain(WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=True, prefetch_inputs=True)), True)
    assert torch.equal(want, got)


def test_reshape_copy_notes_the_write(cuda):
    """A non-contiguous 3-D x makes add_lora_packed copy it (reshape): the
    engine notes the copy itself, and the result equals strict order."""
    dev = torch.device("cuda", 0)
    T, d, r = 128, 1024, 16
    g = torch.Generator(device=dev).manual_seed(7)
    wa = torch.randn(4, 1, r, d, device=dev, dtype=torch.bfloat16, generator=g) * 0.02
    wb = torch.randn(4, 1, d, r, device=dev, dtype=torch.bfloat16, generator=g) * 0.02
    xb = torch.randn(2, d, T // 2, device=dev, dtype=torch.bfloat16, generator=g) * 0.1
    x = xb.transpose(1, 2)  # [2, T/2, d], not contiguous
    ids = torch.as_tensor(zipf_ids(4, T, seed=8), device=dev)
    y0 = torch.randn(T, d, device=dev, dtype=torch.bfloat16, generator=g) * 0.1
    outs = []
    for cfg in (WarpPipeConfig(max_tokens=4096), WarpPipeConfig(max_tokens=4096, prefetch_weights=True,
                                                               prefetch_inputs=True)):
        eng = WarpPipeEngine(cfg)
        y = y0.clone()
        assert eng.build_seg_bounds(ids)
        assert eng.add_lora_packed(y, x, wa, wb, 0.5)
        torch.cuda.synchronize()
        outs.append(y)
    assert torch.equal(outs[0], outs[1])

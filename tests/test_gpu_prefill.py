"""Prefill path: runs of >= 128 tokens of one adapter as tcgen05 GEMMs
(wp_prefill.cu) with the short runs on the decode kernel, against the CPU
oracle (the reference's fp32 per-segment math, oracle/apply.py). Covers the
tile table itself, ranks 16/32/64 in fp16 and bf16, the shapes of the
Llama-7B projections and of the draft model, config 2's prefill mix (8 runs
of 512 tokens), runs that end inside a tile, mixes of long and short runs,
the fallbacks (rank 8, unaligned y), multi-slice calls and CUDA-graph replay.
The reference has no prefill kernel (segments are capped at 32 tokens,
csrc/bridge/warp_pipe_metadata.h:22)."""

import pytest
import torch

from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine
from oracle import apply as oa
from oracle.seg import seg_bounds

pytestmark = pytest.mark.gpu
DTYPES = [torch.float16, torch.bfloat16]


@pytest.fixture(scope="module")
def eng(cuda):
    return WarpPipeEngine(WarpPipeConfig(max_tokens=8192))


def runs(*spec):
    """[(adapter, length), ...] -> token ids."""
    out = []
    for a, n in spec:
        out += [a] * n
    return out


def expected_tiles(idx, min_run=128, tile=128):
    tiles, short = [], []
    i = 0
    while i < len(idx):
        j = i
        while j < len(idx) and idx[j] == idx[i]:
            j += 1
        if idx[i] >= 0:
            n = j - i
            if n >= min_run:
                tiles += [(idx[i], i + s, min(tile, n - s)) for s in range(0, n, tile)]
            else:
                short += [(idx[i], i + s, min(32, n - s)) for s in range(0, n, 32)]
        i = j
    return tiles, short


def check(eng, idx, dtype, d, o, r, n_adapters=8, seed=0, y_offset=None, y_cols=None, prefill=True):
    g = torch.Generator().manual_seed(seed)
    T = len(idx)
    wa = (torch.randn(n_adapters, 1, r, d, generator=g) * 0.02).to(dtype)
    wb = (torch.randn(n_adapters, 1, o, r, generator=g) * 0.02).to(dtype)
    x = (torch.randn(T, d, generator=g) * 0.1).to(dtype)
    y = (torch.randn(T, y_cols or o, generator=g) * 0.1).to(dtype)
    scale = 16.0 / r
    ref = oa.add_lora_grouped(y, x, wa, wb, scale, torch.tensor(idx), y_offset=y_offset or 0)
    yd = y.cuda()
    assert eng.build_seg_bounds(torch.tensor(idx, dtype=torch.int64).cuda(), prefill=prefill)
    if y_offset is None:
        assert eng.add_lora_packed(yd, x.cuda(), wa.cuda(), wb.cuda(), scale)
    else:
        assert eng.add_lora(yd, x.cuda(), wa.cuda(), wb.cuda(), scale, y_offset, o)
    torch.cuda.synchronize()
    rms = float(ref.pow(2).mean().sqrt())
    err = float((yd.float().cpu() - ref).abs().max())
    assert err <= oa.tolerance(dtype) * rms, f"max_abs_err {err:.3e} > {oa.tolerance(dtype) * rms:.3e}"
    assert eng.device_error(clear=True) == 0


def test_tile_tables(eng):
    idx = runs((0, 130), (1, 5), (-1, 7), (2, 300), (3, 127), (4, 1000), (5, 128))
    assert eng.build_seg_bounds(torch.tensor(idx, device="cuda"), prefill=True)
    tiles, short = expected_tiles(idx)
    assert eng.read_seg_table("tiles") == tiles
    assert eng.read_seg_table("short") == short
    # the full table is the reference's, whatever the mode
    assert eng.read_seg_table("live") == [tuple(v) for v in seg_bounds(idx).tolist()]
    assert eng.build_seg_bounds(torch.tensor(idx, device="cuda"), prefill=False)
    assert eng.read_seg_table("tiles") == []


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("r", [16, 32, 64])
def test_prefill_ranks(eng, dtype, r):
    idx = runs((0, 130), (1, 5), (2, 300), (3, 127), (4, 600), (5, 128))
    check(eng, idx, dtype, 1024, 768, r, seed=r)


@pytest.mark.parametrize("d,o", [(4096, 4096), (4096, 11008), (11008, 4096), (768, 3072), (3072, 768)])
def test_prefill_shapes(eng, d, o):
    idx = runs((1, 512), (6, 40), (2, 256), (0, 200))
    check(eng, idx, torch.bfloat16, d, o, 32, seed=d + o)


def test_prefill_mix_config2(eng):
    idx = [a for a in range(8) for _ in range(512)]
    check(eng, idx, torch.bfloat16, 4096, 4096, 32, seed=2)


def test_prefill_auto_mode(cuda):
    # prefill_tokens > 0: a build with at least that many tokens switches to
    # prefill mode by itself; the default (0) never does
    idx = [a for a in range(4) for _ in range(1024)]
    auto = WarpPipeEngine(WarpPipeConfig(max_tokens=8192, prefill_tokens=2048))
    check(auto, idx, torch.bfloat16, 2048, 1024, 16, seed=4, prefill=None)
    assert auto.read_seg_table("tiles") == expected_tiles(idx)[0]
    plain = WarpPipeEngine(WarpPipeConfig(max_tokens=8192))
    check(plain, idx, torch.bfloat16, 2048, 1024, 16, seed=4, prefill=None)
    assert plain.read_seg_table("tiles") == []


def test_prefill_fallbacks(eng):
    idx = runs((0, 300), (1, 20), (2, 256))
    check(eng, idx, torch.bfloat16, 1024, 512, 8, seed=5)  # rank 8: decode kernel on the full table
    check(eng, idx, torch.bfloat16, 1024, 512, 32, seed=6, y_offset=4, y_cols=520)  # unaligned y
    check(eng, idx, torch.bfloat16, 1000, 512, 32, seed=7)  # d not a multiple of 64


def test_prefill_sliced_and_nslice(eng):
    idx = runs((0, 200), (3, 10), (1, 260))
    check(eng, idx, torch.bfloat16, 1024, 512, 32, seed=8, y_offset=512, y_cols=1536)
    g = torch.Generator().manual_seed(9)
    T, d, o, r = len(idx), 1024, 512, 32
    was = [(torch.randn(4, 1, r, d, generator=g) * 0.02).bfloat16() for _ in range(3)]
    wbs = [(torch.randn(4, 1, o, r, generator=g) * 0.02).bfloat16() for _ in range(3)]
    x = (torch.randn(T, d, generator=g) * 0.1).bfloat16()
    y = (torch.randn(T, 3 * o, generator=g) * 0.1).bfloat16()
    yd = y.cuda()
    assert eng.build_seg_bounds(torch.tensor(idx, device="cuda"), prefill=True)
    assert eng.add_lora_packed_nslice(yd, x.cuda(), [w.cuda() for w in was], [w.cuda() for w in wbs], 0.5, [o] * 3)
    torch.cuda.synchronize()
    ref = y.float()
    for s in range(3):
        ref = oa.add_lora_grouped(ref.bfloat16(), x, was[s], wbs[s], 0.5, torch.tensor(idx), y_offset=s * o)
    rms = float(ref.pow(2).mean().sqrt())
    assert float((yd.float().cpu() - ref).abs().max()) <= 2 * oa.tolerance(torch.bfloat16) * rms


def test_prefill_graph_replay(eng):
    dtype, d, o, r = torch.bfloat16, 2048, 1024, 32
    g = torch.Generator().manual_seed(10)
    T = 1024
    wa = (torch.randn(8, 1, r, d, generator=g) * 0.02).to(dtype).cuda()
    wb = (torch.randn(8, 1, o, r, generator=g) * 0.02).to(dtype).cuda()
    x = (torch.randn(T, d, generator=g) * 0.1).to(dtype).cuda()
    y0 = (torch.randn(T, o, generator=g) * 0.1).to(dtype)
    y = y0.cuda()
    idx_buf = torch.zeros(T, dtype=torch.int64, device="cuda")
    first = runs((0, 512), (1, 512))
    idx_buf.copy_(torch.tensor(first))
    assert eng.build_seg_bounds(idx_buf, prefill=True)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        eng.add_lora_packed(y, x, wa, wb, 0.5)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        eng.add_lora_packed(y, x, wa, wb, 0.5)
    for spec in (first, runs((2, 130), (3, 20), (4, 874)), runs((5, 1024)), [a % 8 for a in range(T)]):
        idx_buf.copy_(torch.tensor(spec))
        assert eng.build_seg_bounds(idx_buf, prefill=True)
        y.copy_(y0.cuda())
        graph.replay()
        torch.cuda.synchronize()
        ref = oa.add_lora_grouped(y0, x.cpu(), wa.cpu(), wb.cpu(), 0.5, torch.tensor(spec))
        rms = float(ref.pow(2).mean().sqrt())
        assert float((y.float().cpu() - ref).abs().max()) <= oa.tolerance(dtype) * rms
    assert eng.device_error(clear=True) == 0

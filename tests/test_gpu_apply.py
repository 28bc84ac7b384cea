"""Apply kernels (live add_lora path and registry shrink/expand path) vs the
CPU oracle. Bound: max|Y - Y_ref| <= 5e-3 * RMS(Y_ref) for fp16 and
2e-2 * RMS(Y_ref) for bf16, Y_ref the fp32 per-segment result with no
rounding of H (oracle/apply.py)."""

import ctypes
import random
from pathlib import Path

import numpy as np
import pytest
import torch

from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine
from oracle import apply as oa
from oracle.seg import seg_bounds
from tests.golden.cases import ADD_LORA_CASES, add_lora_inputs, config0_inputs, rank_case_inputs, zipf_ids

pytestmark = pytest.mark.gpu
DTYPES = [torch.float16, torch.bfloat16]
ROOT = Path(__file__).resolve().parent.parent
REF_LIB = ROOT / "oracle" / "_ref" / "libwpref.so"


@pytest.fixture(scope="module", params=["cluster", "split"])
def engine(cuda, request):
    """Both decode kernels: the clustered one and the balanced (split) one."""
    return WarpPipeEngine(WarpPipeConfig(max_tokens=8192, kernel=request.param))


def assert_close(y, y_ref, dtype, what=""):
    y = y.float().cpu()
    y_ref = y_ref.float().cpu()
    rms = float(y_ref.pow(2).mean().sqrt())
    err = float((y - y_ref).abs().max()) if y.numel() else 0.0
    tol = oa.tolerance(dtype) * max(rms, 1e-30)
    assert err <= tol, f"{what}: max_abs_err={err:.3e} > {tol:.3e} (rms {rms:.3e})"


def live_case(engine, idx, dtype, d, o, rank, n_adapters=8, seed=0, y_offset=None, y_cols=None, scale=None):
    g = torch.Generator().manual_seed(seed)
    T = len(idx)
    wa = (torch.randn(n_adapters, 1, rank, d, generator=g) * 0.02).to(dtype)
    wb = (torch.randn(n_adapters, 1, o, rank, generator=g) * 0.02).to(dtype)
    x = (torch.randn(T, d, generator=g) * 0.1).to(dtype)
    y = (torch.randn(T, y_cols or o, generator=g) * 0.1).to(dtype)
    scale = 16.0 / rank if scale is None else scale
    ref = oa.add_lora_grouped(y, x, wa, wb, scale, torch.tensor(idx), y_offset=y_offset or 0)
    yd = y.cuda()
    assert engine.build_seg_bounds(torch.tensor(idx, dtype=torch.int64).cuda())
    if y_offset is None:
        assert engine.add_lora_packed(yd, x.cuda(), wa.cuda(), wb.cuda(), scale)
    else:
        assert engine.add_lora(yd, x.cuda(), wa.cuda(), wb.cuda(), scale, y_offset, o)
    torch.cuda.synchronize()
    return yd, ref


# ---- live path: the reference's index patterns (test_add_lora_packed.py) ----

@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("name", sorted(ADD_LORA_CASES))
def test_add_lora_index_patterns(engine, dtype, name):
    y, ref = live_case(engine, ADD_LORA_CASES[name], dtype, 4096, 4096, 32)
    assert_close(y, ref, dtype, name)


@pytest.mark.parametrize("rank", [8, 16, 32, 64])
@pytest.mark.parametrize("dtype", DTYPES)
def test_add_lora_every_rank(engine, dtype, rank):
    idx = ADD_LORA_CASES["mixed_neg"] + ADD_LORA_CASES["run33"] + list(range(8))
    y, ref = live_case(engine, idx, dtype, 4096, 4096, rank, seed=rank)
    assert_close(y, ref, dtype, f"rank {rank}")


def test_all_negative_leaves_y_untouched(engine):
    idx = [-1] * 8
    g = torch.Generator().manual_seed(0)
    wa = torch.randn(2, 1, 32, 512, generator=g).half().cuda()
    wb = torch.randn(2, 1, 512, 32, generator=g).half().cuda()
    x = torch.randn(8, 512, generator=g).half().cuda()
    y = torch.randn(8, 512, generator=g).half().cuda()
    y0 = y.clone()
    assert engine.build_seg_bounds(torch.tensor(idx).cuda())
    assert engine.add_lora_packed(y, x, wa, wb, 0.5)
    torch.cuda.synchronize()
    assert torch.equal(y, y0)


def test_kernel_matches_reference_golden_numbers(engine, golden):
    """Kernel output vs the numbers of the reference's own Python oracle."""
    for name, idx in ADD_LORA_CASES.items():
        a = add_lora_inputs(idx)
        y = a["y"].cuda()
        assert engine.build_seg_bounds(torch.tensor(idx).cuda())
        assert engine.add_lora_packed(y, a["x"].cuda(), a["wa"].cuda(), a["wb"].cuda(), a["scale"])
        torch.cuda.synchronize()
        dl = (y.float().cpu() - a["y"].float()).double().numpy()
        want = golden[f"add_{name}_cols"]
        rms = float(np.sqrt(np.mean((a["y"].float().numpy()[:, ::8] + want) ** 2)))
        assert np.max(np.abs(dl[:, ::8] - want)) <= 5e-3 * rms + 1e-12, name


@pytest.mark.parametrize("dtype", DTYPES)
def test_segment_reuse_across_layers(engine, dtype):
    """One build_seg_bounds, four layers with different weights
    (test_add_lora_packed.py:116-146)."""
    idx = [0, 0, 0, -1, 1, 1, 1, 1, 1, 2, 2]
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(len(idx), 4096, generator=g) * 0.1).to(dtype)
    assert engine.build_seg_bounds(torch.tensor(idx).cuda())
    for layer in range(4):
        wa = (torch.randn(8, 1, 32, 4096, generator=g) * 0.02).to(dtype)
        wb = (torch.randn(8, 1, 4096, 32, generator=g) * 0.02).to(dtype)
        y = (torch.randn(len(idx), 4096, generator=g) * 0.1).to(dtype)
        yd = y.cuda()
        assert engine.add_lora_packed(yd, x.cuda(), wa.cuda(), wb.cuda(), 0.5)
        torch.cuda.synchronize()
        assert_close(yd, oa.add_lora_grouped(y, x, wa, wb, 0.5, torch.tensor(idx)), dtype, f"layer {layer}")


@pytest.mark.parametrize("dtype", DTYPES)
def test_sliced_output(engine, dtype):
    idx = [0, 0, 1, 1, 1, -1, 2]
    y, ref = live_case(engine, idx, dtype, 1024, 512, 16, y_offset=512, y_cols=1536)
    assert_close(y, ref, dtype, "slice")
    y, ref = live_case(engine, idx, dtype, 1024, 512, 16, y_offset=4, y_cols=1024)  # unaligned offset
    assert_close(y, ref, dtype, "unaligned slice")


@pytest.mark.parametrize("dtype", DTYPES)
def test_live_shrink_then_expand_halves(engine, dtype):
    """wp_add_lora_shrink + wp_add_lora_expand (the halves a tensor-parallel
    row-parallel layer runs around its all-reduce) equal add_lora, with many
    adapters in the stack."""
    from adapterslotsplusplus_b200 import _lib

    T, d, o, r, L = 200, 4096, 1024, 32, 12
    g = torch.Generator().manual_seed(21)
    wa = (torch.randn(L, 1, r, d, generator=g) * 0.02).to(dtype)
    wb = (torch.randn(L, 1, o, r, generator=g) * 0.02).to(dtype)
    x = (torch.randn(T, d, generator=g) * 0.1).to(dtype)
    y = (torch.randn(T, o, generator=g) * 0.1).to(dtype)
    idx = torch.as_tensor(zipf_ids(L, T, seed=5), dtype=torch.int64)
    ref = oa.add_lora_grouped(y, x, wa, wb, 0.75, idx)
    assert engine.build_seg_bounds(idx.cuda())
    lib, h = _lib.load(), engine.handle
    dt = _lib.WP_DTYPE_BF16 if dtype == torch.bfloat16 else _lib.WP_DTYPE_F16
    H = torch.zeros(T, r, dtype=torch.float32, device="cuda")
    xd, wad, wbd, yd = x.cuda(), wa.cuda(), wb.cuda(), y.cuda()
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.wp_add_lora_shrink(h, H.data_ptr(), xd.data_ptr(), wad.data_ptr(), wad.stride(0), L, 0.75, T, d, r,
                                      d, dt, st), h)
    _lib.check(lib.wp_add_lora_expand(h, yd.data_ptr(), H.data_ptr(), wbd.data_ptr(), wbd.stride(0), L, T, o, r, o, 0,
                                      dt, st), h)
    torch.cuda.synchronize()
    assert_close(yd, ref, dtype, "shrink + expand halves")


@pytest.mark.parametrize("nslices,rank,o,dtype", [(3, 32, 4096, torch.bfloat16), (2, 32, 11008, torch.bfloat16),
                                                   (3, 16, 512, torch.float16), (2, 64, 1024, torch.bfloat16),
                                                   (2, 8, 256, torch.float16), (5, 32, 256, torch.bfloat16)])
@pytest.mark.parametrize("pattern", ["zipf", "prefill", "single"])
def test_packed_nslice(engine, nslices, rank, o, dtype, pattern):
    """add_lora_packed_nslice (one launch per three slices) equals one oracle
    add_lora per slice, each into its own column range of y."""
    d = 4096
    if pattern == "zipf":
        idx = zipf_ids(64, 256, seed=1).tolist()
    elif pattern == "prefill":
        idx = [0] * 300 + [-1] * 20 + [1] * 140 + [2] * 5
    else:
        idx = [3]
    T, L = len(idx), 64
    g = torch.Generator().manual_seed(nslices * 100 + rank)
    wa = [(torch.randn(L, 1, rank, d, generator=g) * 0.02).to(dtype) for _ in range(nslices)]
    wb = [(torch.randn(L, 1, o, rank, generator=g) * 0.02).to(dtype) for _ in range(nslices)]
    x = (torch.randn(T, d, generator=g) * 0.1).to(dtype)
    y = (torch.randn(T, nslices * o, generator=g) * 0.1).to(dtype)
    scale = 0.5
    ref = y.float().clone()
    for s in range(nslices):
        ref = oa.add_lora_grouped(ref, x, wa[s], wb[s], scale, torch.tensor(idx), y_offset=s * o)
    yd = y.cuda()
    assert engine.build_seg_bounds(torch.tensor(idx, dtype=torch.int64).cuda())
    assert engine.add_lora_packed_nslice(yd, x.cuda(), [a.cuda() for a in wa], [b.cuda() for b in wb], scale,
                                         [o] * nslices)
    torch.cuda.synchronize()
    for s in range(nslices):
        assert_close(yd[:, s * o:(s + 1) * o], ref[:, s * o:(s + 1) * o], dtype, f"slice {s}")


@pytest.mark.parametrize("d,o", [(1376, 4096), (4096, 1728), (640, 13824 // 8), (11008, 4096), (8, 8)])
def test_shapes_beyond_reference_caps(engine, d, o):
    rng = np.random.default_rng(d + o)
    idx = np.sort(rng.integers(-1, 6, 77)).tolist()
    y, ref = live_case(engine, idx, torch.bfloat16, d, o, 32, seed=d)
    assert_close(y, ref, torch.bfloat16, f"d={d} o={o}")


@pytest.mark.parametrize("T,resident,rank", [(1, 8, 32), (16, 64, 16), (256, 64, 32), (4096, 512, 64), (4096, 8, 8)])
def test_decode_shapes_zipf(engine, T, resident, rank):
    idx = zipf_ids(resident, T, seed=T).tolist()
    y, ref = live_case(engine, idx, torch.bfloat16, 4096, 4096, rank, n_adapters=resident, seed=T)
    assert_close(y, ref, torch.bfloat16, f"T={T} resident={resident}")


def test_prefill_mix_long_segments(engine):
    idx = [0] * 512 + [1] * 512 + [-1] * 100 + [2] * 700 + [3] * 3
    y, ref = live_case(engine, idx, torch.bfloat16, 4096, 4096, 32, n_adapters=4, seed=3)
    assert_close(y, ref, torch.bfloat16, "prefill mix")


def test_unsorted_tokens(engine):
    rng = np.random.default_rng(5)
    idx = rng.integers(-1, 16, 300).tolist()  # many short runs, ids repeat
    y, ref = live_case(engine, idx, torch.float16, 4096, 4096, 32, n_adapters=16, seed=5)
    assert_close(y, ref, torch.float16, "unsorted")


def test_deterministic(engine):
    idx = zipf_ids(64, 256, seed=1).tolist()
    y1, _ = live_case(engine, idx, torch.bfloat16, 4096, 11008, 32, n_adapters=64, seed=9)
    y2, _ = live_case(engine, idx, torch.bfloat16, 4096, 11008, 32, n_adapters=64, seed=9)
    assert torch.equal(y1, y2)


def test_graph_capture_replays_live_table(engine):
    """Capture with one index set, replay after build_seg_bounds with another
    (test_warp_pipe_graph_capture.py:39-129)."""
    dtype = torch.float16
    g = torch.Generator().manual_seed(0)
    wa = (torch.randn(8, 1, 32, 4096, generator=g) * 0.02).to(dtype).cuda()
    wb = (torch.randn(8, 1, 4096, 32, generator=g) * 0.02).to(dtype).cuda()
    x = (torch.randn(16, 4096, generator=g) * 0.1).to(dtype).cuda()
    y_base = (torch.randn(16, 4096, generator=g) * 0.1).to(dtype).cuda()
    idx_buf = torch.zeros(16, dtype=torch.int64, device="cuda")
    y_buf = torch.zeros_like(y_base)
    cap, rep = ADD_LORA_CASES["capture"], ADD_LORA_CASES["replay"]
    idx_buf.copy_(torch.tensor(cap))
    assert engine.build_seg_bounds(idx_buf)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            y_buf.copy_(y_base)
            engine.add_lora_packed(y_buf, x, wa, wb, 0.5)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    y_buf.copy_(y_base)
    with torch.cuda.graph(graph):
        assert engine.add_lora_packed(y_buf, x, wa, wb, 0.5)
    for indices in (cap, rep, cap):
        idx_buf.copy_(torch.tensor(indices))
        assert engine.build_seg_bounds(idx_buf)
        y_buf.copy_(y_base)
        graph.replay()
        torch.cuda.synchronize()
        ref = oa.add_lora_grouped(y_base.cpu(), x.cpu(), wa.cpu(), wb.cpu(), 0.5, torch.tensor(indices))
        assert_close(y_buf, ref, dtype, f"replay {indices[:3]}")


def test_graph_survives_scratch_growth(engine):
    """A graph captured with a small call keeps working after an eager call
    with a larger T and d has grown the kernels' scratch (the outgrown
    buffers stay allocated while graphs may hold their addresses)."""
    dtype = torch.bfloat16
    g = torch.Generator().manual_seed(5)
    small_idx = [0] * 5 + [1] * 11
    wa = (torch.randn(4, 1, 32, 1024, generator=g) * 0.02).to(dtype).cuda()
    wb = (torch.randn(4, 1, 1024, 32, generator=g) * 0.02).to(dtype).cuda()
    x = (torch.randn(16, 1024, generator=g) * 0.1).to(dtype).cuda()
    y_base = (torch.randn(16, 1024, generator=g) * 0.1).to(dtype).cuda()
    y_buf = y_base.clone()
    idx_buf = torch.tensor(small_idx, dtype=torch.int64, device="cuda")
    assert engine.build_seg_bounds(idx_buf)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        engine.add_lora_packed(y_buf, x, wa, wb, 0.5)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        assert engine.add_lora_packed(y_buf, x, wa, wb, 0.5)
    # an eager call with far more tokens and a wider d grows the scratch
    big_idx = sorted(zipf_ids(8, 4096, seed=2).tolist())
    yb, refb = live_case(engine, big_idx, dtype, 11008, 1024, 32, n_adapters=8, seed=6)
    assert_close(yb, refb, dtype, "large eager call")
    del yb
    torch.cuda.synchronize()
    assert engine.build_seg_bounds(idx_buf)
    for _ in range(2):
        y_buf.copy_(y_base)
        graph.replay()
        torch.cuda.synchronize()
        ref = oa.add_lora_grouped(y_base.cpu(), x.cpu(), wa.cpu(), wb.cpu(), 0.5, torch.tensor(small_idx))
        assert_close(y_buf, ref, dtype, "replay after growth")


def test_small_and_empty_calls(engine):
    """One token, one adapter; every token without an adapter; a run of 33."""
    for idx in ([3], [-1] * 40, [2] * 33, [0, -1, 1]):
        for dtype in DTYPES:
            yd, ref = live_case(engine, idx, dtype, 512, 768, 16, n_adapters=4, seed=len(idx))
            assert_close(yd, ref, dtype, f"idx {idx[:4]}")
    assert engine.device_error(clear=True) == 0


# ---- registry path: build_segments + shrink + expand --------------------------

@pytest.mark.parametrize("rank", [8, 16, 32, 64])
def test_registry_rank_variants_vs_golden(engine, golden, rank):
    r = rank_case_inputs(rank)
    K = len(r["table"])
    for i in range(K):
        engine.register_adapter(100 + i, r["A"][i].cuda(), r["B"][i].cuda(), r["alpha"], rank=rank)
    engine.build_segments([100 + i for i in range(K)], [s for _, s, _ in r["table"]] + [r["X"].shape[0]])
    T = r["X"].shape[0]
    H = engine.shrink(r["X"].cuda(), 512, rank, T)
    Y = r["Y"].cuda()
    engine.expand(H, Y, 512, rank)
    torch.cuda.synchronize()
    Hg = golden[f"rank{rank}_H"]
    assert np.max(np.abs(H.cpu().numpy() - Hg)) <= 1e-3 * np.sqrt(np.mean(Hg ** 2))
    dl = (Y.float().cpu() - r["Y"].float()).double().numpy()
    want = golden[f"rank{rank}_Ycols"]
    rms = float(np.sqrt(np.mean((r["Y"].float().numpy()[:, ::8] + want) ** 2)))
    assert np.max(np.abs(dl[:, ::8] - want)) <= 5e-3 * rms
    for i in range(K):
        engine.evict_adapter(100 + i)


@pytest.mark.parametrize("dtype", DTYPES)
def test_config0_both_paths(engine, dtype):
    c = config0_inputs(dtype)
    T = c["X"].shape[0]
    _, Y_ref = oa.apply_segments(c["Y"], c["X"], c["table"], lambda i: c["A"][i], lambda i: c["B"][i],
                                 lambda i: c["alpha"])
    # registry path
    for i in range(8):
        engine.register_adapter(i, c["A"][i].cuda(), c["B"][i].cuda(), c["alpha"], rank=16)
    runs = seg_bounds(c["ids"].numpy())
    engine.build_segments([int(a) for a, _, _ in runs], [int(s) for _, s, _ in runs] + [T])
    Y = c["Y"].cuda()
    H = engine.shrink(c["X"].cuda(), 4096, 16, T)
    engine.expand(H, Y, 4096, 16)
    torch.cuda.synchronize()
    assert_close(Y, Y_ref, dtype, "config0 registry")
    assert engine.read_seg_table("registry") == [tuple(int(v) for v in r) for r in runs]
    # live path on the stacked layout
    y = c["Y"].cuda()
    assert engine.build_seg_bounds(c["ids"].cuda())
    assert engine.read_seg_table("live") == [tuple(int(v) for v in r) for r in runs]
    assert engine.add_lora_packed(y, c["X"].cuda(), c["A"].unsqueeze(1).cuda(), c["B"].unsqueeze(1).cuda(), c["alpha"])
    torch.cuda.synchronize()
    assert_close(y, Y_ref, dtype, "config0 live")
    for i in range(8):
        engine.evict_adapter(i)


@pytest.mark.parametrize("dtype", DTYPES)
def test_registry_stress_random_subsets(engine, dtype):
    """25 iterations, K=32 pool, random subsets and 1..64 tokens per adapter
    (test_concurrent_adapters.py:29-73; segments beyond 32 tokens included)."""
    torch.manual_seed(0)
    rng = random.Random(0)
    K, R, D, O = 32, 32, 4096, 4096
    A = (torch.randn(K, R, D) * 0.02).to(dtype)
    B = (torch.randn(K, O, R) * 0.02).to(dtype)
    Ad, Bd = A.cuda(), B.cuda()
    for i in range(K):
        engine.register_adapter(i, Ad[i], Bd[i], 0.5)
    for it in range(25):
        active = rng.sample(range(K), rng.randint(1, K))
        offs = [0]
        for _ in active:
            offs.append(offs[-1] + rng.randint(1, 64))
        T = offs[-1]
        engine.build_segments(active, offs)
        X = (torch.randn(T, D) * 0.1).to(dtype)
        Y0 = (torch.randn(T, O) * 0.1).to(dtype)
        H = engine.shrink(X.cuda(), D, R, T)
        Y = Y0.cuda()
        engine.expand(H, Y, O, R)
        torch.cuda.synchronize()
        table = [(a, offs[i], offs[i + 1] - offs[i]) for i, a in enumerate(active)]
        H_ref, Y_ref = oa.apply_segments(Y0, X, table, lambda i: A[i], lambda i: B[i], lambda i: 0.5)
        assert_close(H, H_ref, torch.float16, f"iter {it} H")
        assert_close(Y, Y_ref, dtype, f"iter {it} Y")
    for i in range(K):
        engine.evict_adapter(i)


def test_eviction_under_load(engine):
    """40 register/use/evict cycles over 4 reused ids
    (tests/stress/test_eviction_under_load.py:31-65)."""
    rng = random.Random(1)
    for cycle in range(40):
        ids = [0, 1, 2, 3]
        A = [(torch.randn(32, 1024) * 0.02).half().cuda() for _ in ids]
        B = [(torch.randn(1024, 32) * 0.02).half().cuda() for _ in ids]
        for i in ids:
            engine.register_adapter(i, A[i], B[i], 0.5)
        active = rng.sample(ids, rng.randint(1, 4))
        offs = [0]
        for _ in active:
            offs.append(offs[-1] + rng.randint(1, 20))
        T = offs[-1]
        engine.build_segments(active, offs)
        X = (torch.randn(T, 1024) * 0.1).half()
        Y0 = (torch.randn(T, 1024) * 0.1).half()
        Y = Y0.cuda()
        engine.expand(engine.shrink(X.cuda(), 1024, 32, T), Y, 1024, 32)
        for i in ids:
            engine.evict_adapter(i)
        torch.cuda.synchronize()
        table = [(a, offs[k], offs[k + 1] - offs[k]) for k, a in enumerate(active)]
        _, Y_ref = oa.apply_segments(Y0, X, table, lambda i: A[i].cpu(), lambda i: B[i].cpu(), lambda i: 0.5)
        assert_close(Y, Y_ref, torch.float16, f"cycle {cycle}")


def test_registry_errors(engine):
    with pytest.raises(RuntimeError):
        engine.build_segments([12345], [0, 4])  # unknown id
    with pytest.raises(RuntimeError):
        engine.build_segments([0, 1], [0, 4])  # K+1 mismatch
    A = torch.zeros(32, 256, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):
        engine.register_adapter(1, A, torch.zeros(256, 32, dtype=torch.float32, device="cuda"), 1.0)


@pytest.mark.skipif(not REF_LIB.exists(), reason="oracle/_ref/libwpref.so not built")
def test_live_path_matches_reference_kernels_fp16(engine):
    """fp16 rank-32 live path: ours vs the reference's own DSAK kernels on the
    same inputs, both against the fp32 oracle (the reference rounds H to
    fp16, so it is checked with the reference suite's 0.05 bound)."""
    ref = ctypes.CDLL(str(REF_LIB))
    out = (ctypes.c_int32 * 768)()
    num = ctypes.c_int32()
    for name in ("mixed_neg", "run33", "many_short", "replay"):
        idx = ADD_LORA_CASES[name]
        g = torch.Generator().manual_seed(3)
        wa = (torch.randn(8, 1, 32, 4096, generator=g) * 0.02).half()
        wb = (torch.randn(8, 1, 4096, 32, generator=g) * 0.02).half()
        x = (torch.randn(len(idx), 4096, generator=g) * 0.1).half()
        y0 = (torch.randn(len(idx), 4096, generator=g) * 0.1).half()
        y_ref = oa.add_lora_grouped(y0, x, wa, wb, 0.5, torch.tensor(idx))
        xd, wad, wbd, di = x.cuda(), wa.cuda(), wb.cuda(), torch.tensor(idx).cuda()
        y_theirs = y0.cuda()
        torch.cuda.synchronize()
        assert ref.ref_seg_bounds(ctypes.c_void_p(di.data_ptr()), len(idx), out, ctypes.byref(num)) == 0
        assert ref.ref_add_lora_r32(ctypes.c_void_p(y_theirs.data_ptr()), ctypes.c_void_p(xd.data_ptr()),
                                    ctypes.c_void_p(wad.data_ptr()), ctypes.c_int64(wad.stride(0)),
                                    ctypes.c_void_p(wbd.data_ptr()), ctypes.c_int64(wbd.stride(0)),
                                    ctypes.c_float(0.5), 4096, 4096, None) == 0
        y_ours = y0.cuda()
        assert engine.build_seg_bounds(di)
        assert engine.add_lora_packed(y_ours, xd, wad, wbd, 0.5)
        torch.cuda.synchronize()
        err_theirs = float((y_theirs.float().cpu() - y_ref).abs().max())
        assert err_theirs < 0.05, name
        assert_close(y_ours, y_ref, torch.float16, name)
        assert float((y_ours.float().cpu() - y_ref).abs().max()) <= err_theirs + 1e-3

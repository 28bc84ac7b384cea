"""Draft-step integration: a small decoder whose LoRA projections run the
grouped apply over an AdapterPool (adapterslotsplusplus_b200/draft.py),
against the same decoder with a plain-torch per-token LoRA, eager and
replayed from a CUDA graph (the reference captures its draft step the same
way, benchmarks/kernel/bench_graph_capture.py:47-103)."""

import pytest
import torch

from adapterslotsplusplus_b200 import AdapterPool, WarpPipeConfig, WarpPipeEngine
from adapterslotsplusplus_b200.draft import DraftDecoder

pytestmark = pytest.mark.gpu


def _setup(layers=2, tenants=4, seqs=8, lookahead=4, rank=16):
    dev = torch.device("cuda", 0)
    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=4096))
    model = DraftDecoder(layers=layers, hidden=256, heads=4, inter=512, vocab=0, device=dev)
    dims = model.dims()
    pool = AdapterPool(eng, num_slots=tenants + 2, dims=dims, rank=rank, max_adapters=64)
    g = torch.Generator().manual_seed(1)
    A = [[] for _ in dims]
    B = [[] for _ in dims]
    ids_all = [3, 7, 11, 20][:tenants]
    for t in range(32):
        w = [((torch.randn(rank, d, generator=g) * 0.05).bfloat16(), (torch.randn(o, rank, generator=g) * 0.05).bfloat16())
             for d, o in dims]
        pool.register_host(t, pool.pack(w))
        for p, (a, b) in enumerate(w):
            A[p].append(a)
            B[p].append(b)
    torch_lora = {"A": [torch.stack(a).to(dev) for a in A], "B": [torch.stack(b).to(dev) for b in B]}
    ids = torch.tensor(sorted(ids_all * (seqs * lookahead)), dtype=torch.int64, device=dev)
    torch_lora["ids"] = ids
    x = (torch.randn(ids.numel(), 256, generator=g) * 0.5).bfloat16().to(dev)
    return eng, model, pool, torch_lora, ids, x, lookahead


# Both forwards are bf16 end to end and round every projection output once
# each, independently: after two layers their difference is rounding noise
# carried through the norms and the attention (about one bf16 ulp per layer
# at the largest activations), so the draft-level bound is wider than the
# per-call 2e-2 that tests/test_gpu_apply.py holds every kernel call to.
DRAFT_TOL = 6e-2


def _close(a, b, tol=DRAFT_TOL):
    a, b = a.float(), b.float()
    rms = float(b.pow(2).mean().sqrt())
    return float((a - b).abs().max()) <= tol * rms, float((a - b).abs().max()) / rms


def test_draft_step_pool_matches_torch_lora():
    eng, model, pool, tl, ids, x, la = _setup()
    pool.prepare(ids.tolist())
    assert pool.build_seg_bounds(ids)
    out_pool = model.forward(x, la, lora="pool", pool=pool, scale=2.0)
    out_torch = model.forward(x, la, lora="torch", torch_lora=tl, scale=2.0)
    out_base = model.forward(x, la, lora="none")
    torch.cuda.synchronize()
    ok, rel = _close(out_pool, out_torch)
    assert ok, rel
    # the LoRA changes the output (the comparison is not vacuous)
    assert not _close(out_base, out_torch, 1e-3)[0]
    assert eng.device_error(clear=True) == 0


def test_draft_step_graph_replay_with_new_tenants():
    eng, model, pool, tl, ids, x, la = _setup()
    pool.prepare(ids.tolist())
    pool.build_seg_bounds(ids)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        model.forward(x, la, lora="pool", pool=pool, scale=2.0)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = model.forward(x, la, lora="pool", pool=pool, scale=2.0)
    for tenants in ([3, 7, 11, 20], [1, 2, 30, 31], [5, 6, 7, 8]):
        new_ids = torch.tensor(sorted(tenants * (ids.numel() // 4)), dtype=torch.int64, device="cuda")
        pool.prepare(new_ids.tolist())
        pool.build_seg_bounds(new_ids)
        graph.replay()
        torch.cuda.synchronize()
        tl["ids"] = new_ids
        ref = model.forward(x, la, lora="torch", torch_lora=tl, scale=2.0)
        ok, rel = _close(out, ref)
        assert ok, (tenants, rel)

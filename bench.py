"""Benchmark: grouped multi-LoRA apply per decode step.

Workload: a Llama-2-7B-shaped stack, 32 layers x 7
LoRA projections (q,k,v,o: 4096->4096; gate,up: 4096->11008; down:
11008->4096), rank 32, bf16, 64 resident adapters, 256 decode tokens, adapter
popularity Zipf(1.1) with seed 1 (stable-sorted ids). One build_seg_bounds
per step, then the 224 add_lora calls of the step replayed from one CUDA
graph. Weights are random (seeded), activations synthetic.

Metric: LoRA apply us per decode step (lower is better) and the HBM GB/s it
implies against the measured peak. One JSON line on rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-sweep]

With N > 1 (launched under torch.distributed.run, one rank per GPU) the same
step runs tensor-parallel over the N GPUs the way vLLM shards LoRA layers:
column-parallel projections (q, k, v, gate, up) expand their own out_features
slice; row-parallel ones (o, down) shrink their d_in slice and add their
share into the base layer's partial output, which the base model's
all-reduce completes (--row-mode partial, the default; "fused" sums the
ranks' [T, r] partials over NVLink peer memory inside the apply launch,
"nccl" all-reduces them with NCCL). Strong scaling; the time is the max over
ranks. The line carries `tp_parity` (layer 0's q, o and down against the
unsharded single-GPU result on the same box) and per-kind launch times.

  python bench.py --config3 [--gpus N]

times BASELINE config 3 (13B shapes, rank 64, 512 tokens, 128 resident),
tensor-parallel over the N GPUs, and prints its own JSON line.

  python bench.py --profile-case q|gate|down [--launches 12] [--kernel auto|cluster|split|tc]

runs a few launches of one projection of the step and exits (a small case
for profilers).

--impl reference times the reference's CPU implementation of the path (its
torch per-segment fp32 math, tests/correctness/reference_bgmv.py:4-18,
restated in oracle/apply.py) on the host cores, on a bounded sample of the
same workload (a few layers, extrapolated to 32). Its `reference_gpu` key
times the reference's own CUDA kernels (built from its sources into
oracle/_ref) on the same step in fp16; our line's `fp16_step` is the same
step through this library.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from tests.golden.cases import zipf_ids  # noqa: E402  (seeded Zipf id generator)

LAYERS = 32
HIDDEN = 4096
INTER = 11008
RANK = 32
TOKENS = 256
RESIDENT = 64
SEED = 1
# (name, d_in, d_out, input activation, tensor-parallel kind)
PROJS = [("q", HIDDEN, HIDDEN, "h", "col"), ("k", HIDDEN, HIDDEN, "h", "col"), ("v", HIDDEN, HIDDEN, "h", "col"),
         ("o", HIDDEN, HIDDEN, "attn", "row"), ("gate", HIDDEN, INTER, "h", "col"), ("up", HIDDEN, INTER, "h", "col"),
         ("down", INTER, HIDDEN, "inter", "row")]
WORKLOAD = "llama2-7b decode step: 32 layers x 7 LoRA projections, rank 32, bf16, 64 resident, 256 tokens, Zipf(1.1) seed 1"
METRIC = "LoRA apply us/decode-step (HBM GB/s vs peak), 7B x 32 layers, r32, 64 resident, T=256"


def algorithmic_bytes(U: int, T: int, d: int, o: int, r: int, elt: int = 2) -> tuple[int, int]:
    """(shrink bytes, expand bytes) of one projection call: each active
    adapter's A and B once, x read, y read and written. H stays on chip (the
    fused kernel reduces it in distributed shared memory)."""
    shrink = U * d * r * elt + T * d * elt
    expand = U * o * r * elt + 2 * T * o * elt
    return shrink, expand


def step_bytes(U: int, T: int, r: int = RANK, world: int = 1, exchange: bool = False) -> tuple[int, int]:
    """Algorithmic bytes of one step on one rank of a tensor-parallel group of
    `world` (world = 1: the whole model). Column-parallel projections split
    B and y along out_features; row-parallel ones split x and A along d_in
    (with `exchange`, plus the [T, r] fp32 partials, counted as read + write)."""
    s = e = 0
    for _, d, o, _, kind in PROJS:
        if world > 1 and kind == "col":
            o = o // world
        elif world > 1:
            d = d // world
        bs, be = algorithmic_bytes(U, T, d, o, r)
        s += bs
        e += be
        if world > 1 and kind == "row" and exchange:
            e += 2 * T * r * 4
    return s * LAYERS, e * LAYERS


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {}


class ClockSampler:
    """SM clocks and throttle reasons of GPU `index`, sampled every ~5 ms
    through NVML (read-only queries) while the `with` block runs: the timed
    region of a step is tens of ms, shorter than nvidia-smi's start-up.
    Falls back to `nvidia-smi -lms 50` when NVML is not importable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvml.h)
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.nvml = None
        self.stop = threading.Event()
        self.samples: list[tuple[float, int]] = []  # (SM MHz, reason bits)
        self.max_mhz = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self.nvml = (pynvml, h)
            self.samples.append(self._nvml_sample())
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _nvml_sample(self):
        pynvml, h = self.nvml
        mhz = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
        try:
            bits = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
        except AttributeError:
            bits = int(pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h))
        return mhz, bits

    def _poll(self):
        while not self.stop.wait(0.005):
            try:
                self.samples.append(self._nvml_sample())
            except Exception:
                return

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.nvml is not None:
            self.stop.set()
            self.thread.join(timeout=1)
            try:
                self.samples.append(self._nvml_sample())
                self.nvml[0].nvmlShutdown()
            except Exception:
                pass
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], self.max_mhz, set()
        for mhz, bits in self.samples:
            sm.append(mhz)
            for n, b in self.REASONS.items():
                if bits & b:
                    reasons.add(n)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvml" if self.nvml is not None else "nvidia-smi"}


# ---------------------------------------------------------------------------
# workload


def make_ids(resident: int, T: int = TOKENS, seed: int = SEED) -> np.ndarray:
    return zipf_ids(resident, T, seed=seed)


class Stack:
    """Device-resident stacked LoRA weights + activations of the 7B stack, as
    rank `rank` of a tensor-parallel group of `world` holds them."""

    def __init__(self, device, resident, layers=LAYERS, T=TOKENS, dtype=torch.bfloat16, seed=0, rank=0, world=1):
        g = torch.Generator(device=device).manual_seed(seed + 1000 * rank)
        self.layers = []
        for _ in range(layers):
            L = {}
            for name, d, o, _, kind in PROJS:
                dl, ol = d, o
                if world > 1 and kind == "col":
                    ol = o // world
                elif world > 1:
                    dl = d // world
                wa = torch.randn(resident, 1, RANK, dl, device=device, dtype=dtype, generator=g) * 0.02
                wb = torch.randn(resident, 1, ol, RANK, device=device, dtype=dtype, generator=g) * 0.02
                L[name] = (wa, wb, torch.zeros(T, ol, device=device, dtype=dtype))
            dh = HIDDEN // world if world > 1 else HIDDEN
            di = INTER // world if world > 1 else INTER
            L["x"] = {"h": torch.randn(T, HIDDEN, device=device, dtype=dtype, generator=g) * 0.1,
                      "attn": torch.randn(T, dh, device=device, dtype=dtype, generator=g) * 0.1,
                      "inter": torch.randn(T, di, device=device, dtype=dtype, generator=g) * 0.1}
            self.layers.append(L)

    def calls(self):
        for L in self.layers:
            for name, d, o, src, kind in PROJS:
                wa, wb, y = L[name]
                yield kind, y, L["x"][src], wa, wb


def capture(fn, warm=2):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warm):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def time_graph(g, pre, iters):
    """Device time of `iters` replays (pre() runs before each, eagerly)."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(iters):
        if pre is not None:
            pre()
        g.replay()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters  # ms


def tp_parity(eng, tpa, device, rank, world, scale, idx_dev):
    """Tensor-parallel results of layer 0's q (column-parallel), o and down
    (row-parallel) against an fp32 torch computation of the unsharded call on
    the same GPU, on identical inputs (every rank draws the full weights from
    one seed and keeps its shard). Row-parallel partial outputs (bf16, as the
    kernel wrote them) are summed in fp32 with an all-reduce, as the base
    layer's all-reduce would; the rounding of that sum back to bf16 is the
    base model's, not the LoRA kernel's, and is left out. Returns, on every
    rank, max-abs error / RMS per projection and whether all ranks hold
    bit-identical full outputs."""
    import torch.distributed as dist

    from adapterslotsplusplus_b200.tp import shard_column, shard_row, shard_row_input

    g = torch.Generator(device=device).manual_seed(77)
    out = {}
    same = True
    for name, d, o, _, kind in [p for p in PROJS if p[0] in ("q", "o", "down")]:
        wa = torch.randn(RESIDENT, 1, RANK, d, device=device, dtype=torch.bfloat16, generator=g) * 0.02
        wb = torch.randn(RESIDENT, 1, o, RANK, device=device, dtype=torch.bfloat16, generator=g) * 0.02
        x = torch.randn(TOKENS, d, device=device, dtype=torch.bfloat16, generator=g) * 0.1
        y0 = torch.randn(TOKENS, o, device=device, dtype=torch.bfloat16, generator=g) * 0.1
        # fp32 reference of the unsharded call on this GPU (plain torch)
        ids = idx_dev.long()
        h32 = torch.einsum("td,trd->tr", x.float(), wa[ids, 0].float()) * scale
        ref = y0.float() + torch.einsum("tr,tor->to", h32, wb[ids, 0].float())
        del h32
        if kind == "col":
            a, b = rank * (o // world), (rank + 1) * (o // world)
            ys = y0[:, a:b].contiguous()
            assert tpa.column_parallel(ys, x, wa, shard_column(wb, rank, world), scale)
            parts = [torch.empty_like(ys) for _ in range(world)]
            dist.all_gather(parts, ys)
            full = torch.cat(parts, dim=1)
        else:
            if tpa.row_mode == "partial":
                # the base layer's bias-like share goes to rank 0 only
                yp = y0.clone() if rank == 0 else torch.zeros_like(y0)
                assert tpa.row_parallel(yp, shard_row_input(x, rank, world), shard_row(wa, rank, world), wb, scale)
                ypf = yp.float()
                dist.all_reduce(ypf)
                full = ypf
            else:
                full = y0.clone()
                assert tpa.row_parallel(full, shard_row_input(x, rank, world), shard_row(wa, rank, world), wb, scale)
        torch.cuda.synchronize()
        rms = float(ref.pow(2).mean().sqrt())
        err = float((full.float() - ref).abs().max()) / rms
        # bit-identity across ranks: compare every rank's output with rank 0's
        r0 = full.clone()
        dist.broadcast(r0, src=0)
        diff = torch.tensor([int(not torch.equal(r0, full))], device=device)
        dist.all_reduce(diff)
        same = same and int(diff.item()) == 0
        out[name] = round(err, 6)
    return {"max_abs_err_over_rms": out, "bound": 2e-2, "ok": all(v <= 2e-2 for v in out.values()) and same,
            "ranks_bit_identical": same, "row_mode": tpa.row_mode,
            "against": "fp32 torch result of the unsharded call on the same inputs and GPU"}


def run_ours(args, rank, world, local_rank):
    from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    # prefetch_weights + prefetch_inputs: the serving contract (adapter
    # weights are static during a step, and the kernel right before a LoRA
    # call never writes its x) lets each apply launch stream weights and x,
    # and run its shrink, while the previous launch finishes. The serving
    # hooks (punica_wrapper.py, vllm_punica.py) build their engine with the
    # same settings; the step without them is reported as `strict_order`,
    # with weights only as `weights_prefetch_only`.
    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=True, prefetch_inputs=True), device=device)
    plan = eng.apply_plan(torch.bfloat16, RANK)
    scale = 16.0 / RANK

    ids = make_ids(RESIDENT)
    U = int(np.unique(ids).size)
    idx_dev = torch.as_tensor(ids, device=device)
    stack = Stack(device, RESIDENT, rank=rank, world=world)
    calls = list(stack.calls())
    tpa = None
    parity = None
    if world > 1:
        # tensor parallel over the N GPUs (vLLM's sharding): column-parallel
        # projections expand their own output columns; row-parallel ones
        # add their d_in slice's share into the partial output (row_mode
        # "partial"), or exchange the partial H ("fused" / "nccl")
        from adapterslotsplusplus_b200.tp import TensorParallelApply

        tpa = TensorParallelApply(eng, row_mode=args.row_mode)
        eng.build_seg_bounds(idx_dev)
        parity = tp_parity(eng, tpa, device, rank, world, scale, idx_dev)

    def run(kinds=("col", "row")):
        def f():
            for kind, y, x, wa, wb in calls:
                if kind not in kinds:
                    continue
                if tpa is None:
                    eng.add_lora_packed(y, x, wa, wb, scale)
                elif kind == "col":
                    tpa.column_parallel(y, x, wa, wb, scale)
                else:
                    tpa.row_parallel(y, x, wa, wb, scale)
        return f

    seg = lambda: eng.build_seg_bounds(idx_dev)  # noqa: E731
    seg()
    g_full = capture(run())

    for _ in range(args.warmup):
        seg()
        g_full.replay()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()

    with ClockSampler(local_rank) as clk:
        ms = time_graph(g_full, seg, args.steps)  # the step: segmenter + 224 apply launches
        ms_apply = time_graph(g_full, None, args.steps)  # the 224 apply launches alone
    torch.cuda.synchronize()
    per_kind = {}
    if world > 1 or args.per_kind:
        # column- and row-parallel launches timed apart (each kind's calls of
        # the step in a graph of their own)
        for kind in ("col", "row"):
            gk = capture(run((kind,)), warm=1)
            n = sum(1 for c in calls if c[0] == kind)
            per_kind[kind] = time_graph(gk, None, args.steps) * 1e3 / n
            del gk
    outside_ms = ms - ms_apply  # this rank's time outside the apply graph
    if world > 1:
        t = torch.tensor([ms, ms_apply, per_kind.get("col", 0.0), per_kind.get("row", 0.0), outside_ms],
                         device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, ms_apply, per_kind["col"], per_kind["row"], outside_ms = t.tolist()

    # e2e through the public API: token ids from pinned host memory, the step,
    # and a read back of one output row, all on the stream, every step.
    ids_host = torch.as_tensor(ids).pin_memory()
    out_host = torch.empty(calls[-1][1].size(-1), dtype=torch.bfloat16).pin_memory()
    y_last = calls[-1][1]

    def e2e_step():
        idx_dev.copy_(ids_host, non_blocking=True)
        eng.build_seg_bounds(idx_dev)
        g_full.replay()
        out_host.copy_(y_last[0], non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(args.steps):
        e2e_step()
    en.record()
    torch.cuda.synchronize()
    e2e_ms = max(st.elapsed_time(en), (time.perf_counter() - t0) * 1e3) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())

    exchange = tpa is not None and tpa.row_mode != "partial"
    shr_b, exp_b = step_bytes(U, TOKENS, world=world, exchange=exchange)
    total_b = (shr_b + exp_b) * world  # whole job: every rank's share of the step
    peaks = measured_peaks()
    hbm = peaks.get("hbm_gbs")
    peak_src = "measured" if hbm else "fallback"
    hbm = hbm or 6650.0
    # dominant kernel: the apply kernel (one launch per call; the segmenter is
    # one launch per step). Per launch: the mean over the calls of the step on
    # one rank.
    dom = eng.last_apply_kernel() or "apply_kernel"
    launches_per_step = LAYERS * len(PROJS)
    if tpa is not None and tpa.row_mode == "nccl":
        apply_launches = launches_per_step + 2 * LAYERS * sum(1 for p in PROJS if p[4] == "row")
    else:
        apply_launches = launches_per_step
    per_launch_ms = ms_apply / launches_per_step
    per_launch_b = total_b / world / launches_per_step
    achieved = per_launch_b / (per_launch_ms * 1e-3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists() and world == 1:
        try:
            traffic = json.loads(tf.read_text()).get(dom)
        except Exception:
            traffic = None
    if tpa is None:
        tp_desc = "single GPU"
    elif tpa.row_mode == "partial":
        tp_desc = ("tensor-parallel: column-parallel projections split B and y; row-parallel ones add their "
                   "d_in slice's share into the base layer's partial output (vLLM RowParallelLinearWithLoRA), "
                   "completed by the base model's all-reduce, which is not LoRA work and is not timed")
    else:
        tp_desc = f"tensor-parallel, row-parallel partial H summed over the ranks ({tpa.row_mode})"

    result = {
        "metric": METRIC,
        "value": round(ms * 1e3, 2),
        "unit": "us/step",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random weights and activations, Zipf(1.1) routing)",
        "config": {"workload": WORKLOAD, "layers": LAYERS, "projections": len(PROJS), "rank": RANK,
                   "resident_adapters": RESIDENT, "active_adapters": U, "tokens": TOKENS,
                   "parallelism": f"tp{world}" if world > 1 else "single", "tp": tp_desc,
                   "l2": "inputs exceed L2 (10.2 GB of adapter weights per step), no flush needed"},
        "step_gbs": round(total_b / (ms * 1e-3) / 1e9, 1),
        "step_frac_of_hbm": round(total_b / (ms * 1e-3) / 1e9 / hbm / world, 4),
        "step_bytes": total_b,
        "kernels_ms_per_step": {dom: round(ms_apply, 4), "segmenter_and_gaps": round(ms - ms_apply, 4)},
        "apply_plan": {"cluster": plan[0], "ctas": plan[1]},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm,
                     "peak_source": peak_src, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "traffic": traffic, "algorithmic_bytes_per_launch": int(per_launch_b),
                     "launch_us": round(per_launch_ms * 1e3, 3)},
        "e2e": {"value": round(e2e_ms * 1e3, 2), "unit": "us/step", "h2d_bytes_per_step": int(ids.nbytes),
                "d2h_bytes_per_step": int(out_host.numel() * 2),
                "path": "WarpPipeEngine.build_seg_bounds + graph of the step's apply calls; per step the token "
                        "ids come from pinned host memory and one output row goes back. The activations and "
                        "outputs stay on the device, as they do for a LoRA hook inside a served model (" + tp_desc + ")"},
        "gpu_launches": args.steps * (1 + apply_launches),
        "clocks": clk.summary(),
    }
    if per_kind:
        result["per_kind_us_per_launch"] = {k: round(v, 3) for k, v in per_kind.items()}
        result["per_kind_us_per_launch"]["outside_graph_us_per_step"] = round(outside_ms * 1e3, 2)
    if parity is not None:
        result["tp_parity"] = parity
    del g_full, stack, calls
    if tpa is not None:
        tpa.close()
    torch.cuda.empty_cache()
    return eng, result


def fp16_step(device, steps):
    """The headline step in fp16 (the reference kernels' only type), for the
    side-by-side with the reference's own GPU kernels that the reference arm
    (`--impl reference`, key `reference_gpu`) times on the same workload."""
    from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine

    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=True, prefetch_inputs=True), device=device)
    idx = torch.as_tensor(make_ids(RESIDENT), device=device)
    stack = Stack(device, RESIDENT, dtype=torch.float16)
    calls = list(stack.calls())

    def step():
        for _, y, x, wa, wb in calls:
            eng.add_lora_packed(y, x, wa, wb, 16.0 / RANK)

    eng.build_seg_bounds(idx)
    g = capture(step, warm=1)
    for _ in range(3):
        g.replay()
    ms = time_graph(g, lambda: eng.build_seg_bounds(idx), steps)
    del g, stack, calls, eng
    torch.cuda.empty_cache()
    return {"us_per_step": round(ms * 1e3, 2), "dtype": "fp16"}


def strict_order(device, steps, prefetch_weights=False):
    """The step without the serving contract's prefetch: prefetch_weights off
    (strict stream order: no load of a launch starts before the previous
    launch has finished), or weights only (x and the shrink wait for the
    previous launch)."""
    from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine

    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=prefetch_weights), device=device)
    ids = make_ids(RESIDENT)
    idx = torch.as_tensor(ids, device=device)
    stack = Stack(device, RESIDENT)
    calls = list(stack.calls())
    scale = 16.0 / RANK

    def step():
        for _, y, x, wa, wb in calls:
            eng.add_lora_packed(y, x, wa, wb, scale)

    eng.build_seg_bounds(idx)
    g = capture(step, warm=1)
    for _ in range(3):
        g.replay()
    ms = time_graph(g, lambda: eng.build_seg_bounds(idx), steps)
    del g, stack, calls, eng
    torch.cuda.empty_cache()
    return {"us_per_step": round(ms * 1e3, 2), "prefetch_weights": prefetch_weights, "prefetch_inputs": False}


def fused_slices(eng, device, steps):
    """The same step with the projections that share an input fused the way
    vLLM packs them (q/k/v and gate/up through add_lora_packed_nslice): 4
    launches per layer instead of 7, identical bytes and results."""
    stack = Stack(device, RESIDENT)
    scale = 16.0 / RANK
    yqkv = torch.zeros(TOKENS, 3 * HIDDEN, device=device, dtype=torch.bfloat16)
    ygu = torch.zeros(TOKENS, 2 * INTER, device=device, dtype=torch.bfloat16)

    def step():
        for L in stack.layers:
            xs = L["x"]
            eng.add_lora_packed_nslice(yqkv, xs["h"], [L[n][0] for n in "qkv"], [L[n][1] for n in "qkv"], scale,
                                       [HIDDEN] * 3)
            wa, wb, y = L["o"]
            eng.add_lora_packed(y, xs["attn"], wa, wb, scale)
            eng.add_lora_packed_nslice(ygu, xs["h"], [L["gate"][0], L["up"][0]], [L["gate"][1], L["up"][1]],
                                       scale, [INTER] * 2)
            wa, wb, y = L["down"]
            eng.add_lora_packed(y, xs["inter"], wa, wb, scale)

    eng.build_seg_bounds(torch.as_tensor(make_ids(RESIDENT), device=device))
    g = capture(step)
    for _ in range(3):
        g.replay()
    ms = time_graph(g, None, steps)
    U = int(np.unique(make_ids(RESIDENT)).size)
    shr_b, exp_b = step_bytes(U, TOKENS)
    del g, stack
    torch.cuda.empty_cache()
    return {"apply_us_per_step": round(ms * 1e3, 2), "launches_per_step": 4 * LAYERS,
            "step_gbs": round((shr_b + exp_b) / (ms * 1e-3) / 1e9, 1),
            "path": "add_lora_packed_nslice for q/k/v and gate/up, add_lora_packed for o and down"}


def sweep_resident(eng, device, counts, steps):
    """Flatness: us/step and roofline-normalised time vs resident adapters."""
    out = []
    scale = 16.0 / RANK
    hbm = measured_peaks().get("hbm_gbs", 6650.0)
    for resident in counts:
        ids = make_ids(resident)
        U = int(np.unique(ids).size)
        idx = torch.as_tensor(ids, device=device)
        stack = Stack(device, resident, seed=resident)
        calls = list(stack.calls())

        def step():
            for _, y, x, wa, wb in calls:
                eng.add_lora_packed(y, x, wa, wb, scale)

        eng.build_seg_bounds(idx)
        g = capture(step, warm=1)
        for _ in range(2):
            g.replay()
        ms = time_graph(g, lambda: eng.build_seg_bounds(idx), steps)
        sb, eb = step_bytes(U, TOKENS)
        roof_ms = (sb + eb) / (hbm * 1e9) * 1e3
        out.append({"resident": resident, "active": U, "us_per_step": round(ms * 1e3, 1),
                    "gb_per_step": round((sb + eb) / 1e9, 3), "roofline_us": round(roof_ms * 1e3, 1),
                    "time_over_roofline": round(ms / roof_ms, 3)})
        del g, stack, calls
        torch.cuda.empty_cache()
    if out:
        base = out[0]
        for r in out:
            r["raw_growth"] = round(r["us_per_step"] / base["us_per_step"], 3)
            r["normalised_growth"] = round(r["time_over_roofline"] / base["time_over_roofline"], 3)
    return out


# ---------------------------------------------------------------------------
# CPU legs (oracle port of the reference's torch per-segment path)


def cpu_reference_layers(n_layers: int, resident: int = RESIDENT, threads: int | None = None, reps: int = 1):
    """Time the reference's CPU math on n_layers layers of the workload.
    Returns (seconds per layer, threads used)."""
    from oracle.apply import reference_bgmv_expand, reference_bgmv_shrink
    from oracle.seg import seg_bounds

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    ids = make_ids(resident)
    table = seg_bounds(ids)
    g = torch.Generator().manual_seed(0)
    weights = []
    for _ in range(n_layers):
        L = {}
        for name, d, o, *_ in PROJS:
            L[name] = ((torch.randn(resident, RANK, d, generator=g) * 0.02).bfloat16(),
                       (torch.randn(resident, o, RANK, generator=g) * 0.02).bfloat16(),
                       (torch.randn(TOKENS, d, generator=g) * 0.1).bfloat16(),
                       torch.zeros(TOKENS, o, dtype=torch.bfloat16))
        weights.append(L)
    scale = 16.0 / RANK

    def one_layer(L):
        for name, d, o, *_ in PROJS:
            wa, wb, x, y = L[name]
            yf = y.float()
            for aid, s, n in table:
                h = reference_bgmv_shrink(x[s:s + n], wa[aid], scale)
                yf[s:s + n] = reference_bgmv_expand(h, wb[aid], yf[s:s + n])
            y.copy_(yf)

    one_layer(weights[0])  # warm-up
    t0 = time.perf_counter()
    for _ in range(reps):
        for L in weights:
            one_layer(L)
    dt = (time.perf_counter() - t0) / (reps * n_layers)
    return dt, threads


def reference_gpu(steps: int, warmup: int):
    """The reference's own CUDA kernels (warp_pipe_r32.cu, built from the
    reference's sources into oracle/_ref/libwpref.so by oracle/build_ref.sh)
    on the same decode step in fp16, their only type: one
    build_seg_bounds_kernel, then per call bgmv_shrink_dsak + bgmv_expand_dsak
    (WarpPipeExtension::add_lora_packed, warp_pipe_bindings.cpp:195-234),
    the 224 calls replayed from one CUDA graph. Config 1 fits every limit of
    those kernels (T = 256, d and o multiples of 256, rank 32)."""
    import ctypes

    so = ROOT / "oracle" / "_ref" / "libwpref.so"
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    if not so.exists():
        return {"unavailable": "oracle/_ref/libwpref.so was not built (reference sources absent at build time)"}
    lib = ctypes.CDLL(str(so))
    lib.ref_seg_bounds.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    lib.ref_add_lora_r32.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                                             ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    ids = make_ids(RESIDENT)
    idx = torch.as_tensor(ids, device=device, dtype=torch.int64)
    table = (ctypes.c_int32 * (3 * 256))()
    num = ctypes.c_int32()
    if lib.ref_seg_bounds(idx.data_ptr(), len(ids), table, ctypes.byref(num)) != 0:
        return {"unavailable": "reference build_seg_bounds refused the table"}
    stack = Stack(device, RESIDENT, dtype=torch.float16)
    calls = list(stack.calls())
    scale = 16.0 / RANK

    def step():
        st = torch.cuda.current_stream().cuda_stream
        for _, y, x, wa, wb in calls:
            rc = lib.ref_add_lora_r32(y.data_ptr(), x.data_ptr(), wa.data_ptr(), wa.stride(0), wb.data_ptr(),
                                      wb.stride(0), scale, x.size(-1), y.size(-1), st)
            if rc != 0:
                raise RuntimeError(f"ref_add_lora_r32 failed ({rc})")

    step()  # first call allocates the reference's buffers (outside capture)
    torch.cuda.synchronize()
    g = capture(step, warm=1)
    for _ in range(max(3, warmup)):
        g.replay()
    ms = time_graph(g, None, steps)
    U = int(np.unique(ids).size)
    sb, eb = step_bytes(U, TOKENS)
    del g, stack, calls
    torch.cuda.empty_cache()
    return {"us_per_step": round(ms * 1e3, 2), "dtype": "fp16", "segments": int(num.value),
            "step_gbs": round((sb + eb) / (ms * 1e-3) / 1e9, 1),
            "kernels": "reference build_seg_bounds once (outside the graph) + 224 x (bgmv_shrink_dsak_r32, "
                       "bgmv_expand_dsak_r32) in a CUDA graph",
            "compare_with": "our line's fp16_step.us_per_step (same workload, fp16)"}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    for _ in range(args.warmup):
        cpu_reference_layers(1, reps=1)
    per_layer = []
    threads = os.cpu_count() or 1
    for _ in range(args.steps):
        dt, threads = cpu_reference_layers(1, reps=1)
        per_layer.append(dt)
    us = float(np.median(per_layer)) * LAYERS * 1e6
    sample = f"1 of {LAYERS} layers (7 projections) per step, extrapolated x{LAYERS}"
    try:
        gpu = reference_gpu(args.steps, args.warmup)
    except Exception as exc:  # reported, never fatal to the CPU arm
        gpu = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
    return {
        "metric": METRIC, "value": round(us, 1), "unit": "us/step", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(us / 1e3, 3), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD, "parallelism": "cpu"},
        "cpu_baseline": {"value": round(us, 1), "unit": "us/step", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(us, 1), "unit": "us/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_gpu": gpu,
    }


def prefill_mix(device, iters=10):
    """BASELINE config 2's prefill mix on one 4096 -> 4096 projection: 4096
    tokens in 8 contiguous 512-token runs (8 adapters), rank 32, bf16. Device
    us per call (CUDA graph of one call over 8 rotating weight sets) and the
    HBM GB/s of its algorithmic bytes, for the tcgen05 prefill path (runs as
    128-token GEMM tiles, build_seg_bounds(prefill=True)) and for the decode
    kernels on 32-token pieces (prefill=False)."""
    from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine

    T, n_ad = 4096, 8
    ids = np.repeat(np.arange(n_ad), T // n_ad).astype(np.int64)
    g = torch.Generator(device=device).manual_seed(3)
    sets = [(torch.randn(n_ad, 1, RANK, HIDDEN, device=device, dtype=torch.bfloat16, generator=g) * 0.02,
             torch.randn(n_ad, 1, HIDDEN, RANK, device=device, dtype=torch.bfloat16, generator=g) * 0.02)
            for _ in range(8)]
    x = torch.randn(T, HIDDEN, device=device, dtype=torch.bfloat16, generator=g) * 0.1
    y = torch.zeros(T, HIDDEN, device=device, dtype=torch.bfloat16)
    sb, eb = algorithmic_bytes(n_ad, T, HIDDEN, HIDDEN, RANK)
    hbm = measured_peaks().get("hbm_gbs") or 6650.0
    out = {}
    for name, kern, prefill in (("tcgen05_prefill", "auto", True), ("decode_cluster", "cluster", False),
                                ("decode_split", "split", False)):
        eng = WarpPipeEngine(WarpPipeConfig(max_tokens=T, prefetch_weights=True, prefetch_inputs=True, kernel=kern), device=device)
        eng.build_seg_bounds(torch.as_tensor(ids, device=device), prefill=prefill)

        def step():
            for wa, wb in sets:
                eng.add_lora_packed(y, x, wa, wb, 16.0 / RANK)

        gr = capture(step, warm=1)
        ms = time_graph(gr, None, iters) / len(sets)
        gbs = (sb + eb) / (ms * 1e-3) / 1e9
        out[name] = {"us_per_call": round(ms * 1e3, 2), "gbs": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 3)}
        del gr, eng
    return {"tokens": T, "runs": f"{n_ad} x {T // n_ad}", "d": HIDDEN, "o": HIDDEN, "rank": RANK,
            "algorithmic_mb": round((sb + eb) / 1e6, 1), "per_path": out}


def prefill_profile_case(args):
    """A few prefill-path launches of config 2's mix (for profilers)."""
    from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine

    device = torch.device("cuda", 0)
    T, n_ad = 4096, 8
    ids = np.repeat(np.arange(n_ad), T // n_ad).astype(np.int64)
    g = torch.Generator(device=device).manual_seed(3)
    sets = [(torch.randn(n_ad, 1, RANK, HIDDEN, device=device, dtype=torch.bfloat16, generator=g) * 0.02,
             torch.randn(n_ad, 1, HIDDEN, RANK, device=device, dtype=torch.bfloat16, generator=g) * 0.02)
            for _ in range(4)]
    x = torch.randn(T, HIDDEN, device=device, dtype=torch.bfloat16, generator=g) * 0.1
    y = torch.zeros(T, HIDDEN, device=device, dtype=torch.bfloat16)
    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=T, prefetch_weights=True, prefetch_inputs=True), device=device)
    eng.build_seg_bounds(torch.as_tensor(ids, device=device), prefill=True)
    for i in range(args.launches):
        wa, wb = sets[i % len(sets)]
        eng.add_lora_packed(y, x, wa, wb, 16.0 / RANK)
    torch.cuda.synchronize()
    print(json.dumps({"prefill_profile_case": "8 x 512 tokens, d = o = 4096, r32", "calls": args.launches}))


def config2_sweep(device, iters=5, ranks=(8, 16, 32, 64), residents=(1, 8, 64, 512), tokens=(1, 16, 256, 4096),
                  routings=("uniform", "zipf")):
    """one 4096 -> 4096 projection, bf16, rank x resident
    adapters x tokens x routing (uniform or Zipf(1.1), stable-sorted ids).
    Per case: device us per call (a CUDA graph of calls over rotating weight
    sets, together larger than L2 where the resident set allows it), the
    algorithmic GB/s and its fraction of the measured HBM bandwidth. Compact
    rows: [rank, resident, tokens, routing, active, us, GB/s, frac]."""
    from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine

    d = o = HIDDEN
    hbm = measured_peaks().get("hbm_gbs") or 6650.0
    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=True, prefetch_inputs=True), device=device)
    rows = []
    g = torch.Generator(device=device).manual_seed(2)
    for r in ranks:
        for resident in residents:
            set_bytes = resident * (d + o) * r * 2
            nsets = int(min(16, max(2, -(-300_000_000 // set_bytes))))
            sets = [(torch.randn(resident, 1, r, d, device=device, dtype=torch.bfloat16, generator=g) * 0.02,
                     torch.randn(resident, 1, o, r, device=device, dtype=torch.bfloat16, generator=g) * 0.02)
                    for _ in range(nsets)]
            for T in tokens:
                x = torch.randn(T, d, device=device, dtype=torch.bfloat16, generator=g) * 0.1
                y = torch.zeros(T, o, device=device, dtype=torch.bfloat16)
                for routing in routings:
                    if routing == "zipf":
                        ids = zipf_ids(resident, T, seed=SEED)
                    else:
                        ids = np.sort(np.random.default_rng(0).integers(0, resident, T), kind="stable")
                    U = int(np.unique(ids).size)
                    eng.build_seg_bounds(torch.as_tensor(ids, device=device))

                    def step():
                        for wa, wb in sets:
                            eng.add_lora_packed(y, x, wa, wb, 16.0 / r)

                    gr = capture(step, warm=1)
                    ms = time_graph(gr, None, iters) / nsets
                    del gr
                    sb, eb = algorithmic_bytes(U, T, d, o, r)
                    gbs = (sb + eb) / (ms * 1e-3) / 1e9
                    rows.append([r, resident, T, routing, U, round(ms * 1e3, 2), round(gbs, 1), round(gbs / hbm, 3)])
                del x, y
            del sets
            torch.cuda.empty_cache()
    del eng
    return {"d": d, "o": o, "dtype": "bf16", "columns": ["rank", "resident", "tokens", "routing", "active",
                                                         "us_per_call", "gbs", "frac_of_hbm"], "rows": rows}


def config4(device, steps: int = 200, warmup: int = 10, seed: int = 4):
    """multi-tenant draft-LoRA step with adapter churn.
    Draft shapes: 12 layers, hidden 768, intermediate 3072; every tenant owns
    a rank-16 LoRA on q, k, v, o, gate, up, down (84 projections, 6.8 MB per
    tenant). 1024 tenants live in page-locked host memory (one blob each,
    6.95 GB) behind a 128-slot GPU AdapterPool. A step applies 32 tenants x 8
    sequences x 4 lookahead tokens = 1024 tokens through all 84 projections
    (one build_seg_bounds_pool, the 84 calls replayed from a CUDA graph). Cold
    tenants arrive as a Poisson process at 0.05 per step (default_rng(4)) and
    replace a random active tenant one step later.

    Two runs of the same arrival sequence: on demand (the step that first
    uses a cold tenant copies it; the stream waits) and scheduler-aware
    prefetch (the arrival is written to the bridge as queued (is_hot) and
    PrefetchPolicy prefetches it on the pool's copy stream while the current
    step runs). Reports device us per step (CUDA events on the step stream),
    warm vs cold steps, cold misses and the prefetch-overlap fraction
    1 - (cold_prefetch - warm) / (cold_on_demand - warm)."""
    from adapterslotsplusplus_b200 import AdapterPool, WarpPipeConfig, WarpPipeEngine
    from adapterslotsplusplus_b200.scheduler_bridge import PrefetchPolicy

    layers, hid, inter, r = 12, 768, 3072, 16
    tenants_total, slots, active_n, T = 1024, 128, 32, 4 * 8 * 32
    per_layer = [("q", hid, hid, "h"), ("k", hid, hid, "h"), ("v", hid, hid, "h"), ("o", hid, hid, "a"),
                 ("gate", hid, inter, "h"), ("up", hid, inter, "h"), ("down", inter, hid, "i")]
    dims = [(d, o) for _ in range(layers) for _, d, o, _ in per_layer]
    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=True, prefetch_inputs=True), device=device)
    pool = AdapterPool(eng, slots, dims, rank=r, dtype=torch.bfloat16, max_adapters=tenants_total)
    sb = pool.slot_bytes
    # host store: one page-locked allocation, one blob per tenant; contents
    # from 8 random GPU-made blobs (the copies move full-size blobs)
    host = torch.empty(tenants_total, sb, dtype=torch.uint8, pin_memory=True)
    g = torch.Generator(device=device).manual_seed(seed)
    protos = []
    for _ in range(8):
        blob = torch.zeros(sb, dtype=torch.uint8, device=device)
        for (d, o), (a_off, b_off) in zip(dims, pool.layout):
            blob[a_off:a_off + r * d * 2].copy_((torch.randn(r * d, device=device, generator=g) * 0.02)
                                                 .bfloat16().view(torch.uint8))
            blob[b_off:b_off + o * r * 2].copy_((torch.randn(o * r, device=device, generator=g) * 0.02)
                                                 .bfloat16().view(torch.uint8))
        protos.append(blob)
    for i in range(tenants_total):
        host[i].copy_(protos[i % 8], non_blocking=True)
    torch.cuda.synchronize()
    for i in range(tenants_total):
        pool.register_host(i, host[i])
    xs = {"h": torch.randn(T, hid, device=device, dtype=torch.bfloat16, generator=g) * 0.1,
          "a": torch.randn(T, hid, device=device, dtype=torch.bfloat16, generator=g) * 0.1,
          "i": torch.randn(T, inter, device=device, dtype=torch.bfloat16, generator=g) * 0.1}
    ys = [torch.zeros(T, o, device=device, dtype=torch.bfloat16) for _, o in dims]
    srcs = [src for _ in range(layers) for *_, src in per_layer]
    idx_buf = torch.zeros(T, dtype=torch.int64, device=device)

    def apply_all():
        for p in range(len(dims)):
            pool.add_lora(p, ys[p], xs[srcs[p]], 1.0)

    rng = np.random.default_rng(seed)
    first_active = [int(v) for v in rng.choice(tenants_total, active_n, replace=False)]
    total_steps = warmup + steps
    arrivals = rng.poisson(0.05, total_steps)  # cold arrivals announced at each step
    arrival_ids = [[int(v) for v in rng.choice(tenants_total, k, replace=False)] if k else [] for k in arrivals]
    replace_at = [[int(v) for v in rng.integers(0, active_n, k)] if k else [] for k in arrivals]

    def token_ids(active):
        return torch.as_tensor(np.repeat(np.sort(np.asarray(active)), T // active_n), dtype=torch.int64)

    # capture the 84 apply calls once (the pool's stacks never move)
    pool.prepare(first_active)
    idx_buf.copy_(token_ids(first_active))
    pool.build_seg_bounds(idx_buf)
    graph = capture(apply_all, warm=1)

    def run(mode):
        # a fresh pool state per mode: the first active set resident (an empty
        # step first, so no slot counts as read by the step in flight)
        torch.cuda.synchronize()
        pool.prepare([])
        for i in range(tenants_total):
            pool.evict(i)
            pool.register_host(i, host[i])
        pool.prepare(first_active)
        torch.cuda.synchronize()
        policy = PrefetchPolicy(pool, budget=8, min_priority=1.0) if mode == "prefetch" else None
        active = list(first_active)
        pending = []  # (position, tenant) to swap in at the next step
        times, cold_flags, misses = [], [], 0
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(total_steps)]
        for step in range(total_steps):
            cold = bool(pending)
            for pos, tid in pending:
                if tid not in active:
                    active[pos] = tid
            pending = []
            st, en = evs[step]
            st.record()
            m = pool.prepare(active)
            idx_buf.copy_(token_ids(active), non_blocking=True)
            pool.build_seg_bounds(idx_buf)
            graph.replay()
            en.record()
            if step >= warmup:
                misses += m
                cold_flags.append(cold)
            # the scheduler admits this step's arrivals; they run next step
            new = [t for t in arrival_ids[step] if t not in active]
            pending = list(zip(replace_at[step][:len(new)], new))
            if policy is not None:
                hot = {t for _, t in pending}
                n = tenants_total
                bridge = {"num_active_adapters": n, "is_hot": [1 if i in hot else 0 for i in range(n)],
                          "whittle_scores": [0.0] * n, "lambda_hat": [0.0] * n, "gwar_pred_next3": [0.0] * n}
                policy.tick(bridge, protected=active)
            # a serving loop reads the step's output (sampled draft tokens)
            # before it schedules the next step
            en.synchronize()
        torch.cuda.synchronize()
        times = [evs[i][0].elapsed_time(evs[i][1]) * 1e3 for i in range(warmup, total_steps)]
        warm = [t for t, c in zip(times, cold_flags) if not c]
        coldt = [t for t, c in zip(times, cold_flags) if c]
        return {"us_per_step": round(float(np.mean(times)), 1), "warm_us": round(float(np.median(warm)), 1),
                "cold_us": round(float(np.mean(coldt)), 1) if coldt else None, "cold_steps": len(coldt),
                "cold_misses": int(misses), "prefetch_issued": policy.issued if policy else 0}

    # one tenant's host -> device copy, alone
    cs = torch.cuda.Stream()
    dst = torch.empty(sb, dtype=torch.uint8, device=device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(cs):
        e0.record()
        for i in range(4):
            dst.copy_(host[i], non_blocking=True)
        e1.record()
    torch.cuda.synchronize()
    copy_us = e0.elapsed_time(e1) * 1e3 / 4

    on_demand = run("on_demand")
    prefetch = run("prefetch")
    overlap = None
    if on_demand["cold_us"] and prefetch["cold_us"] and on_demand["cold_us"] > on_demand["warm_us"]:
        overlap = 1.0 - (prefetch["cold_us"] - prefetch["warm_us"]) / (on_demand["cold_us"] - on_demand["warm_us"])
        overlap = round(max(0.0, min(1.0, overlap)), 3)
    U = active_n
    step_bytes = 0
    for d, o in dims:
        sb_, eb_ = algorithmic_bytes(U, T, d, o, r)
        step_bytes += sb_ + eb_
    del graph, ys, xs, pool, host
    torch.cuda.empty_cache()
    return {"config": "4 (draft: 12 layers, h768, i3072, 32 tenants x r16 x 7 projections, 1024 tokens; 1024 "
                      "host tenants, 128 GPU slots, Poisson cold arrivals 0.05/step, default_rng(4))",
            "steps": steps, "tenant_bytes": sb, "copy_us_per_tenant": round(copy_us, 1),
            "step_gb": round(step_bytes / 1e9, 3), "on_demand": on_demand, "prefetch": prefetch,
            "prefetch_overlap_fraction": overlap}


def draft_step(device, iters: int = 20):
    """The multi-tenant draft step of config 4 end to end: a 12-layer draft
    decoder (hidden 768, 12 heads, intermediate 3072, LM head 32000; random
    init, bf16) over 32 tenants x 8 sequences x 4 lookahead tokens = 1024
    tokens, every projection's draft-LoRA (rank 16) applied by one grouped
    call over a 128-slot AdapterPool, the step replayed from a CUDA graph
    (adapterslotsplusplus_b200/draft.py). Device us per draft step: base
    model only, with the grouped LoRA, and with a plain-torch per-token
    gather of the same adapters (the stock path it replaces)."""
    from adapterslotsplusplus_b200 import AdapterPool, WarpPipeConfig, WarpPipeEngine
    from adapterslotsplusplus_b200.draft import DraftDecoder

    tenants, seqs, la, r = 32, 8, 4, 16
    T = tenants * seqs * la
    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=True, prefetch_inputs=True), device=device)
    model = DraftDecoder(layers=12, hidden=768, heads=12, inter=3072, vocab=32000, device=device)
    dims = model.dims()
    pool = AdapterPool(eng, 128, dims, rank=r, max_adapters=1024)
    g = torch.Generator(device=device).manual_seed(5)
    A = [torch.randn(tenants, r, d, device=device, generator=g).mul_(0.02).bfloat16() for d, _ in dims]
    B = [torch.randn(tenants, o, r, device=device, generator=g).mul_(0.02).bfloat16() for _, o in dims]
    blobs = []
    for t in range(tenants):
        blob = torch.empty(pool.slot_bytes, dtype=torch.uint8, pin_memory=True)
        pool.fill(blob, [(A[p][t].cpu(), B[p][t].cpu()) for p in range(len(dims))])
        pool.register_host(t, blob)
        blobs.append(blob)
    ids = torch.as_tensor(np.repeat(np.arange(tenants), seqs * la), dtype=torch.int64, device=device)
    tl = {"ids": ids, "A": A, "B": B}
    x = torch.randn(T, 768, device=device, generator=g).mul_(0.5).bfloat16()
    pool.prepare(ids.tolist())
    pool.build_seg_bounds(ids)
    out = {}
    for mode in ("none", "pool", "torch"):
        gr = capture(lambda: model.forward(x, la, lora=mode, pool=pool, scale=1.0, torch_lora=tl), warm=1)
        for _ in range(3):
            gr.replay()
        out[mode] = round(time_graph(gr, None, iters) * 1e3, 1)
        del gr
    del pool, blobs, model, A, B
    torch.cuda.empty_cache()
    return {"workload": "draft decoder 12 x (h768, 12 heads, i3072) + LM head 32000, 1024 tokens = 32 tenants x 8 "
                        "sequences x 4 lookahead, 84 rank-16 LoRA projections, CUDA graph",
            "us_per_step": {"base_only": out["none"], "grouped_lora": out["pool"], "torch_gather_lora": out["torch"]},
            "lora_us_per_step": round(out["pool"] - out["none"], 1),
            "torch_lora_us_per_step": round(out["torch"] - out["none"], 1)}


def config3(args, rank, world, local_rank):
    """a Llama-2-13B-shaped stack (40 layers, hidden 5120,
    intermediate 13824), rank 64, bf16, 128 resident adapters, 512 tokens,
    Zipf(1.1), tensor-parallel over the N GPUs (column-parallel q/k/v/gate/up,
    row-parallel o/down as --row-mode says). Four distinct layer
    weight sets (6.4 GB per GPU at N = 1, far larger than L2) are cycled over
    the 40 layers, so every launch streams its weights from HBM. One JSON
    line on rank 0: us per step (max over ranks) and the per-GPU HBM GB/s."""
    from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine

    layers, hid, inter, r, resident, T = 40, 5120, 13824, 64, 128, 512
    projs = [("q", hid, hid, "h", "col"), ("k", hid, hid, "h", "col"), ("v", hid, hid, "h", "col"),
             ("o", hid, hid, "attn", "row"), ("gate", hid, inter, "h", "col"), ("up", hid, inter, "h", "col"),
             ("down", inter, hid, "inter", "row")]
    device = torch.device("cuda", local_rank)
    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=True, prefetch_inputs=True), device=device)
    g = torch.Generator(device=device).manual_seed(3 + 1000 * rank)
    sets = []
    for _ in range(4):
        L = {}
        for name, d, o, _, kind in projs:
            dl = d // world if (world > 1 and kind == "row") else d
            ol = o // world if (world > 1 and kind == "col") else o
            L[name] = (torch.randn(resident, 1, r, dl, device=device, dtype=torch.bfloat16, generator=g) * 0.02,
                       torch.randn(resident, 1, ol, r, device=device, dtype=torch.bfloat16, generator=g) * 0.02,
                       torch.zeros(T, ol, device=device, dtype=torch.bfloat16))
        sets.append(L)
    xs = {"h": torch.randn(T, hid, device=device, dtype=torch.bfloat16, generator=g) * 0.1,
          "attn": torch.randn(T, hid // world, device=device, dtype=torch.bfloat16, generator=g) * 0.1,
          "inter": torch.randn(T, inter // world, device=device, dtype=torch.bfloat16, generator=g) * 0.1}
    ids = zipf_ids(resident, T, seed=SEED)
    U = int(np.unique(ids).size)
    eng.build_seg_bounds(torch.as_tensor(ids, device=device))
    tpa = None
    if world > 1:
        from adapterslotsplusplus_b200.tp import TensorParallelApply

        tpa = TensorParallelApply(eng, row_mode=args.row_mode)
    scale = 1.0

    def step():
        for li in range(layers):
            L = sets[li % 4]
            for name, d, o, src, kind in projs:
                wa, wb, y = L[name]
                if tpa is None:
                    eng.add_lora_packed(y, xs[src], wa, wb, scale)
                elif kind == "col":
                    tpa.column_parallel(y, xs[src], wa, wb, scale)
                else:
                    tpa.row_parallel(y, xs[src], wa, wb, scale)

    gr = capture(step)
    for _ in range(max(3, args.warmup)):
        gr.replay()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ms = time_graph(gr, None, args.steps)
    if world > 1:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    per_gpu = 0
    for name, d, o, src, kind in projs:
        dl = d // world if (world > 1 and kind == "row") else d
        ol = o // world if (world > 1 and kind == "col") else o
        sb, eb = algorithmic_bytes(U, T, dl, ol, r)
        per_gpu += sb + eb
    per_gpu *= layers
    peaks = measured_peaks()
    hbm = peaks.get("hbm_gbs") or 6650.0
    del gr
    if tpa is not None:
        tpa.close()
    del sets, xs
    torch.cuda.empty_cache()
    return {"config": "3 (llama2-13b: 40 layers, r64, bf16, 128 resident, 512 tokens, Zipf(1.1))",
            "n_gpus": world, "parallelism": f"tp{world}" if world > 1 else "single",
            "row_mode": args.row_mode if world > 1 else None,
            "us_per_step": round(ms * 1e3, 1), "launches_per_step": layers * len(projs),
            "active_adapters": U, "bytes_per_gpu_per_step": int(per_gpu),
            "gbs_per_gpu": round(per_gpu / (ms * 1e-3) / 1e9, 1),
            "frac_of_hbm": round(per_gpu / (ms * 1e-3) / 1e9 / hbm, 4)}


def profile_case(args):
    """A few launches of one projection of the workload, for profilers: the
    decode-step call shape (T = 256, Zipf routing over 64 resident adapters,
    rank 32) with 8 rotating weight sets (larger than L2 together)."""
    from adapterslotsplusplus_b200 import WarpPipeConfig, WarpPipeEngine

    shapes = {"q": (HIDDEN, HIDDEN), "gate": (HIDDEN, INTER), "down": (INTER, HIDDEN)}
    d, o = shapes[args.profile_case]
    device = torch.device("cuda", 0)
    eng = WarpPipeEngine(WarpPipeConfig(max_tokens=4096, prefetch_weights=True, prefetch_inputs=True, kernel=args.kernel), device=device)
    g = torch.Generator(device=device).manual_seed(0)
    sets = [(torch.randn(RESIDENT, 1, RANK, d, device=device, dtype=torch.bfloat16, generator=g) * 0.02,
             torch.randn(RESIDENT, 1, o, RANK, device=device, dtype=torch.bfloat16, generator=g) * 0.02)
            for _ in range(8)]
    x = torch.randn(TOKENS, d, device=device, dtype=torch.bfloat16, generator=g) * 0.1
    y = torch.zeros(TOKENS, o, device=device, dtype=torch.bfloat16)
    eng.build_seg_bounds(torch.as_tensor(make_ids(args.profile_resident), device=device))
    torch.cuda.synchronize()
    for i in range(args.launches):
        wa, wb = sets[i % len(sets)]
        eng.add_lora_packed(y, x, wa, wb, 16.0 / RANK)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": args.profile_case, "launches": args.launches, "kernel": eng.last_apply_kernel(),
                      "cluster": eng.last_apply_cluster(), "resident": args.profile_resident,
                      "d": d, "o": o, "tokens": TOKENS, "rank": RANK}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--cpu-layers", type=int, default=2, help="layers in the cpu_baseline sample")
    ap.add_argument("--profile-case", choices=["q", "gate", "down"], default=None,
                    help="run a few launches of one projection (for profilers) and exit")
    ap.add_argument("--profile-resident", type=int, default=RESIDENT,
                    help="resident adapters of --profile-case (Zipf routing over them)")
    ap.add_argument("--launches", type=int, default=12, help="launches of --profile-case")
    ap.add_argument("--kernel", choices=["auto", "cluster", "split"], default="auto",
                    help="apply kernel of --profile-case")
    ap.add_argument("--prefill-mix", action="store_true", help="time config 2's prefill mix per kernel and exit")
    ap.add_argument("--prefill-profile", action="store_true",
                    help="run --launches prefill-path calls of config 2's mix (for profilers) and exit")
    ap.add_argument("--config3", action="store_true",
                    help="time BASELINE config 3 (13B, r64, T=512, tensor-parallel over the N GPUs) and exit")
    ap.add_argument("--config4", action="store_true",
                    help="time BASELINE config 4 (draft-LoRA churn over a pinned-host pool) and exit")
    ap.add_argument("--row-mode", choices=["partial", "fused", "nccl"], default="partial",
                    help="row-parallel layers under tensor parallelism (N > 1)")
    ap.add_argument("--per-kind", action="store_true", help="also time column/row-parallel launches apart at N = 1")
    ap.add_argument("--no-extras", action="store_true",
                    help="only the headline step (no flatness, config 2 / 3, prefill or fused-slice keys)")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args)
        return
    if args.prefill_mix:
        print(json.dumps(prefill_mix(torch.device("cuda", 0))), flush=True)
        return
    if args.prefill_profile:
        prefill_profile_case(args)
        return
    if args.config4:
        dev0 = torch.device("cuda", 0)
        print(json.dumps({"config4": config4(dev0, steps=args.steps * 10), "draft_step": draft_step(dev0)}), flush=True)
        return
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    if args.config3:
        if world > 1:
            torch.cuda.set_device(local_rank)
            os.environ.setdefault("NCCL_DEBUG", "WARN")
            torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
        res = config3(args, rank, world, local_rank)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        if rank == 0:
            print(json.dumps(res), flush=True)
        return
    if world > 1:
        torch.cuda.set_device(local_rank)
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep NCCL's banner off stdout (one JSON line)
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    eng, result = run_ours(args, rank, world, local_rank)
    device = torch.device("cuda", local_rank)
    if not args.no_extras:
        # config 3 (13B, r64, T = 512) on the same N GPUs, in the same line
        result["config3"] = config3(args, rank, world, local_rank)
    if rank == 0 and world == 1 and not args.no_extras:
        if not args.no_sweep:
            result["flatness"] = sweep_resident(eng, device, [1, 8, 64, 128, 512], max(3, args.steps // 4))
            result["config2_sweep"] = config2_sweep(device)
        result["fused_slices"] = fused_slices(eng, device, max(3, args.steps // 2))
        result["strict_order"] = strict_order(device, max(3, args.steps // 2))
        result["weights_prefetch_only"] = strict_order(device, max(3, args.steps // 2), prefetch_weights=True)
        result["fp16_step"] = fp16_step(device, max(3, args.steps // 2))
        result["prefill_mix"] = prefill_mix(device)
        result["config4"] = config4(device)
        result["draft_step"] = draft_step(device)
    if rank == 0 and world == 1:
        dt, threads = cpu_reference_layers(args.cpu_layers)
        result["cpu_baseline"] = {"value": round(dt * LAYERS * 1e6, 1), "unit": "us/step", "cores": threads,
                                  "kind": "port",
                                  "sample": f"{args.cpu_layers} of {LAYERS} layers timed, extrapolated x{LAYERS}"}
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()

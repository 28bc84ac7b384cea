"""Seeded input generators shared by the golden-fixture scripts and the tests.

Shapes and distributions follow the reference's own tests and the
configurations of the benchmark:
  * config 0: d = o = 4096, rank 16, 8 adapters, 64 tokens, fp16; token ids
    uniform (seed 0), stable-sorted; X ~ N(0,1), A_i ~ N(0, 1/4096),
    B_i ~ N(0, 1/16), Y ~ N(0,1), alpha = 2.0;
  * ADD_LORA_CASES: the index patterns of
    tests/correctness/test_add_lora_packed.py:78-109 and
    test_warp_pipe_graph_capture.py:54-55 (weights * 0.02, activations * 0.1,
    scale 16/32, as there);
  * RANK_CASES: tests/unit/test_rank_variants.py:24-27 (K = 3 adapters x 17
    tokens, d = o = 512, weights * 0.02, activations * 0.1, alpha 16/rank).
All tensors are generated on the CPU; callers move them to a device.
"""

from __future__ import annotations

import numpy as np
import torch

ADD_LORA_CASES = {
    "mixed_neg": [0, 0, 0, 0, -1, -1, 2, 2, 2, 1, 1, 1, 1, 1, 1, 1],
    "run32": [3] * 32,
    "all_neg": [-1] * 8,
    "run33": [5] * 33,
    "many_short": list(range(8)) * 4,
    "run8": [4] * 8,
    "run9": [4] * 9,
    "capture": [0, 0, 0, 0, 1, 1, 1, 1, -1, -1, 2, 2, 2, 2, 2, 2],
    "replay": [3, 3, 5, 5, 5, 5, 5, 5, 5, 5, 5, 5, 5, 5, -1, 6],
}
ADD_LORA_DIM = 256
ADD_LORA_RANK = 32
ADD_LORA_NUM = 8
RANK_CASES = (8, 16, 32, 64)


def input_checksum(d: dict) -> float:
    s = 0.0
    for k in sorted(d):
        v = d[k]
        if isinstance(v, torch.Tensor) and v.is_floating_point():
            s += float(v.double().abs().sum())
    return s


def config0_inputs(dtype=torch.float16) -> dict:
    T, D, O, R, K = 64, 4096, 4096, 16, 8
    ids = torch.randint(0, K, (T,), generator=torch.Generator().manual_seed(0))
    ids_sorted, perm = torch.sort(ids, stable=True)
    g = torch.Generator().manual_seed(1)
    X = torch.randn(T, D, generator=g)[perm]
    A = (torch.randn(K, D, R, generator=g) * (1.0 / 4096) ** 0.5).transpose(1, 2).contiguous()  # [K, R, D]
    B = (torch.randn(K, R, O, generator=g) * (1.0 / 16) ** 0.5).transpose(1, 2).contiguous()  # [K, O, R]
    Y = torch.randn(T, O, generator=g)
    from oracle.seg import seg_bounds  # run-length table of the sorted ids

    table = [tuple(int(v) for v in row) for row in seg_bounds(ids_sorted.numpy())]
    return {"ids": ids_sorted, "X": X.to(dtype), "A": A.to(dtype), "B": B.to(dtype), "Y": Y.to(dtype),
            "alpha": 2.0, "table": table}


def add_lora_inputs(idx, dtype=torch.float16, dim=ADD_LORA_DIM, rank=ADD_LORA_RANK, seed=0) -> dict:
    g = torch.Generator().manual_seed(seed)
    T = len(idx)
    wa = (torch.randn(ADD_LORA_NUM, 1, rank, dim, generator=g) * 0.02).to(dtype)
    wb = (torch.randn(ADD_LORA_NUM, 1, dim, rank, generator=g) * 0.02).to(dtype)
    x = (torch.randn(T, dim, generator=g) * 0.1).to(dtype)
    y = (torch.randn(T, dim, generator=g) * 0.1).to(dtype)
    return {"wa": wa, "wb": wb, "x": x, "y": y, "scale": 16.0 / rank}


def rank_case_inputs(rank, dtype=torch.float16, K=3, per=17, dim=512) -> dict:
    g = torch.Generator().manual_seed(100 + rank)
    A = (torch.randn(K, rank, dim, generator=g) * 0.02).to(dtype)
    B = (torch.randn(K, dim, rank, generator=g) * 0.02).to(dtype)
    X = (torch.randn(K * per, dim, generator=g) * 0.1).to(dtype)
    Y = (torch.randn(K * per, dim, generator=g) * 0.1).to(dtype)
    table = [(i, i * per, per) for i in range(K)]
    return {"A": A, "B": B, "X": X, "Y": Y, "alpha": 16.0 / rank, "table": table}


def zipf_ids(num_resident: int, T: int, seed: int, s: float = 1.1) -> np.ndarray:
    """Zipf(s) adapter popularity, weights 1/(i+1)^s normalised
    (benchmarks/sota/drivers/vllm_v1_throughput_driver.py:18-24), ids drawn
    with numpy default_rng(seed) and stable-sorted."""
    w = 1.0 / np.power(np.arange(1, num_resident + 1, dtype=np.float64), s)
    w /= w.sum()
    ids = np.random.default_rng(seed).choice(num_resident, T, p=w)
    return np.sort(ids, kind="stable").astype(np.int64)

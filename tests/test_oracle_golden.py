"""The CPU oracle against the reference's own golden numbers (no GPU).

tests/golden/golden_apply.npz was produced by the reference's own Python
oracle functions (tests/golden/make_golden.py); seg_bounds_ref.json, when
present, by the reference's own build_seg_bounds kernel on a B200
(tests/golden/make_ref_seg_golden.py).
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import apply as oa
from oracle.seg import SEG_TOKENS, seg_bounds, seg_bounds_loop, segment_table
from tests.golden.cases import (ADD_LORA_CASES, RANK_CASES, add_lora_inputs, config0_inputs, input_checksum,
                                rank_case_inputs)

GOLD = Path(__file__).resolve().parent / "golden"


def _close(a, b, tol):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    assert a.shape == b.shape
    assert np.max(np.abs(a - b)) <= tol, np.max(np.abs(a - b))


def test_config0_oracle_matches_reference_golden(golden):
    c = config0_inputs()
    assert input_checksum(c) == pytest.approx(float(golden["cfg0_input_sum"]), rel=1e-12)
    _, Y = oa.apply_segments(c["Y"], c["X"], c["table"], lambda i: c["A"][i], lambda i: c["B"][i],
                             lambda i: c["alpha"])
    delta = (Y - c["Y"].float()).double().numpy()
    _close(delta.sum(1), golden["cfg0_row_sum"], 1e-6)
    _close((delta ** 2).sum(1), golden["cfg0_row_sq"], 1e-6 * float(golden["cfg0_row_sq"].max()))
    _close(delta[:, ::16], golden["cfg0_cols"], 1e-5)


@pytest.mark.parametrize("name", sorted(ADD_LORA_CASES))
def test_add_lora_oracle_matches_reference_golden(golden, name):
    idx = ADD_LORA_CASES[name]
    a = add_lora_inputs(idx)
    assert input_checksum(a) == pytest.approx(float(golden[f"add_{name}_input_sum"]), rel=1e-12)
    for fn in (oa.reference_add_lora, oa.add_lora_grouped):
        y = fn(a["y"], a["x"], a["wa"], a["wb"], a["scale"], torch.tensor(idx))
        dl = (y - a["y"].float()).double().numpy()
        _close(dl[:, ::8], golden[f"add_{name}_cols"], 1e-6)
        _close(dl.sum(1), golden[f"add_{name}_row_sum"], 1e-5)


@pytest.mark.parametrize("rank", RANK_CASES)
def test_rank_variant_oracle_matches_reference_golden(golden, rank):
    r = rank_case_inputs(rank)
    assert input_checksum(r) == pytest.approx(float(golden[f"rank{rank}_input_sum"]), rel=1e-12)
    H, Y = oa.apply_segments(r["Y"], r["X"], r["table"], lambda i: r["A"][i], lambda i: r["B"][i],
                             lambda i: r["alpha"])
    _close(H.numpy(), golden[f"rank{rank}_H"], 1e-6)
    dl = (Y - r["Y"].float()).double().numpy()
    _close(dl[:, ::8], golden[f"rank{rank}_Ycols"], 1e-6)
    _close(dl.sum(1), golden[f"rank{rank}_Yrow_sum"], 1e-5)


# ---- segmenter restatement --------------------------------------------------

KNOWN = {
    # test_add_lora_packed.py:78-109 patterns with their tables under the
    # rule of build_seg_bounds_kernel (warp_pipe_r32.cu:461-512)
    "mixed_neg": [(0, 0, 4), (2, 6, 3), (1, 9, 7)],
    "run32": [(3, 0, 32)],
    "all_neg": [],
    "run33": [(5, 0, 32), (5, 32, 1)],
    "run8": [(4, 0, 8)],
    "run9": [(4, 0, 9)],
    "capture": [(0, 0, 4), (1, 4, 4), (2, 10, 6)],
    "replay": [(3, 0, 2), (5, 2, 12), (6, 15, 1)],
}


@pytest.mark.parametrize("name", sorted(KNOWN))
def test_seg_bounds_known_answers(name):
    got = [tuple(r) for r in seg_bounds(ADD_LORA_CASES[name]).tolist()]
    assert got == KNOWN[name]


def test_seg_bounds_many_short_runs():
    t = seg_bounds(list(range(8)) * 4)
    assert t.shape == (32, 3)
    assert (t[:, 2] == 1).all() and (t[:, 1] == np.arange(32)).all()


def test_seg_bounds_vectorised_equals_loop():
    rng = np.random.default_rng(0)
    for trial in range(400):
        T = int(rng.integers(0, 700))
        kind = trial % 4
        if kind == 0:
            idx = rng.integers(-1, 4, T)
        elif kind == 1:
            idx = np.sort(rng.integers(-2, 9, T))
        elif kind == 2:
            idx = np.repeat(rng.integers(-1, 6, max(1, T // 37 + 1)), 37)[:T]
        else:
            idx = np.full(T, int(rng.integers(-1, 3)))
        a, b = seg_bounds(idx), seg_bounds_loop(idx)
        assert a.shape == b.shape and (a == b).all()
        if T:
            assert (a[:, 2] <= SEG_TOKENS).all() and (a[:, 2] >= 1).all()


def test_seg_bounds_int64_ids_cast_like_reference():
    # ids are compared as int64 and stored as int32 (warp_pipe_r32.cu:476,507)
    big = [2 ** 33 + 1] * 3 + [1] * 2
    t = seg_bounds(big)
    assert t.tolist() == [[int(np.int64(2 ** 33 + 1).astype(np.int32)), 0, 3], [1, 3, 2]]


def test_segment_table_restatement():
    assert segment_table([0, 1, 2], [0, 1, 32, 34]).tolist() == [[0, 0, 1], [1, 1, 31], [2, 32, 2]]
    with pytest.raises(RuntimeError):
        segment_table([0, 1], [0, 4])


def test_seg_bounds_reference_kernel_fixture():
    """Tables produced by the reference's own kernel on a B200 (T <= 256)."""
    p = GOLD / "seg_bounds_ref.json"
    if not p.exists():
        pytest.skip("seg_bounds_ref.json not generated yet")
    cases = json.loads(p.read_text())
    assert len(cases) >= 20
    for c in cases:
        got = seg_bounds(c["idx"]).tolist()
        assert got == c["table"], c["name"]

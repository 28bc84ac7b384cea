"""Generate tests/golden/golden_apply.npz with the REFERENCE's own Python oracle.

Run in a checkout where the reference (vac014/AdapterSlotsPlusPlus) is
available (WP_REFERENCE_ROOT, else a checkout named "reference" beside this
repository's directory):

    python tests/golden/make_golden.py

It imports the reference's own functions, unmodified:
  * reference_bgmv_shrink / reference_bgmv_expand from
    tests/correctness/reference_bgmv.py:4-18;
  * reference_add_lora from tests/correctness/test_add_lora_packed.py:35-45
    (extracted with `ast`, because importing that file would import the
    reference's CUDA extension).
Inputs are regenerated from the seeds recorded below (torch CPU RNG), so the
fixture stores only input checksums plus the expected outputs: full arrays for
small cases (H), and for Y deltas per-row sums/sums of squares plus a
column sample. The tests check oracle/apply.py against these
numbers; they never read the reference at run time.
"""

from __future__ import annotations

import ast
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
from tests.golden.cases import (  # noqa: E402
    ADD_LORA_CASES, RANK_CASES, config0_inputs, add_lora_inputs, rank_case_inputs, input_checksum,
)

COL_STRIDE = 8  # column sample of the small cases (row sums cover every column)
REF = Path(os.environ.get("WP_REFERENCE_ROOT", str(Path(__file__).resolve().parents[3] / "reference")))


def load_reference_functions():
    spec = importlib.util.spec_from_file_location("ref_bgmv", REF / "tests/correctness/reference_bgmv.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    src = (REF / "tests/correctness/test_add_lora_packed.py").read_text()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "reference_add_lora")
    ns = {"torch": torch}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "reference_add_lora", "exec"), ns)
    return mod.reference_bgmv_shrink, mod.reference_bgmv_expand, ns["reference_add_lora"]


def main():
    shrink, expand, add_lora = load_reference_functions()
    out = {}

    # config 0: per-segment registry-path math (test_bgmv_correctness.py:38-44 form, no H rounding)
    c = config0_inputs()
    Y = c["Y"].float().clone()
    for aid, s, n in c["table"]:
        h = shrink(c["X"][s:s + n], c["A"][aid], c["alpha"])
        Y[s:s + n] = expand(h, c["B"][aid], c["Y"][s:s + n])
    delta = (Y - c["Y"].float()).numpy()
    out["cfg0_input_sum"] = np.array(input_checksum(c), dtype=np.float64)
    out["cfg0_row_sum"] = delta.astype(np.float64).sum(1)
    out["cfg0_row_sq"] = (delta.astype(np.float64) ** 2).sum(1)
    out["cfg0_cols"] = delta[:, ::16].astype(np.float32)

    # add_lora index patterns (test_add_lora_packed.py:78-109) at d = o = 256, r = 32
    for name, idx in ADD_LORA_CASES.items():
        a = add_lora_inputs(idx)
        ref = add_lora(a["y"], a["x"], a["wa"], a["wb"], a["scale"], torch.tensor(idx))
        dl = (ref - a["y"].float()).numpy().astype(np.float64)
        out[f"add_{name}_cols"] = dl[:, ::COL_STRIDE].astype(np.float32)
        out[f"add_{name}_row_sum"] = dl.sum(1)
        out[f"add_{name}_row_sq"] = (dl ** 2).sum(1)
        out[f"add_{name}_input_sum"] = np.array(input_checksum(a), dtype=np.float64)

    # rank variants (test_rank_variants.py:24-27): K=3 adapters x 17 tokens, d = o = 512
    for rank in RANK_CASES:
        r = rank_case_inputs(rank)
        Y = r["Y"].float().clone()
        H = torch.zeros(r["X"].shape[0], rank)
        for aid, s, n in r["table"]:
            h = shrink(r["X"][s:s + n], r["A"][aid], r["alpha"])
            H[s:s + n] = h
            Y[s:s + n] = expand(h, r["B"][aid], r["Y"][s:s + n])
        out[f"rank{rank}_H"] = H.numpy().astype(np.float32)
        dl = (Y - r["Y"].float()).numpy().astype(np.float64)
        out[f"rank{rank}_Ycols"] = dl[:, ::COL_STRIDE].astype(np.float32)
        out[f"rank{rank}_Yrow_sum"] = dl.sum(1)
        out[f"rank{rank}_input_sum"] = np.array(input_checksum(r), dtype=np.float64)

    np.savez_compressed(HERE / "golden_apply.npz", **out)
    print(f"wrote {HERE / 'golden_apply.npz'} ({(HERE / 'golden_apply.npz').stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()

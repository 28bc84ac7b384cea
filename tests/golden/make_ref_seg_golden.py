"""Generate tests/golden/seg_bounds_ref.json with the REFERENCE's own
build_seg_bounds_kernel (csrc/kernels/warp_pipe_r32.cu:461-512), run on a GPU.

Needs oracle/_ref/libwpref.so (built from the reference's kernel sources by
oracle/build_ref.sh) and a CUDA device:

    python tests/golden/make_ref_seg_golden.py [OUT.json]

Index vectors: the reference tests' own patterns (test_add_lora_packed.py:78-109,
test_warp_pipe_graph_capture.py:54-55) plus seeded random, sorted, Zipf and
long-run vectors of up to 256 tokens (the reference kernel's limit).
"""

from __future__ import annotations

import ctypes
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
from tests.golden.cases import ADD_LORA_CASES, zipf_ids  # noqa: E402


def index_cases():
    cases = [(f"ref_{k}", list(v)) for k, v in ADD_LORA_CASES.items()]
    rng = np.random.default_rng(2024)
    for T in (1, 2, 31, 32, 33, 64, 65, 100, 128, 200, 255, 256):
        cases.append((f"uniform_T{T}", rng.integers(-1, 6, T).tolist()))
        cases.append((f"sorted_T{T}", np.sort(rng.integers(-1, 50, T)).tolist()))
        cases.append((f"zipf_T{T}", zipf_ids(64, T, seed=T).tolist()))
        cases.append((f"runs70_T{T}", np.repeat(rng.integers(-1, 4, T // 70 + 1), 70)[:T].tolist()))
    cases.append(("all_one_256", [9] * 256))
    cases.append(("alternating_256", [i % 2 for i in range(256)]))
    return cases


def main(out_path: Path):
    lib = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libwpref.so"))
    out = (ctypes.c_int32 * 768)()
    num = ctypes.c_int32()
    result = []
    for name, idx in index_cases():
        d = torch.tensor(idx, dtype=torch.int64, device="cuda")
        torch.cuda.synchronize()
        rc = lib.ref_seg_bounds(ctypes.c_void_p(d.data_ptr()), ctypes.c_int(len(idx)), out, ctypes.byref(num))
        assert rc == 0, (name, rc)
        table = [[out[3 * i], out[3 * i + 1], out[3 * i + 2]] for i in range(num.value)]
        result.append({"name": name, "idx": idx, "table": table})
    out_path.write_text(json.dumps(result))
    print(f"wrote {out_path}: {len(result)} cases")


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else HERE / "seg_bounds_ref.json")

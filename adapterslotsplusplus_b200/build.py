"""Build recipe for libwp_b200.so (sm_100a), in-tree.

Compiles every CUDA source under ``csrc/`` with nvcc for
``-gencode arch=compute_100a,code=sm_100a`` and links a plain shared
library with an ``extern "C"`` ABI (include/wp_api.h). NCCL comes from the
nvidia-nccl wheel that PyTorch ships; its directory is baked in as an rpath.

Usage:  python -m adapterslotsplusplus_b200.build   (or build() from Python)
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB_NAME = "libwp_b200.so"
LIB_PATH = PKG / LIB_NAME
SOURCES = ["wp_segment.cu", "wp_apply.cu", "wp_apply_split.cu", "wp_prefill.cu", "wp_api.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libwp_b200.so")


def nccl_paths() -> tuple[str, str]:
    """(include dir, lib dir) of the NCCL that PyTorch loads."""
    import importlib.util

    spec = importlib.util.find_spec("nvidia.nccl")
    if spec is not None and spec.submodule_search_locations:
        root = Path(list(spec.submodule_search_locations)[0])
        if (root / "include" / "nccl.h").exists() and (root / "lib").exists():
            return str(root / "include"), str(root / "lib")
    if Path("/usr/include/nccl.h").exists():
        return "/usr/include", "/usr/lib/x86_64-linux-gnu"
    raise RuntimeError("nccl.h not found (nvidia-nccl wheel or /usr/include)")


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    lib_t = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [INCLUDE / "wp_api.h"]
    return any(p.stat().st_mtime > lib_t for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile libwp_b200.so next to this file (no-op when up to date)."""
    if not force and not _stale():
        return LIB_PATH
    nvcc = _nvcc()
    inc, libdir = nccl_paths()
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    common = [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(INCLUDE), "-I", inc,
              *os.environ.get("WP_NVCC_EXTRA", "").split()]
    from concurrent.futures import ThreadPoolExecutor

    cmds = []
    objs = []
    for src in SOURCES:
        obj = objdir / (Path(src).stem + ".o")
        cmds.append([*common, "-c", str(CSRC / src), "-o", str(obj)])
        objs.append(str(obj))
        if verbose:
            print(" ".join(cmds[-1]), file=sys.stderr)
    # the sources compile independently: one nvcc per source, in parallel
    with ThreadPoolExecutor(max_workers=len(cmds)) as pool:
        for f in [pool.submit(subprocess.run, c, check=True) for c in cmds]:
            f.result()
    ncclso = Path(libdir) / "libnccl.so.2"
    link = [
        nvcc, *ARCH, "-shared", "-o", str(LIB_PATH) + ".tmp", *objs,
        "-Xlinker", f"-rpath={libdir}", "-Xlinker", "-l:libnccl.so.2" if ncclso.exists() else "-lnccl",
        "-L", libdir,
    ]
    if verbose:
        print(" ".join(link), file=sys.stderr)
    subprocess.run(link, check=True)
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))

"""Build ``libclef_b200.so`` in-tree with nvcc for sm_100a.

    python -m deciax_b200.build          # or deciax_b200.build.build()

The library links the NCCL shipped with the PyTorch wheel (``nvidia-nccl-cu12``)
so that it shares one libnccl with ``torch.distributed``.  nvcc cross-compiles,
so this runs on a machine without a GPU.
"""

from __future__ import annotations

import importlib.util
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libclef_b200.so"
INCLUDE = PKG.parent / "include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def nccl_paths() -> tuple[Path, Path]:
    spec = importlib.util.find_spec("nvidia.nccl")
    if spec and spec.submodule_search_locations:
        root = Path(list(spec.submodule_search_locations)[0])
        if (root / "include" / "nccl.h").exists():
            return root / "include", root / "lib"
    if Path("/usr/include/nccl.h").exists():
        return Path("/usr/include"), Path("/usr/lib/x86_64-linux-gnu")
    raise RuntimeError("NCCL headers not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "clef_b200.h"]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    inc, lib = nccl_paths()
    cmd = [
        nvcc(),
        *ARCH,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "-shared",
        f"-I{INCLUDE}",
        f"-I{inc}",
        str(CSRC / "clef.cu"),
        "-o",
        str(LIB) + ".tmp",
        f"-L{lib}",
        "-l:libnccl.so.2",
        f"-Xlinker=-rpath,{lib}",
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr[-8000:]}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)

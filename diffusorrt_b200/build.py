"""Build libdiffusorrt_b200.so in-tree with nvcc for sm_100a.

    python -m diffusorrt_b200.build [--verbose]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT = PKG / "libdiffusorrt_b200.so"
SOURCES = [CSRC / "capi.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "diffusorrt_b200.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found")
    return exe


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in SOURCES + HEADERS)


def nccl_include() -> list[str]:
    """Include path of nccl.h (types only: the library resolves NCCL at run time)."""
    try:
        import nvidia.nccl  # the NCCL that torch.distributed loads

        for base in nvidia.nccl.__path__:
            if (Path(base) / "include" / "nccl.h").exists():
                return ["-I", str(Path(base) / "include")]
    except ImportError:
        pass
    if Path("/usr/include/nccl.h").exists():
        return []
    raise RuntimeError("nccl.h not found")


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", *nccl_include(),
           "-o", str(tmp), *map(str, SOURCES), "-ldl"]
    if verbose:
        cmd.insert(1, "-Xptxas")
        cmd.insert(2, "-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=str(PKG))
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))

"""Build recipe for libdflashcuda.so (sm_100a only, in-tree output).

    python dflash-swift_b200/build.py [--force] [--ptxas-verbose]

One nvcc invocation over the single translation unit csrc/libdflashcuda.cu; the CUDA
runtime is linked statically and the driver API is resolved at run time, so the
library loads on machines without a GPU driver (the C-ABI symbol checks run there).
"""
from __future__ import annotations

import argparse
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "libdflashcuda.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def up_to_date() -> bool:
    return OUT.exists() and all(OUT.stat().st_mtime >= s.stat().st_mtime for s in sources())


def build(force: bool = False, ptxas_verbose: bool = False, extra=()) -> Path:
    if not force and up_to_date():
        return OUT
    cmd = ["nvcc", *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           f"-I{ROOT / 'include'}", str(CSRC / "libdflashcuda.cu"), "-o", str(OUT), "-cudart", "static",
           "-diag-suppress", "550", *extra]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    subprocess.run(cmd, check=True)
    return OUT


HOST = PKG / "host"
HOST_OUT = PKG / "libdflashkit.so"


def cuda_home() -> Path:
    import shutil
    nvcc = shutil.which("nvcc")
    return Path(nvcc).resolve().parent.parent if nvcc else Path("/usr/local/cuda")


def build_host(force: bool = False) -> Path:
    """libdflashkit.so: the C++ host interface (host/dflashkit.{hpp,cpp}) over
    libdflashcuda.so, linked against the shared CUDA runtime for its allocations."""
    srcs = sorted(HOST.glob("*.cpp")) + sorted(HOST.glob("*.hpp")) + sorted((ROOT / "include").glob("*.h"))
    if not force and HOST_OUT.exists() and OUT.exists() and all(
            HOST_OUT.stat().st_mtime >= s.stat().st_mtime for s in srcs + [OUT]):
        return HOST_OUT
    cuda = cuda_home()
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", "-Werror",
           f"-I{ROOT / 'include'}", f"-I{cuda / 'include'}", str(HOST / "dflashkit.cpp"), "-o", str(HOST_OUT),
           f"-L{PKG}", "-ldflashcuda", f"-L{cuda / 'lib64'}", "-lcudart",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{cuda / 'lib64'}"]
    subprocess.run(cmd, check=True)
    return HOST_OUT


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(a.force, a.ptxas_verbose))
    print(build_host(a.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())

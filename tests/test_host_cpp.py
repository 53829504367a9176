"""The C++ host interface (dflash-swift_b200/host/dflashkit.hpp) through its own test
program, tests/host/test_dflashkit.cpp: the CPU cases here (tree plan, accepted path,
eligibility, swap semantics, argument errors), the GPU cases on a B200 (the quantized
linear layer and the gated-delta rollbacks against the oracle)."""
from __future__ import annotations

import importlib.util
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "dflash-swift_b200"
SRC = ROOT / "tests" / "host" / "test_dflashkit.cpp"
EXE = ROOT / "tests" / "host" / "_build" / "test_dflashkit"


def _build_module():
    spec = importlib.util.spec_from_file_location("dflash_build", PKG / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _binary() -> Path:
    build = _build_module()
    if not build.OUT.exists():  # never rebuild the CUDA library under a process that has it loaded
        build.build()
    kit = build.build_host()
    oracle = ROOT / "oracle" / "liboracle.so"
    deps = [SRC, kit, oracle, PKG / "host" / "dflashkit.hpp"]
    if EXE.exists() and all(EXE.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return EXE
    EXE.parent.mkdir(parents=True, exist_ok=True)
    cuda = build.cuda_home()
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", f"-I{PKG / 'host'}", f"-I{ROOT / 'include'}",
           f"-I{cuda / 'include'}", str(SRC), "-o", str(EXE), f"-L{PKG}", "-ldflashkit", "-ldflashcuda",
           f"-L{oracle.parent}", "-loracle", f"-L{cuda / 'lib64'}", "-lcudart",
           f"-Wl,-rpath,{PKG}", f"-Wl,-rpath,{oracle.parent}", f"-Wl,-rpath,{cuda / 'lib64'}"]
    subprocess.run(cmd, check=True)
    return EXE


def _run(mode: str) -> subprocess.CompletedProcess:
    return subprocess.run([str(_binary()), mode], capture_output=True, text=True, timeout=600)


def test_host_cpp_cpu_cases():
    r = _run("cpu")
    print(r.stdout, r.stderr)
    assert r.returncode == 0, r.stderr
    assert "0 failures" in r.stdout


@pytest.mark.gpu
def test_host_cpp_gpu_cases(cuda):
    r = _run("gpu")
    print(r.stdout, r.stderr)
    assert r.returncode == 0, r.stderr
    assert "0 failures" in r.stdout

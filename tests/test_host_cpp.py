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


def _dump_stack(d: Path, cfg, plan, w, state, context, hidden, proposals, keep, max_len):
    """blob.bin + manifest.txt for the program's `stack` mode: every buffer of the shard
    (256-byte aligned in the blob) and the descriptor's fields."""
    import torch
    blob, lines = bytearray(), []

    def put(name, t):
        raw = t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()
        off = (len(blob) + 255) // 256 * 256
        blob.extend(b"\0" * (off - len(blob)))
        lines.append(f"tensor {name} {off} {len(raw)}")
        blob.extend(raw)

    def putq(name, q):
        put(name + ".w", q.w)
        put(name + ".scales", q.scales)
        put(name + ".biases", q.biases)
        lines.append(f"qweight {name} {q.N} {q.K}")

    for i, (L, S) in enumerate(zip(w["layers"], state["layers"])):
        gdn = L["kind"] == "gdn"
        lines.append(f"layer {i} {0 if gdn else 1}")
        p = f"L{i}."
        put(p + "ln", L["ln"])
        put(p + "post_ln", L["post_ln"])
        names = ("in_proj", "out_proj") if gdn else ("qkv", "o_proj")
        for n in names + ("gate_up", "down"):
            putq(p + n, L[n])
        for n in (("conv", "a_log", "dt_bias", "gdn_norm") if gdn else ("q_norm", "k_norm")):
            put(p + n, L[n])
        for n, t in S.items():
            put(p + n, t)
    put("final_norm", w["final_norm"])
    putq("lm_head", w["lm_head"])
    put("hidden", hidden)
    put("proposals", proposals)
    fields = dict(hidden=cfg.hidden, block=cfg.block, gdn_heads=plan.gdn_heads,
                  gdn_key_heads=plan.gdn_key_heads or plan.gdn_heads, gdn_dk=cfg.gdn_dk, gdn_dv=cfg.gdn_dv,
                  conv_kernel=cfg.conv_kernel, attn_heads=plan.attn_heads, kv_heads=plan.kv_heads,
                  head_dim=cfg.head_dim, rotary_dim=cfg.rotary_dim, max_len=max_len, rope_theta=cfg.rope_theta,
                  eps=cfg.eps, group=cfg.group, bits=cfg.bits, context=context, keep=keep)
    lines += [f"cfg {k} {v!r}" for k, v in fields.items()]
    (d / "blob.bin").write_bytes(bytes(blob))
    (d / "manifest.txt").write_text("\n".join(lines) + "\n")


@pytest.mark.gpu
def test_host_cpp_drives_the_stack_object(cuda, tmp_path):
    """A C++ host runs one verify round through the C-ABI stack object alone (create,
    verify, forward, commit, advance) over a TP=1 tiny stack; its output, target tokens,
    accept count and the committed state equal, bit for bit, what the Python orchestration
    (verify_stack.VerifyStack) computes over the same buffers."""
    import sys
    from dataclasses import replace
    import numpy as np
    import torch
    sys.path.insert(0, str(PKG))
    import verify_stack as vs
    cfg = vs.TINY
    state = vs.build_rank_state(replace(cfg, block=3 * cfg.block), vs.shard_plan(cfg, 0, 1), 0, cuda)
    py = vs.VerifyStack(cfg, 0, 1, seed=0, device=cuda, state=state)
    hidden = vs.make_block(cfg, 0, cuda)
    proposals = torch.arange(7, 7 + cfg.block - 1, dtype=torch.int32, device=cuda)
    keep = 5
    max_len = next(S["cache_k"].shape[1] for S in py.state["layers"] if "cache_k" in S)
    _dump_stack(tmp_path, cfg, py.plan, py.w, py.state, py.context, hidden, proposals, keep, max_len)
    tok, acc = py.verify(hidden, proposals)
    want = {"out": py.out.clone(), "tokens": tok.clone(), "accepted": acc.clone()}
    py.commit(list(range(keep)))
    py.advance(keep)
    torch.cuda.synchronize()
    for i, S in enumerate(py.state["layers"]):
        for k, t in S.items():
            want[f"L{i}.{k}"] = t
    r = subprocess.run([str(_binary()), "stack", str(tmp_path)], capture_output=True, text=True, timeout=600)
    print(r.stdout, r.stderr)
    assert r.returncode == 0, r.stderr
    assert "0 failures" in r.stdout
    blob = (tmp_path / "result.bin").read_bytes()
    got = {}
    for line in (tmp_path / "result.txt").read_text().split("\n"):
        if line:
            name, off, n = line.split()
            got[name] = np.frombuffer(blob[int(off):int(off) + int(n)], dtype=np.uint8)
    assert set(got) == set(want)
    for name, t in want.items():
        assert np.array_equal(got[name], t.contiguous().cpu().view(torch.uint8).numpy().reshape(-1)), name

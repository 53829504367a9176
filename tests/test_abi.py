"""C-ABI surface tests that need no GPU: the library loads, exports every symbol the
header declares, and rejects bad arguments with the documented statuses before any
CUDA call is made."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "dflash_cuda.h"
HEADERS = sorted((ROOT / "include").glob("*.h"))
LIB = ROOT / "dflash-swift_b200" / "libdflashcuda.so"

FAKE = 0x10000  # a 16-byte aligned non-null pointer value; never dereferenced by these calls


def declared_functions():
    text = "\n".join(h.read_text() for h in HEADERS)
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dflash_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_expected_surface(dc):
    names = declared_functions()
    assert set(names) == set(dc.EXPORTED)


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (dflash_[a-z0-9_]+)\b", out))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, f"declared but not exported: {missing}"


def test_version_and_status_strings(dc):
    text = HEADER.read_text()
    assert dc.lib.dflash_version() == int(re.search(r"#define DFLASH_VERSION (\d+)", text).group(1))
    assert dc.lib.dflash_status_string(0) == b"ok"
    for st in range(1, 8):
        assert dc.lib.dflash_status_string(st) not in (b"ok", b"unknown status")
    assert dc.lib.dflash_status_string(99) == b"unknown status"


def _qmm(dc, M=8, N=4096, K=1024, group=64, bits=4, x=FAKE, w=FAKE, s=FAKE, b=FAKE, y=FAKE, ws=FAKE,
         ws_bytes=None):
    if ws_bytes is None:
        ws_bytes = dc.qmm_workspace_bytes(M, N, K, group, bits)
    return dc.lib.dflash_qmm(x, w, s, b, y, M, N, K, group, bits, ws, ws_bytes, None)


@pytest.mark.parametrize("kw,status", [
    (dict(M=17), 2), (dict(M=0), 2), (dict(bits=3), 2), (dict(bits=2), 2), (dict(group=96), 2),
    (dict(group=16), 2), (dict(K=1000), 1), (dict(N=0), 1), (dict(K=0), 1), (dict(x=0), 1), (dict(w=0), 1),
    (dict(s=0), 1), (dict(b=0), 1), (dict(y=0), 1), (dict(x=FAKE + 2), 3), (dict(w=FAKE + 4), 3),
    (dict(ws=0), 7), (dict(ws_bytes=16), 7), (dict(ws=FAKE + 8), 7),
])
def test_qmm_argument_errors(dc, kw, status):
    assert _qmm(dc, **kw) == status
    assert dc.last_error()


def test_qmm_noalloc_argument_errors(dc):
    """The no-allocation entry point validates like dflash_qmm, and rejects a shape
    whose scratch would not fit its static array before touching the GPU."""
    f = dc.lib.dflash_qmm_noalloc
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, 17, 4096, 1024, 64, 4, None) == 2
    assert f(0, FAKE, FAKE, FAKE, FAKE, 8, 4096, 1024, 64, 4, None) == 1
    assert f(FAKE + 2, FAKE, FAKE, FAKE, FAKE, 8, 4096, 1024, 64, 4, None) == 3
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, 16, 4096, 1 << 20, 64, 4, None) == 2
    assert "static" in dc.last_error() and "dflash_qmm" in dc.last_error()
    assert dc.qmm_workspace_bytes(16, 4096, 209664, 32, 4) <= 8 << 20 < dc.qmm_workspace_bytes(16, 4096, 209920, 32, 4)


def test_qmm_supported_table(dc):
    f = dc.lib.dflash_qmm_supported
    for bits in (4, 8):
        for g in (32, 64, 128):
            assert f(17408, 5120, g, bits) == 1
    assert f(4096, 1024, 64, 3) == 0
    assert f(4096, 1024, 96, 4) == 0
    assert f(4096, 1000, 64, 4) == 0
    assert f(0, 1024, 64, 4) == 0
    # wider than the reference's gate (N >= 4096, K % 512 == 0, group 64 only)
    assert f(2048, 1088, 64, 4) == 1
    assert f(17, 64, 32, 8) == 1


def test_workspace_size_is_shape_bounded(dc):
    """The workspace holds x packets for every stage along K: independent of N, growing
    with M (one or two n-tiles of 8 rows) and K, zero for shapes the kernel rejects."""
    a = dc.qmm_workspace_bytes(8, 17408, 5120, 64, 4)
    assert a == dc.qmm_workspace_bytes(8, 5120, 5120, 64, 4) == dc.qmm_workspace_bytes(1, 248320, 5120, 64, 4)
    # 20 stages of 256 k; per stage 4 units x 8 rows x 128 B of fp16 x plus 4 x 8 x 16 B of sums
    assert a == 20 * (4 * 8 * 128 + 4 * 8 * 16)
    assert dc.qmm_workspace_bytes(16, 17408, 5120, 64, 4) == 2 * a
    assert dc.qmm_workspace_bytes(8, 17408, 17408, 64, 4) > a
    assert dc.qmm_workspace_bytes(8, 17408, 5120, 64, 8) > a
    assert dc.qmm_workspace_bytes(8, 0, 5120, 64, 4) == 0
    assert dc.qmm_workspace_bytes(17, 17408, 5120, 64, 4) == 0
    assert dc.qmm_workspace_bytes(8, 17408, 5000, 64, 4) == 0


def _gdn_step(dc, T=8, H=4, dk=128, dv=128, si=FAKE, so=FAKE * 2, q=FAKE, k=FAKE, v=FAKE, a=FAKE, b=FAKE, out=0):
    return dc.lib.dflash_gdn_step(si, so, q, k, v, a, b, out, T, H, dk, dv, 1.0, None)


@pytest.mark.parametrize("kw,status", [
    (dict(T=0), 2), (dict(T=65), 2), (dict(dk=96), 2), (dict(dk=256), 2), (dict(dv=48), 2), (dict(dv=0), 2),
    (dict(H=0), 1), (dict(si=0), 1), (dict(k=0), 1), (dict(so=FAKE), 1), (dict(si=FAKE + 4), 3),
    (dict(out=FAKE, q=0), 1),
])
def test_gdn_step_argument_errors(dc, kw, status):
    assert _gdn_step(dc, **kw) == status


def test_gdn_replay_argument_errors(dc):
    r = dc.lib.dflash_gdn_replay
    ok_args = (FAKE, FAKE * 2, FAKE, FAKE, FAKE, FAKE)
    assert r(*ok_args, None, 0, 8, 2, 4, 128, 128, None) == 1          # keep 0
    assert r(*ok_args, None, 9, 8, 2, 4, 128, 128, None) == 1          # keep > width
    assert r(*ok_args, None, 3, 65, 2, 4, 128, 128, None) == 1         # width > 64
    assert r(*ok_args, None, 3, 8, 0, 4, 128, 128, None) == 1          # layers 0
    rows = (ctypes.c_int32 * 3)(0, 1, 8)                               # row outside [0, width)
    assert r(*ok_args, rows, 3, 8, 2, 4, 128, 128, None) == 1
    assert "rows[2]=8" in dc.last_error()
    assert r(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, None, 3, 8, 2, 4, 128, 128, None) == 1  # aliasing


def test_conv_rollback_argument_errors(dc):
    c = dc.lib.dflash_gdn_conv_rollback
    assert c(FAKE, FAKE, FAKE, None, 3, 8, 2, 3, 64, None) == 1        # aliasing
    assert c(FAKE, FAKE * 2, FAKE, None, 0, 8, 2, 3, 64, None) == 1    # keep 0
    assert c(FAKE, FAKE * 2, FAKE, None, 3, 8, 2, 0, 64, None) == 1    # kc1 0
    rows = (ctypes.c_int32 * 2)(0, -1)
    assert c(FAKE, FAKE * 2, FAKE, rows, 2, 8, 2, 3, 64, None) == 1


def test_bounded_wait_hook_argument_errors(dc):
    assert dc.lib.dflash_test_bounded_wait(0, None) == 1
    assert dc.lib.dflash_test_bounded_wait(10 ** 12, None) == 1


def test_last_error_is_thread_local(dc):
    import threading
    assert _qmm(dc, M=17) == 2
    main_msg = dc.last_error()
    seen = {}

    def worker():
        seen["before"] = dc.last_error()
        _qmm(dc, bits=3)
        seen["after"] = dc.last_error()

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert seen["before"] == ""
    assert "bits" in seen["after"]
    assert dc.last_error() == main_msg


def test_stack_argument_errors(dc):
    L = dc.lib
    # conv width outside 1..8, channels not divisible into the parts, null pointers
    assert L.dflash_stack_conv_silu(FAKE, 96, FAKE, FAKE, FAKE, 8, 96, 9, 3, None) == 2
    assert L.dflash_stack_conv_silu(FAKE, 96, FAKE, FAKE, FAKE, 8, 96, 4, 5, None) == 1
    assert L.dflash_stack_conv_silu(None, 96, FAKE, FAKE, FAKE, 8, 96, 4, 3, None) == 1
    # attention: unsupported head dim, rotary dims, cache overflow, ragged GQA grouping
    args = dict(ld=4096, M=8, hq=4, hkv=2, d=256, rot=64, pos0=0, max_len=64)
    def prep(**kw):
        a = {**args, **kw}
        return L.dflash_stack_attn_prep(FAKE, a["ld"], FAKE, FAKE, FAKE, FAKE, a["M"], a["hq"], a["hkv"], a["d"],
                                        a["rot"], a["pos0"], a["max_len"], 1e-6, 1e4, None)
    def dec(**kw):
        a = {**args, **kw}
        return L.dflash_stack_attn_decode(FAKE, a["ld"], FAKE, FAKE, FAKE, a["M"], a["hq"], a["hkv"], a["d"],
                                          a["pos0"], a["max_len"], 0.1, None)
    assert prep(d=96) == 2 and prep(rot=32) == 2 and prep(rot=320) == 2
    assert prep(pos0=60) == 1 and prep(ld=100) == 1
    assert dec(hq=3) == 1 and dec(pos0=57) == 1 and dec(d=32) == 2
    assert L.dflash_stack_add_rmsnorm(FAKE, None, FAKE, FAKE, 0, 64, 1e-6, None) == 1
    assert L.dflash_stack_silu_mul(FAKE, None, 8, 64, None) == 1
    assert L.dflash_stack_gdn_gates(FAKE, FAKE, FAKE, 8, FAKE, FAKE, None, FAKE, 8, 4, 128, None) == 1
    assert L.dflash_stack_gated_norm(FAKE, FAKE, 8, FAKE, FAKE, 8, 0, 128, 1e-6, None) == 1


def test_qmm_ex_tp_and_accept_argument_errors(dc):
    import ctypes
    L = dc.lib
    ws = dc.qmm_workspace_bytes(8, 1024, 1024, 64, 4)
    bases = (ctypes.c_void_p * 2)(FAKE, FAKE + 0x1000)

    def ex(**kw):
        o = dc.QmmOptions(kw.get("swiglu", 0), kw.get("push", 0), kw.get("rank", 0), kw.get("world", 1),
                          kw.get("set", 0), ctypes.cast(bases, ctypes.c_void_p) if kw.get("bases", True) else None,
                          kw.get("keys", None))
        return L.dflash_qmm_ex(FAKE, FAKE, FAKE, FAKE, kw.get("y", FAKE), 8, kw.get("N", 1024), 1024, 64, 4, FAKE, ws,
                               ctypes.addressof(o), None)

    assert ex(push=1, world=2, rank=2) == 1            # rank outside world
    assert ex(push=1, world=2, set=2) == 1
    assert ex(push=1, world=2, bases=False) == 1
    assert ex(push=1, world=2, N=1020) == 2            # pushing needs N % 8 == 0
    assert ex(push=1, world=2, keys=FAKE) == 1         # push and argmax are exclusive
    assert ex(keys=FAKE + 4) == 3                      # keys 8-byte aligned
    assert ex(y=0) == 1                                # no destination at all
    assert L.dflash_qmm_ex(FAKE, FAKE, FAKE, FAKE, FAKE, 8, 1024, 1020, 4, 4, FAKE, ws, None, None) == 2
    # accept
    assert L.dflash_accept(None, FAKE, 7, FAKE, FAKE, None) == 1
    assert L.dflash_accept(FAKE, None, 7, FAKE, FAKE, None) == 1
    assert L.dflash_accept(FAKE, FAKE, -1, FAKE, FAKE, None) == 1
    # exchange
    assert L.dflash_tp_exchange_bytes(9, 8, 5120) == 0 and L.dflash_tp_exchange_bytes(0, 8, 5120) == 0
    assert L.dflash_tp_exchange_bytes(8, 8, 5120) == 256 + 2 * 8 * 8 * 5120 // 2 * 8
    assert L.dflash_tp_push(FAKE, bases, 2, 2, 8, 5120, 0, None) == 1
    assert L.dflash_tp_push(FAKE, bases, 0, 2, 8, 5121, 0, None) == 3
    assert L.dflash_tp_push(FAKE + 2, bases, 0, 2, 8, 5120, 0, None) == 3
    assert L.dflash_stack_add_rmsnorm_reduce(FAKE, FAKE, 2, 2, FAKE, FAKE, 8, 5120, 1e-6, None) == 1
    assert L.dflash_stack_add_rmsnorm_reduce(FAKE, FAKE, 2, 0, FAKE, FAKE, 8, 5122, 1e-6, None) == 2
    assert L.dflash_stack_gdn_conv_gates(FAKE, 144, FAKE, FAKE, FAKE, FAKE, 8, FAKE, FAKE, FAKE, FAKE, 8, 1, 48, 4,
                                         None) == 2


def test_tree_entry_argument_errors(dc):
    """Tree rounds: a parent list is required, at most 32 rows, then the chain checks."""
    L = dc.lib
    cg = lambda parents, M=8, dk=128: L.dflash_stack_gdn_conv_gates_tree(
        FAKE, 3 * 4 * dk + 8, FAKE, FAKE, FAKE, FAKE, 8, FAKE, FAKE, FAKE, FAKE, M, 4, dk, 4, parents, None)
    assert cg(None) == 1 and cg(FAKE, M=33) == 1 and cg(FAKE, dk=48) == 2
    prep = lambda parents, M=8, d=256: L.dflash_stack_attn_prep_tree(
        FAKE, 4096, FAKE, FAKE, FAKE, FAKE, M, 4, 2, d, 64, 0, 64, 1e-6, 1e4, parents, None)
    assert prep(None) == 1 and prep(FAKE, M=40) == 1 and prep(FAKE, d=96) == 2
    dec = lambda parents, M=8, hq=4: L.dflash_stack_attn_decode_tree(
        FAKE, 4096, FAKE, FAKE, FAKE, M, hq, 2, 256, 0, 64, 0.1, parents, None)
    assert dec(None) == 1 and dec(FAKE, M=33) == 1 and dec(FAKE, hq=3) == 1
    step = lambda parents, T=8, dk=128, out=FAKE: L.dflash_gdn_step_tree(
        FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, parents, out, T, 4, dk, 128, 1.0, None)
    assert step(None) == 1 and step(FAKE, out=None) == 1
    assert step(FAKE, T=33) == 2 and step(FAKE, T=0) == 2 and step(FAKE, dk=96) == 2
    assert L.dflash_gdn_step_tree(FAKE + 4, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 8, 4, 128, 128, 1.0,
                                  None) == 3


def test_kv_compact_argument_errors(dc):
    L = dc.lib
    rows = lambda *r: (ctypes.c_int32 * len(r))(*r)
    kv = lambda ck=FAKE, cv=FAKE + 0x100000, layers=1, stride=0, d=128, pos0=30, max_len=40, r=rows(0, 2, 5), \
        keep=3: L.dflash_stack_kv_compact(ck, cv, layers, stride, 2, d, pos0, max_len, r, keep, None)
    assert kv(cv=FAKE) == 1                              # k and v must be distinct caches
    assert kv(r=rows(0, 2, 10)) == 1                     # pos0 + 10 is past max_len
    assert kv(r=rows(0, -1, 2)) == 1
    assert kv(keep=0) == 1 and kv(keep=33) == 1
    assert kv(layers=2, stride=100) == 1                 # layers would overlap
    assert kv(layers=2, stride=2 * 40 * 128 + 4) == 3    # layer stride not 16-byte aligned
    assert kv(d=96) == 2
    assert kv(ck=FAKE + 8) == 3
    assert L.dflash_stack_kv_compact(FAKE, FAKE + 0x100000, 1, 0, 2, 128, 30, 40, None, 3, None) == 1


def test_qmm_host_workspace_and_argument_errors(dc):
    L = dc.lib
    for (M, N, K, g, b) in [(8, 17408, 5120, 64, 4), (1, 4096, 1024, 32, 8), (16, 5120, 17408, 128, 4)]:
        base = L.dflash_qmm_workspace_bytes(M, N, K, g, b)
        r256 = lambda v: (v + 255) // 256 * 256
        assert L.dflash_qmm_host_workspace_bytes(M, N, K, g, b) == base + r256(2 * M * K) + r256(2 * M * N)
    assert L.dflash_qmm_host_workspace_bytes(17, 4096, 1024, 64, 4) == 0
    assert L.dflash_qmm_host_workspace_bytes(8, 4096, 1000, 64, 4) == 0
    need = L.dflash_qmm_host_workspace_bytes(8, 4096, 1024, 64, 4)
    h = lambda x=FAKE, w=FAKE, y=FAKE, ws=FAKE, nbytes=need, M=8, bits=4: L.dflash_qmm_host(
        x, w, FAKE, FAKE, y, M, 4096, 1024, 64, bits, ws, nbytes, None)
    assert h(x=None) == 1 and h(y=None) == 1
    assert h(w=FAKE + 4) == 3
    assert h(nbytes=need - 1) == 7 and h(ws=None) == 7 and h(ws=FAKE + 8) == 7
    assert h(M=17) == 2 and h(bits=3) == 2


def test_bias_add_argument_errors(dc):
    L = dc.lib
    assert L.dflash_bias_add(None, FAKE, 8, 4096, None) == 1
    assert L.dflash_bias_add(FAKE, None, 8, 4096, None) == 1
    assert L.dflash_bias_add(FAKE, FAKE, 0, 4096, None) == 1
    assert L.dflash_bias_add(FAKE, FAKE, 8, 0, None) == 1


def test_accept_tree_argument_errors(dc):
    L = dc.lib
    assert L.dflash_accept_tree(None, FAKE, FAKE, 8, FAKE, FAKE, FAKE, None) == 1
    assert L.dflash_accept_tree(FAKE, FAKE, FAKE, 0, FAKE, FAKE, FAKE, None) == 1
    assert L.dflash_accept_tree(FAKE, FAKE, FAKE, 33, FAKE, FAKE, FAKE, None) == 1
    assert L.dflash_accept_tree(FAKE, FAKE, FAKE, 8, FAKE, None, FAKE, None) == 1


def test_grouped_key_head_argument_errors(dc):
    L = dc.lib
    step = lambda heads=8, kh=4: L.dflash_gdn_step_grouped(FAKE, FAKE + 0x100000, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE,
                                                           8, heads, kh, 128, 128, 1.0, None)
    assert step(kh=3) == 1 and step(kh=0) == 1 and step(kh=16) == 1
    tree = lambda kh: L.dflash_gdn_step_tree_grouped(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 8, 8, kh, 128,
                                                     128, 1.0, None)
    assert tree(3) == 1 and tree(0) == 1
    replay = lambda kh: L.dflash_gdn_replay_grouped(FAKE, FAKE + 0x100000, FAKE, FAKE, FAKE, FAKE, None, 4, 8, 2, 8,
                                                    kh, 128, 128, None)
    assert replay(5) == 1 and replay(0) == 1
    cg = lambda heads=8, kh=4, ld=(2 * 4 + 8) * 64, M=8, parents=None, dk=64: L.dflash_stack_gdn_conv_gates_grouped(
        FAKE, ld, FAKE, FAKE, FAKE, FAKE, 16, FAKE, FAKE, FAKE, FAKE, M, heads, kh, dk, 4, parents, None)
    assert cg(kh=3) == 1 and cg(ld=100) == 1 and cg(M=33, parents=FAKE) == 1
    assert cg(dk=48, ld=(2 * 4 + 8) * 48) == 2


def test_attention_ex_argument_errors(dc):
    L = dc.lib
    prep = lambda M=8, pos0=0, parents=None, position=None, d=256: L.dflash_stack_attn_prep_ex(
        FAKE, 4096, FAKE, FAKE, FAKE, FAKE, M, 4, 2, d, 64, pos0, 64, 1e-6, 1e4, parents, position, None)
    assert prep(pos0=60) == 1                       # host position past the cache
    assert prep(M=33, parents=FAKE) == 1            # a tree has at most 32 rows
    assert prep(d=96, position=FAKE) == 2
    dec = lambda M=8, pos0=0, parents=None, position=None, hq=4: L.dflash_stack_attn_decode_ex(
        FAKE, 4096, FAKE, FAKE, FAKE, M, hq, 2, 256, pos0, 64, 0.1, parents, position, None)
    assert dec(pos0=57) == 1 and dec(M=33, parents=FAKE) == 1 and dec(hq=3, position=FAKE) == 1


def test_no_cpu_path_anywhere(tmp_path):
    """The product fails loudly without the CUDA library or a CUDA device: the binding
    refuses to import when libdflashcuda.so is missing, and the verify stack refuses a
    CPU device (there is no CPU fallback to run instead)."""
    import subprocess
    import sys
    code = ("import os, sys; os.environ['DFLASH_CUDA_LIB'] = sys.argv[1]; sys.path.insert(0, sys.argv[2])\n"
            "try:\n    import dflashcuda\nexcept ImportError as e:\n    print('refused:', e)\n")
    r = subprocess.run([sys.executable, "-c", code, str(tmp_path / "missing.so"), str(ROOT / "dflash-swift_b200")],
                       capture_output=True, text=True, timeout=120)
    assert "refused:" in r.stdout and "no CPU fallback" in r.stdout
    import verify_stack as vs
    with pytest.raises(RuntimeError, match="no CPU path"):
        vs.VerifyStack(vs.TINY, device="cpu")

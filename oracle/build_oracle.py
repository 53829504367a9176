"""Build recipe for the CPU checkers (TEST INFRASTRUCTURE; nothing here is shipped).

1. ``oracle/liboracle.so`` from this project's own C restatement
   (``qmm_oracle.c``, ``gdn_oracle.c``).
2. When the reference tree is present (this container only; the GPU box receives the
   prebuilt files), ``oracle/_ref/libref_metal_qmm.so``: the reference's own small-M
   Metal kernel text, extracted from the Swift string literals that hold it
   (Sources/DFlashKit/SmallMQuantizedMatmul.swift:55-71 unpack snippets and :80-165
   kernel body) and assembled the way ``SmallMQuantizedMatmul.source(tiles:)`` and the
   kernel table (:174-187) assemble it, then compiled for host cores against
   ``ref_metal/metal_shim.hpp``.  Nothing from the reference is written outside
   ``oracle/_ref/`` (git-ignored).

Usage: ``python oracle/build_oracle.py [--reference DIR]``.
"""
from __future__ import annotations

import argparse
import os
import re
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"
KERNEL_SWIFT = Path("Sources/DFlashKit/SmallMQuantizedMatmul.swift")


def build_oracle_lib() -> Path:
    out = HERE / "liboracle.so"
    srcs = [HERE / "qmm_oracle.c", HERE / "gdn_oracle.c"]
    if out.exists() and all(out.stat().st_mtime >= s.stat().st_mtime for s in srcs):
        return out
    cmd = ["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off",
           *map(str, srcs), "-o", str(out), "-lm"]
    subprocess.run(cmd, check=True)
    return out


def _swift_literal_after(text: str, anchor: str) -> str:
    """Return the body of the first Swift multi-line string literal after `anchor`."""
    i = text.index(anchor)
    start = text.index('"""', i) + 3
    end = text.index('"""', start)
    return text[start:end]


def _ternary_literal(text: str, name: str) -> tuple[str, str]:
    """`let name = tiles == 2 ? <literal> : ""` -> (literal for tiles==2, for tiles==1)."""
    i = text.index(f"let {name} =")
    seg = text[i:text.index("\n\n", i) if "\n\n" in text[i:] else len(text)]
    q = seg.index("?")
    after = seg[q + 1:].lstrip()
    if after.startswith('"""'):
        lit = after[3:after.index('"""', 3)]
    else:
        m = re.match(r'"((?:[^"\\]|\\.)*)"', after)
        lit = m.group(1)
    return lit, ""


def extract_kernel_sources(reference: Path) -> dict[tuple[int, int], str]:
    text = (reference / KERNEL_SWIFT).read_text()
    # the `4:` and `8:` keys of the unpack table each open one literal
    unpack = {b: _swift_literal_after(text[text.index(f'{b}: """'):], f"{b}: ") for b in (4, 8)}
    src_fn = text.index("private static func source(tiles: Int)")
    fn_text = text[src_fn:]
    body = _swift_literal_after(fn_text, "return ")
    pieces = {n: _ternary_literal(fn_text, n)
              for n in ("secondTileMMA", "secondTileDeclare", "secondTileStore", "secondTileLoad")}
    out = {}
    for bits in (4, 8):
        for tiles in (1, 2):
            s = body
            for n, (two, one) in pieces.items():
                s = s.replace(f"\\({n})", two if tiles == 2 else one)
            s = s.replace("\\(tiles)", str(tiles))
            s = s.replace("__UNPACK__", unpack[bits])
            assert "\\(" not in s, "unresolved Swift interpolation"
            # threadgroup arrays are shared by the running threadgroup's threads
            s = re.sub(r"threadgroup\s+(\w+)\s+(\w+)\[([^\]]+)\];", r"static \1 \2[\3];", s)
            out[(bits, tiles)] = s
    return out


def build_ref(reference: Path) -> Path | None:
    if not (reference / KERNEL_SWIFT).exists():
        return None
    REF_OUT.mkdir(exist_ok=True)
    for (bits, tiles), src in extract_kernel_sources(reference).items():
        (REF_OUT / f"metal_{bits}_{tiles}.inc").write_text(src)
    out = REF_OUT / "libref_metal_qmm.so"
    cmd = ["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-pthread", "-ffp-contract=off",
           "-w", f"-I{REF_OUT}", f"-I{HERE / 'ref_metal'}", str(HERE / "ref_metal" / "harness.cpp"),
           "-o", str(out)]
    subprocess.run(cmd, check=True)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DFLASH_REFERENCE_DIR", "/root/reference"))
    a = ap.parse_args(argv)
    print("oracle:", build_oracle_lib())
    ref = build_ref(Path(a.reference))
    print("reference kernel:", ref if ref else "reference tree absent; using prebuilt oracle/_ref if any")
    return 0


if __name__ == "__main__":
    sys.exit(main())

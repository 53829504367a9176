"""Generates tests/golden/qmm_ref_*.npz from the reference's own small-M kernel.

The outputs come from oracle/_ref/libref_metal_qmm.so: the Metal kernel text of
Sources/DFlashKit/SmallMQuantizedMatmul.swift (unpack :55-71, body :80-165, dispatch
:210-224) compiled for host cores by oracle/build_oracle.py, in the container where the
reference tree is mounted.  Inputs are not stored: they are regenerated from the seeds
by oracle.make_qmm_case, and a SHA-256 of each input tensor is stored so a drifting
generator or quantizer is caught instead of silently changing the case.

Cases: the reference test's shape (N=4096, K=1024; SmallMQuantizedMatmulTests.swift:
33-34, 82-92) at rows 8 and 16 (4-bit) and 8 (8-bit), plus a small shape (N=512,
K=512) at rows 1, 5 and 9 for both widths.  The reference kernel hard-codes group 64.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "oracle"))
import oracle as O  # noqa: E402

CASES = [
    # (M, N, K, bits, seed_x, seed_w)
    (8, 4096, 1024, 4, 0, 1),
    (16, 4096, 1024, 4, 0, 1),
    (8, 4096, 1024, 8, 0, 1),
    (1, 512, 512, 4, 5, 6),
    (5, 512, 512, 4, 5, 6),
    (9, 512, 512, 4, 5, 6),
    (1, 512, 512, 8, 5, 6),
    (5, 512, 512, 8, 5, 6),
    (9, 512, 512, 8, 5, 6),
]
GROUP = 64


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def case_name(M, N, K, bits, sx, sw) -> str:
    return f"qmm_ref_m{M}_n{N}_k{K}_b{bits}_s{sx}{sw}.npz"


def main() -> int:
    if not O.ref_available():
        print("oracle/_ref/libref_metal_qmm.so missing: run oracle/build_oracle.py where the reference is mounted")
        return 1
    for M, N, K, bits, sx, sw in CASES:
        x, wq, s, b = O.make_qmm_case(M, N, K, GROUP, bits, seed_x=sx, seed_w=sw)
        y = O.ref_metal_qmm(x, wq, s, b, bits)
        np.savez_compressed(HERE / case_name(M, N, K, bits, sx, sw), M=M, N=N, K=K, group=GROUP, bits=bits,
                            seed_x=sx, seed_w=sw, y_ref=y,
                            sha_x=digest(x), sha_w=digest(wq), sha_s=digest(s), sha_b=digest(b))
        print("wrote", case_name(M, N, K, bits, sx, sw))
    return 0


if __name__ == "__main__":
    sys.exit(main())

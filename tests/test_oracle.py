"""CPU tests of the oracle itself: pinned against the reference's own kernel.

The golden fixtures hold outputs of the reference's small-M Metal kernel text compiled
for host cores (tests/golden/make_golden.py).  The oracle's bf16-dequant flavour
restates that kernel's arithmetic (SmallMQuantizedMatmul.swift:59-71) with fp64
accumulation, so after rounding to bf16 it must agree to within one bf16 ulp
everywhere; anything else means a packing, indexing or dequant mistake.
"""
from __future__ import annotations

import glob
from pathlib import Path

import numpy as np
import pytest

GOLDEN = sorted(glob.glob(str(Path(__file__).parent / "golden" / "qmm_ref_*.npz")))


def _load_case(O, path):
    g = np.load(path)
    M, N, K, group, bits = (int(g[k]) for k in ("M", "N", "K", "group", "bits"))
    x, wq, s, b = O.make_qmm_case(M, N, K, group, bits, seed_x=int(g["seed_x"]), seed_w=int(g["seed_w"]))
    import hashlib
    for name, arr in (("x", x), ("w", wq), ("s", s), ("b", b)):
        assert hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest() == str(g[f"sha_{name}"]), \
            f"regenerated input {name} differs from the one the golden was made from"
    return (M, N, K, group, bits), (x, wq, s, b), g["y_ref"]


def test_golden_fixtures_present():
    assert len(GOLDEN) >= 9


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: Path(p).stem)
def test_oracle_matches_reference_kernel_golden(O, path):
    (M, N, K, group, bits), (x, wq, s, b), y_ref = _load_case(O, path)
    y = O.bf16_bits(O.qmm_f64(x, wq, s, b, group, bits, O.FLAVOUR_BF16DQ))
    ulp = np.abs(y.astype(np.int32) - y_ref.astype(np.int32))
    assert ulp.max() <= 1, f"oracle vs reference kernel: {ulp.max()} bf16 ulps"
    assert (ulp == 0).mean() > 0.99
    # the exact-dequant flavour (what the CUDA kernel computes) is within the
    # reference test's tolerance of the reference kernel too
    assert O.closeness(O.bits_to_f32(y_ref), O.qmm_f64(x, wq, s, b, group, bits)) <= 1e-2


@pytest.mark.parametrize("path", GOLDEN[:1], ids=lambda p: Path(p).stem)
def test_negative_control_wrong_nibble_order_fails(O, path):
    """A kernel that read the nibbles high-first would still produce a plausible
    tensor; the golden comparison must reject it."""
    (M, N, K, group, bits), (x, wq, s, b), y_ref = _load_case(O, path)
    assert bits == 4
    swapped = np.zeros_like(wq)
    for t in range(8):
        swapped |= ((wq >> np.uint32(4 * t)) & np.uint32(15)) << np.uint32(4 * (7 - t))
    y_bad = O.qmm_f64(x, swapped, s, b, group, bits)
    assert O.closeness(O.bits_to_f32(y_ref), y_bad) > 1e-2


@pytest.mark.parametrize("path", GOLDEN[:1], ids=lambda p: Path(p).stem)
def test_negative_control_wrong_group_size_fails(O, path):
    (M, N, K, group, bits), (x, wq, s, b), y_ref = _load_case(O, path)
    # read the same scales as if the groups were 128 wide
    s2 = np.ascontiguousarray(s[:, ::2])
    b2 = np.ascontiguousarray(b[:, ::2])
    y_bad = O.qmm_f64(x, wq, s2, b2, 128, bits)
    assert O.closeness(O.bits_to_f32(y_ref), y_bad) > 1e-2


@pytest.mark.skipif(not __import__("oracle").ref_available(), reason="reference kernel not compiled here")
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [1, 6, 8, 12, 16])
def test_oracle_matches_reference_kernel_live(O, bits, M):
    x, wq, s, b = O.make_qmm_case(M, 96, 512, 64, bits, seed_x=11, seed_w=7)
    y_ref = O.ref_metal_qmm(x, wq, s, b, bits)
    y = O.bf16_bits(O.qmm_f64(x, wq, s, b, 64, bits, O.FLAVOUR_BF16DQ))
    assert np.abs(y.astype(np.int32) - y_ref.astype(np.int32)).max() <= 1


def test_packing_is_low_nibble_first(O):
    """Hand-built word: codes 0..7 at k = 0..7 must pack as 0x76543210
    (SmallMQuantizedMatmul.swift:57-61: value t is (p >> 4t) & 15)."""
    K, group = 64, 64
    w = np.zeros((1, K), dtype=np.float32)
    w[0, :8] = np.arange(8, dtype=np.float32)
    w[0, 8:] = 15.0
    wq, s, b = O.quantize(w, group, 4, refine=False)
    assert O.bits_to_f32(s)[0, 0] == 1.0 and O.bits_to_f32(b)[0, 0] == 0.0
    assert wq[0, 0] == 0x76543210
    deq = O.dequantize(wq, s, b, K, group, 4)
    assert np.array_equal(deq, w)


def test_packing_8bit_byte_order(O):
    K, group = 64, 64
    w = np.zeros((1, K), dtype=np.float32)
    w[0, :4] = [1, 2, 3, 4]
    w[0, 4] = 0.0
    w[0, 5:] = 255.0
    wq, s, b = O.quantize(w, group, 8, refine=False)
    assert wq[0, 0] == 0x04030201
    assert np.array_equal(O.dequantize(wq, s, b, K, group, 8), w)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("refine", [True, False])
def test_quantizer_error_bound(O, bits, group, refine):
    """Each dequantised value is within half a step of the original plus bf16 rounding
    of scale and bias: |w - deq| <= |s|/2 + ulp terms.  The refined (MLX) quantizer
    trades range for an exactly representable edge, so values at the far edge may be
    clamped by up to one more step: its bound is |s|."""
    r = np.random.Generator(np.random.PCG64(3))
    w = r.standard_normal((16, 512), dtype=np.float32) * np.float32(0.02)
    wq, s, b = O.quantize(w, group, bits, refine)
    deq = O.dequantize(wq, s, b, 512, group, bits)
    sf = np.repeat(np.abs(O.bits_to_f32(s)), group, axis=1)
    bf = np.repeat(np.abs(O.bits_to_f32(b)), group, axis=1)
    levels = (1 << bits) - 1
    bound = (1.0 if refine else 0.5) * sf + (2 ** -8) * (levels * sf + bf) + 1e-7
    assert np.all(np.abs(w - deq) <= bound)


def test_refined_quantizer_represents_zero_exactly(O):
    """MLX's refinement makes the larger-magnitude edge exactly representable, which
    puts 0 on the grid: q0 * s + b == 0 for q0 = -edge/s (up to bf16 rounding of s)."""
    r = np.random.Generator(np.random.PCG64(4))
    w = r.standard_normal((8, 256), dtype=np.float32)
    wq, s, b = O.quantize(w, 64, 4, True)
    sf, bf = O.bits_to_f32(s).astype(np.float64), O.bits_to_f32(b).astype(np.float64)
    q0 = -bf / sf
    assert np.all(np.abs(q0 - np.rint(q0)) < 0.05)


def test_cpu_restatement_matches_f64(O):
    x, wq, s, b = O.make_qmm_case(8, 300, 1024, 64, 4)
    y, used = O.qmm_cpu(x, wq, s, b, 64, 4)
    assert used >= 1
    assert O.closeness(O.bits_to_f32(y), O.qmm_f64(x, wq, s, b, 64, 4)) <= 4e-3


def test_closeness_measure_matches_reference_definition(O):
    ref = np.array([[0.5, -3.0]])
    assert O.closeness(ref + np.array([[0.0, 0.06]]), ref) == pytest.approx(0.02)
    small = np.array([[0.1, -0.2]])
    assert O.closeness(small + 0.01, small) == pytest.approx(0.01)

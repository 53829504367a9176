"""Python face of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import this module, and
only as the checker or the timed CPU baseline.  The CUDA product path never does.

Wraps ``liboracle.so`` (this project's C restatement, see qmm_oracle.c and
gdn_oracle.c for the reference citations) and, when present,
``_ref/libref_metal_qmm.so`` (the reference's own small-M Metal kernel text compiled
for host cores by build_oracle.py).  Also holds the seeded input generators shared by
tests and bench: numpy PCG64, x seed 0, W seed 1, gated-delta seed 2; bf16 through
ml_dtypes.
"""
from __future__ import annotations

import ctypes
import subprocess
import sys
from pathlib import Path

import ml_dtypes
import numpy as np

HERE = Path(__file__).resolve().parent
BF16 = ml_dtypes.bfloat16

FLAVOUR_EXACT = 0    # fp32 q*s+b (stock quantizedMatmul semantics)
FLAVOUR_BF16DQ = 1   # bf16(q*s+b) (reference Metal kernel, SmallMQuantizedMatmul.swift:59)

_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_c_i = ctypes.c_int

_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        so = HERE / "liboracle.so"
        if not so.exists():
            subprocess.run([sys.executable, str(HERE / "build_oracle.py")], check=True)
        L = ctypes.CDLL(str(so))
        L.oracle_quantize_affine.argtypes = [_f32p, _c_i, _c_i, _c_i, _c_i, _c_i, _u32p, _u16p, _u16p]
        L.oracle_quantize_affine.restype = None
        L.oracle_dequantize.argtypes = [_u32p, _u16p, _u16p, _c_i, _c_i, _c_i, _c_i, _c_i, _f32p]
        L.oracle_dequantize.restype = None
        L.oracle_qmm_f64.argtypes = [_u16p, _u32p, _u16p, _u16p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _f64p]
        L.oracle_qmm_f64.restype = None
        L.oracle_qmm_bf16_fp32acc.argtypes = [_u16p, _u32p, _u16p, _u16p, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i, _c_i,
                                              _c_i, _u16p]
        L.oracle_qmm_bf16_fp32acc.restype = _c_i
        L.oracle_gdn_recurrence.argtypes = [_f32p, ctypes.c_void_p, _u16p, _u16p, _f32p, _f32p, ctypes.c_void_p,
                                            _c_i, _c_i, _c_i, _c_i, ctypes.c_double, _f64p, ctypes.c_void_p]
        L.oracle_gdn_recurrence.restype = None
        L.oracle_conv_window.argtypes = [_u16p, _u16p, ctypes.c_void_p, _c_i, _c_i, _c_i, _u16p]
        L.oracle_conv_window.restype = None
        _lib = L
    return _lib


def ref_available() -> bool:
    return (HERE / "_ref" / "libref_metal_qmm.so").exists()


def ref():
    """The reference's Metal kernel text compiled for host cores (None if not built)."""
    global _ref
    if _ref is None and ref_available():
        R = ctypes.CDLL(str(HERE / "_ref" / "libref_metal_qmm.so"))
        R.ref_metal_qmm.argtypes = [_u16p, _u32p, _u16p, _u16p, _u16p, _c_i, _c_i, _c_i, _c_i]
        R.ref_metal_qmm.restype = _c_i
        _ref = R
    return _ref


# ----------------------------------------------------------------------------- bf16 helpers

def bf16_bits(a: np.ndarray) -> np.ndarray:
    """float array -> bf16 bit patterns (uint16), round to nearest even."""
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32).astype(BF16).view(np.uint16))


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------- qmm

def quantize(w: np.ndarray, group: int, bits: int, refine: bool = True):
    """MLX affine quantisation of fp32 [N, K] -> (packed u32 [N, K*bits/32], scales u16, biases u16)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    wq = np.zeros((N, K * bits // 32), dtype=np.uint32)
    s = np.zeros((N, K // group), dtype=np.uint16)
    b = np.zeros((N, K // group), dtype=np.uint16)
    lib().oracle_quantize_affine(w, N, K, group, bits, int(refine), wq, s, b)
    return wq, s, b


def dequantize(wq, s, b, K: int, group: int, bits: int, flavour: int = FLAVOUR_EXACT) -> np.ndarray:
    N = wq.shape[0]
    out = np.empty((N, K), dtype=np.float32)
    lib().oracle_dequantize(np.ascontiguousarray(wq), np.ascontiguousarray(s), np.ascontiguousarray(b), N, K, group,
                            bits, flavour, out)
    return out


def qmm_f64(x_bits, wq, s, b, group: int, bits: int, flavour: int = FLAVOUR_EXACT) -> np.ndarray:
    """fp64 y[M, N] of x . deq(W)^T."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    M, K = x_bits.shape
    N = wq.shape[0]
    y = np.empty((M, N), dtype=np.float64)
    lib().oracle_qmm_f64(x_bits, np.ascontiguousarray(wq), np.ascontiguousarray(s), np.ascontiguousarray(b), M, N, K,
                         group, bits, flavour, y)
    return y


def qmm_cpu(x_bits, wq, s, b, group: int, bits: int, n_begin: int = 0, n_end=None, threads: int = 0, out=None):
    """The timed CPU restatement: fp32 accumulate, bf16 out, OpenMP over N.
    Returns (y bits [M, N], threads used)."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    M, K = x_bits.shape
    N = wq.shape[0]
    n_end = N if n_end is None else n_end
    y = out if out is not None else np.zeros((M, N), dtype=np.uint16)
    used = lib().oracle_qmm_bf16_fp32acc(x_bits, wq, s, b, M, N, K, group, bits, n_begin, n_end, threads, y)
    return y, used


def ref_metal_qmm(x_bits, wq, s, b, bits: int) -> np.ndarray:
    """Reference Metal kernel on host cores: group 64 only, K % 512 == 0, rows 1..16."""
    R = ref()
    if R is None:
        raise RuntimeError("oracle/_ref/libref_metal_qmm.so is not built")
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    M, K = x_bits.shape
    N = wq.shape[0]
    out = np.zeros((M, N), dtype=np.uint16)
    rc = R.ref_metal_qmm(x_bits, np.ascontiguousarray(wq), np.ascontiguousarray(s), np.ascontiguousarray(b), out, M, N,
                         K, bits)
    if rc != 0:
        raise ValueError(f"reference kernel has no variant for M={M} K={K} bits={bits}")
    return out


def make_x(M: int, K: int, seed_x: int = 0, x_scale: float = 1.0) -> np.ndarray:
    """x ~ N(0, x_scale) as bf16 bits [M, K] (numpy PCG64)."""
    rx = np.random.Generator(np.random.PCG64(seed_x))
    return bf16_bits(rx.standard_normal((M, K), dtype=np.float32) * np.float32(x_scale))


def make_weights(N: int, K: int, group: int, bits: int, seed_w: int = 1, w_scale: float = 0.02,
                 refine: bool = True):
    """W ~ N(0, w_scale) [N, K] quantized with the MLX affine scheme."""
    rw = np.random.Generator(np.random.PCG64(seed_w))
    w = rw.standard_normal((N, K), dtype=np.float32) * np.float32(w_scale)
    return quantize(w, group, bits, refine)


def make_qmm_case(M: int, N: int, K: int, group: int, bits: int, seed_x: int = 0, seed_w: int = 1,
                  x_scale: float = 1.0, w_scale: float = 0.02, refine: bool = True):
    """Seeded inputs of the benchmark configs: x ~ N(0, x_scale) bf16 [M, K];
    W ~ N(0, w_scale) [N, K] quantized (MLX affine)."""
    x = make_x(M, K, seed_x, x_scale)
    wq, s, b = make_weights(N, K, group, bits, seed_w, w_scale, refine)
    return x, wq, s, b


def closeness(y, ref) -> float:
    """max|y - ref| / max(max|ref|, 1): the reference test's measure
    (Tests/DFlashKitTests/SmallMQuantizedMatmulTests.swift:65-80)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(y - ref)) / max(float(np.max(np.abs(ref))), 1.0))


# ----------------------------------------------------------------------------- gated delta

def gdn_recurrence(s0, k_bits, v_bits, alpha, beta, n_rows: int, rows=None, q_bits=None, q_scale: float = 1.0):
    """One layer: s0 fp32 [H, dv, dk]; k [T, H, dk]; v [T, H, dv]; alpha/beta [T, H].
    Returns (state fp64 [H, dv, dk], outputs fp64 [n_rows, H, dv] or None)."""
    s0 = np.ascontiguousarray(s0, dtype=np.float32)
    H, dv, dk = s0.shape
    s_out = np.empty_like(s0, dtype=np.float64)
    o = np.empty((n_rows, H, dv), dtype=np.float64) if q_bits is not None else None
    rows_arr = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    lib().oracle_gdn_recurrence(
        s0,
        None if q_bits is None else np.ascontiguousarray(q_bits, dtype=np.uint16).ctypes.data,
        np.ascontiguousarray(k_bits, dtype=np.uint16), np.ascontiguousarray(v_bits, dtype=np.uint16),
        np.ascontiguousarray(alpha, dtype=np.float32), np.ascontiguousarray(beta, dtype=np.float32),
        None if rows_arr is None else rows_arr.ctypes.data, n_rows, H, dk, dv, float(q_scale), s_out,
        None if o is None else o.ctypes.data)
    return s_out, o


def conv_window(window_bits, conv_in_bits, keep: int, rows=None) -> np.ndarray:
    window_bits = np.ascontiguousarray(window_bits, dtype=np.uint16)
    kc1, C = window_bits.shape
    out = np.empty_like(window_bits)
    rows_arr = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    lib().oracle_conv_window(window_bits, np.ascontiguousarray(conv_in_bits, dtype=np.uint16),
                             None if rows_arr is None else rows_arr.ctypes.data, keep, kc1, C, out)
    return out


def make_gdn_case(layers: int, width: int, heads: int, dk: int, dv: int, seed: int = 2, state_scale: float = 0.1):
    """Seeded capture of one verify round (config 5 distributions): q/v ~ N(0,1) bf16,
    k ~ N(0,1) L2-normalised per head then bf16, alpha ~ U(0.9, 1), beta ~ U(0, 1),
    snapshot ~ N(0, state_scale) fp32."""
    r = np.random.Generator(np.random.PCG64(seed))
    snap = (r.standard_normal((layers, heads, dv, dk), dtype=np.float32) * np.float32(state_scale))
    q = r.standard_normal((layers, width, heads, dk), dtype=np.float32)
    k = r.standard_normal((layers, width, heads, dk), dtype=np.float32)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = r.standard_normal((layers, width, heads, dv), dtype=np.float32)
    alpha = r.uniform(0.9, 1.0, (layers, width, heads)).astype(np.float32)
    beta = r.uniform(0.0, 1.0, (layers, width, heads)).astype(np.float32)
    return dict(snapshot=np.ascontiguousarray(snap), q=bf16_bits(q), k=bf16_bits(k), v=bf16_bits(v),
                alpha=alpha, beta=beta)


# ----------------------------------------------------------------------------- accept

def accepted_prefix(logits_bits, proposals):
    """Greedy accept of a verify round (DFlashSpeculativeGenerator.swift:555-571):
    target tokens = argmax over the vocabulary of each row of the bf16 logits (first
    index among equal maxima, as argMax does), match[i] = proposals[i] == tokens[i] for
    i < drafts, accepted = sum(cumprod(match)).  Returns (tokens int32 [drafts + 1],
    accepted)."""
    logits = bits_to_f32(np.asarray(logits_bits, dtype=np.uint16))
    tokens = np.argmax(logits, axis=-1).astype(np.int32)
    proposals = np.asarray(proposals, dtype=np.int32)
    drafts = proposals.shape[0]
    assert logits.shape[0] == drafts + 1
    match = (proposals == tokens[:drafts]).astype(np.int32)
    return tokens, int(np.cumprod(match).sum())

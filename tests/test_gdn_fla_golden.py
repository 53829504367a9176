"""Gated-delta parity pinned to an independent implementation.

tests/golden/gdn_fla_*.npz hold what flash-linear-attention's plain PyTorch recurrence
(fla 0.5.1, `naive_recurrent_gated_delta_rule`) computes on seeded config-5-shaped
inputs (made by tests/golden/make_gdn_golden.py): the state after each kept prefix of a
round, and the per-position outputs.  They fix the convention the reference's un-vendored
fork leaves open (decay first, then the delta rule; alpha = exp(g); o_t = S_t q_t):
  * CPU: the fp64 oracle reproduces them, and the other order (delta rule, then decay)
    does not (negative control);
  * GPU: dflash_gdn_step over the whole round and dflash_gdn_replay of every kept prefix
    reproduce the fp32 states within 1e-4 of the largest value (the north star's replay
    bound), and the step's bf16 outputs within their rounding.
"""
from __future__ import annotations

import glob
import hashlib
from pathlib import Path

import numpy as np
import pytest

FIXTURES = sorted(glob.glob(str(Path(__file__).parent / "golden" / "gdn_fla_*.npz")))
REL = 1e-4      # fp32 states
OUT_REL = 4e-3  # the step's bf16 outputs: one bf16 rounding (2^-9 relative) of each value


def rel(got, want) -> float:
    got, want = np.asarray(got, dtype=np.float64), np.asarray(want, dtype=np.float64)
    return float(np.abs(got - want).max() / np.abs(want).max())


def load(O, path):
    z = np.load(path)
    L, W, H, dk, dv, seed = (int(v) for v in z["case"])
    c = O.make_gdn_case(L, W, H, dk, dv, seed=seed)
    for key in ("snapshot", "q", "k", "v", "alpha", "beta"):
        assert hashlib.sha256(np.ascontiguousarray(c[key]).tobytes()).hexdigest() == str(z[f"sha_{key}"]), key
    return z, c, (L, W, H, dk, dv), [int(k) for k in z["keeps"]], float(z["q_scale"])


def test_fixtures_present():
    assert len(FIXTURES) == 2


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: Path(p).stem)
def test_oracle_matches_fla(O, path):
    z, c, (L, W, H, dk, dv), keeps, qs = load(O, path)
    for layer in range(L):
        for keep in keeps:
            s, _ = O.gdn_recurrence(c["snapshot"][layer], c["k"][layer], c["v"][layer], c["alpha"][layer],
                                    c["beta"][layer], keep)
            assert rel(s, z[f"state_keep{keep}"][layer]) <= 1e-5, (layer, keep)
        _, o = O.gdn_recurrence(c["snapshot"][layer], c["k"][layer], c["v"][layer], c["alpha"][layer],
                                c["beta"][layer], W, q_bits=c["q"][layer], q_scale=qs)
        assert rel(o, z["o"][layer]) <= 1e-5, layer


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: Path(p).stem)
def test_other_update_order_is_rejected(O, path):
    """Negative control: applying the decay after the delta rule, S <- alpha (S + beta (v -
    S k) k^T), is a different recurrence, and the fixtures tell the two apart."""
    z, c, (L, W, H, dk, dv), keeps, _ = load(O, path)
    f = O.bits_to_f32
    S = c["snapshot"][0].astype(np.float64)
    k, v = f(c["k"][0]).astype(np.float64), f(c["v"][0]).astype(np.float64)
    for t in range(W):
        for h in range(H):
            u = c["beta"][0, t, h] * (v[t, h] - S[h] @ k[t, h])
            S[h] = c["alpha"][0, t, h] * (S[h] + np.outer(u, k[t, h]))
    assert rel(S, z[f"state_keep{W}"][0]) > 100 * REL


def _dev(a, d):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).to(d).view(torch.bfloat16)
    return torch.from_numpy(a).to(d)


@pytest.mark.gpu
@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: Path(p).stem)
def test_step_matches_fla(dc, O, cuda, path):
    import torch
    z, c, (L, W, H, dk, dv), keeps, qs = load(O, path)
    for layer in range(L):
        snap = _dev(c["snapshot"][layer], cuda)
        state = torch.empty_like(snap)
        out = torch.empty((W, H, dv), dtype=torch.bfloat16, device=cuda)
        dc.gdn_step(snap, state, _dev(c["q"][layer], cuda), _dev(c["k"][layer], cuda), _dev(c["v"][layer], cuda),
                    _dev(c["alpha"][layer], cuda), _dev(c["beta"][layer], cuda), out=out, q_scale=qs)
        torch.cuda.synchronize()
        assert rel(state.cpu().numpy(), z[f"state_keep{W}"][layer]) <= REL, layer
        assert rel(out.float().cpu().numpy(), z["o"][layer]) <= OUT_REL, layer
    assert dc.device_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: Path(p).stem)
def test_replay_matches_fla(dc, O, cuda, path):
    import torch
    z, c, (L, W, H, dk, dv), keeps, _ = load(O, path)
    snap = _dev(c["snapshot"], cuda)
    for keep in keeps:
        state = torch.full_like(snap, float("nan"))
        dc.gdn_replay(snap, state, _dev(c["k"], cuda), _dev(c["v"], cuda), _dev(c["alpha"], cuda),
                      _dev(c["beta"], cuda), keep=keep)
        torch.cuda.synchronize()
        assert rel(state.cpu().numpy(), z[f"state_keep{keep}"]) <= REL, keep
    assert dc.device_error() == 0

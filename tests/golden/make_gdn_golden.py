"""Generates tests/golden/gdn_fla_*.npz: the gated-delta recurrence as an independent,
published implementation computes it, for pinning this project's oracle and kernels.

The reference's capture/replay lives in an un-vendored fork (random1st/mlx-swift-lm,
branch dflash-multilayer-tap); its tests pin only properties (replay(keep) equals a
committed forward over keep positions, GatedDeltaRollbackTests.swift:84-111).  The
recurrence's convention (decay applied before the delta rule, the gate as a log-decay)
is fixed here against flash-linear-attention's plain PyTorch recurrence,
`fla.ops.gated_delta_rule.naive.naive_recurrent_gated_delta_rule` (fla 0.5.1, installed
in this image), which this script RUNS; nothing of it is copied.  fla's recurrence per
head, in its own layout (state h [dk, dv]):
    h <- h * exp(g_t);  u = beta_t (v_t - h^T k_t);  h <- h + k_t u^T;  o_t = h^T (scale q_t)
which is this project's S [dv, dk] = h^T with alpha = exp(g).

Inputs are not stored: they come from oracle.make_gdn_case(seed) (config 5's
distributions: k L2-normalised then bf16, alpha ~ U(0.9, 1), beta ~ U(0, 1)); a SHA-256
of each input is stored so a drifting generator is caught.  Stored outputs (fp32): the
state after each kept prefix (keep in KEEPS) and the per-position outputs o of the full
round.

    python tests/golden/make_gdn_golden.py
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "oracle"))
import oracle as O  # noqa: E402

# (layers, width, heads, dk, dv, seed): config 5's head size (128 x 128, width 8) on a
# few heads, and a smaller head size
CASES = [(1, 8, 2, 128, 128, 71), (2, 8, 2, 64, 64, 72)]
KEEPS = (1, 3, 8)
Q_SCALE = 0.5  # a non-default scale, so that the output convention is pinned too


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def name(case) -> str:
    L, W, H, dk, dv, seed = case
    return f"gdn_fla_l{L}_w{W}_h{H}_dk{dk}_dv{dv}_s{seed}.npz"


def fla_round(c, layer: int, keep: int):
    """fla's recurrence over the first `keep` positions of one layer, from the snapshot."""
    import torch
    from fla.ops.gated_delta_rule.naive import naive_recurrent_gated_delta_rule as fla

    f32 = lambda bits: torch.from_numpy(O.bits_to_f32(bits[layer, :keep]).copy())[None]  # [1, T, H, d]
    q, k, v = f32(c["q"]), f32(c["k"]), f32(c["v"])
    g = torch.from_numpy(np.log(c["alpha"][layer, :keep].astype(np.float64)).astype(np.float32))[None]
    beta = torch.from_numpy(c["beta"][layer, :keep].copy())[None]
    h0 = torch.from_numpy(c["snapshot"][layer].copy()).transpose(-1, -2).contiguous()[None]  # [1, H, dk, dv]
    o, h = fla(q, k, v, beta, g, scale=Q_SCALE, initial_state=h0, output_final_state=True)
    state = h[0].transpose(-1, -2).contiguous().numpy()  # [H, dv, dk]
    return state.astype(np.float32), o[0].numpy().astype(np.float32)  # o: [T, H, dv]


def main() -> None:
    for case in CASES:
        L, W, H, dk, dv, seed = case
        c = O.make_gdn_case(L, W, H, dk, dv, seed=seed)
        out = {"case": np.array(case, dtype=np.int64), "keeps": np.array(KEEPS, dtype=np.int64),
               "q_scale": np.array(Q_SCALE, dtype=np.float64)}
        for key in ("snapshot", "q", "k", "v", "alpha", "beta"):
            out[f"sha_{key}"] = np.array(sha(c[key]))
        for keep in KEEPS:
            out[f"state_keep{keep}"] = np.stack([fla_round(c, layer, keep)[0] for layer in range(L)])
        out["o"] = np.stack([fla_round(c, layer, W)[1] for layer in range(L)])  # [L, W, H, dv]
        np.savez_compressed(HERE / name(case), **out)
        print("wrote", name(case))


if __name__ == "__main__":
    main()

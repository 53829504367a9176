"""GPU tests of the gated-delta step (capture) and rollback replay.

The property the reference's rollback tests pin (GatedDeltaRollbackTests.swift:84-111):
after a round of `width` positions is rolled back to `keep`, the recurrent state equals
what a committed forward over those `keep` positions leaves.  Here: replay(keep) from
the snapshot vs dflash_gdn_step over the first `keep` positions (same device
arithmetic, so bit-identical), and both vs the fp64 oracle within 1e-4 relative.  The
reference's negative controls (no rollback; a rollback one position too deep,
:131-162) must diverge by more than its 2e-3 bound.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 1e-4


def dev(a, d):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).to(d).view(torch.bfloat16)
    return torch.from_numpy(a).to(d)


def rel_err(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.abs(got - want).max() / max(1.0, np.abs(want).max()))


def step_layer(dc, d, c, layer, T, with_out=True):
    import torch
    snap = dev(c["snapshot"][layer], d)
    out_state = torch.empty_like(snap)
    H, dk = c["k"].shape[2], c["k"].shape[3]
    dv = c["v"].shape[3]
    o = torch.empty((T, H, dv), dtype=torch.bfloat16, device=d) if with_out else None
    dc.gdn_step(snap, out_state, dev(c["q"][layer, :T], d), dev(c["k"][layer, :T], d), dev(c["v"][layer, :T], d),
                dev(c["alpha"][layer, :T], d), dev(c["beta"][layer, :T], d), out=o, q_scale=dk ** -0.5)
    torch.cuda.synchronize()
    return out_state, o


@pytest.mark.parametrize("dk,dv,H", [(128, 128, 4), (32, 32, 2), (64, 128, 3)])
@pytest.mark.parametrize("T", [1, 3, 8, 16])
def test_step_matches_oracle(dc, O, cuda, dk, dv, H, T):
    c = O.make_gdn_case(1, T, H, dk, dv, seed=2)
    st, o = step_layer(dc, cuda, c, 0, T)
    want_s, want_o = O.gdn_recurrence(c["snapshot"][0], c["k"][0], c["v"][0], c["alpha"][0], c["beta"][0], T,
                                      q_bits=c["q"][0], q_scale=dk ** -0.5)
    assert rel_err(st.cpu().numpy(), want_s) <= REL
    assert rel_err(o.float().cpu().numpy(), want_o) <= 1e-2  # bf16 outputs


@pytest.mark.parametrize("decays", ["halving", "vanishing", "zero", "none"])
def test_decay_extremes_over_long_rounds(dc, O, cuda, decays):
    """64 positions whose decays halve the state at every position (2^-64 of it left at the
    end), drop it to 1e-30 or to 0 at once, or never decay it: the step stays within the
    fp64 oracle's tolerance and the replay reproduces it bit for bit."""
    import torch
    T, H, dk, dv = 64, 2, 128, 128
    c = O.make_gdn_case(1, T, H, dk, dv, seed=9)
    a = c["alpha"]
    if decays == "halving":
        a[:] = 0.5
    elif decays == "vanishing":
        a[:, ::7] = 1e-30
    elif decays == "zero":
        a[:, 5::11] = 0.0
    else:
        a[:] = 1.0
    c["alpha"] = np.ascontiguousarray(a, dtype=np.float32)
    st, _ = step_layer(dc, cuda, c, 0, T, with_out=False)
    want, _ = O.gdn_recurrence(c["snapshot"][0], c["k"][0], c["v"][0], c["alpha"][0], c["beta"][0], T)
    assert rel_err(st.cpu().numpy(), want) <= REL
    snap = dev(c["snapshot"], cuda)
    replayed = torch.empty_like(snap)
    dc.gdn_replay(snap, replayed, dev(c["k"], cuda), dev(c["v"], cuda), dev(c["alpha"], cuda), dev(c["beta"], cuda),
                  keep=T)
    torch.cuda.synchronize()
    assert torch.equal(replayed[0], st)


@pytest.mark.parametrize("keep", [1, 3, 7, 8])
def test_replay_equals_committed_forward(dc, O, cuda, keep):
    import torch
    L, W, H, dk, dv = 3, 8, 4, 128, 128
    c = O.make_gdn_case(L, W, H, dk, dv, seed=5)
    snap = dev(c["snapshot"], cuda)
    replayed = torch.empty_like(snap)
    dc.gdn_replay(snap, replayed, dev(c["k"], cuda), dev(c["v"], cuda), dev(c["alpha"], cuda), dev(c["beta"], cuda),
                  keep=keep)
    torch.cuda.synchronize()
    for layer in range(L):
        committed, _ = step_layer(dc, cuda, c, layer, keep, with_out=False)
        assert torch.equal(replayed[layer], committed), f"layer {layer}: replay and committed step differ"
        want, _ = O.gdn_recurrence(c["snapshot"][layer], c["k"][layer], c["v"][layer], c["alpha"][layer],
                                   c["beta"][layer], keep)
        assert rel_err(replayed[layer].cpu().numpy(), want) <= REL


@pytest.mark.parametrize("rolled,committed_to,label", [
    (8, 3, "an un-rolled-back state must not look committed"),
    (4, 3, "a rollback one position too deep must not look committed"),
])
def test_negative_controls_diverge(dc, O, cuda, rolled, committed_to, label):
    import torch
    L, W, H, dk, dv = 2, 8, 4, 128, 128
    c = O.make_gdn_case(L, W, H, dk, dv, seed=6)
    snap = dev(c["snapshot"], cuda)
    replayed = torch.empty_like(snap)
    dc.gdn_replay(snap, replayed, dev(c["k"], cuda), dev(c["v"], cuda), dev(c["alpha"], cuda), dev(c["beta"], cuda),
                  keep=rolled)
    torch.cuda.synchronize()
    for layer in range(L):
        want, _ = O.gdn_recurrence(c["snapshot"][layer], c["k"][layer], c["v"][layer], c["alpha"][layer],
                                   c["beta"][layer], committed_to)
        assert rel_err(replayed[layer].cpu().numpy(), want) > 2e-3, label


@pytest.mark.parametrize("rows", [[0, 1, 3, 5], [0, 2], [0], [0, 4, 5, 7, 2]])
def test_tree_rollback_rows(dc, O, cuda, rows):
    """rollbackGatedDeltaTree keeps a scattered set of rows (SpeculativeTreeTests.swift:170-225)."""
    import torch
    L, W, H, dk, dv = 2, 8, 4, 128, 128
    c = O.make_gdn_case(L, W, H, dk, dv, seed=7)
    snap = dev(c["snapshot"], cuda)
    out = torch.empty_like(snap)
    dc.gdn_replay(snap, out, dev(c["k"], cuda), dev(c["v"], cuda), dev(c["alpha"], cuda), dev(c["beta"], cuda),
                  keep=len(rows), rows=rows)
    torch.cuda.synchronize()
    for layer in range(L):
        want, _ = O.gdn_recurrence(c["snapshot"][layer], c["k"][layer], c["v"][layer], c["alpha"][layer],
                                   c["beta"][layer], len(rows), rows=rows)
        assert rel_err(out[layer].cpu().numpy(), want) <= REL
    if rows != list(range(len(rows))):
        chain, _ = O.gdn_recurrence(c["snapshot"][0], c["k"][0], c["v"][0], c["alpha"][0], c["beta"][0], len(rows))
        assert rel_err(out[0].cpu().numpy(), chain) > 2e-3


@pytest.mark.parametrize("keep", [1, 2, 3, 6])
@pytest.mark.parametrize("rows", [None, "tree"])
@pytest.mark.parametrize("channels", [64, 12288, 100])
def test_conv_window_rollback_bit_exact(dc, O, cuda, keep, rows, channels):
    import torch
    L, W, kc1 = 3, 8, 3
    r = np.random.Generator(np.random.PCG64(9))
    window = O.bf16_bits(r.standard_normal((L, kc1, channels), dtype=np.float32))
    conv_in = O.bf16_bits(r.standard_normal((L, W, channels), dtype=np.float32))
    rl = None if rows is None else [0, 2, 3, 5, 6, 7][:keep]
    out = torch.empty((L, kc1, channels), dtype=torch.bfloat16, device=cuda)
    dc.gdn_conv_rollback(dev(window, cuda), out, dev(conv_in, cuda), keep=keep, rows=rl)
    torch.cuda.synchronize()
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    for layer in range(L):
        want = O.conv_window(window[layer], conv_in[layer], keep, rows=rl)
        assert np.array_equal(got[layer], want)


@pytest.mark.parametrize("keep", [1, 4, 8])
def test_config5_full_size(dc, O, cuda, keep):
    """48 layers x 32 heads x 128 x 128 fp32 state; the oracle checks
    three layers and four heads of each."""
    import torch
    L, W, H, dk, dv = 48, 8, 32, 128, 128
    c = O.make_gdn_case(L, W, H, dk, dv, seed=2)
    snap = dev(c["snapshot"], cuda)
    out = torch.empty_like(snap)
    dc.gdn_replay(snap, out, dev(c["k"], cuda), dev(c["v"], cuda), dev(c["alpha"], cuda), dev(c["beta"], cuda),
                  keep=keep)
    torch.cuda.synchronize()
    heads = [0, 7, 19, 31]
    for layer in (0, 23, 47):
        want, _ = O.gdn_recurrence(c["snapshot"][layer][heads], c["k"][layer][:, heads], c["v"][layer][:, heads],
                                   c["alpha"][layer][:, heads], c["beta"][layer][:, heads], keep)
        assert rel_err(out[layer][heads].cpu().numpy(), want) <= REL
    assert dc.device_error() == 0


@pytest.mark.parametrize("dk,dv,H,Hk,width,rows", [
    (128, 128, 32, 32, 8, None),
    (128, 128, 32, 8, 8, [0, 2, 3, 5, 6]),
    (64, 64, 48, 48, 12, [0, 2, 3, 5, 8, 9, 11]),
    (32, 32, 100, 25, 5, None),
    (128, 64, 20, 4, 64, None),
])
def test_multi_layer_replay_matches_per_layer_steps(dc, O, cuda, dk, dv, H, Hk, width, rows):
    """A replay of several layers over a subset of a round's positions (shared key heads
    included) equals, layer by layer, a step over those positions gathered: bit for bit,
    and the oracle within tolerance."""
    import torch
    L = 3
    keep = len(rows) if rows else width
    c = O.make_gdn_case(L, width, H, dk, dv, seed=11)
    if Hk != H:  # one key head per group of H / Hk value heads
        c["k"] = np.ascontiguousarray(c["k"][:, :, ::H // Hk])
        c["q"] = np.ascontiguousarray(c["q"][:, :, ::H // Hk])
    snap = dev(c["snapshot"], cuda)
    out = torch.empty_like(snap)
    dc.gdn_replay(snap, out, dev(c["k"], cuda), dev(c["v"], cuda), dev(c["alpha"], cuda), dev(c["beta"], cuda),
                  keep=keep, rows=rows)
    torch.cuda.synchronize()
    assert dc.device_error() == 0
    sel = rows if rows else list(range(width))
    for layer in range(L):
        g = {key: np.ascontiguousarray(c[key][layer][sel]) for key in ("q", "k", "v", "alpha", "beta")}
        st = torch.empty_like(snap[layer])
        dc.gdn_step(snap[layer], st, dev(g["q"], cuda), dev(g["k"], cuda), dev(g["v"], cuda), dev(g["alpha"], cuda),
                    dev(g["beta"], cuda))
        torch.cuda.synchronize()
        assert torch.equal(out[layer], st), f"layer {layer}"
    heads = [0, H // 3, H - 1]
    kh = [h // (H // Hk) for h in heads]
    layer = L - 1
    want, _ = O.gdn_recurrence(c["snapshot"][layer][heads], c["k"][layer][sel][:, kh], c["v"][layer][sel][:, heads],
                               c["alpha"][layer][sel][:, heads], c["beta"][layer][sel][:, heads], keep)
    assert rel_err(out[layer][heads].cpu().numpy(), want) <= REL


@pytest.mark.parametrize("dk,dv", [(128, 128), (64, 64), (32, 32)])
@pytest.mark.parametrize("T", [1, 8, 29])
def test_row_layouts_agree_bit_for_bit(dc, O, cuda, dk, dv, T):
    """A step over few heads runs one state row per thread (its grid would leave SMs idle
    with four) and one over many heads four rows per thread; the heads they share get the
    same state and outputs, bit for bit."""
    import torch
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    tiles = dv // 32
    small = max(1, (2 * sms) // (4 * tiles))           # at most 2 x SMs blocks of 32 rows
    big = (2 * sms) // tiles + 1                        # more than that
    c = O.make_gdn_case(1, T, big, dk, dv, seed=13)

    def run(H):
        g = {key: dev(np.ascontiguousarray(c[key][0][:, :H]), cuda) for key in ("q", "k", "v", "alpha", "beta")}
        snap = dev(np.ascontiguousarray(c["snapshot"][0][:H]), cuda)
        st = torch.empty_like(snap)
        o = torch.empty((T, H, dv), dtype=torch.bfloat16, device=cuda)
        dc.gdn_step(snap, st, g["q"], g["k"], g["v"], g["alpha"], g["beta"], out=o, q_scale=dk ** -0.5)
        torch.cuda.synchronize()
        return st, o

    st_s, o_s = run(small)
    st_b, o_b = run(big)
    assert torch.equal(st_s, st_b[:small])
    assert torch.equal(o_s, o_b[:, :small])
    assert dc.device_error() == 0

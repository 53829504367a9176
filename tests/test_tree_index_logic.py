"""The index logic of the tree and shared-key-head kernels, restated on the CPU.

The tree kernels derive everything from a device parent list with bit operations: the
path mask and depth of a row (tree_walk, csrc/common.cuh), each recurrence block's leaf,
path rows and owned rows (gdn_kernel<CH, true>, csrc/gdn.cu), each conv tap's source
(gdn_conv_gates_kernel, csrc/stack.cu) and the accepted-path walk (accept_tree_kernel).
This file transcribes that logic line for line and checks it against the host plan
(dflash-swift_b200/tree.py) on random trees of 1..32 rows: the blocks' paths are the plan's
paths, every row is written by exactly one block, the taps are the last kc inputs of the
row's history, the walk accepts the plan's rows; and that the decode kernel's split online
softmax with hidden keys at -inf (a finite exponent base while a range has seen no visible
key, weight 0 for a range that never does) is the softmax over the visible keys.  It also
checks that the grouped conv
kernel's channel and output maps tile [0, C) and the output exactly.  The GPU tests check
the kernels themselves; this pins the algorithm they implement.
"""
from __future__ import annotations

import itertools
import random

import numpy as np

from tree import SpeculativeTreePlan, accepted_path


def tree_parent(par, r):
    """tree_parent (csrc/common.cuh): an entry outside [0, r) makes the row a root."""
    p = par[r] if r > 0 else -1
    return p if 0 <= p < r else -1


def tree_walk(par, t):
    """tree_walk (csrc/common.cuh): the row's path mask and depth."""
    path, depth, r = 0, 0, t
    for _ in range(32):
        if r < 0:
            break
        path |= 1 << r
        r = tree_parent(par, r)
        depth += r >= 0
    return path, depth


def gdn_tree_blocks(par, width):
    """gdn_kernel<CH, true> (csrc/gdn.cu), warp 0: per block z, the z-th leaf's path rows
    and the rows it writes (those no earlier leaf's path holds); None when z has no leaf."""
    paths = [tree_walk(par, lane)[0] if lane < width else 0 for lane in range(32)]
    pars = [tree_parent(par, lane) if lane < width else -1 for lane in range(32)]
    has_child = 0
    for p in pars:  # __reduce_or_sync
        if p >= 0:
            has_child |= 1 << p
    leaves = 0  # __ballot_sync
    for lane in range(32):
        if lane < width and not (has_child >> lane) & 1:
            leaves |= 1 << lane
    blocks = []
    for z in range(width):
        m = leaves
        for _ in range(z):
            if not m:
                break
            m &= m - 1
        if not m:
            blocks.append(None)
            continue
        leaf = (m & -m).bit_length() - 1  # __ffs - 1
        mine = paths[leaf]
        earlier = leaves & ((1 << leaf) - 1)
        taken = 0
        for lane in range(32):
            if (earlier >> lane) & 1:
                taken |= paths[lane]
        blocks.append(([lane for lane in range(32) if (mine >> lane) & 1], mine & ~taken))
    return blocks


def conv_taps(par, t, KC, parents=True):
    """gdn_conv_gates_kernel (csrc/stack.cu): tap i of row t reads x row back[KC-1-i], or
    window row depth + i once the history has left the block."""
    back = [t] + [0] * (KC - 1)
    for s in range(1, KC):
        back[s] = -1 if back[s - 1] < 0 else (tree_parent(par, back[s - 1]) if parents else back[s - 1] - 1)
    depth = sum(1 for s in range(1, KC) if back[s] >= 0)
    return [("x", back[KC - 1 - i]) if back[KC - 1 - i] >= 0 else ("w", depth + i) for i in range(KC)]


def accept_tree(target, par, tokens, rows):
    """accept_tree_kernel (csrc/stack.cu): one ballot per step over the current row's
    children holding the target's token; the lowest such row is taken."""
    row, path = 0, [0]
    for _ in range(1, rows):
        hits = [lane for lane in range(rows) if tree_parent(par, lane) == row and tokens[lane] == target[row]]
        if not hits:
            break
        row = min(hits)
        path.append(row)
    return path, target[row]


def test_tree_index_logic_matches_the_host_plan():
    random.seed(0)
    for _ in range(3000):
        n = random.randint(1, 32)
        par = [-1] + [random.randint(0, r - 1) for r in range(1, n)]
        plan = SpeculativeTreePlan(par)
        blocks = gdn_tree_blocks(par, n)
        owned = [0] * n
        got_paths = []
        for b in blocks:
            if b is None:
                continue
            rows, own = b
            got_paths.append(rows)
            for r in range(n):
                owned[r] += (own >> r) & 1
        assert got_paths == plan.paths, par
        assert owned == [1] * n, par
        for t in range(n):
            KC = random.randint(2, 4)
            hist = [("w", i) for i in range(KC - 1)] + [("x", a) for a in plan.ancestors(t)]
            assert conv_taps(par, t, KC) == hist[-KC:], (par, t, KC)
            path, depth = tree_walk(par, t)
            assert depth == plan.depths[t] and path == sum(1 << a for a in plan.ancestors(t))
        tokens = [random.randint(0, 3) for _ in range(n)]
        target = [random.randint(0, 3) for _ in range(n)]
        assert accept_tree(target, par, tokens, n) == accepted_path(tokens, plan, target)


def test_chain_taps_are_the_original_formula():
    for t in range(32):
        for KC in (2, 3, 4):
            old = [("x", t + i - (KC - 1)) if t + i - (KC - 1) >= 0 else ("w", t + i) for i in range(KC)]
            assert conv_taps(None, t, KC, parents=False) == old


def test_malformed_parent_lists_stay_in_range():
    random.seed(1)
    for _ in range(2000):
        n = random.randint(1, 32)
        par = [random.randint(-3, 40) for _ in range(n)]
        for t in range(n):
            path, depth = tree_walk(par, t)
            assert 0 < path < (1 << n) and 0 <= depth < n
            for KC in (2, 3, 4):
                for kind, i in conv_taps(par, t, KC):
                    assert (0 <= i < n) if kind == "x" else (0 <= i < KC - 1)
        for b in gdn_tree_blocks(par, n):
            if b is not None:
                assert all(0 <= r < n for r in b[0])


def test_grouped_conv_maps_tile_channels_and_output():
    """gdn_conv_gates_grouped_kernel (csrc/stack.cu): slot -> (part, head), its first
    channel c0 and output offset y0; every channel is read and every output element written
    exactly once."""
    for Hk, g, dk, M in itertools.product((1, 2, 3, 4), (1, 2, 3), (32, 64, 128), (1, 5, 8)):
        H = Hk * g
        slots = 2 * Hk + H
        C = slots * dk
        chan, outs = set(), set()
        for t in range(M):
            for slot in range(slots):
                part = 0 if slot < Hk else 1 if slot < 2 * Hk else 2
                h = slot - part * Hk
                assert 0 <= h < (Hk if part < 2 else H)
                c0 = part * Hk * dk + h * dk
                part_heads = Hk if part < 2 else H
                y0 = part * M * Hk * dk + (t * part_heads + h) * dk
                for lane in range(32):
                    for j in range(dk // 32):
                        c = c0 + lane + 32 * j
                        assert 0 <= c < C
                        if t == 0:
                            chan.add(c)
                        o = y0 + lane + 32 * j
                        assert 0 <= o < M * C and o not in outs
                        outs.add(o)
        assert chan == set(range(C)) and len(outs) == M * C
        # value head h reads key head h // g in the recurrence kernel
        for h in range(H):
            assert h // (H // Hk) < Hk


def decode_split_softmax(scores, values, visible_mask, pos0, t, split=4, chunk=256):
    """attn_decode_kernel (csrc/stack.cu) for one token and head: the keys 0 .. pos0 + t cut
    into `split` CTA ranges, an online softmax per range in chunks with hidden keys at -inf
    and a finite exponent base while no key is visible, then the merge of the ranges'
    (max, sum, p V) with weight 0 for a range whose max stayed -inf."""
    n = pos0 + t + 1
    parts = []
    for rank in range(split):
        k0, k1 = n * rank // split, n * (rank + 1) // split
        m, l, acc = -np.inf, 0.0, np.zeros(values.shape[1])
        for c0 in range(k0, k1, chunk):
            j = np.arange(c0, min(k1, c0 + chunk))
            b = j - pos0
            s = np.where((b >= 0) & ~visible_mask[np.clip(b, 0, None)] if visible_mask is not None else False,
                         -np.inf, scores[j])
            mnew = max(m, s.max())
            base = 0.0 if mnew == -np.inf else mnew
            p = np.exp(s - base)
            corr = np.exp(m - base)
            l = l * corr + p.sum()
            acc = acc * corr + p @ values[j]
            m = mnew
        parts.append((m, l, acc))
    mx = max(m for m, _, _ in parts)
    f = [0.0 if m == -np.inf else np.exp(m - mx) for m, _, _ in parts]
    den = sum(fr * l for fr, (_, l, _) in zip(f, parts))
    return sum(fr * acc for fr, (_, _, acc) in zip(f, parts)) / den


def test_decode_masking_and_merge_are_the_masked_softmax():
    """Including ranges whose keys are all hidden (a row deep in the block, pos0 = 0)."""
    rng = np.random.default_rng(3)
    for _ in range(300):
        M = int(rng.integers(1, 17))
        par = [-1] + [int(rng.integers(0, r)) for r in range(1, M)]
        pos0 = int(rng.choice([0, 1, 5, 300, 700]))
        n_keys = pos0 + M
        scores_all = rng.standard_normal(n_keys) * 3
        values = rng.standard_normal((n_keys, 4))
        for t in range(M):
            path, _ = tree_walk(par, t)
            visible = np.array([(path >> b) & 1 == 1 for b in range(M)])
            got = decode_split_softmax(scores_all, values, visible, pos0, t)
            keys = list(range(pos0)) + [pos0 + a for a in range(M) if visible[a]]
            w = np.exp(scores_all[keys] - scores_all[keys].max())
            want = (w / w.sum()) @ values[keys]
            assert np.allclose(got, want, rtol=1e-10, atol=1e-12), (par, pos0, t)
            chain = decode_split_softmax(scores_all, values, None, pos0, t)
            keys = list(range(pos0 + t + 1))
            w = np.exp(scores_all[keys] - scores_all[keys].max())
            assert np.allclose(chain, (w / w.sum()) @ values[keys], rtol=1e-10, atol=1e-12)

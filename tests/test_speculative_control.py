"""The end-to-end control of the reference's bench (`dflash-bench --control`,
Sources/dflash-bench/main.swift:146-187): speculative decoding emits exactly the tokens
plain greedy decoding emits.

Run on the stack reference (oracle/stack_ref.py) with its commit step, for chain rounds
(verify 8 rows, accept the matching prefix, roll the gated-delta state and conv window
back to it) and tree rounds (verify a drafted tree, walk the accepted path with the
shipped host walk, roll back to it and move its attention cache entries into place).
This pins the round semantics the CUDA stack implements — forward at a moving context,
accept, rollback over the accepted rows, cache compaction — by the token sequence, and
checks the final hidden state behind every emitted token against greedy's (observed
bit-identical; the bar is 1e-4 because the reference keeps the recurrent state in fp64
within a round and in fp32 between rounds).  Negative controls: committing every
verified row instead of the accepted ones (hidden states 9e-2 off greedy's), and
committing a tree path as if it were the first rows of a chain (other tokens), both
leave greedy.  The model is the parity stack (TINY) with a random bf16 embedding table
standing in for the target's (the stack takes hidden states).
"""
from __future__ import annotations

import sys
from dataclasses import replace
from pathlib import Path

import numpy as np
import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))

import verify_stack as vs  # noqa: E402
from tree import SpeculativeTreePlan, accepted_path  # noqa: E402

CFG = replace(vs.TINY, context=4, block=32)  # caches of 36 positions, 4 already filled
ROWS = 8                                     # rows verified per round
N_TOKENS = 16
FIRST = 17


@pytest.fixture(scope="module")
def model():
    plan = vs.shard_plan(CFG, 0, 1)
    w = vs.build_rank_weights(CFG, plan, 0, "cpu")
    gen = torch.Generator().manual_seed(5)
    emb = torch.randn(CFG.vocab, CFG.hidden, generator=gen).to(torch.bfloat16).float()
    return plan, w, emb


def _fresh_state(plan):
    return vs.build_rank_state(CFG, plan, 0, "cpu")


def _round(model, state, ctx, tokens, parents=None):
    import stack_ref
    plan, w, emb = model
    r = stack_ref.forward(CFG, plan, w, state, emb[tokens], parents=parents, context=ctx)
    target, accepted = stack_ref.lm_head_accept(plan, w, r["out"], tokens[1:])
    return r, [int(t) for t in target], accepted


def closeness(y, ref) -> float:
    y, ref = np.asarray(y, dtype=np.float64), np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(y - ref)) / max(float(np.max(np.abs(ref))), 1.0))


@pytest.fixture(scope="module")
def greedy(model):
    """Plain greedy decoding, one token per forward, committed each step: the tokens and
    the final hidden state behind each."""
    import stack_ref
    state, ctx, tok, out, hid = _fresh_state(model[0]), CFG.context, FIRST, [], []
    for _ in range(N_TOKENS + ROWS):
        r, target, _ = _round(model, state, ctx, [tok])
        stack_ref.commit(state, r, [0], ctx)
        ctx += 1
        tok = target[0]
        out.append(tok)
        hid.append(r["out"][0])
    return out, torch.stack(hid)


def _speculative_chain(model, greedy, wrong_at, commit_all=False):
    """Chain rounds whose drafts are the greedy continuation with one wrong token at
    wrong_at[round] (None: no wrong token)."""
    import stack_ref
    greedy = greedy[0]
    state, ctx, anchor, out, rnd = _fresh_state(model[0]), CFG.context, FIRST, [], 0
    accepts, hid = [], []
    while len(out) < N_TOKENS:
        p = len(out)
        drafts = list(greedy[p:p + ROWS - 1])
        bad = wrong_at[rnd % len(wrong_at)]
        if bad is not None:
            drafts[bad] = (drafts[bad] + 1) % CFG.vocab
        r, target, acc = _round(model, state, ctx, [anchor] + drafts)
        keep = ROWS if commit_all else acc + 1
        stack_ref.commit(state, r, list(range(keep)), ctx)
        out += drafts[:acc] + [target[acc]]
        hid += [r["out"][i] for i in range(acc + 1)]
        ctx += acc + 1
        anchor = target[acc]
        accepts.append(acc)
        rnd += 1
    return out[:N_TOKENS], torch.stack(hid)[:N_TOKENS], accepts


BRANCHY = [-1, 0, 0, 1, 1, 2, 3, 5]  # paths [0, 1, 3, 6], [0, 1, 4], [0, 2, 5, 7]


def _speculative_tree(model, greedy, cut, as_chain=False):
    """Tree rounds on BRANCHY: the greedy continuation sits on the path 0-2-5-7 (so the
    accepted rows are not the block's first rows), the other rows hold wrong tokens;
    cut[round] = k keeps only the first k continuation tokens right."""
    import stack_ref
    greedy = greedy[0]
    plan = SpeculativeTreePlan(BRANCHY)
    state, ctx, anchor, out, rnd = _fresh_state(model[0]), CFG.context, FIRST, [], 0
    depths, hid = [], []
    while len(out) < N_TOKENS:
        p = len(out)
        g = greedy[p:p + 3]
        k = cut[rnd % len(cut)]
        tokens = [anchor] + [(g[0] + 1 + i) % CFG.vocab for i in range(ROWS - 1)]  # all wrong
        for depth, row in enumerate((2, 5, 7)):
            if depth < k:
                tokens[row] = g[depth]
        r, target, _ = _round(model, state, ctx, tokens, parents=BRANCHY)
        rows, bonus = accepted_path(tokens, plan, target)
        commit_rows = list(range(len(rows))) if as_chain else rows
        stack_ref.commit(state, r, commit_rows, ctx)
        out += [tokens[row] for row in rows[1:]] + [bonus]
        hid += [r["out"][row] for row in rows]
        ctx += len(rows)
        anchor = bonus
        depths.append(len(rows) - 1)
        rnd += 1
    return out[:N_TOKENS], torch.stack(hid)[:N_TOKENS], depths


def test_chain_rounds_emit_the_greedy_sequence(model, greedy):
    out, hid, accepts = _speculative_chain(model, greedy, wrong_at=[3, None, 0, 5, 1])
    assert out == greedy[0][:N_TOKENS]
    assert closeness(hid, greedy[1][:N_TOKENS]) <= 1e-4
    assert max(accepts) == ROWS - 1 and min(accepts) == 0  # full, partial and empty rounds ran


def test_tree_rounds_emit_the_greedy_sequence(model, greedy):
    out, hid, depths = _speculative_tree(model, greedy, cut=[3, 1, 2, 0])
    assert out == greedy[0][:N_TOKENS]
    assert closeness(hid, greedy[1][:N_TOKENS]) <= 1e-4
    assert set(depths) >= {0, 1, 2, 3}


def test_committing_rejected_rows_leaves_greedy(model, greedy):
    out, hid, _ = _speculative_chain(model, greedy, wrong_at=[3, None, 0, 5, 1], commit_all=True)
    assert out != greedy[0][:N_TOKENS] or closeness(hid, greedy[1][:N_TOKENS]) > 1e-2


def test_committing_a_tree_path_as_chain_rows_leaves_greedy(model, greedy):
    out, hid, _ = _speculative_tree(model, greedy, cut=[3, 1, 2, 0], as_chain=True)
    assert out != greedy[0][:N_TOKENS] or closeness(hid, greedy[1][:N_TOKENS]) > 1e-2


def test_greedy_sequence_is_not_constant(greedy):
    assert len(set(greedy[0])) > 4


# ----------------------------------------------------------------------------- CUDA stack (GPU)

@pytest.mark.gpu
def test_cuda_stack_speculative_rounds_emit_its_greedy_sequence(cuda):
    """The same control on the CUDA stack: greedy is a one-row stack committing every
    token; chain rounds and tree rounds run on eight-row stacks with the drafts built as
    above, committing the accepted rows (commit + advance).  On the device a row's
    arithmetic does not depend on the other rows of its block (each matmul row
    accumulates in a fixed order, norms and attention are per row, the replay runs the
    step's own per-position update), so the sequences agree; committing every verified
    row instead leaves greedy."""
    plan = vs.shard_plan(CFG, 0, 1)
    w = vs.build_rank_weights(CFG, plan, 0, cuda)
    gen = torch.Generator().manual_seed(5)
    emb = torch.randn(CFG.vocab, CFG.hidden, generator=gen).to(torch.bfloat16).to(cuda)

    def make(rows, tree=False):
        cfg = replace(CFG, block=rows)  # caches stay sized for CFG (36 positions)
        return vs.VerifyStack(cfg, 0, 1, device=cuda, weights=w, state=vs.build_rank_state(CFG, plan, 0, cuda),
                              tree=tree)

    g1 = make(1)
    greedy, ghid, tok = [], [], FIRST
    for _ in range(N_TOKENS + ROWS):
        target, _ = g1.verify(emb[[tok]], torch.zeros(0, dtype=torch.int32, device=cuda))
        g1.commit([0])
        g1.advance(1)
        tok = int(target[0].item())
        greedy.append(tok)
        ghid.append(g1.out[0].float().cpu())
    ghid = torch.stack(ghid)
    assert len(set(greedy)) > 4

    def chain(commit_all=False):
        s8 = make(ROWS)
        out, hid, anchor, rnd = [], [], FIRST, 0
        while len(out) < N_TOKENS:
            p = len(out)
            drafts = list(greedy[p:p + ROWS - 1])
            bad = [3, None, 0, 5, 1][rnd % 5]
            if bad is not None:
                drafts[bad] = (drafts[bad] + 1) % CFG.vocab
            target, acc = s8.verify(emb[[anchor] + drafts], torch.tensor(drafts, dtype=torch.int32, device=cuda))
            acc, target = int(acc.item()), target.tolist()
            s8.commit(list(range(ROWS if commit_all else acc + 1)))
            s8.advance(acc + 1)
            out += drafts[:acc] + [target[acc]]
            hid += [s8.out[i].float().cpu() for i in range(acc + 1)]
            anchor = target[acc]
            rnd += 1
        return out[:N_TOKENS], torch.stack(hid)[:N_TOKENS]

    def tree():
        st = make(ROWS, tree=True)
        st.set_tree(BRANCHY)
        out, hid, anchor, rnd = [], [], FIRST, 0
        while len(out) < N_TOKENS:
            p = len(out)
            g = greedy[p:p + 3]
            k = [3, 1, 2, 0][rnd % 4]
            tokens = [anchor] + [(g[0] + 1 + i) % CFG.vocab for i in range(ROWS - 1)]
            for depth, row in enumerate((2, 5, 7)):
                if depth < k:
                    tokens[row] = g[depth]
            rows, bonus = st.verify_tree(emb[tokens], tokens)
            st.commit(rows)
            st.advance(len(rows))
            out += [tokens[r] for r in rows[1:]] + [bonus]
            hid += [st.out[r].float().cpu() for r in rows]
            anchor = bonus
            rnd += 1
        return out[:N_TOKENS], torch.stack(hid)[:N_TOKENS]

    out, hid = chain()
    assert out == greedy[:N_TOKENS]
    assert closeness(hid, ghid[:N_TOKENS]) <= 1e-2
    out, hid = tree()
    assert out == greedy[:N_TOKENS]
    assert closeness(hid, ghid[:N_TOKENS]) <= 1e-2
    out, hid = chain(commit_all=True)
    assert out != greedy[:N_TOKENS] or closeness(hid, ghid[:N_TOKENS]) > 1e-2

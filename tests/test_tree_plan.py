"""Speculative tree plans (host logic of a tree verify round), checked against the
properties the reference pins (Tests/DFlashKitTests/SpeculativeTreeTests.swift), and the
accepted path fed to the gated-delta replay oracle as its row list."""
from __future__ import annotations

import numpy as np
import pytest

import tree as T

#  0 ─┬─ 1 ─┬─ 3 ─── 5
#     │     └─ 4
#     └─ 2
FORKED = [-1, 0, 0, 1, 1, 3]
ROW_TOKENS = [11, 23, 37, 41, 37, 53]


def test_depths_follow_the_tree_not_row_order():
    assert T.SpeculativeTreePlan(FORKED).depths == [0, 1, 1, 2, 2, 3]


def test_every_leaf_becomes_one_root_path():
    plan = T.SpeculativeTreePlan(FORKED)
    assert {tuple(p) for p in plan.paths} == {(0, 1, 3, 5), (0, 1, 4), (0, 2)}
    assert plan.path_length == 4
    for row, src in enumerate(plan.row_sources):
        assert plan.paths[src.path][src.depth] == row


def test_attention_mask_shows_ancestors_and_nothing_else():
    mask = T.SpeculativeTreePlan(FORKED).attention_mask(prefix=2)
    assert mask.shape == (6, 8)
    assert mask[:, :2].all()
    assert [j for j in range(6) if mask[5, 2 + j]] == [0, 1, 3, 5]   # not the cousins 2 and 4
    assert [j for j in range(6) if mask[2, 2 + j]] == [0, 2]


def test_positions_come_from_depth():
    assert T.SpeculativeTreePlan(FORKED).positions(10).tolist() == [10, 11, 11, 12, 12, 13]


def test_chain_plan_is_the_degenerate_tree():
    plan = T.SpeculativeTreePlan.chain(4)
    assert plan.parents == [-1, 0, 1, 2] and plan.paths == [[0, 1, 2, 3]]
    assert plan.is_root_path([0, 1, 2]) and not plan.is_root_path([0, 2])
    mask = plan.attention_mask(0)
    assert (mask == np.tril(np.ones((4, 4), dtype=bool))).all()  # a chain's mask is causal


def test_bad_parents_are_rejected():
    for parents in ([0, 0], [-1, 1], [-1, 0, 3]):
        with pytest.raises(ValueError):
            T.SpeculativeTreePlan(parents)


@pytest.mark.parametrize("targets,rows,bonus", [
    ([37, 99, 71, 99, 99, 99], [0, 2], 71),        # into the second branch, then nothing drafted
    ([99, 11, 22, 33, 44, 55], [0], 99),           # no child holds the target's token
    ([23, 41, 0, 53, 0, 67], [0, 1, 3, 5], 67),    # the whole deep branch
])
def test_accepted_path(targets, rows, bonus):
    plan = T.SpeculativeTreePlan(FORKED)
    got_rows, got_bonus = T.accepted_path(ROW_TOKENS, plan, targets)
    assert got_rows == rows and got_bonus == bonus
    assert plan.is_root_path(got_rows)


@pytest.mark.parametrize("targets", [[23, 41, 0, 53, 0, 67], [37, 99, 71, 99, 99, 99]])
def test_rollback_rows_replay_the_accepted_path(O, targets):
    """The replay over the accepted rows of a tree capture equals the recurrence run as a
    plain chain over those rows' inputs in path order (the rollback property the
    reference checks against a committed forward)."""
    plan = T.SpeculativeTreePlan(FORKED)
    rows, _ = T.accepted_path(ROW_TOKENS, plan, targets)
    keep, row_list = T.rollback_arguments(rows)
    c = O.make_gdn_case(1, plan.rows, 4, 32, 32, seed=11)
    tree_state, _ = O.gdn_recurrence(c["snapshot"][0], c["k"][0], c["v"][0], c["alpha"][0], c["beta"][0], keep,
                                     rows=row_list)
    chain_state, _ = O.gdn_recurrence(c["snapshot"][0], c["k"][0][row_list], c["v"][0][row_list],
                                      c["alpha"][0][row_list], c["beta"][0][row_list], keep)
    assert np.array_equal(tree_state, chain_state)

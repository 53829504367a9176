"""Speculative tree rounds through the verify stack.

The property the reference pins (Tests/DFlashKitTests/SpeculativeTreeTests.swift:119-140):
each row of a tree-verify forward equals the plain (chain) forward of its root-to-row
path; a chain verify of the same rows in row order does not (:145-165); after the round,
rolling back to the accepted path leaves the state a committed forward of that path would
(:170-225).

CPU: the stack reference (oracle/stack_ref.py) run as a tree against its own chain
forward of every path, bit for bit (row arithmetic is independent of the other rows), and
the host tree plan against the reference's path bookkeeping.  GPU: each tree kernel
against its chain kernel on the gathered path rows (the same bits where the arithmetic is
the same; attention within bf16 rounding, its key ranges split differently), the KV
compaction against a gather, and the CUDA stack in tree mode against the reference
(<= 2e-2 closeness, the tolerance of the chain stack test), including graph replay with a
new tree and the commit of an accepted path.
"""
from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))

import verify_stack as vs  # noqa: E402
from tree import SpeculativeTreePlan  # noqa: E402


# 8-row trees (TINY's block): branching at the anchor and below, a deep chain, a star.
TREES = {
    "branchy": [-1, 0, 0, 1, 1, 2, 3, 5],
    "chain": [-1, 0, 1, 2, 3, 4, 5, 6],
    "star": [-1, 0, 0, 0, 0, 0, 0, 0],
    "two_deep": [-1, 0, 1, 0, 3, 1, 5, 2],
}


def closeness(y, ref) -> float:
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(y - ref)) / max(float(np.max(np.abs(ref))), 1.0))


# ----------------------------------------------------------------------------- reference (CPU)

@pytest.mark.parametrize("name", sorted(TREES))
def test_reference_paths_match_the_host_plan(name):
    """The reference's path bookkeeping and the shipped plan agree: ancestors, leaf paths
    in row order, depths (rotary positions)."""
    import stack_ref
    parents = TREES[name]
    plan = SpeculativeTreePlan(parents)
    anc, paths = stack_ref.tree_paths(parents, len(parents))
    assert paths == plan.paths
    assert anc == [plan.ancestors(r) for r in range(plan.rows)]
    assert [len(a) - 1 for a in anc] == plan.depths


def test_reference_tree_forward_with_a_chain_tree_is_the_chain_forward():
    import stack_ref
    cfg = vs.TINY
    plan = vs.shard_plan(cfg, 0, 1)
    w = vs.build_rank_weights(cfg, plan, 0, "cpu")
    st = vs.build_rank_state(cfg, plan, 0, "cpu")
    hidden = vs.make_block(cfg, 0, "cpu")
    a = stack_ref.forward(cfg, plan, w, st, hidden)
    b = stack_ref.forward(cfg, plan, w, st, hidden, parents=TREES["chain"])
    assert torch.equal(a["out"], b["out"])


@pytest.fixture(scope="module")
def tiny_tree_reference():
    import stack_ref
    cfg = vs.TINY
    plan = vs.shard_plan(cfg, 0, 1)
    w = vs.build_rank_weights(cfg, plan, 0, "cpu")
    st = vs.build_rank_state(cfg, plan, 0, "cpu")
    hidden = vs.make_block(cfg, 3, "cpu")
    parents = TREES["branchy"]
    tree = stack_ref.forward(cfg, plan, w, st, hidden, parents=parents)
    chains = {tuple(p): stack_ref.forward(cfg, plan, w, st, hidden[p]) for p in SpeculativeTreePlan(parents).paths}
    return dict(cfg=cfg, plan=plan, w=w, st=st, hidden=hidden, parents=parents, tree=tree, chains=chains)


def test_reference_tree_rows_equal_their_path_chains(tiny_tree_reference):
    """SpeculativeTreeTests.swift:119-140 on the stack reference: every row of every path,
    the final hidden state and the attention cache entries, bit for bit."""
    r = tiny_tree_reference
    cfg, tree = r["cfg"], r["tree"]
    for path, chain in r["chains"].items():
        path = list(path)
        assert torch.equal(tree["out"][path], chain["out"]), path
        for ai in range(len(tree["cache_k"])):
            for key in ("cache_k", "cache_v"):
                got = tree[key][ai][:, [cfg.context + t for t in path]]
                want = chain[key][ai][:, cfg.context:cfg.context + len(path)]
                assert torch.equal(got, want), (path, key)


def test_reference_row_order_chain_is_not_the_tree(tiny_tree_reference):
    """The negative control (SpeculativeTreeTests.swift:145-165): verifying the tree's rows
    as a chain in row order gets the rows whose path is not 0..r wrong."""
    import stack_ref
    r = tiny_tree_reference
    chain = stack_ref.forward(r["cfg"], r["plan"], r["w"], r["st"], r["hidden"])
    plan = SpeculativeTreePlan(r["parents"])
    for row in range(plan.rows):
        same = torch.equal(chain["out"][row], r["tree"]["out"][row])
        assert same == (plan.ancestors(row) == list(range(row + 1))), row


def test_reference_commit_of_a_tree_path_is_the_path_chain(tiny_tree_reference, O):
    """Replaying the tree round's capture over an accepted path gives the state a chain
    forward of that path leaves, and the rebuilt conv window is that chain's window, bit
    for bit (rollbackGatedDeltaTree, SpeculativeTreeTests.swift:170-225)."""
    import stack_ref
    bits = lambda t: stack_ref._bits(t.to(torch.bfloat16))  # values already bf16-exact
    r = tiny_tree_reference
    cfg, tree = r["cfg"], r["tree"]
    kc1 = cfg.conv_kernel - 1
    gdn_states = [S for S in r["st"]["layers"] if "snapshot" in S]
    for path, chain in r["chains"].items():
        for keep in range(1, len(path) + 1):
            rows = list(path[:keep])
            for gi, S in enumerate(gdn_states):
                q, k, v = tree["qkv"][gi]
                s, _ = O.gdn_recurrence(S["snapshot"].numpy(), bits(k), bits(v), tree["alpha"][gi].numpy(),
                                        tree["beta"][gi].numpy(), keep, rows=rows)
                if keep == len(path):
                    assert np.array_equal(s.astype(np.float32), chain["state"][gi].numpy()), (path, gi)
                win = O.conv_window(bits(S["window"]), bits(tree["conv_in"][gi]), keep, rows)
                hist = torch.cat([S["window"].float(), chain["conv_in"][gi][:keep]])[-kc1:]
                assert np.array_equal(win, bits(hist)), (path, keep, gi)


def test_reference_tree_at_tp2_matches_tp1(tmp_path, tiny_tree_reference):
    """The tree round sharded over two gloo ranks (column / row shards, all-reduce after
    the row-sharded projections) matches the one-rank tree round, and dropping the
    all-reduce does not."""
    import stack_workers
    from dataclasses import asdict
    from test_verify_stack import _run_ranks, free_port
    r = tiny_tree_reference
    ref = r["tree"]["out"].numpy()
    errs = {}
    for drop in (False, True):
        out = tmp_path / f"tree_tp2_drop{int(drop)}.pt"
        port = free_port()
        codes = _run_ranks(stack_workers.gloo_reference_rank, 2,
                           lambda k: (k, 2, port, str(out), asdict(vs.TINY), drop, r["parents"], 3))
        assert codes == [0, 0], codes
        errs[drop] = closeness(torch.load(out)["out"].numpy(), ref)
    assert errs[False] <= 3e-2
    assert errs[True] > max(0.05, 10 * errs[False])


# ----------------------------------------------------------------------------- kernels (GPU)

def _gather_rows(t, rows):
    return t[rows].contiguous()


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(TREES))
@pytest.mark.parametrize("heads,dk,kc", [(4, 64, 4), (32, 128, 4), (3, 32, 2)])
def test_conv_gates_tree_is_the_chain_of_each_path(dc, cuda, name, heads, dk, kc):
    parents = TREES[name]
    M = len(parents)
    gen = torch.Generator(device=cuda).manual_seed(heads + kc)
    C = 3 * heads * dk
    x = torch.randn(M, C + 4 * heads * dk + 2 * heads, generator=gen, device=cuda).to(torch.bfloat16)
    win = torch.randn(kc - 1, C, generator=gen, device=cuda).to(torch.bfloat16)
    w = (0.5 * torch.randn(C, kc, generator=gen, device=cuda)).to(torch.bfloat16)
    a_log = torch.randn(heads, generator=gen, device=cuda)
    dt = torch.randn(heads, generator=gen, device=cuda)
    par = torch.tensor(parents, dtype=torch.int32, device=cuda)
    got = torch.empty(3, M, heads, dk, dtype=torch.bfloat16, device=cuda)
    al, be = (torch.empty(M, heads, device=cuda) for _ in range(2))
    dc.stack_gdn_conv_gates(x, win, w, got, x[:, C + 4 * heads * dk:], a_log, dt, al, be, heads, dk, parents=par)
    for path in SpeculativeTreePlan(parents).paths:
        xp = _gather_rows(x, path)
        want = torch.empty(3, len(path), heads, dk, dtype=torch.bfloat16, device=cuda)
        alw, bew = (torch.empty(len(path), heads, device=cuda) for _ in range(2))
        dc.stack_gdn_conv_gates(xp, win, w, want, xp[:, C + 4 * heads * dk:], a_log, dt, alw, bew, heads, dk)
        torch.cuda.synchronize()
        assert torch.equal(got[:, path], want), path
        assert torch.equal(al[path], alw) and torch.equal(be[path], bew), path


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(TREES))
@pytest.mark.parametrize("heads,dk", [(4, 128), (32, 128), (2, 64)])
def test_gdn_step_tree_is_the_chain_of_each_path(dc, O, cuda, name, heads, dk):
    """Every row's output equals a chain step over its path from the same snapshot (the
    same device arithmetic), and matches the recurrence oracle along that path."""
    parents = TREES[name]
    T, dv = len(parents), dk
    c = O.make_gdn_case(1, T, heads, dk, dv, seed=11)
    t = lambda a: (torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(cuda).view(torch.bfloat16)
                   if a.dtype == np.uint16 else torch.from_numpy(np.ascontiguousarray(a)).to(cuda))
    snap, q, k, v, al, be = (t(c[key][0]) for key in ("snapshot", "q", "k", "v", "alpha", "beta"))
    par = torch.tensor(parents, dtype=torch.int32, device=cuda)
    out = torch.zeros(T, heads, dv, dtype=torch.bfloat16, device=cuda)
    dc.gdn_step_tree(snap, q, k, v, al, be, par, out, q_scale=1.0 / math.sqrt(dk))
    torch.cuda.synchronize()
    for path in SpeculativeTreePlan(parents).paths:
        st = torch.empty_like(snap)
        want = torch.empty(len(path), heads, dv, dtype=torch.bfloat16, device=cuda)
        dc.gdn_step(snap, st, *(_gather_rows(a, path) for a in (q, k, v, al, be)), out=want,
                    q_scale=1.0 / math.sqrt(dk))
        torch.cuda.synchronize()
        assert torch.equal(out[path], want), path
        _, o = O.gdn_recurrence(c["snapshot"][0], c["k"][0], c["v"][0], c["alpha"][0], c["beta"][0], len(path),
                                rows=path, q_bits=c["q"][0], q_scale=1.0 / math.sqrt(dk))
        assert closeness(out[path].float().cpu().numpy(), o) <= 1e-2, path
    assert dc.device_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(TREES))
@pytest.mark.parametrize("hq,hkv,d,rot,pos0", [(4, 2, 64, 64, 24), (24, 4, 256, 64, 300), (8, 8, 128, 128, 0)])
def test_attention_tree_is_the_chain_of_each_path(dc, cuda, name, hq, hkv, d, rot, pos0):
    """Prep: the same q and cache entries as a chain prep of the path (rotary position
    pos0 + depth).  Decode: the output of a chain decode of the path, within bf16 rounding.
    pos0 = 0 makes whole CTA key ranges hold only hidden keys."""
    parents = TREES[name]
    M = len(parents)
    gen = torch.Generator(device=cuda).manual_seed(hq + d + pos0)
    max_len = pos0 + M
    qkv0 = torch.randn(M, (2 * hq + 2 * hkv) * d, generator=gen, device=cuda).to(torch.bfloat16)
    qn = (1.0 + 0.1 * torch.randn(d, generator=gen, device=cuda)).to(torch.bfloat16)
    kn = (1.0 + 0.1 * torch.randn(d, generator=gen, device=cuda)).to(torch.bfloat16)
    ck0 = torch.randn(hkv, max_len, d, generator=gen, device=cuda).to(torch.bfloat16)
    cv0 = torch.randn(hkv, max_len, d, generator=gen, device=cuda).to(torch.bfloat16)
    par = torch.tensor(parents, dtype=torch.int32, device=cuda)
    qkv, ck, cv = qkv0.clone(), ck0.clone(), cv0.clone()
    dc.stack_attn_prep(qkv, qn, kn, ck, cv, hq, hkv, rot, pos0, 1e-6, 1e4, parents=par)
    out = torch.empty(M, hq * d, dtype=torch.bfloat16, device=cuda)
    dc.stack_attn_decode(qkv, ck, cv, out, hq, hkv, pos0, 1.0 / math.sqrt(d), parents=par)
    for path in SpeculativeTreePlan(parents).paths:
        n = len(path)
        qkv_p, ck_p, cv_p = _gather_rows(qkv0, path), ck0.clone(), cv0.clone()
        dc.stack_attn_prep(qkv_p, qn, kn, ck_p, cv_p, hq, hkv, rot, pos0, 1e-6, 1e4)
        out_p = torch.empty(n, hq * d, dtype=torch.bfloat16, device=cuda)
        dc.stack_attn_decode(qkv_p, ck_p, cv_p, out_p, hq, hkv, pos0, 1.0 / math.sqrt(d))
        torch.cuda.synchronize()
        assert torch.equal(qkv[path], qkv_p), path
        slots = [pos0 + t for t in path]
        assert torch.equal(ck[:, slots], ck_p[:, pos0:pos0 + n]) and torch.equal(cv[:, slots], cv_p[:, pos0:pos0 + n])
        assert closeness(out[path].float().cpu().numpy(), out_p.float().cpu().numpy()) <= 1e-2, path


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [[0, 2, 5], [0, 1, 3, 4], [0], [0, 1, 2, 3, 4, 5, 6, 7], [0, 3, 4, 6]])
def test_kv_compact_moves_the_accepted_rows(dc, cuda, rows):
    hkv, max_len, d, pos0 = 3, 40, 128, 30
    gen = torch.Generator(device=cuda).manual_seed(len(rows))
    ck = torch.randn(2, hkv, max_len, d, generator=gen, device=cuda).to(torch.bfloat16)
    cv = torch.randn(2, hkv, max_len, d, generator=gen, device=cuda).to(torch.bfloat16)
    want_k, want_v = ck.clone(), cv.clone()
    src = [pos0 + r for r in rows]
    want_k[:, :, pos0:pos0 + len(rows)] = ck[:, :, src]
    want_v[:, :, pos0:pos0 + len(rows)] = cv[:, :, src]
    dc.stack_kv_compact(ck, cv, pos0, rows)  # both layers at once
    torch.cuda.synchronize()
    assert torch.equal(ck, want_k) and torch.equal(cv, want_v)
    one_k, one_v = ck[1].clone(), cv[1].clone()  # one layer, rows moved back in place: a no-op
    dc.stack_kv_compact(one_k, one_v, pos0, list(range(len(rows))))
    torch.cuda.synchronize()
    assert torch.equal(one_k, ck[1]) and torch.equal(one_v, cv[1])


@pytest.mark.gpu
@pytest.mark.parametrize("seed", range(6))
def test_accept_tree_matches_the_host_walk(dc, cuda, seed):
    """dflash_accept_tree against tree.accepted_path on random trees of 1..32 rows, with
    targets that mostly follow a drafted child (deep walks) and drafted tokens that repeat
    across siblings (the first child in row order must win)."""
    from tree import accepted_path
    rng = np.random.default_rng(seed)
    for rows in (1, 2, 8, 16, 32):
        parents = [-1] + [int(rng.integers(0, r)) for r in range(1, rows)]
        plan = SpeculativeTreePlan(parents)
        tokens = [int(t) for t in rng.integers(0, 4, rows)]
        target = []
        for r in range(rows):
            kids = plan.children[r]
            follow = kids and rng.random() < 0.8
            target.append(tokens[int(rng.choice(kids))] if follow else int(rng.integers(100, 200)))
        want_rows, want_next = accepted_path(tokens, plan, target)
        t = lambda v: torch.tensor(v, dtype=torch.int32, device=cuda)
        path = torch.full((rows,), -7, dtype=torch.int32, device=cuda)
        n, nxt = t([0]), t([0])
        dc.accept_tree(t(target), t(parents), t(tokens), path, n, nxt)
        torch.cuda.synchronize()
        got = path[:int(n.item())].tolist()
        assert got == want_rows and int(nxt.item()) == want_next, (rows, parents, tokens, target)


# ----------------------------------------------------------------------------- CUDA stack (GPU)

@pytest.mark.gpu
def test_cuda_stack_tree_matches_reference_and_replays_a_new_tree(cuda):
    import stack_ref
    cfg = vs.TINY
    stack = vs.VerifyStack(cfg, 0, 1, seed=0, device=cuda, tree=True)
    hidden = vs.make_block(cfg, 3, cuda)
    for name in ("branchy", "two_deep"):
        stack.set_tree(TREES[name])
        out = stack.forward(hidden).float().cpu()
        torch.cuda.synchronize()
        ref = stack_ref.forward(cfg, stack.plan, stack.w, stack.state, hidden, parents=TREES[name])
        assert closeness(out.numpy(), ref["out"].numpy()) <= 2e-2, name
        for gi in range(len(ref["qkv"])):
            assert closeness(stack.capture_qkv[gi].float().cpu().numpy(), ref["qkv"][gi].numpy()) <= 2e-2
            assert closeness(stack.capture_alpha[gi].cpu().numpy(), ref["alpha"][gi].numpy()) <= 2e-2
    # the device walk of the round equals the host walk over the round's target tokens
    from tree import accepted_path
    drafted = [11, 23, 37, 41, 37, 53, 5, 9]
    rows, nxt = stack.verify_tree(hidden, drafted)
    target = stack.tokens.cpu().tolist()
    assert (rows, nxt) == accepted_path(drafted, stack.tree_plan, target)
    # a graph captured under one tree replays another: the kernels read the parent list
    stack.set_tree(TREES["star"])
    g = stack.capture(hidden)
    stack.set_tree(TREES["branchy"])
    eager = stack.forward(hidden).clone()
    stack.out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(stack.out, eager)
    del g


@pytest.mark.gpu
def test_cuda_stack_tree_commit_is_the_path_chain(cuda):
    """After a tree round and commit(path): every gated-delta state, conv window and the
    attention cache entries context .. context + keep - 1 match the reference's chain
    forward of the path."""
    import stack_ref
    cfg = vs.TINY
    parents = TREES["branchy"]
    path = [0, 1, 4]
    stack = vs.VerifyStack(cfg, 0, 1, seed=0, device=cuda, tree=True)
    pre = {i: {k: v.clone() for k, v in S.items()} for i, S in enumerate(stack.state["layers"])}
    hidden = vs.make_block(cfg, 3, cuda)
    stack.set_tree(parents)
    stack.forward(hidden)
    stack.commit(path)
    torch.cuda.synchronize()
    ref = stack_ref.forward(cfg, stack.plan, stack.w, {"layers": [pre[i] for i in sorted(pre)]}, hidden[path])
    gi = ai = 0
    kc1 = cfg.conv_kernel - 1
    for li, (L, S) in enumerate(zip(stack.w["layers"], stack.state["layers"])):
        if L["kind"] == "gdn":
            s, sr = S["snapshot"].cpu().numpy(), ref["state"][gi].numpy()
            assert np.max(np.abs(s - sr)) / np.max(np.abs(sr)) <= 2e-2, gi
            want_win = torch.cat([pre[li]["window"].float().cpu(), ref["conv_in"][gi]])[-kc1:]
            assert closeness(S["window"].float().cpu().numpy(), want_win.numpy()) <= 2e-2, gi
            gi += 1
        else:
            for key in ("cache_k", "cache_v"):
                got = S[key].float().cpu()[:, cfg.context:cfg.context + len(path)]
                want = ref[key][ai][:, cfg.context:cfg.context + len(path)]
                assert closeness(got.numpy(), want.numpy()) <= 2e-2, key
            ai += 1

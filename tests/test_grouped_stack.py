"""The verify stack with shared gated-delta key heads (TINY_GROUPED: 2 key heads for 4
value heads, as the reference's fixture has, Tests/DFlashKitTests/TinyHybridTarget.swift:27-30).

Value head h reads key head h / (H / Hk).  CPU: the stack reference on the grouped model
equals, bit for bit, the reference on the ungrouped model whose q and k rows (in_proj, conv
weights, conv window) are the key heads' repeated per value head; the shard plan tiles
the grouped in_proj; two gloo ranks match one; a grouped checkpoint loads back to the
same shards.  GPU: the CUDA stack against the reference."""
from __future__ import annotations

import sys
from dataclasses import asdict, replace
from pathlib import Path

import numpy as np
import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))

import verify_stack as vs  # noqa: E402

CFG = vs.TINY_GROUPED


def closeness(y, ref) -> float:
    y, ref = np.asarray(y, dtype=np.float64), np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(y - ref)) / max(float(np.max(np.abs(ref))), 1.0))


def _expand(cfg, w, st):
    """Weights and state of the ungrouped model equal to the grouped one: the key heads'
    q / k rows repeated per value head (in_proj rows, conv weight rows, window columns)."""
    H, Hk, dk = cfg.gdn_heads, cfg.gdn_kheads, cfg.gdn_dk
    g = H // Hk

    def rep_rows(t, off):  # rows [off, off + Hk dk) -> per value head
        blk = t[off:off + Hk * dk]
        return blk.unflatten(0, (Hk, dk)).repeat_interleave(g, dim=0).flatten(0, 1)

    w2 = {**w, "layers": []}
    for L in w["layers"]:
        L = dict(L)
        if L["kind"] == "gdn":
            q = L["in_proj"]
            parts = lambda t: torch.cat([rep_rows(t, 0), rep_rows(t, Hk * dk), t[2 * Hk * dk:]]).contiguous()
            L["in_proj"] = vs.Quant(parts(q.w), parts(q.scales), parts(q.biases), q.group, q.bits)
            L["conv"] = parts(L["conv"])
        w2["layers"].append(L)
    st2 = {"layers": []}
    for S in st["layers"]:
        S = dict(S)
        if "window" in S:
            S["window"] = torch.cat([rep_rows(S["window"].t(), 0).t(), rep_rows(S["window"].t(), Hk * dk).t(),
                                     S["window"][:, 2 * Hk * dk:]], dim=1).contiguous()
        st2["layers"].append(S)
    return w2, st2


@pytest.fixture(scope="module")
def grouped_reference():
    import stack_ref
    plan = vs.shard_plan(CFG, 0, 1)
    w = vs.build_rank_weights(CFG, plan, 0, "cpu")
    st = vs.build_rank_state(CFG, plan, 0, "cpu")
    hidden = vs.make_block(CFG, 0, "cpu")
    return plan, w, st, hidden, stack_ref.forward(CFG, plan, w, st, hidden)


def test_grouped_reference_is_the_ungrouped_one_on_repeated_key_heads(grouped_reference):
    import stack_ref
    plan, w, st, hidden, r = grouped_reference
    ucfg = replace(CFG, gdn_key_heads=0)
    w2, st2 = _expand(CFG, w, st)
    u = stack_ref.forward(ucfg, vs.shard_plan(ucfg, 0, 1), w2, st2, hidden)
    assert torch.equal(r["out"], u["out"])
    for gi in range(len(r["state"])):
        assert torch.equal(r["state"][gi], u["state"][gi])
    # and the grouping matters: pairing value heads with other key heads changes the result
    w3 = {**w, "layers": [dict(L) for L in w["layers"]]}
    for L in w3["layers"]:
        if L["kind"] == "gdn":
            q = L["in_proj"]
            dk = CFG.gdn_dk
            swap = lambda t: torch.cat([t[dk:2 * dk], t[:dk], t[2 * dk:]])  # key heads 0 and 1 trade q rows
            L["in_proj"] = vs.Quant(swap(q.w), swap(q.scales), swap(q.biases), q.group, q.bits)
    assert closeness(stack_ref.forward(CFG, plan, w3, st, hidden)["out"].numpy(), r["out"].numpy()) > 1e-2


@pytest.mark.parametrize("world", [1, 2])
def test_grouped_shards_tile_the_in_projection(world):
    H, Hk, dk, dv = CFG.gdn_heads, CFG.gdn_kheads, CFG.gdn_dk, CFG.gdn_dv
    hits = np.zeros(2 * Hk * dk + 2 * H * dv + 2 * H, dtype=np.int64)
    for r in range(world):
        p = vs.shard_plan(CFG, r, world)
        assert p.gdn_key_heads == Hk // world and p.gdn_key_head0 == r * Hk // world
        for a, b in vs._ranges_gdn_in(CFG, p):
            hits[a:b] += 1
    assert (hits == 1).all()
    with pytest.raises(ValueError):
        vs.shard_plan(CFG, 0, 4)  # 2 key heads do not split over 4 ranks


def test_grouped_tp2_over_gloo_matches_tp1(tmp_path, grouped_reference):
    import stack_workers
    from test_verify_stack import _run_ranks, free_port
    ref = grouped_reference[4]["out"].numpy()
    errs = {}
    for drop in (False, True):
        out = tmp_path / f"grouped_tp2_{int(drop)}.pt"
        port = free_port()
        codes = _run_ranks(stack_workers.gloo_reference_rank, 2, lambda k: (k, 2, port, str(out), asdict(CFG), drop))
        assert codes == [0, 0], codes
        errs[drop] = closeness(torch.load(out)["out"].numpy(), ref)
    assert errs[False] <= 3e-2
    assert errs[True] > max(0.05, 10 * errs[False])


@pytest.mark.parametrize("world", [1, 2])
def test_grouped_checkpoint_loads_to_the_same_shards(tmp_path, world):
    import mlx_checkpoint as mc
    full = vs.build_rank_weights(CFG, vs.shard_plan(CFG, 0, 1), 0, "cpu")
    mc.save_stack_checkpoint(tmp_path, CFG, full)
    config, tensors = mc.load_directory(tmp_path)
    assert mc.stack_config_from_json(config, context=CFG.context, block=CFG.block) == CFG
    for r in range(world):
        plan = vs.shard_plan(CFG, r, world)
        got, want = mc.stack_from_checkpoint(CFG, plan, config, tensors, "cpu"), vs.build_rank_weights(CFG, plan, 0,
                                                                                                      "cpu")
        for La, Lb in zip(got["layers"], want["layers"]):
            for k, v in Lb.items():
                if isinstance(v, torch.Tensor):
                    assert torch.equal(La[k], v), k
                elif isinstance(v, vs.Quant):
                    assert torch.equal(La[k].w, v.w) and torch.equal(La[k].scales, v.scales), k


@pytest.mark.gpu
def test_cuda_grouped_stack_matches_reference(cuda, grouped_reference):
    import stack_ref
    stack = vs.VerifyStack(CFG, 0, 1, seed=0, device=cuda)
    hidden = vs.make_block(CFG, 0, cuda)
    # The stack's pre-round state was drawn by the CUDA generator, whose draws differ from the
    # CPU generator's for the same seed: the commit reference must start from these bits.
    pre = {"layers": [{k: v.cpu().clone() for k, v in S.items()} for S in stack.state["layers"]]}
    out = stack.forward(hidden).float().cpu()
    torch.cuda.synchronize()
    ref = stack_ref.forward(CFG, stack.plan, stack.w, stack.state, hidden)
    assert closeness(out.numpy(), ref["out"].numpy()) <= 2e-2
    for gi in range(len(ref["state"])):
        s, sr = stack.state_out[gi].cpu().numpy(), ref["state"][gi].numpy()
        assert np.max(np.abs(s - sr)) / np.max(np.abs(sr)) <= 2e-2
    stack.commit(list(range(5)))  # replay over grouped key heads: the state after 5 rows
    torch.cuda.synchronize()
    ref5 = stack_ref.forward(CFG, stack.plan, stack.w, pre, hidden[:5])
    gi = 0
    for S in stack.state["layers"]:
        if "snapshot" in S:
            s, sr = S["snapshot"].cpu().numpy(), ref5["state"][gi].numpy()
            assert np.max(np.abs(s - sr)) / np.max(np.abs(sr)) <= 2e-2
            gi += 1

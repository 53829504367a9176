"""dflash_stack: the verify stack as one C-ABI object (include/dflash_stack.h), for hosts that
drive a verify round through libdflashcuda alone (the reference's generator runs its verify
forward, LM head and accept in-process, DFlashSpeculativeGenerator.swift:389-398 and
:555-571, and rolls back with rollbackGatedDeltaRound, :455-460).

CPU: the creation checks reject bad descriptors before any CUDA call.  GPU: over the same
shard weights and a copy of the same state, the object computes exactly the bits the Python
orchestration (verify_stack.VerifyStack) computes, round after round: forward, verify
(tokens and accept count), commit of a partially accepted round, advance, next round.
"""
from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))

import verify_stack as vs  # noqa: E402


def test_create_rejects_bad_descriptors(dc):
    h = ctypes.c_void_p()
    assert dc.lib.dflash_stack_create(None, 0, ctypes.byref(h)) == dc.DFLASH_ERR_INVALID_ARGUMENT
    layers = (dc.StackLayer * 1)()
    d = dc.StackDesc()
    d.layers, d.hidden, d.block, d.world, d.rank, d.group, d.bits = 1, 256, 8, 1, 0, 64, 4
    d.layer = layers
    d.final_norm = 0x10000
    d.max_len = 64
    for field, value in (("block", 17), ("world", 0), ("rank", 1), ("bits", 3)):
        bad = dc.StackDesc.from_buffer_copy(d)
        setattr(bad, field, value)
        assert dc.lib.dflash_stack_create(ctypes.byref(bad), 0, ctypes.byref(h)) == dc.DFLASH_ERR_INVALID_ARGUMENT
    two = dc.StackDesc.from_buffer_copy(d)
    two.world = 2  # no exchange bases
    assert dc.lib.dflash_stack_create(ctypes.byref(two), 0, ctypes.byref(h)) == dc.DFLASH_ERR_INVALID_ARGUMENT
    assert "exchange" in dc.last_error()
    # the layer has no tensors: its shapes are checked before anything is allocated
    assert dc.lib.dflash_stack_create(ctypes.byref(d), 0, ctypes.byref(h)) == dc.DFLASH_ERR_INVALID_ARGUMENT
    assert dc.lib.dflash_stack_create(ctypes.byref(d), 60, ctypes.byref(h)) == dc.DFLASH_ERR_INVALID_ARGUMENT
    assert "max_len" in dc.last_error()


def _clone_state(state):
    return {"layers": [{k: v.clone() for k, v in S.items()} for S in state["layers"]]}


def _same(a, b):
    return torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a,
                       b.view(torch.int16) if b.dtype == torch.bfloat16 else b)


@pytest.mark.gpu
@pytest.mark.parametrize("cfg", [vs.TINY, vs.TINY_GROUPED, vs.TP_CHECK], ids=["tiny", "grouped", "tp_check"])
def test_stack_object_matches_the_python_orchestration(dc, cuda, cfg):
    from dataclasses import replace
    # caches with room for the rounds below (each round's block rows land past the committed ones)
    state = vs.build_rank_state(replace(cfg, block=3 * cfg.block), vs.shard_plan(cfg, 0, 1), 0, cuda)
    py = vs.VerifyStack(cfg, 0, 1, seed=0, device=cuda, state=state)
    cstate = _clone_state(py.state)
    cs = dc.CStack(cfg, py.plan, py.w, cstate, py.context)
    try:
        hidden = vs.make_block(cfg, 0, cuda)
        out_c = torch.empty_like(py.out)
        for rnd in range(2):
            out_py = py.forward(hidden).clone()
            cs.forward(hidden, out_c)
            torch.cuda.synchronize()
            assert _same(out_c, out_py), f"forward, round {rnd}"
            proposals = torch.arange(7, 7 + cfg.block - 1, dtype=torch.int32, device=cuda)
            tok_py, acc_py = py.verify(hidden, proposals)
            tok_c = torch.empty_like(tok_py)
            acc_c = torch.empty_like(acc_py)
            cs.verify(hidden, proposals, tok_c, acc_c)
            torch.cuda.synchronize()
            assert torch.equal(tok_c, tok_py) and torch.equal(acc_c, acc_py), f"verify, round {rnd}"
            keep = 5 - rnd  # a partially accepted round: commit, advance
            py.commit(list(range(keep)))
            py.advance(keep)
            cs.commit(keep)
            cs.advance(keep)
            torch.cuda.synchronize()
            assert cs.context == py.context
            for S, C in zip(py.state["layers"], cstate["layers"]):
                for k in S:
                    assert _same(C[k], S[k]), (rnd, k)
        # a round allocates nothing: the forward records into a CUDA graph and replays the same bits
        eager = torch.empty_like(out_c)
        cs.forward(hidden, eager)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        graphed = torch.empty_like(out_c)
        with torch.cuda.graph(g):
            cs.forward(hidden, graphed)
        g.replay()
        torch.cuda.synchronize()
        assert _same(graphed, eager)
        del g
        assert dc.device_error() == 0
    finally:
        cs.close()

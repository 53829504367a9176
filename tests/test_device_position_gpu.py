"""A verify round captured once and replayed across a decode loop: with device_position the
attention kernels read the cache position from device memory (dflash_stack_attn_prep_ex /
dflash_stack_attn_decode_ex), so after commit + advance the same CUDA graph runs at the new
context.  Each replay must give the bits of an eager forward at that context, and a
position past the cache must be refused by the kernels' own check (no write, the
DFLASH_DEVERR_POSITION bit raised)."""
from __future__ import annotations

from dataclasses import replace

import pytest
import torch

import verify_stack as vs

pytestmark = pytest.mark.gpu


def test_one_graph_serves_a_decode_loop(cuda):
    cfg = replace(vs.TINY, context=4)
    caches = replace(cfg, block=32)  # attention caches of 36 positions
    plan = vs.shard_plan(cfg, 0, 1)
    w = vs.build_rank_weights(cfg, plan, 0, cuda)

    def make(device_position):
        return vs.VerifyStack(cfg, 0, 1, device=cuda, weights=w, state=vs.build_rank_state(caches, plan, 0, cuda),
                              device_position=device_position)

    graphed, eager = make(True), make(False)
    hidden = vs.make_block(cfg, 0, cuda)
    graph = graphed.capture(hidden)
    for _ in range(4):
        eager.forward(hidden)
        graphed.out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(graphed.out, eager.out), graphed.context
        for s in (graphed, eager):
            s.commit([0, 1, 2])
            s.advance(3)
    del graph
    assert graphed.context == eager.context == cfg.context + 12


def test_a_position_past_the_cache_is_refused(dc, cuda):
    M, hq, hkv, d, max_len = 8, 4, 2, 64, 16
    gen = torch.Generator(device=cuda).manual_seed(1)
    qkv = torch.randn(M, (2 * hq + 2 * hkv) * d, generator=gen, device=cuda).to(torch.bfloat16)
    norm = torch.ones(d, dtype=torch.bfloat16, device=cuda)
    ck = torch.randn(hkv, max_len, d, generator=gen, device=cuda).to(torch.bfloat16)
    cv = torch.randn_like(ck)
    ck0, cv0, qkv0 = ck.clone(), cv.clone(), qkv.clone()
    out = torch.zeros(M, hq * d, dtype=torch.bfloat16, device=cuda)
    assert dc.device_error() == 0
    position = torch.tensor([max_len - M + 1], dtype=torch.int32, device=cuda)
    dc.stack_attn_prep(qkv, norm, norm, ck, cv, hq, hkv, 64, 0, 1e-6, 1e4, position=position)
    dc.stack_attn_decode(qkv, ck, cv, out, hq, hkv, 0, 0.125, position=position)
    torch.cuda.synchronize()
    assert dc.device_error() == dc.DEVERR_POSITION
    assert torch.equal(ck, ck0) and torch.equal(cv, cv0) and torch.equal(qkv, qkv0) and not out.any()
    position.fill_(max_len - M)  # the last position that fits
    dc.stack_attn_prep(qkv, norm, norm, ck, cv, hq, hkv, 64, 0, 1e-6, 1e4, position=position)
    dc.stack_attn_decode(qkv, ck, cv, out, hq, hkv, 0, 0.125, position=position)
    torch.cuda.synchronize()
    assert dc.device_error() == 0 and torch.isfinite(out.float()).all() and out.any()

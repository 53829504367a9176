"""Gated-delta layers whose q and k have fewer heads than v (the target's Qwen3.5
configuration allows linear_num_key_heads < linear_num_value_heads; the reference's fixture
has 2 key heads for 4 value heads, Tests/DFlashKitTests/TinyHybridTarget.swift:27-30).

Value head h reads key head h / (H / Hk).  Each grouped entry point must give the bits of
the ungrouped one run on q, k (and their conv channels) repeated per value head: the
arithmetic per value head is the same, only where q and k are read from differs.  The
recurrence is also checked against the fp64 oracle on the repeated inputs."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _repeat_heads(t, group, axis):
    return t.repeat_interleave(group, dim=axis).contiguous()


@pytest.mark.parametrize("H,Hk,dk", [(4, 2, 128), (32, 16, 128), (8, 1, 64)])
def test_grouped_step_replay_and_tree_equal_repeated_key_heads(dc, O, cuda, H, Hk, dk):
    T, dv, g = 8, dk, H // Hk
    gen = torch.Generator(device=cuda).manual_seed(H + Hk)
    snap = 0.1 * torch.randn(H, dv, dk, generator=gen, device=cuda)
    q = torch.randn(T, Hk, dk, generator=gen, device=cuda).to(torch.bfloat16)
    k = torch.nn.functional.normalize(torch.randn(T, Hk, dk, generator=gen, device=cuda), dim=-1).to(torch.bfloat16)
    v = torch.randn(T, H, dv, generator=gen, device=cuda).to(torch.bfloat16)
    alpha = 0.9 + 0.1 * torch.rand(T, H, generator=gen, device=cuda)
    beta = torch.rand(T, H, generator=gen, device=cuda)
    qr, kr = _repeat_heads(q, g, 1), _repeat_heads(k, g, 1)
    scale = 1.0 / math.sqrt(dk)

    st_g, st_u = torch.empty_like(snap), torch.empty_like(snap)
    o_g = torch.empty(T, H, dv, dtype=torch.bfloat16, device=cuda)
    o_u = torch.empty_like(o_g)
    dc.gdn_step(snap, st_g, q, k, v, alpha, beta, out=o_g, q_scale=scale)
    dc.gdn_step(snap, st_u, qr, kr, v, alpha, beta, out=o_u, q_scale=scale)

    rows = [0, 2, 3, 6]
    rp_g, rp_u = torch.empty_like(snap), torch.empty_like(snap)
    dc.gdn_replay(snap[None], rp_g[None], k[None], v[None], alpha[None], beta[None], keep=4, rows=rows)
    dc.gdn_replay(snap[None], rp_u[None], kr[None], v[None], alpha[None], beta[None], keep=4, rows=rows)

    parents = torch.tensor([-1, 0, 0, 1, 1, 2, 3, 5], dtype=torch.int32, device=cuda)
    tr_g, tr_u = torch.empty_like(o_g), torch.empty_like(o_g)
    dc.gdn_step_tree(snap, q, k, v, alpha, beta, parents, tr_g, q_scale=scale)
    dc.gdn_step_tree(snap, qr, kr, v, alpha, beta, parents, tr_u, q_scale=scale)
    torch.cuda.synchronize()
    assert torch.equal(st_g, st_u) and torch.equal(o_g, o_u)
    assert torch.equal(rp_g, rp_u)
    assert torch.equal(tr_g, tr_u)

    bits = lambda t: t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    want, _ = O.gdn_recurrence(snap.cpu().numpy(), bits(kr), bits(v), alpha.cpu().numpy(), beta.cpu().numpy(), T)
    got = st_g.cpu().numpy().astype(np.float64)
    assert np.abs(got - want).max() / np.abs(want).max() <= 1e-4
    assert dc.device_error() == 0


@pytest.mark.parametrize("H,Hk,dk,kc", [(4, 2, 64, 4), (32, 16, 128, 4), (6, 3, 32, 2)])
@pytest.mark.parametrize("tree", [False, True])
def test_grouped_conv_gates_equal_repeated_key_channels(dc, cuda, H, Hk, dk, kc, tree):
    M, g = 8, H // Hk
    gen = torch.Generator(device=cuda).manual_seed(H * kc + tree)
    Cg = (2 * Hk + H) * dk
    x = torch.randn(M, Cg + 2 * H, generator=gen, device=cuda).to(torch.bfloat16)  # [q | k | v | b | a]
    win = torch.randn(kc - 1, Cg, generator=gen, device=cuda).to(torch.bfloat16)
    w = (0.5 * torch.randn(Cg, kc, generator=gen, device=cuda)).to(torch.bfloat16)
    a_log = torch.randn(H, generator=gen, device=cuda)
    dt = torch.randn(H, generator=gen, device=cuda)
    parents = torch.tensor([-1, 0, 0, 1, 1, 2, 3, 5], dtype=torch.int32, device=cuda) if tree else None

    def expand(t, axis):  # channels [q | k | v] with q, k per key head -> per value head
        q, k, v = torch.split(t, [Hk * dk, Hk * dk, H * dk], dim=axis)
        rep = lambda u: u.unflatten(axis, (Hk, dk)).repeat_interleave(g, dim=axis).flatten(axis, axis + 1)
        return torch.cat([rep(q), rep(k), v], dim=axis).contiguous()

    xu = torch.cat([expand(x[:, :Cg], 1), x[:, Cg:]], dim=1).contiguous()
    ab_g, ab_u = x[:, Cg:], xu[:, 3 * H * dk:]
    yg = torch.empty(M * Cg, dtype=torch.bfloat16, device=cuda)
    al_g, be_g = (torch.empty(M, H, device=cuda) for _ in range(2))
    dc.stack_gdn_conv_gates(x, win, w, yg, ab_g, a_log, dt, al_g, be_g, H, dk, parents=parents, k_heads=Hk)
    yu = torch.empty(3, M, H, dk, dtype=torch.bfloat16, device=cuda)
    al_u, be_u = (torch.empty(M, H, device=cuda) for _ in range(2))
    dc.stack_gdn_conv_gates(xu, expand(win, 1), expand(w, 0), yu, ab_u, a_log, dt, al_u, be_u, H, dk,
                            parents=parents)
    torch.cuda.synchronize()
    qg, kg, vg = torch.split(yg, [M * Hk * dk, M * Hk * dk, M * H * dk])
    assert torch.equal(_repeat_heads(qg.view(M, Hk, dk), g, 1), yu[0])
    assert torch.equal(_repeat_heads(kg.view(M, Hk, dk), g, 1), yu[1])
    assert torch.equal(vg.view(M, H, dk), yu[2])
    assert torch.equal(al_g, al_u) and torch.equal(be_g, be_u)

"""LM head with the fused argmax, and the greedy accept of a verify round
(acceptedPrefix, Sources/DFlashKit/DFlashSpeculativeGenerator.swift:555-571).

CPU: the oracle's accept restatement on hand-built cases (leading run, first mismatch,
no drafts, ties resolved to the first index).  GPU: the fused argmax equals the first
index of the maximum of the logits the same kernel writes (bit-identical bf16), its
maximum logit is within the qmm tolerance of the fp64 oracle, and dflash_accept
matches the oracle's accept on planted proposals — at a ragged vocabulary and at the
target's 248,320."""
from __future__ import annotations

import numpy as np
import pytest


def _bits(a):
    import ml_dtypes
    return np.asarray(a, dtype=np.float32).astype(ml_dtypes.bfloat16).view(np.uint16)


def test_oracle_accept_leading_run(O):
    logits = np.full((4, 6), -1.0, dtype=np.float32)
    for i, t in enumerate([2, 5, 1, 3]):
        logits[i, t] = 1.0
    tokens, acc = O.accepted_prefix(_bits(logits), [2, 5, 0])
    assert tokens.tolist() == [2, 5, 1, 3] and acc == 2
    assert O.accepted_prefix(_bits(logits), [2, 5, 1])[1] == 3
    assert O.accepted_prefix(_bits(logits), [0, 5, 1])[1] == 0          # later matches do not count
    assert O.accepted_prefix(_bits(logits[:1]), [])[1] == 0             # no drafts


def test_oracle_accept_ties_take_first_index(O):
    logits = np.zeros((2, 5), dtype=np.float32)
    logits[0, [1, 3]] = 2.0
    logits[1, [0, 4]] = 2.0
    tokens, acc = O.accepted_prefix(_bits(logits), [1])
    assert tokens.tolist() == [1, 0] and acc == 1


def _run(dc, O, cuda, M, V, K, group, bits, seed):
    import torch
    import verify_stack as vs
    gen = torch.Generator(device=cuda).manual_seed(seed)
    q = vs.random_quant(gen, V, K, group, bits, cuda)
    x = torch.randn(M, K, generator=gen, device=cuda).to(torch.bfloat16)
    y = dc.qmm(x, q.w, q.scales, q.biases, group, bits)
    keys = dc.lm_head_argmax(x, q.w, q.scales, q.biases, group, bits)
    torch.cuda.synchronize()
    tok = (~(keys & 0xFFFFFFFF).to(torch.int64)) & 0xFFFFFFFF
    want = torch.argmax(y.float(), dim=1)  # first index of the maximum
    assert torch.equal(tok, want)
    # the winning logit against the fp64 oracle on a sample of rows around it
    xb = x.view(torch.int16).cpu().numpy().view(np.uint16)
    wq = q.w.cpu().numpy().view(np.uint32)
    s = q.scales.view(torch.int16).cpu().numpy().view(np.uint16)
    b = q.biases.view(torch.int16).cpu().numpy().view(np.uint16)
    cols = np.unique(np.concatenate([want.cpu().numpy(), np.arange(0, V, max(1, V // 512))]))
    ref = O.qmm_f64(xb, wq[cols], s[cols], b[cols], group, bits)
    got = y.float().cpu().numpy()[:, cols]
    assert O.closeness(got, ref) <= 1e-2
    return y, keys


@pytest.mark.gpu
@pytest.mark.parametrize("M,V,K,group,bits", [(8, 4099 * 8, 1024, 64, 4), (5, 2000, 512, 32, 8),
                                              (8, 248320, 5120, 64, 4)])
def test_lm_head_argmax_and_accept(dc, O, cuda, M, V, K, group, bits):
    import torch
    y, keys = _run(dc, O, cuda, M, V, K, group, bits, seed=M + V)
    ybits = y.view(torch.int16).cpu().numpy().view(np.uint16)
    tokens_ref, _ = O.accepted_prefix(ybits, np.zeros(M - 1, dtype=np.int32))
    for plant in range(M):  # proposals agreeing up to `plant`, then one wrong token
        prop = tokens_ref[:M - 1].copy()
        if plant < M - 1:
            prop[plant] = (prop[plant] + 1) % V
        t_ref, acc_ref = O.accepted_prefix(ybits, prop)
        tokens, acc = dc.accept(keys, torch.from_numpy(prop).to(cuda))
        torch.cuda.synchronize()
        assert tokens.cpu().numpy().tolist() == t_ref.tolist()
        assert int(acc.item()) == acc_ref == min(plant, M - 1)

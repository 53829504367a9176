"""CPU reference of the tensor-parallel verify stack (TEST INFRASTRUCTURE ONLY).

Only tests/ import this module, as the checker of dflash-swift_b200/verify_stack.py.
It runs one rank's shard of the hybrid gated-delta / attention stack on the CPU in
fp32 (fp64 for the projections), rounding to bf16 exactly where the CUDA path stores
bf16, so the two agree up to accumulation order.  The projections go through the
pinned qmm oracle (``oracle.qmm_f64``, MLX affine dequantisation w = s*q + b,
Sources/DFlashKit/SmallMQuantizedMatmul.swift:59) and the recurrence through the pinned
gated-delta oracle (``oracle.gdn_recurrence``: S <- aS; u = v - Sk; S <- S + b u k^T;
o = S q, the update the reference replays in rollbackGatedDeltaRound,
DFlashSpeculativeGenerator.swift:455-460).  The layer glue (RMSNorm, the causal conv,
q/k L2 normalisation and gates, gated output norm, rotary attention with an output
gate, SiLU MLP) restates the Qwen3.5-style target that the reference's verify forward
calls (DFlashSpeculativeGenerator.swift:397); that model is in an external MLX fork not
present in the reference tree, so this part of the stack is parity unpinned beyond
its self-consistency (TP=P equals TP=1).

Weights and state come in the layout of verify_stack.build_rank_weights /
build_rank_state (torch tensors, any device; copied to the CPU here).
"""
from __future__ import annotations

import math
from typing import Callable, Optional

import numpy as np
import torch

import oracle as O


def rb(t: torch.Tensor) -> torch.Tensor:
    """Round fp32 to bf16 and back (a bf16 store)."""
    return t.to(torch.bfloat16).to(torch.float32)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to("cpu").contiguous().view(torch.int16).numpy().view(np.uint16)


def qmm(x: torch.Tensor, q) -> torch.Tensor:
    """rb(x . deq(W)^T) through the fp64 qmm oracle.  x: fp32 holding bf16 values [M, K]."""
    y = O.qmm_f64(_bits(x.to(torch.bfloat16)), q.w.detach().cpu().contiguous().numpy().view(np.uint32),
                  _bits(q.scales), _bits(q.biases), q.group, q.bits)
    return rb(torch.from_numpy(y).to(torch.float32))


def add_rmsnorm(resid: torch.Tensor, delta: Optional[torch.Tensor], w: torch.Tensor, eps: float) -> torch.Tensor:
    if delta is not None:
        resid += delta
    rs = torch.rsqrt(resid.pow(2).mean(dim=1, keepdim=True) + eps)
    return rb(resid * rs * w.float())


def silu(t: torch.Tensor) -> torch.Tensor:
    return t / (1.0 + torch.exp(-t))


def tree_paths(parents, M: int):
    """For block rows with parent list `parents` (-1: a root; an entry outside [0, r) is
    treated as -1): each row's root-to-row path (root first), and one path per leaf, the
    leaves in row order.  A chain is parents = [-1, 0, 1, ...]."""
    par = [int(p) if 0 <= int(p) < r else -1 for r, p in enumerate(parents)]
    assert len(par) == M
    anc = []
    for r in range(M):
        path = [r]
        while par[path[-1]] >= 0:
            path.append(par[path[-1]])
        anc.append(path[::-1])
    has_child = {p for p in par if p >= 0}
    leaves = [r for r in range(M) if r not in has_child]
    return anc, [anc[r] for r in leaves]


def conv_silu(x: torch.Tensor, window: torch.Tensor, w: torch.Tensor, parents=None) -> torch.Tensor:
    """x [M, C]; window [kc-1, C] (older first); w [C, kc], last tap on the current row.
    Row t convolves the window followed by the rows before it (a chain) or by its
    root-to-t path (a tree with parent list `parents`)."""
    M = x.shape[0]
    kc = w.shape[1]
    anc, _ = tree_paths(parents if parents is not None else [-1] + list(range(M - 1)), M)
    out = torch.zeros_like(x)
    for t in range(M):
        hist = torch.cat([window.float(), x[anc[t]]], dim=0)
        seg = hist[-kc:]  # the last kc inputs of t's history; the last one is x[t]
        out[t] = (seg * w.float().t()).sum(dim=0)
    return rb(silu(out))


def l2norm_heads(v: torch.Tensor) -> torch.Tensor:
    """v [M, h, d] -> rb(v / sqrt(sum v^2 + 1e-6)) per head."""
    return rb(v * torch.rsqrt(v.pow(2).sum(dim=-1, keepdim=True) + 1e-6))


def gdn_gates(ab: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor, h: int):
    b, a = ab[:, :h], ab[:, h:2 * h]
    x = a + dt_bias.float()
    sp = torch.where(x > 20.0, x, torch.log1p(torch.exp(x)))
    alpha = torch.exp(-torch.exp(a_log.float()) * sp)
    beta = 1.0 / (1.0 + torch.exp(-b))
    return alpha, beta


def gdn_step(snapshot: torch.Tensor, q, k, v, alpha, beta, q_scale: float):
    """Through the C oracle: returns (state fp32 [h, dv, dk], o rb [M, h, dv])."""
    M = q.shape[0]
    s, o = O.gdn_recurrence(snapshot.detach().cpu().float().numpy(), _bits(k.to(torch.bfloat16)),
                            _bits(v.to(torch.bfloat16)), alpha.numpy(), beta.numpy(), M,
                            q_bits=_bits(q.to(torch.bfloat16)), q_scale=q_scale)
    return torch.from_numpy(s).to(torch.float32), rb(torch.from_numpy(o).to(torch.float32))


def gated_norm(o: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """o [M, h, dv]; z [M, h*dv]."""
    M, h, dv = o.shape
    rs = torch.rsqrt(o.pow(2).mean(dim=-1, keepdim=True) + eps)
    return rb((o * rs * w.float()).reshape(M, h * dv) * silu(z))


def rope(v: torch.Tensor, rot: int, theta: float, pos: torch.Tensor) -> torch.Tensor:
    """Rotate-half over the first rot dims of v [M, h, d]; frequency theta^(-2i/rot)."""
    half = rot // 2
    i = torch.arange(half, dtype=torch.float32)
    inv = torch.exp2(-(2.0 * i / rot) * math.log2(theta))
    ang = pos.float()[:, None] * inv[None, :]  # [M, half]
    cs, sn = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    out = v.clone()
    a, b = v[..., :half], v[..., half:rot]
    out[..., :half] = a * cs - b * sn
    out[..., half:rot] = b * cs + a * sn
    return out


def head_rmsnorm(v: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return rb(v * torch.rsqrt(v.pow(2).mean(dim=-1, keepdim=True) + eps) * w.float())


def attention(q, gate, cache_k, cache_v, pos0: int, scale: float, visible=None):
    """q, gate [M, hq, d]; caches [hkv, L, d] (fp32 holding bf16).  Token t sees keys
    0 .. pos0 + t, or (a tree) keys 0 .. pos0 - 1 and pos0 + a for the block rows a in
    visible[t].  Returns rb(softmax(q K^T scale) V * sigmoid(gate)) [M, hq*d]."""
    M, hq, d = q.shape
    hkv = cache_k.shape[0]
    out = torch.zeros(M, hq, d)
    for h in range(hq):
        kv = h // (hq // hkv)
        for t in range(M):
            keys = list(range(pos0 + t + 1)) if visible is None else list(range(pos0)) + [pos0 + a for a in visible[t]]
            s = (cache_k[kv, keys].double() @ q[t, h].double()) * scale
            p = torch.softmax(s, dim=0)
            out[t, h] = (p @ cache_v[kv, keys].double()).float()
    return rb(out * torch.sigmoid(gate)).reshape(M, hq * d)


def forward(cfg, plan, weights: dict, state: dict, hidden: torch.Tensor,
            all_reduce: Optional[Callable[[torch.Tensor], None]] = None, parents=None,
            context: Optional[int] = None) -> dict:
    """One rank's verify forward over the M = hidden.shape[0] block rows.  Returns the final
    hidden states and, per layer, the capture and state the CUDA stack produces
    (gated-delta conv output, alpha, beta, state after the block; attention cache rows
    written).  With a tree parent list (`parents`, the tree round of mtpTreePlanKey) every
    row computes what a chain over its root-to-row path computes: convolution and
    recurrence along the path, rotary position context + depth, attention to the prefix
    and the path's rows; the state entry is then None (the state after a tree round is the
    replay of the accepted path).  `context`: tokens already in the attention caches
    (cfg.context when not given); the block's rows go to cache rows context + row."""
    all_reduce = all_reduce or (lambda t: None)
    M, H = hidden.shape[0], cfg.hidden
    ctx = cfg.context if context is None else int(context)
    anc, paths = tree_paths(parents, M) if parents is not None else (None, None)
    eps = cfg.eps
    resid = torch.zeros(M, H)
    delta = hidden.detach().cpu().float()
    cap = {"qkv": [], "alpha": [], "beta": [], "state": [], "cache_k": [], "cache_v": [], "conv_in": []}
    h, dk, dv = plan.gdn_heads, cfg.gdn_dk, cfg.gdn_dv
    d, hq, hkv = cfg.head_dim, plan.attn_heads, plan.kv_heads
    cpu = lambda t: t.detach().cpu()
    for L, S in zip(weights["layers"], state["layers"]):
        L = {k: (cpu(v) if isinstance(v, torch.Tensor) else v) for k, v in L.items()}
        normed = add_rmsnorm(resid, delta, L["ln"], eps)
        if L["kind"] == "gdn":
            # q and k have hk heads, each read by h / hk consecutive value heads
            hk = getattr(plan, "gdn_key_heads", 0) or h
            C = (2 * hk + h) * dk
            proj = qmm(normed, L["in_proj"])
            cap["conv_in"].append(proj[:, :C])
            conv = conv_silu(proj[:, :C], cpu(S["window"]), L["conv"], parents)
            q = conv[:, :hk * dk].reshape(M, hk, dk)
            k = conv[:, hk * dk:2 * hk * dk].reshape(M, hk, dk)
            v = conv[:, 2 * hk * dk:].reshape(M, h, dk)
            q, k = l2norm_heads(q), l2norm_heads(k)
            qr, kr = q.repeat_interleave(h // hk, dim=1), k.repeat_interleave(h // hk, dim=1)
            ab = proj[:, 2 * hk * dk + 2 * h * dv:]
            alpha, beta = gdn_gates(ab, L["a_log"], L["dt_bias"], h)
            if parents is None:
                st, o = gdn_step(cpu(S["snapshot"]), qr, kr, v, alpha, beta, 1.0 / math.sqrt(dk))
            else:  # each row's output from the first leaf's path (row order) that holds it
                st, o, done = None, torch.zeros(M, h, dv), set()
                for path in paths:
                    _, op = gdn_step(cpu(S["snapshot"]), qr[path], kr[path], v[path], alpha[path], beta[path],
                                     1.0 / math.sqrt(dk))
                    for i, r in enumerate(path):
                        if r not in done:
                            o[r] = op[i]
                            done.add(r)
            cap["qkv"].append(torch.stack([q, k, v]) if hk == h else (q, k, v))
            cap["alpha"].append(alpha)
            cap["beta"].append(beta)
            cap["state"].append(st)
            z = proj[:, 2 * hk * dk + h * dv:2 * hk * dk + 2 * h * dv]
            part = qmm(gated_norm(o, z, L["gdn_norm"], eps), L["out_proj"])
        else:
            qkv = qmm(normed, L["qkv"])
            q = qkv[:, :hq * d].reshape(M, hq, d)
            gate = qkv[:, hq * d:2 * hq * d].reshape(M, hq, d)
            kn = qkv[:, 2 * hq * d:2 * hq * d + hkv * d].reshape(M, hkv, d)
            vn = qkv[:, 2 * hq * d + hkv * d:].reshape(M, hkv, d)
            pos = ctx + (torch.arange(M) if parents is None else torch.tensor([len(a) - 1 for a in anc]))
            q = rb(rope(head_rmsnorm(q, L["q_norm"], eps), cfg.rotary_dim, cfg.rope_theta, pos))
            kn = rb(rope(head_rmsnorm(kn, L["k_norm"], eps), cfg.rotary_dim, cfg.rope_theta, pos))
            ck, cv = cpu(S["cache_k"]).float().clone(), cpu(S["cache_v"]).float().clone()
            ck[:, ctx:ctx + M] = kn.transpose(0, 1)
            cv[:, ctx:ctx + M] = vn.transpose(0, 1)
            cap["cache_k"].append(ck)
            cap["cache_v"].append(cv)
            part = qmm(attention(q, gate, ck, cv, ctx, 1.0 / math.sqrt(d), anc), L["o_proj"])
        all_reduce(part)
        delta = rb(part)
        normed = add_rmsnorm(resid, delta, L["post_ln"], eps)
        gu = qmm(normed, L["gate_up"])
        I = plan.inter
        act = rb(silu(gu[:, :I]) * gu[:, I:])
        part = qmm(act, L["down"])
        all_reduce(part)
        delta = rb(part)
    out = add_rmsnorm(resid, delta, cpu(weights["final_norm"]), eps)
    return {"out": out, "resid": resid, **cap}


def commit(state: dict, result: dict, rows, context: int) -> None:
    """Make a round's accepted rows (anchor first) the committed state, in place, as
    rollbackGatedDeltaRound / Tree do (DFlashSpeculativeGenerator.swift:453-460): each
    gated-delta snapshot becomes the recurrence over those rows from it
    (``oracle.gdn_recurrence``), each conv window the last kc-1 rows of [window || their
    conv inputs] (``oracle.conv_window``), and each attention cache holds their k and v at
    rows context .. context + keep - 1.  `result` is this round's forward()."""
    rows = [int(r) for r in rows]
    keep = len(rows)
    gi = ai = 0
    for S in state["layers"]:
        if "snapshot" in S:
            q, k, v = result["qkv"][gi]
            k = k.repeat_interleave(v.shape[1] // k.shape[1], dim=1)  # shared key heads, per value head
            s, _ = O.gdn_recurrence(S["snapshot"].detach().cpu().float().numpy(), _bits(k.to(torch.bfloat16)),
                                    _bits(v.to(torch.bfloat16)), result["alpha"][gi].numpy(),
                                    result["beta"][gi].numpy(), keep, rows=rows)
            S["snapshot"].copy_(torch.from_numpy(s.astype(np.float32)))
            win = O.conv_window(_bits(S["window"]), _bits(result["conv_in"][gi].to(torch.bfloat16)), keep, rows)
            S["window"].copy_(torch.from_numpy(win.view(np.int16)).view(torch.bfloat16))
            gi += 1
        else:
            for key in ("cache_k", "cache_v"):
                src = result[key][ai][:, [context + r for r in rows]]
                S[key][:, context:context + keep] = src.to(S[key].dtype)
            ai += 1


def _order_key(v: np.ndarray) -> np.ndarray:
    """uint32 keys ordering float32 values as the floats order."""
    u = v.astype(np.float32).view(np.uint32)
    return np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint64)


def lm_head_accept(plan, weights: dict, out: torch.Tensor, proposals, combine=None):
    """The LM head of this rank's vocabulary shard (rb logits through the qmm oracle),
    each row's largest logit with its lowest global index as a 64-bit key (value order
    high, ~index low), `combine` taking the maximum over the ranks (identity at TP=1),
    then the greedy accept (acceptedPrefix, DFlashSpeculativeGenerator.swift:555-571).
    Returns (tokens int32 [M], accepted)."""
    logits = qmm(out.detach().cpu().float(), weights["lm_head"]).numpy()  # [M, vocab_r]
    idx = np.argmax(logits, axis=1)  # first index of the maximum
    val = logits[np.arange(logits.shape[0]), idx]
    keys = (_order_key(val) << np.uint64(32)) | (~(idx + plan.vocab0).astype(np.uint32)).astype(np.uint64)
    if combine is not None:
        keys = combine(keys)
    tokens = (~(keys & np.uint64(0xFFFFFFFF)).astype(np.uint32)).astype(np.int32)
    proposals = np.asarray(proposals, dtype=np.int32)
    match = (proposals == tokens[:len(proposals)]).astype(np.int32)
    return tokens, int(np.cumprod(match).sum())

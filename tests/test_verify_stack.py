"""Tensor-parallel verify stack: shard planning (CPU), TP=2 over gloo against TP=1 on the
CPU reference, and the CUDA stack against that reference on the GPU.

Tolerances: closeness = max|y - ref| / max(max|ref|, 1) (the reference's qmm test
measure).  The CUDA stack against the CPU reference of the same shard: <= 2e-2 on the
final hidden states after 4 layers (bf16 stores at every kernel boundary; the two sides
differ only in accumulation order, amplified through the RMSNorms).  TP=2 against TP=1:
<= 3e-2 (the partial sums are rounded to bf16 before the all-reduce).
"""
from __future__ import annotations

import math
import multiprocessing as mp
import socket
import sys
import tempfile
from dataclasses import asdict
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(Path(__file__).resolve().parent))

import verify_stack as vs  # noqa: E402


def closeness(y, ref) -> float:
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(y - ref)) / max(float(np.max(np.abs(ref))), 1.0))


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ----------------------------------------------------------------------------- planning (CPU)

@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_config4_shard_plan(world):
    cfg = vs.CONFIG4
    plans = [vs.shard_plan(cfg, r, world) for r in range(world)]
    assert sum(p.gdn_heads for p in plans) == cfg.gdn_heads
    assert sum(p.attn_heads for p in plans) == cfg.attn_heads
    assert sum(p.inter for p in plans) == cfg.intermediate
    q_per_kv = cfg.attn_heads // cfg.kv_heads
    for p in plans:
        # every q head of the rank reads a kv head the rank holds
        for h in range(p.attn_head0, p.attn_head0 + p.attn_heads):
            assert p.kv_head0 <= h // q_per_kv < p.kv_head0 + p.kv_heads
        assert (p.inter % cfg.group, (p.gdn_heads * cfg.gdn_dv) % cfg.group,
                (p.attn_heads * cfg.head_dim) % cfg.group) == (0, 0, 0)
    if world == 8:  # 4 kv heads over 8 ranks: each kv head on two ranks
        assert [p.kv_head0 for p in plans] == [0, 0, 1, 1, 2, 2, 3, 3]
        assert all(p.kv_heads == 1 for p in plans)


def test_shard_plan_rejects_uneven_splits():
    with pytest.raises(ValueError):
        vs.shard_plan(vs.CONFIG4, 0, 3)
    with pytest.raises(ValueError):
        vs.shard_plan(vs.StackConfig(intermediate=17408 + 64 * 7), 0, 8)
    with pytest.raises(ValueError):
        vs.shard_plan(vs.CONFIG4, 2, 2)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_column_shards_tile_the_global_rows(world):
    """Across ranks, the kept rows of the column-sharded projections cover every global
    row exactly once (kv rows excepted when they are replicated)."""
    cfg = vs.CONFIG4
    n_in = 2 * cfg.gdn_heads * cfg.gdn_dk + 2 * cfg.gdn_heads * cfg.gdn_dv + 2 * cfg.gdn_heads
    for fn, total in ((vs._ranges_gdn_in, n_in), (vs._ranges_gate_up, 2 * cfg.intermediate)):
        hits = np.zeros(total, dtype=np.int64)
        for r in range(world):
            for a, b in fn(cfg, vs.shard_plan(cfg, r, world)):
                hits[a:b] += 1
        assert (hits == 1).all()
    d = cfg.head_dim
    hits = np.zeros(2 * cfg.attn_heads * d, dtype=np.int64)
    for r in range(world):
        for a, b in vs._ranges_attn_qkv(cfg, vs.shard_plan(cfg, r, world))[:2]:
            hits[a:b] += 1
    assert (hits == 1).all()


def test_quant_row_and_col_slices():
    gen = torch.Generator().manual_seed(5)
    q = vs.random_quant(gen, 64, 512, 64, 4, "cpu")
    assert (q.N, q.K) == (64, 512) and q.w.shape == (64, 64) and q.scales.shape == (64, 8)
    r = q.rows([(0, 8), (32, 40)])
    assert torch.equal(r.w, torch.cat([q.w[:8], q.w[32:40]]))
    c = q.cols(128, 256)
    assert (c.N, c.K) == (64, 128) and torch.equal(c.scales, q.scales[:, 2:4])
    with pytest.raises(ValueError):
        q.cols(32, 128)


def test_config4_weight_bytes_per_rank():
    """Streamed bytes per forward: the packed weights, scales and biases of every
    projection (about 13.7 GB at TP=1), split evenly by TP except the replicated kv rows."""
    cfg = vs.CONFIG4
    H, I, G = cfg.hidden, cfg.intermediate, cfg.group

    def qbytes(N, K):
        return N * K // 2 + 2 * 2 * N * (K // G)

    gdn = qbytes(4 * 4096 + 64, H) + qbytes(H, 4096)
    attn = qbytes(2 * 6144 + 2 * 1024, H) + qbytes(H, 6144)
    mlp = qbytes(2 * I, H) + qbytes(H, I)
    total = 48 * gdn + 16 * attn + 64 * mlp
    assert 13.0e9 < total < 14.5e9


# ----------------------------------------------------------------------------- gloo ranks (CPU)

def _run_ranks(target, world, args_fn, timeout=240):
    """Run the ranks as spawned processes; all of them together get `timeout` seconds,
    after which any still alive are killed (and reported with exit code None)."""
    import time
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=target, args=args_fn(r)) for r in range(world)]
    for p in procs:
        p.start()
    deadline = time.monotonic() + timeout
    for p in procs:
        p.join(max(0.0, deadline - time.monotonic()))
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    return codes


@pytest.fixture(scope="module")
def tiny_tp1_reference():
    import stack_ref
    cfg = vs.TINY
    plan = vs.shard_plan(cfg, 0, 1)
    w = vs.build_rank_weights(cfg, plan, 0, "cpu")
    st = vs.build_rank_state(cfg, plan, 0, "cpu")
    r = stack_ref.forward(cfg, plan, w, st, vs.make_block(cfg, 0, "cpu"))
    r["tokens"], _ = stack_ref.lm_head_accept(plan, w, r["out"], list(range(cfg.block - 1)))
    return r


@pytest.mark.parametrize("world", [2, 4])
def test_tp_gloo_matches_tp1_and_dropped_reduce_diverges(tmp_path, tiny_tp1_reference, world):
    """TP=2, and TP=4 where the 2 kv heads are replicated over pairs of ranks."""
    import stack_workers
    ref = tiny_tp1_reference["out"].numpy()
    results = {}
    for drop in (False, True):
        out = tmp_path / f"tp{world}_drop{int(drop)}.pt"
        port = free_port()
        codes = _run_ranks(stack_workers.gloo_reference_rank, world,
                           lambda r: (r, world, port, str(out), asdict(vs.TINY), drop))
        assert codes == [0] * world, codes
        res = torch.load(out)
        results[drop] = res["out"].numpy()
        if not drop:  # the vocabulary-sharded LM head's argmax, combined over the ranks
            tok_tp = res["tokens"].numpy()
    err, err_drop = closeness(results[False], ref), closeness(results[True], ref)
    print(f"TP={world} vs TP=1: {err:.3e}; without the all-reduce: {err_drop:.3e}")
    assert err <= 3e-2
    assert err_drop > max(0.05, 10 * err)
    # same tokens as TP=1 wherever TP=1's top logit is not within the TP rounding of a rival
    assert (tok_tp == tiny_tp1_reference["tokens"]).mean() >= 0.75


def test_tp_check_config_at_eight_gloo_ranks_matches_tp1():
    """The stack bench.py checks TP = N against at N = 2, 4, 8 (one q head, one gated-delta
    head and 128 MLP units per rank at 8, each kv head replicated over four ranks): the
    CPU reference of its 8-rank shards, summed by a real all-reduce, is TP = 1's function."""
    import stack_ref
    import stack_workers
    cfg = vs.TP_CHECK
    plan = vs.shard_plan(cfg, 0, 1)
    ref = stack_ref.forward(cfg, plan, vs.build_rank_weights(cfg, plan, 0, "cpu"), vs.build_rank_state(cfg, plan, 0, "cpu"),
                            vs.make_block(cfg, 0, "cpu"))["out"].numpy()
    out = Path(tempfile.mkdtemp()) / "tp8.pt"
    port = free_port()
    codes = _run_ranks(stack_workers.gloo_reference_rank, 8, lambda r: (r, 8, port, str(out), asdict(cfg), False))
    assert codes == [0] * 8, codes
    assert closeness(torch.load(out)["out"].numpy(), ref) <= 3e-2


def test_reference_stack_is_self_consistent(tiny_tp1_reference):
    """The CPU reference's pieces: outputs finite, normalised rows, alpha in (0, 1)."""
    r = tiny_tp1_reference
    assert torch.isfinite(r["out"]).all()
    rms = r["out"].pow(2).mean(dim=1).sqrt()
    assert (rms > 0.5).all() and (rms < 2.0).all()
    for a in r["alpha"]:
        assert ((a > 0) & (a < 1)).all()
    for qkv in r["qkv"]:
        n = qkv[1].float().pow(2).sum(-1).sqrt()  # k rows are unit length
        assert torch.allclose(n, torch.ones_like(n), atol=1e-2)


# ----------------------------------------------------------------------------- CUDA stack (GPU)

@pytest.mark.gpu
def test_cuda_stack_tp1_matches_reference(cuda):
    import stack_ref
    cfg = vs.TINY
    stack = vs.VerifyStack(cfg, 0, 1, seed=0, device=cuda)
    hidden = vs.make_block(cfg, 0, cuda)
    out = stack.forward(hidden).float().cpu()
    torch.cuda.synchronize()
    plan = stack.plan
    ref = stack_ref.forward(cfg, plan, stack.w, stack.state, hidden)
    assert closeness(out.numpy(), ref["out"].numpy()) <= 2e-2
    # the capture the rollback consumes, and the state after the block
    for gi in range(len(ref["qkv"])):
        assert closeness(stack.capture_qkv[gi].float().cpu().numpy(), ref["qkv"][gi].numpy()) <= 2e-2
        assert closeness(stack.capture_alpha[gi].cpu().numpy(), ref["alpha"][gi].numpy()) <= 2e-2
        assert closeness(stack.capture_beta[gi].cpu().numpy(), ref["beta"][gi].numpy()) <= 2e-2
        s, sr = stack.state_out[gi].cpu().numpy(), ref["state"][gi].numpy()
        assert np.max(np.abs(s - sr)) / np.max(np.abs(sr)) <= 2e-2
    ai = 0
    for L, S in zip(stack.w["layers"], stack.state["layers"]):
        if L["kind"] == "attn":
            for key in ("cache_k", "cache_v"):
                got = S[key].float().cpu()[:, :cfg.context + cfg.block]
                want = ref[key][ai][:, :cfg.context + cfg.block]
                assert closeness(got.numpy(), want.numpy()) <= 2e-2
            ai += 1


@pytest.mark.gpu
@pytest.mark.parametrize("heads,dk,kc,M", [(32, 128, 4, 8), (4, 64, 4, 16), (3, 32, 2, 1)])
def test_conv_gates_kernel_equals_separate_kernels(dc, cuda, heads, dk, kc, M):
    gen = torch.Generator(device=cuda).manual_seed(heads + dk)
    C = 3 * heads * dk
    x = torch.randn(M, C + 4 * heads * dk + 2 * heads, generator=gen, device=cuda).to(torch.bfloat16)
    win = torch.randn(kc - 1, C, generator=gen, device=cuda).to(torch.bfloat16)
    w = (0.5 * torch.randn(C, kc, generator=gen, device=cuda)).to(torch.bfloat16)
    ab = x[:, C + heads * dk * 4 - 0:]
    a_log = torch.randn(heads, generator=gen, device=cuda)
    dt = torch.randn(heads, generator=gen, device=cuda)
    want = torch.empty(3, M, heads, dk, dtype=torch.bfloat16, device=cuda)
    al1, be1 = (torch.empty(M, heads, device=cuda) for _ in range(2))
    dc.stack_conv_silu(x, win, w, want, channels=C, parts=3)
    dc.stack_gdn_gates(want[0], want[1], ab, a_log, dt, al1, be1)
    got = torch.empty_like(want)
    al2, be2 = (torch.empty(M, heads, device=cuda) for _ in range(2))
    dc.stack_gdn_conv_gates(x, win, w, got, ab, a_log, dt, al2, be2, heads, dk)
    torch.cuda.synchronize()
    assert torch.equal(got, want) and torch.equal(al1, al2) and torch.equal(be1, be2)


@pytest.mark.gpu
def test_qmm_swiglu_input_equals_separate_silu_mul(dc, O, cuda):
    """dflash_qmm_ex with x_swiglu gives the same bits as dflash_stack_silu_mul followed by
    dflash_qmm (the down projection of the MLP)."""
    M, I, N = 8, 2048, 1024
    gen = torch.Generator(device=cuda).manual_seed(3)
    gu = torch.randn(M, 2 * I, generator=gen, device=cuda).to(torch.bfloat16)
    q = vs.random_quant(gen, N, I, 64, 4, cuda)
    act = torch.empty(M, I, dtype=torch.bfloat16, device=cuda)
    dc.stack_silu_mul(gu, act)
    want = dc.qmm(act, q.w, q.scales, q.biases, 64, 4)
    got = dc.qmm_ex(gu, q.w, q.scales, q.biases, 64, 4, swiglu=True)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("via", ["push_kernel", "qmm_epilogue"])
@pytest.mark.parametrize("H", [512, 5120, 12288])
def test_peer_exchange_two_ranks_in_one_process(dc, cuda, via, H):
    """The exchange protocol with two 'ranks' emulated by two buffers on one GPU (each
    push completes before the sums are read, so nothing waits on another kernel): both
    buffers' reducing norms equal add_rmsnorm with delta = bf16(y0 + y1), for two
    consecutive exchanges (both slot sets) and a third that reuses set 0.  H = 5120 is the
    config-4 hidden size (four float4 per thread of a norm CTA, 512 two, 12288 eight: the
    slices' loads are batched four, two and two at a time)."""
    M, K = 8, 1024
    gen = torch.Generator(device=cuda).manual_seed(4)
    ex = [dc.PeerExchange(2, M, H) for _ in range(2)]
    ptrs = [e.ptr for e in ex]
    for r in range(2):
        ex[r].connect_local(r, ptrs)
    q = [vs.random_quant(gen, H, K, 64, 4, cuda) for _ in range(2)]
    w = (1.0 + 0.1 * torch.randn(H, generator=gen, device=cuda)).to(torch.bfloat16)
    resid0 = torch.randn(M, H, generator=gen, device=cuda)
    resid = [resid0.clone(), resid0.clone()]
    want_resid = resid0.clone()
    try:
        for step in range(3):
            s = step % 2
            xs = [torch.randn(M, K, generator=gen, device=cuda).to(torch.bfloat16) for _ in range(2)]
            ys = [dc.qmm(xs[r], q[r].w, q[r].scales, q[r].biases, 64, 4) for r in range(2)]
            for r in range(2):
                if via == "push_kernel":
                    ex[r].push(ys[r], s)
                else:
                    dc.qmm_ex(xs[r], q[r].w, q[r].scales, q[r].biases, 64, 4, exchange=ex[r], set_=s)
            outs = [torch.empty(M, H, dtype=torch.bfloat16, device=cuda) for _ in range(2)]
            for r in range(2):
                dc.stack_add_rmsnorm_reduce(resid[r], ex[r], s, w, outs[r], 1e-6)
            delta = (ys[0].float() + ys[1].float()).to(torch.bfloat16)
            want = torch.empty(M, H, dtype=torch.bfloat16, device=cuda)
            dc.stack_add_rmsnorm(want_resid, delta, w, want, 1e-6)
            torch.cuda.synchronize()
            assert dc.device_error() == 0
            for r in range(2):
                assert torch.equal(outs[r], want), (step, r)
                assert torch.equal(resid[r], want_resid), (step, r)
    finally:
        for e in ex:
            e.close()


@pytest.mark.gpu
def test_cuda_stack_verify_round_tp1(dc, cuda):
    """forward + LM head argmax + accept: the tokens are the first maximum of the logits
    the plain qmm writes for the stack's output, the accept count follows the planted
    proposals, and the captured round replays the same tokens."""
    cfg = vs.TINY
    stack = vs.VerifyStack(cfg, 0, 1, seed=0, device=cuda)
    hidden = vs.make_block(cfg, 0, cuda)
    out = stack.forward(hidden).clone()
    q = stack.w["lm_head"]
    want = torch.argmax(dc.qmm(out, q.w, q.scales, q.biases, q.group, q.bits).float(), dim=1).to(torch.int32)
    for plant in range(cfg.block):
        prop = want[:cfg.block - 1].clone()
        if plant < cfg.block - 1:
            prop[plant] = (prop[plant] + 1) % cfg.vocab
        tokens, acc = stack.verify(hidden, prop)
        torch.cuda.synchronize()
        assert torch.equal(tokens, want) and int(acc.item()) == min(plant, cfg.block - 1)
    g = stack.capture(hidden, want[:cfg.block - 1].clone())
    stack.tokens.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(stack.tokens, want) and int(stack.accepted.item()) == cfg.block - 1
    del g


@pytest.mark.gpu
def test_accept_reduce_two_vocabulary_shards_in_one_process(dc, cuda):
    """Keys of two vocabulary shards, pushed into two emulated ranks' key exchanges,
    reduce to the tokens of the unsharded LM head (ties resolved to the lowest index)."""
    M, V, K = 8, 2048, 512
    gen = torch.Generator(device=cuda).manual_seed(6)
    q = vs.random_quant(gen, V, K, 64, 4, cuda)
    x = torch.randn(M, K, generator=gen, device=cuda).to(torch.bfloat16)
    full = dc.lm_head_argmax(x, q.w, q.scales, q.biases, 64, 4)
    want = ((~(full & 0xFFFFFFFF)) & 0xFFFFFFFF).to(torch.int32)
    ex = [dc.PeerExchange(2, M, 4) for _ in range(2)]
    try:
        for r in range(2):
            ex[r].connect_local(r, [e.ptr for e in ex])
        for step in range(2):  # twice, so the epochs move on
            for r in range(2):
                half = q.rows([(r * V // 2, (r + 1) * V // 2)])
                keys = dc.lm_head_argmax(x, half.w, half.scales, half.biases, 64, 4, index_base=r * V // 2)
                ex[r].push(keys.view(torch.bfloat16).view(M, 4), 0)
            prop = want[:M - 1].clone()
            prop[3] += 1
            for r in range(2):
                tokens, acc = dc.accept_reduce(ex[r], 0, prop)
                torch.cuda.synchronize()
                assert torch.equal(tokens, want) and int(acc.item()) == 3
        assert dc.device_error() == 0
    finally:
        for e in ex:
            e.close()


@pytest.mark.gpu
def test_cuda_stack_graph_replay_equals_eager(cuda):
    cfg = vs.TINY
    stack = vs.VerifyStack(cfg, 0, 1, seed=1, device=cuda)
    hidden = vs.make_block(cfg, 1, cuda)
    eager = stack.forward(hidden).clone()
    g = stack.capture(hidden)
    stack.out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(stack.out, eager)
    del g


@pytest.mark.gpu
def test_cuda_stack_config4_shapes_run(cuda):
    """Config-4 layer shapes (hidden 5120, MLP 17408, 32 x 128 gated-delta heads, 24 x 256
    q heads with 4 kv heads) for one gated-delta and one attention layer: the forward is
    finite and its graph replay is bit-identical to eager."""
    from dataclasses import replace
    cfg = replace(vs.CONFIG4, layers=4, attn_interval=2, context=256)
    stack = vs.VerifyStack(cfg, 0, 1, seed=2, device=cuda)
    hidden = vs.make_block(cfg, 2, cuda)
    eager = stack.forward(hidden).clone()
    assert torch.isfinite(eager.float()).all()
    g = stack.capture(hidden)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(stack.out, eager)
    del g


@pytest.mark.gpu
def test_cuda_tp_check_stack_matches_reference(cuda):
    """The benchmark's TP check stack at TP = 1 on the GPU against the CPU reference."""
    import stack_ref
    cfg = vs.TP_CHECK
    stack = vs.VerifyStack(cfg, 0, 1, seed=0, device=cuda)
    hidden = vs.make_block(cfg, 0, cuda)
    out = stack.forward(hidden).float().cpu().numpy()
    torch.cuda.synchronize()
    ref = stack_ref.forward(cfg, stack.plan, stack.w, stack.state, hidden)["out"].numpy()
    assert closeness(out, ref) <= 2e-2


@pytest.mark.gpu
def test_cuda_stack_tp2_matches_tp1_reference(cuda, tmp_path):
    """TP=2 on two GPUs, all-reduce over peer memory and through NCCL: both match the TP=1
    reference, agree bit for bit with each other (a two-term bf16 sum rounds once either
    way), and graph replay equals eager."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import stack_ref
    import stack_workers
    cfg = vs.TINY
    plan = vs.shard_plan(cfg, 0, 1)
    w = vs.build_rank_weights(cfg, plan, 0, cuda)
    st = vs.build_rank_state(cfg, plan, 0, cuda)
    ref = stack_ref.forward(cfg, plan, w, st, vs.make_block(cfg, 0, cuda))["out"].numpy()
    res = {}
    for mode in ("peer", "nccl"):
        out = tmp_path / f"tp2_{mode}.pt"
        port = free_port()
        codes = _run_ranks(stack_workers.nccl_stack_rank, 2, lambda r: (r, 2, port, str(out), asdict(cfg), mode))
        assert codes == [0, 0], (mode, codes)
        res[mode] = torch.load(out)
        assert res[mode]["device_error"] == 0
        assert torch.equal(res[mode]["eager"], res[mode]["graphed"])
        assert torch.equal(res[mode]["tokens"], res[mode]["graphed_tokens"])
        assert closeness(res[mode]["eager"].float().numpy(), ref) <= 3e-2
    assert torch.equal(res["peer"]["eager"], res["nccl"]["eager"])
    assert torch.equal(res["peer"]["tokens"], res["nccl"]["tokens"])


# ----------------------------------------------------------------------------- decode attention (GPU)
@pytest.mark.gpu
@pytest.mark.parametrize("hq,hkv,M,ctx", [(3, 1, 8, 1024), (6, 1, 8, 700), (24, 4, 8, 1024), (12, 2, 8, 300),
                                          (4, 2, 1, 40)])
def test_decode_attention_matches_fp32_reference(dc, cuda, hq, hkv, M, ctx):
    """dflash_stack_attn_decode against plain fp32 attention: token t of the block sees the
    cached keys 0 .. ctx + t (its own and earlier block rows included), head h reads kv head
    h / (hq / hkv), and the output is gated by sigmoid(gate).  The shapes cover both cluster
    widths (8 CTAs per kv head and token when the grid is small, 4 otherwise) and one or
    two passes over a CTA's keys."""
    d = 256
    g = torch.Generator(device=cuda).manual_seed(hq * 100 + hkv * 10 + M)
    max_len = ctx + M + 16
    qkv = torch.randn(M, (2 * hq + 2 * hkv) * d, generator=g, device=cuda).to(torch.bfloat16)
    ck = torch.randn(hkv, max_len, d, generator=g, device=cuda).to(torch.bfloat16)
    cv = torch.randn(hkv, max_len, d, generator=g, device=cuda).to(torch.bfloat16)
    out = torch.empty(M, hq * d, dtype=torch.bfloat16, device=cuda)
    scale = d ** -0.5
    dc.stack_attn_decode(qkv, ck, cv, out, hq, hkv, ctx, scale)
    torch.cuda.synchronize()
    q = qkv[:, :hq * d].float().view(M, hq, d)
    gate = qkv[:, hq * d:2 * hq * d].float().view(M, hq, d)
    want = torch.empty(M, hq, d, device=cuda)
    for t in range(M):
        for h in range(hq):
            j = h // (hq // hkv)
            k = ck[j, :ctx + t + 1].float()
            v = cv[j, :ctx + t + 1].float()
            p = torch.softmax((k @ q[t, h]) * scale, dim=0)
            want[t, h] = (p @ v) * torch.sigmoid(gate[t, h])
    assert closeness(out.float().view(M, hq, d).cpu().numpy(), want.cpu().numpy()) <= 1e-2
    assert dc.device_error() == 0

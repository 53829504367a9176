"""Rank bodies for the multi-process verify-stack tests (spawned children).

gloo ranks run the CPU reference of one shard (oracle/stack_ref.py) with a real
all-reduce; nccl ranks run the CUDA stack (dflash-swift_b200/verify_stack.py) on one
GPU each.  Each child writes its rank-0 result to `out_path` with torch.save."""
from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT / "oracle"), str(ROOT / "dflash-swift_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def _init(backend: str, rank: int, world: int, port: int, device=None):
    import torch.distributed as dist
    kw = dict(device_id=device) if device is not None else {}
    dist.init_process_group(backend, init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), **kw)
    return dist


def gloo_reference_rank(rank: int, world: int, port: int, out_path: str, cfg_kw: dict, drop_reduce: bool,
                        parents=None, hidden_seed: int = 0):
    import torch
    import verify_stack as vs
    import stack_ref
    dist = _init("gloo", rank, world, port)
    try:
        cfg = vs.StackConfig(**cfg_kw)
        plan = vs.shard_plan(cfg, rank, world)
        w = vs.build_rank_weights(cfg, plan, 0, "cpu")
        st = vs.build_rank_state(cfg, plan, 0, "cpu")
        hidden = vs.make_block(cfg, hidden_seed, "cpu")

        def reduce(t):
            if not drop_reduce:
                dist.all_reduce(t)

        r = stack_ref.forward(cfg, plan, w, st, hidden, all_reduce=reduce, parents=parents)

        def combine(keys):  # max over the ranks: unsigned keys as signed with the sign bit flipped
            import numpy as np
            t = torch.from_numpy((keys ^ np.uint64(1 << 63)).view(np.int64).copy())
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return t.numpy().view(np.uint64) ^ np.uint64(1 << 63)

        tokens, acc = stack_ref.lm_head_accept(plan, w, r["out"], list(range(cfg.block - 1)), combine=combine)
        if rank == 0:
            torch.save({"out": r["out"], "tokens": torch.from_numpy(tokens)}, out_path)
    finally:
        dist.destroy_process_group()


def nccl_stack_rank(rank: int, world: int, port: int, out_path: str, cfg_kw: dict, allreduce: str = "peer"):
    import torch
    import verify_stack as vs
    torch.cuda.set_device(rank)
    dev = torch.device(f"cuda:{rank}")
    dist = _init("nccl", rank, world, port, device=dev)
    try:
        cfg = vs.StackConfig(**cfg_kw)
        stack = vs.VerifyStack(cfg, rank, world, seed=0, device=dev, group=dist.group.WORLD, allreduce=allreduce)
        hidden = vs.make_block(cfg, 0, dev)
        eager = stack.forward(hidden).clone()
        g = stack.capture(hidden)
        g.replay()
        torch.cuda.synchronize(dev)
        graphed = stack.out.clone()
        del g
        proposals = torch.arange(cfg.block - 1, dtype=torch.int32, device=dev)
        tokens, acc = stack.verify(hidden, proposals)
        tokens, acc = tokens.clone(), acc.clone()
        g = stack.capture(hidden, proposals)
        g.replay()
        torch.cuda.synchronize(dev)
        graphed_tokens = stack.tokens.clone()
        del g
        stack.graph = None
        import dflashcuda
        dev_err = dflashcuda.device_error()
        stack.close()
        if rank == 0:
            torch.save({"eager": eager.cpu(), "graphed": graphed.cpu(), "device_error": dev_err, "tokens": tokens.cpu(),
                        "graphed_tokens": graphed_tokens.cpu(), "accepted": int(acc.item())}, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()

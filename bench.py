"""Benchmark of the small-M quantized matmul (BASELINE config 2 at M=8).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one dflash_qmm call: x bf16 [8, 5120] against a 4-bit group-64 MLX-packed
W [17408, 5120] (the MLP gate/up projection of the 27B target) -> y bf16 [8, 17408].
Inputs are seeded synthetic data with the config's distributions (x ~ N(0,1),
W ~ N(0, 0.02)), resident in HBM before the timed region.  L2 is defeated by rotating
through enough distinct weight copies that every step streams its weights from HBM
(> 4x the 126 MB L2).  The timed region replays a CUDA graph of the K launches and is
bracketed by a barrier and device synchronisation; the time is the max over ranks.

Multi-GPU (torchrun, one rank per GPU): every rank runs its own copy of the workload
(the path shards with no collective), so scaling is weak and `value` is the job total.
Beside that line, a job of N > 1 GPUs runs BASELINE config 4 tensor-parallel over its N
GPUs (`verify_stack_config4_tp<N>`: a TP = N vs TP = 1 correctness gate, then the
64-layer verify forward and round timed from CUDA graphs, max over ranks).

--impl reference times this project's CPU restatement of the reference arithmetic
(oracle/qmm_oracle.c) on the host cores: the reference's own path is Metal/MLX and
cannot run on this machine.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "dflash-swift_b200"))

METRIC = "M=8 4-bit qmatmul µs and HBM GB/s (% of 8 TB/s); M=8/M=1 time ratio"
M, N, K, GROUP, BITS = 8, 17408, 5120, 64, 4
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 1024 * 1024
PROFILE_SUMMARY = ROOT / "profiles" / "qmm_m8_k5120_n17408_4b_g64.json"
KERNELS_PER_CALL = 2  # prep (x packets: fp16 fragment order + segment sums), main (weight stream)
WARM_LAUNCHES = 2000  # untimed launches before each timed region (~35 ms of device work)


def algorithmic_bytes(m: int, n: int = N, k: int = K, group: int = GROUP, bits: int = BITS) -> int:
    """Packed W + bf16 scales + bf16 biases + x + y, each moved once."""
    return n * k * bits // 8 + 2 * n * (k // group) * 2 + m * k * 2 + m * n * 2


def config(m: int = M) -> dict:
    return {"workload": "qmm_config2_gate_up", "M": m, "N": N, "K": K, "bits": BITS, "group_size": GROUP,
            "x": "bf16 N(0,1)", "w": "N(0,0.02) MLX affine 4-bit g64",
            "l2": "rotating distinct weight copies totalling > 4x L2 per pass",
            "algorithmic_bytes_per_step": algorithmic_bytes(m)}


def measured_peak():
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the GPU works."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = set(int(g) for g in gpu_indices)
        self.proc = None
        self.out = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50"], stdout=self.out, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.flush()
        rows = []
        for line in Path(self.out.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                if int(parts[0]) in self.gpus:
                    rows.append(parts)
            except ValueError:
                continue
        os.unlink(self.out.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------------------- GPU arm

def to_dev(a, dev):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).to(dev).view(torch.bfloat16)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).to(dev)
    return torch.from_numpy(a).to(dev)


def weight_copies(dev, wq, s, b):
    """Enough distinct copies of (W, scales, biases) that consecutive steps never hit L2."""
    import torch
    per = wq.nbytes + s.nbytes + b.nbytes
    n = max(2, -(-4 * L2_BYTES // per) + 1)
    w0, s0, b0 = to_dev(wq, dev), to_dev(s, dev), to_dev(b, dev)
    copies = [(w0, s0, b0)] + [(w0.clone(), s0.clone(), b0.clone()) for _ in range(n - 1)]
    torch.cuda.synchronize()
    return copies


def time_graph(dc, dev, x_d, copies, y_d, ws, steps, warmup, m):
    """Capture one launch per weight copy into a CUDA graph (plus a graph of the remainder
    launches) so that the timed replays cover exactly `steps` launches. Every graph that the
    timed region replays is replayed untimed first (its upload and first-launch cost stay
    outside the timing), and at least `warmup` launches run before the timed region."""
    import torch
    stream = torch.cuda.Stream(dev)
    R = len(copies)

    def capture(count):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            # prime once outside capture (one-time kernel attribute setup)
            dc.qmm(x_d[:m], copies[0][0], copies[0][1], copies[0][2], GROUP, BITS, out=y_d[:m], workspace=ws,
                   stream=stream)
        stream.synchronize()
        with torch.cuda.graph(g, stream=stream):
            for i in range(count):
                w, s, b = copies[i % R]
                dc.qmm(x_d[:m], w, s, b, GROUP, BITS, out=y_d[:m], workspace=ws, stream=stream)
        return g

    full = capture(R)
    rest_n = steps % R
    rest = capture(rest_n) if rest_n else None
    # at least `warmup` launches, and at least WARM_LAUNCHES, so that the GPU left idle by
    # the host-side set-up before this call is back at its working clocks when timing starts
    with torch.cuda.stream(stream):
        for _ in range(max(1, -(-max(warmup, WARM_LAUNCHES) // R))):
            full.replay()
        if rest is not None:
            rest.replay()
    stream.synchronize()
    return stream, full, rest, steps // R


def run_ours(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import dflashcuda as dc
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O  # seeded input generation (and the CPU baseline below)

    x = O.make_x(16, K, seed_x=0)
    wq, s, b = O.make_weights(N, K, GROUP, BITS, seed_w=1)
    copies = weight_copies(dev, wq, s, b)
    x_d = to_dev(x, dev)
    y_d = torch.empty((16, N), dtype=torch.bfloat16, device=dev)
    ws = dc.Workspace(dc.qmm_workspace_bytes(16, N, K, GROUP, BITS), dev)

    # correctness gate before timing
    dc.qmm(x_d[:M], copies[0][0], copies[0][1], copies[0][2], GROUP, BITS, out=y_d[:M], workspace=ws)
    torch.cuda.synchronize()
    rows = np.arange(0, N, 97)
    err = O.closeness(y_d[:M].float().cpu().numpy()[:, rows], O.qmm_f64(x[:M], wq[rows], s[rows], b[rows], GROUP, BITS))
    if err > 1e-2:
        raise SystemExit(f"parity gate failed before timing: closeness {err}")

    def timed(m, steps, warmup, sample_clocks=False):
        stream, full, rest, reps = time_graph(dc, dev, x_d, copies, y_d, ws, steps, warmup, m)
        sampler = None
        if sample_clocks and rank == 0:
            sampler = ClockSampler(gpu_ids(world))
            sampler.start()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        # An untimed replay queued ahead of the start event keeps the GPU busy while the host
        # enqueues the timed replays, so the graph-launch latency of the host does not land
        # inside the timed region (it would after the idle synchronize above).
        with torch.cuda.stream(stream):
            full.replay()
        t0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(reps):
                full.replay()
            if rest is not None:
                rest.replay()
        t1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        clocks = sampler.stop() if sampler else None
        ms = t0.elapsed_time(t1)
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, clocks

    ms8, clocks = timed(M, args.steps, args.warmup, sample_clocks=True)
    ms1, _ = timed(1, args.steps, args.warmup)
    us8 = ms8 * 1e3 / args.steps
    us1 = ms1 * 1e3 / args.steps
    m_sweep = None
    if world == 1:  # BASELINE config 2 asks for every M in 1..8 (M = 1 and 8 timed above)
        sweep_steps = max(200, min(args.steps, 4000))
        m_sweep = {}
        try:
            for m in range(1, 9):
                us = us1 if m == 1 else us8 if m == M else timed(m, sweep_steps, args.warmup)[0] * 1e3 / sweep_steps
                m_sweep[m] = {"us": round(us, 3), "GBs": round(algorithmic_bytes(m) / (us * 1e-6) / 1e9, 1)}
        except Exception as exc:  # a side measurement: never costs the main line
            m_sweep["error"] = repr(exc)[:300]
    bytes8 = algorithmic_bytes(M)
    per_gpu_gbs = bytes8 / (us8 * 1e-6) / 1e9
    value = world * per_gpu_gbs

    e2e = e2e_through_abi(dc, dev, x, copies, args, world)
    try:  # the one-call host-buffer entry point, checked bit for bit before it is timed
        want = []
        for (w_, s_, b_) in copies:
            dc.qmm(x_d[:M], w_, s_, b_, GROUP, BITS, out=y_d[:M], workspace=ws)
            want.append(y_d[:M].cpu())
        e2e_host = e2e_host_entry(dc, dev, x, copies, args, want)
    except Exception as exc:  # reported; the three-call figure above stands
        e2e_host = {"error": repr(exc)[:300], "ms": float("inf")}
    if world > 1:  # every rank takes both reductions, failed or not
        for rec in (e2e, e2e_host):
            t = torch.tensor([min(rec["ms"], 1e30)], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            rec["ms"] = float(t.item()) if t.item() < 1e30 else float("inf")

    peak, peak_kind = measured_peak()
    traffic = None
    if PROFILE_SUMMARY.exists():
        try:
            traffic = json.loads(PROFILE_SUMMARY.read_text()).get("dram_bytes_per_launch")
        except Exception:
            traffic = None

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(O, x[:M], wq, s, b, budget_s=args.cpu_seconds)
    gdn = fmt = stack4 = stack_tp = None
    if world > 1:  # the tensor-parallel verify stack over the job's GPUs (collectives on every rank)
        try:
            stack_tp = verify_stack_tp(dev, world, rank)
        except Exception as exc:
            stack_tp = {"error": repr(exc)[:300]}
    if world == 1:
        try:
            gdn = gdn_replay_config5(dc, dev, peak)
        except Exception as exc:  # a side measurement: never costs the main line
            gdn = {"error": repr(exc)[:300]}
        try:
            fmt = format_sweep_config3(dc, dev)
        except Exception as exc:  # a side measurement: never costs the main line
            fmt = {"error": repr(exc)[:300]}
        try:
            stack4 = verify_stack_config4(dev)
        except Exception as exc:  # a side measurement: never costs the main line
            stack4 = {"error": repr(exc)[:300]}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(us8 / 1e3, 6), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u4 weights, bf16 x/y, fp32 accumulate", "data": "synthetic",
            "config": config(M),
            "us_per_call": round(us8, 3), "us_per_call_m1": round(us1, 3), "m8_over_m1": round(us8 / us1, 4),
            "pct_of_8TBs": round(100 * per_gpu_gbs / NOMINAL_HBM_GBS, 2),
            "pct_of_measured_hbm": round(100 * per_gpu_gbs / peak, 2),
            "roofline": {"bound": "hbm", "achieved": round(per_gpu_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(per_gpu_gbs / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic, "algorithmic_bytes": bytes8},
            "cpu_baseline": cpu,
            "e2e": e2e_line(e2e, e2e_host, world, bytes8, args.steps),
            "gpu_launches": KERNELS_PER_CALL * args.steps,
            "m_sweep_config2": m_sweep,
            "format_sweep_config3": fmt,
            "gdn_replay_config5": gdn,
            "verify_stack_config4_tp1": stack4,
            f"verify_stack_config4_tp{world}" if world > 1 else "verify_stack_config4_tpN": stack_tp,
            "clocks": clocks,
            "parity_closeness_before_timing": err,
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def gdn_replay_config5(dc, dev, peak, reps=20):
    """BASELINE config 5 beside the main line: the rollback replay of 48 layers x 32 heads
    of fp32 [128, 128] state, keeping 8 of 8 captured positions (seeded q/k/v, k
    L2-normalised, alpha ~ U(0.9, 1), beta ~ U(0, 1)).  A CUDA graph of `reps` replays
    alternating over two (snapshot, state) buffer pairs: each replay reads a 100.7 MB
    snapshot and writes a 100.7 MB state, and consecutive replays touch different pairs
    (403 MB in all against the 126 MB L2), so no replay finds its snapshot in L2."""
    import torch
    L, W, H, dk, dv, keep = 48, 8, 32, 128, 128, 8
    g = torch.Generator(device=dev).manual_seed(2)
    snaps = [0.1 * torch.randn(L, H, dv, dk, generator=g, device=dev) for _ in range(2)]
    outs = [torch.empty_like(snaps[0]) for _ in range(2)]
    k = torch.nn.functional.normalize(torch.randn(L, W, H, dk, generator=g, device=dev), dim=-1).to(torch.bfloat16)
    v = torch.randn(L, W, H, dv, generator=g, device=dev).to(torch.bfloat16)
    alpha = 0.9 + 0.1 * torch.rand(L, W, H, generator=g, device=dev)
    beta = torch.rand(L, W, H, generator=g, device=dev)
    for i in range(2):
        dc.gdn_replay(snaps[i], outs[i], k, v, alpha, beta, keep=keep)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(reps):
            dc.gdn_replay(snaps[i & 1], outs[i & 1], k, v, alpha, beta, keep=keep)
    graph.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / reps
    nbytes = 2 * L * H * dk * dv * 4 + keep * L * H * (dk + dv) * 2 + keep * L * H * 2 * 4
    gbs = nbytes / us / 1e3
    del graph
    return {"us": round(us, 2), "GBs": round(gbs, 1), "algorithmic_bytes": nbytes, "frac_of_peak": round(gbs / peak, 4),
            "device_error": dc.device_error(), "workload": "48 layers x 32 heads x 128 x 128 fp32, keep 8 of 8",
            "l2": "replays alternate over two snapshot/state pairs (403 MB)"}


def verify_stack_config4(dev, steps=20, warmup=3):
    """BASELINE config 4 at TP = 1 beside the main line: the 64-layer verify forward of an
    8-row block (48 gated-delta + 16 attention layers, hidden 5120, MLP 17408, 4-bit g64
    seeded random weights, 1024 cached tokens) and the whole verify round (forward, the
    248,320-row LM head with its argmax, the accept), each replayed from a CUDA graph and
    timed with CUDA events.  The tensor-parallel runs (TP 2 / 4 / 8) use
    dflash-swift_b200/verify_stack.py under torchrun."""
    import torch
    import verify_stack as vs
    cfg = vs.CONFIG4
    stack = vs.VerifyStack(cfg, 0, 1, seed=0, device=dev)
    hidden = vs.make_block(cfg, 0, dev)
    proposals = torch.zeros(cfg.block - 1, dtype=torch.int32, device=dev)

    def timed(g):
        for _ in range(warmup):
            g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) * 1e3 / steps

    g = stack.capture(hidden)
    fwd = timed(g)
    del g
    g = stack.capture(hidden, proposals)
    rnd = timed(g)
    del g
    stack.graph = None
    wbytes = vs.weight_bytes(stack.w)
    out = {"forward_us": round(fwd, 1), "round_us": round(rnd, 1), "tokens_per_s": round(cfg.block / (fwd * 1e-6), 1),
           "weight_bytes": wbytes, "weight_GBs": round(wbytes / (fwd * 1e-6) / 1e9, 1),
           "kernels_per_forward": stack.kernels_per_forward(), "steps": steps}
    del stack
    torch.cuda.empty_cache()
    return out


def verify_stack_tp(dev, world, rank, steps=20, warmup=5):
    """BASELINE config 4 tensor-parallel over the job's N GPUs (N > 1), beside the qmm line.

    First a correctness gate on the same GPUs: verify_stack.TP_CHECK (a small stack that
    shards over 2, 4 and 8 ranks) run at TP = N, its output compared on every rank with the
    same stack run at TP = 1 on that rank's GPU (max|d| / max(max|ref|, 1) <= 3e-2, the
    multi-rank stack tests' bar); a mismatch on any rank fails the entry.  Then the 64-layer
    config-4 verify forward and whole verify round at TP = N, each from a CUDA graph, timed
    with CUDA events and taken as the max over ranks, with the clocks sampled meanwhile.
    Every rank takes the same collective steps in the same order."""
    import torch
    import torch.distributed as dist
    import verify_stack as vs

    def max_over_ranks(v: float) -> float:
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    cfg = vs.TP_CHECK
    one = vs.VerifyStack(cfg, 0, 1, seed=0, device=dev)
    hidden = vs.make_block(cfg, 0, dev)
    ref = one.forward(hidden).float().cpu()
    del one
    tp = vs.VerifyStack(cfg, rank, world, seed=0, device=dev, group=dist.group.WORLD)
    out = tp.forward(hidden).float().cpu()
    torch.cuda.synchronize(dev)
    tp.close()
    del tp
    err = max_over_ranks(float((out - ref).abs().max()) / max(float(ref.abs().max()), 1.0))
    check = {"stack": "TP_CHECK (4 layers, hidden 512, 8 gated-delta / 8 q / 2 kv heads)", "closeness_vs_tp1": err,
             "bar": 3e-2, "ok": err <= 3e-2}
    if not check["ok"]:
        return {"error": "TP = N differs from TP = 1", "tp_check": check}

    cfg = vs.CONFIG4
    stack = vs.VerifyStack(cfg, rank, world, seed=0, device=dev, group=dist.group.WORLD)
    hidden = vs.make_block(cfg, 0, dev)
    proposals = torch.zeros(cfg.block - 1, dtype=torch.int32, device=dev)

    def timed(g, sample):
        for _ in range(warmup):
            g.replay()
        torch.cuda.synchronize(dev)
        sampler = ClockSampler(gpu_ids(world)) if sample and rank == 0 else None
        if sampler:
            sampler.start()
        dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        dist.barrier()
        clocks = sampler.stop() if sampler else None
        return max_over_ranks(e0.elapsed_time(e1) * 1e3 / steps), clocks

    g = stack.capture(hidden)
    fwd, clocks = timed(g, True)
    del g
    g = stack.capture(hidden, proposals)
    rnd, _ = timed(g, False)
    del g
    stack.graph = None
    wbytes = vs.weight_bytes(stack.w)
    kernels = stack.kernels_per_forward()
    stack.close()
    del stack
    torch.cuda.empty_cache()
    return {"tp": world, "forward_us": round(fwd, 1), "round_us": round(rnd, 1),
            "tokens_per_s": round(cfg.block / (fwd * 1e-6), 1), "weight_bytes_per_gpu": wbytes,
            "weight_GBs_per_gpu": round(wbytes / (fwd * 1e-6) / 1e9, 1), "kernels_per_forward": kernels,
            "allreduce": "peer (NVLink stores into the other ranks' exchange buffers)", "steps": steps,
            "timing": "CUDA graph per forward, CUDA events, max over ranks", "clocks": clocks, "tp_check": check}


def _qmm_copies(dev, gen, n, k, group, bits):
    """Seeded random packed weights (the time does not depend on the values) in enough
    distinct copies that a CUDA graph rotating through them never finds one in L2."""
    import verify_stack as vs
    q0 = vs.random_quant(gen, n, k, group, bits, dev)
    return [q0] + [vs.Quant(q0.w.clone(), q0.scales.clone(), q0.biases.clone(), group, bits)
                   for _ in range(max(1, -(-4 * L2_BYTES // q0.nbytes())))]


def _time_qmm(dc, dev, stream, copies, x, y, ws, m, steps):
    """us per dflash_qmm call at M = m: a CUDA graph of one launch per copy, replayed to
    cover about `steps` launches after 3 warm-up replays, timed with CUDA events."""
    import torch
    q0 = copies[0]
    with torch.cuda.stream(stream):
        dc.qmm(x[:m], q0.w, q0.scales, q0.biases, q0.group, q0.bits, out=y[:m], workspace=ws, stream=stream)
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for q in copies:
            dc.qmm(x[:m], q.w, q.scales, q.biases, q.group, q.bits, out=y[:m], workspace=ws, stream=stream)
    reps = max(1, steps // len(copies))
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(reps):
            g.replay()
    e1.record(stream)
    stream.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / (reps * len(copies))


def format_sweep_config3(dc, dev, steps=2000):
    """BASELINE config 3 beside the main line: down-proj (K=17408, N=5120) and attention-out
    (K=6144, N=5120) at bits 4 and 8, groups 32, 64 and 128, M = 1, 4 and 8; and config 1's
    shape (K=4096, N=4096, 4-bit g64, M=8) on the GPU.  `steps` timed launches per point;
    reported as us per call and GB/s of algorithmic bytes."""
    import torch
    out = {}
    stream = torch.cuda.Stream(dev)
    gen = torch.Generator(device=dev).manual_seed(3)
    points = [(5120, 17408, "down", bits, group, (1, 4, 8)) for bits in (4, 8) for group in (32, 64, 128)]
    points += [(5120, 6144, "attn_out", bits, group, (1, 4, 8)) for bits in (4, 8) for group in (32, 64, 128)]
    points += [(4096, 4096, "config1", 4, 64, (8,))]
    for (n, k, name, bits, group, ms) in points:
        x = torch.randn(8, k, generator=gen, device=dev).to(torch.bfloat16)
        y = torch.empty(8, n, dtype=torch.bfloat16, device=dev)
        copies = _qmm_copies(dev, gen, n, k, group, bits)
        ws = dc.Workspace(dc.qmm_workspace_bytes(8, n, k, group, bits), dev)
        for m in ms:
            us = _time_qmm(dc, dev, stream, copies, x, y, ws, m, steps)
            nbytes = algorithmic_bytes(m, n=n, k=k, group=group, bits=bits)
            out[f"{name}_b{bits}_g{group}_m{m}"] = {"us": round(us, 3), "GBs": round(nbytes / (us * 1e-6) / 1e9, 1)}
        del copies, ws
        torch.cuda.empty_cache()
    return out


def gpu_ids(world):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [int(v) for v in vis.split(",") if v.strip().isdigit()]
        return ids[:world] if ids else list(range(world))
    return list(range(world))


# Streams the e2e legs rotate over.  The 278 KB copy of y back to the host takes 8.4 us of
# the single device-to-host copy engine per step; with two streams it and the next steps'
# copies pipeline poorly against the kernels (24.1 us per step), with three better
# (17.9 us), with four they hide behind the kernels entirely (15.6 us, the kernels alone
# on the same streams: 15.2 us).
E2E_STREAMS = 4

E2E_PATHS = {
    "host_entry": "pinned host x -> dflash_qmm_host (C ABI via ctypes: copy in, matmul, copy out queued by one "
                  "library call) -> pinned host y, every step; steps rotate over four streams so copies overlap "
                  "kernels",
    "three_calls": "pinned host x -> device (torch copy) -> dflash_qmm (C ABI via ctypes) -> pinned host y (torch "
                   "copy), every step; steps rotate over four streams so copies overlap kernels",
}


def e2e_line(three, host, world, nbytes, steps):
    """The e2e key: the faster of the two host paths that ran (the one-call host-buffer
    entry point counts only after its bit-exact check); both figures are listed."""
    def fig(rec):
        if "error" in rec or not math.isfinite(rec["ms"]):
            return {"error": rec.get("error", "not finite")}
        return {"value": round(world * nbytes / (rec["ms"] * 1e-3 / steps) / 1e9, 1), "unit": "GB/s",
                "us_per_step": round(rec["ms"] * 1e3 / steps, 3)}
    figs = {"host_entry": fig(host), "three_calls": fig(three)}
    ok = [k for k in ("host_entry", "three_calls") if "value" in figs[k]]
    best = max(ok, key=lambda k: figs[k]["value"]) if ok else "three_calls"
    return {**figs[best], "h2d_bytes_per_step": three["h2d"], "d2h_bytes_per_step": three["d2h"],
            "path": E2E_PATHS[best], "paths": figs}


def e2e_host_entry(dc, dev, x, copies, args, want):
    """Per step ONE library call, dflash_qmm_host through ctypes: it queues the copy of
    pinned host x into its workspace, the matmul and the copy of y to pinned host memory
    on the step's stream.  Steps rotate over E2E_STREAMS streams (each with its own
    workspace and host output), as in e2e_through_abi.  Before timing, one call per weight
    copy must reproduce dflash_qmm's bits (`want`)."""
    import ctypes
    import torch
    streams = [torch.cuda.Stream(dev) for _ in range(E2E_STREAMS)]
    x_h = torch.from_numpy(np.ascontiguousarray(x[:M]).view(np.int16)).view(torch.bfloat16).pin_memory()
    fn = dc.lib.dflash_qmm_host
    lanes = []
    for st in streams:
        ws = dc.Workspace(dc.qmm_host_workspace_bytes(M, N, K, GROUP, BITS), dev)
        y_h = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
        lanes.append({"ws": ws, "y_h": y_h, "stream": st,
                      "args": [(x_h.data_ptr(), w.data_ptr(), s_.data_ptr(), b.data_ptr(), y_h.data_ptr(), M, N, K,
                                GROUP, BITS, ws.buf.data_ptr(), ctypes.c_size_t(ws.nbytes), st.cuda_stream)
                               for (w, s_, b) in copies]})
    R = len(copies)
    torch.cuda.synchronize(dev)
    for r in range(R):
        lane = lanes[r % E2E_STREAMS]
        dc.check(fn(*lane["args"][r]))
        lane["stream"].synchronize()
        if not torch.equal(lane["y_h"], want[r]):
            raise RuntimeError(f"dflash_qmm_host differs from dflash_qmm on weight copy {r}")

    def step(i):
        lane = lanes[i % E2E_STREAMS]
        dc.check(fn(*lane["args"][i % R]))

    for i in range(min(args.warmup, 200)):
        step(i)
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(streams[0])
    for st in streams[1:]:
        st.wait_event(t0)
    for i in range(args.steps):
        step(i)
    for st in streams[1:]:
        done = torch.cuda.Event()
        done.record(st)
        streams[0].wait_event(done)
    t1.record(streams[0])
    torch.cuda.synchronize(dev)
    return {"ms": t0.elapsed_time(t1), "h2d": M * K * 2, "d2h": M * N * 2}


def e2e_through_abi(dc, dev, x, copies, args, world):
    """Per step: pinned host x -> device, dflash_qmm through the C ABI (ctypes, the
    library's entry point itself), device y -> pinned host; CUDA events around the K
    steps.  Steps rotate over E2E_STREAMS streams, each with its own device buffers,
    workspace and host output, so one step's copies overlap another step's kernels, as
    a serving host would pipeline consecutive requests."""
    import ctypes
    import torch
    streams = [torch.cuda.Stream(dev) for _ in range(E2E_STREAMS)]
    x_h = torch.from_numpy(np.ascontiguousarray(x[:M]).view(np.int16)).view(torch.bfloat16).pin_memory()
    lanes = []
    for st in streams:
        lane = {"x_d": torch.empty((M, K), dtype=torch.bfloat16, device=dev),
                "y_d": torch.empty((M, N), dtype=torch.bfloat16, device=dev),
                "y_h": torch.empty((M, N), dtype=torch.bfloat16).pin_memory(),
                "ws": dc.Workspace(dc.qmm_workspace_bytes(M, N, K, GROUP, BITS), dev), "stream": st}
        lane["args"] = [(lane["x_d"].data_ptr(), w.data_ptr(), s_.data_ptr(), b.data_ptr(), lane["y_d"].data_ptr(), M,
                         N, K, GROUP, BITS, lane["ws"].buf.data_ptr(), ctypes.c_size_t(lane["ws"].nbytes),
                         st.cuda_stream) for (w, s_, b) in copies]
        lanes.append(lane)
    R = len(copies)

    def step(i):
        lane = lanes[i % E2E_STREAMS]
        with torch.cuda.stream(lane["stream"]):
            lane["x_d"].copy_(x_h, non_blocking=True)
            dc.check(dc.lib.dflash_qmm(*lane["args"][i % R]))
            lane["y_h"].copy_(lane["y_d"], non_blocking=True)

    for i in range(min(args.warmup, 200)):
        step(i)
    torch.cuda.synchronize(dev)
    steps = args.steps
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(streams[0])
    for st in streams[1:]:
        st.wait_event(t0)
    for i in range(steps):
        step(i)
    for st in streams[1:]:
        done = torch.cuda.Event()
        done.record(st)
        streams[0].wait_event(done)
    t1.record(streams[0])
    torch.cuda.synchronize(dev)
    return {"ms": t0.elapsed_time(t1), "h2d": M * K * 2, "d2h": M * N * 2}


def cpu_baseline(O, x, wq, s, b, budget_s: float):
    """The CPU restatement on all host cores, on a bounded row sample of the same
    workload; reported as algorithmic GB/s of the rows processed."""
    threads = os.cpu_count() or 1
    t = time.perf_counter()
    y, used = O.qmm_cpu(x, wq, s, b, GROUP, BITS, 0, 256, threads)
    per_row = (time.perf_counter() - t) / 256
    n_rows = int(min(N, max(256, budget_s / max(per_row, 1e-9))))
    passes = int(max(1, budget_s / max(per_row * n_rows, 1e-9)))
    t = time.perf_counter()
    for _ in range(passes):
        _, used = O.qmm_cpu(x, wq, s, b, GROUP, BITS, 0, n_rows, threads)
    dt = time.perf_counter() - t
    bytes_rows = algorithmic_bytes(M, n=n_rows) * passes
    # the same restatement on one thread, over a smaller sample (about a tenth of the budget)
    n1 = int(min(N, max(64, 0.1 * budget_s / max(per_row * max(used, 1), 1e-9))))
    t1 = time.perf_counter()
    O.qmm_cpu(x, wq, s, b, GROUP, BITS, 0, n1, 1)
    dt1 = time.perf_counter() - t1
    return {"value": round(bytes_rows / dt / 1e9, 3), "unit": "GB/s", "cores": used, "kind": "port",
            "sample": f"{passes} pass(es) over rows 0..{n_rows} of N={N} (M={M}, K={K}, 4-bit g64), {dt:.2f} s",
            "us_per_call_equiv": round(dt * 1e6 * N / n_rows / passes, 1),
            "single_thread": {"value": round(algorithmic_bytes(M, n=n1) / dt1 / 1e9, 3), "unit": "GB/s",
                              "sample": f"rows 0..{n1}, {dt1:.2f} s on 1 thread"}}


# ----------------------------------------------------------------------------- reference arm

def run_reference(args):
    world, rank, local = dist_env()
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    x = O.make_x(M, K, seed_x=0)
    wq, s, b = O.make_weights(N, K, GROUP, BITS, seed_w=1)
    threads = os.cpu_count() or 1
    t = time.perf_counter()
    O.qmm_cpu(x, wq, s, b, GROUP, BITS, 0, 512, threads)
    per_row = (time.perf_counter() - t) / 512
    total_steps = args.steps + args.warmup
    rows = int(max(1, min(N, args.reference_budget_s / total_steps / max(per_row, 1e-9))))
    out = np.zeros((M, N), dtype=np.uint16)
    for i in range(args.warmup):
        n0 = (i * rows) % (N - rows + 1)
        O.qmm_cpu(x, wq, s, b, GROUP, BITS, n0, n0 + rows, threads, out=out)
    t = time.perf_counter()
    used = threads
    for i in range(args.steps):
        n0 = (i * rows) % (N - rows + 1)
        _, used = O.qmm_cpu(x, wq, s, b, GROUP, BITS, n0, n0 + rows, threads, out=out)
    dt = time.perf_counter() - t
    gbs = algorithmic_bytes(M, n=rows) * args.steps / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 6),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u4 weights, bf16 x/y, fp32 accumulate", "data": "synthetic", "config": config(M),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": used, "kind": "port",
                         "sample": f"each step: {rows} consecutive rows of W (of {N}), M={M}, K={K}"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference path is Metal/MLX on Apple GPUs (unavailable here); this is the project's C "
                "restatement of its arithmetic on all host cores",
    }
    print(json.dumps(line))


def run_profile(args):
    """3 warm-up + 3 profiled launches of config 2 on distinct weight copies (each
    launch streams its weights from HBM).  Used as the ncu target."""
    import torch
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    import dflashcuda as dc
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    m = args.profile_m
    x_d = to_dev(O.make_x(m, K, seed_x=0), dev)
    wq, s, b = O.make_weights(N, K, GROUP, BITS, seed_w=1)
    copies = weight_copies(dev, wq, s, b)
    y_d = torch.empty((m, N), dtype=torch.bfloat16, device=dev)
    ws = dc.Workspace(dc.qmm_workspace_bytes(m, N, K, GROUP, BITS), dev)
    for i in range(6):
        w, sc, bi = copies[i % len(copies)]
        dc.qmm(x_d, w, sc, bi, GROUP, BITS, out=y_d, workspace=ws)
    torch.cuda.synchronize()
    print(f"profile run ok: {6} launches, M={m}, device error {dc.device_error()}")


def run_profile_gdn(args):
    """4 plain rollback replays of BASELINE config 5 (48 layers x 32 heads x 128 x 128 fp32,
    keep 8), alternating over two snapshot/state pairs: the target of a kernel capture of the replay."""
    import torch
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    import dflashcuda as dc
    L, W, H, dk, dv, keep = 48, 8, 32, 128, 128, 8
    g = torch.Generator(device=dev).manual_seed(2)
    snaps = [0.1 * torch.randn(L, H, dv, dk, generator=g, device=dev) for _ in range(2)]
    outs = [torch.empty_like(snaps[0]) for _ in range(2)]
    k = torch.nn.functional.normalize(torch.randn(L, W, H, dk, generator=g, device=dev), dim=-1).to(torch.bfloat16)
    v = torch.randn(L, W, H, dv, generator=g, device=dev).to(torch.bfloat16)
    alpha = 0.9 + 0.1 * torch.rand(L, W, H, generator=g, device=dev)
    beta = torch.rand(L, W, H, generator=g, device=dev)
    for i in range(4):
        dc.gdn_replay(snaps[i & 1], outs[i & 1], k, v, alpha, beta, keep=keep)
    torch.cuda.synchronize()
    print(f"gdn profile run ok: 4 replays, device error {dc.device_error()}")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=2000)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--reference-budget-s", type=float, default=60.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="a few plain launches of the workload for ncu (no graph, no timing line)")
    ap.add_argument("--profile-m", type=int, default=M)
    ap.add_argument("--profile-gdn", action="store_true",
                    help="a few plain rollback replays of config 5 for ncu (no timing line)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.profile_gdn:
        run_profile_gdn(args)
    elif args.profile:
        run_profile(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

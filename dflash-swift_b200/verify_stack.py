"""Tensor-parallel verify forward of a hybrid gated-delta / attention target.

The reference verifies a drafted block with one forward of its Qwen3.5-style target
(`target(verifyInput, cache: targetCache)`, Sources/DFlashKit/DFlashSpeculativeGenerator.swift:397,
with gated-delta capture switched on at :389-393).  That model lives in an external MLX
fork; its shape is fixed here as a 64-layer stack (48 gated-delta + 16 GQA attention
layers, one attention layer per 4, `full_attention_interval`, Tests/DFlashKitTests/
TinyHybridTarget.swift:37) whose every projection is an MLX affine-quantized matmul.

Each rank (one process per GPU) owns a shard of every layer:
  * column-sharded along N (heads / intermediate units): the gated-delta in_proj
    [q | k | v | z | b | a], the attention qkv projection [q | gate | k | v] and the MLP
    gate_up [gate | up];
  * row-sharded along K (group-aligned): gated-delta out_proj, attention o_proj and the
    MLP down projection, whose partial [M, hidden] outputs are summed by one all-reduce.
So a layer has exactly two collectives (after the mixer and after the MLP), 128 per
forward.  The residual stream is fp32 and replicated; everything between the shard
boundaries is rank-local.  The projections run on dflash_qmm, the recurrence on
dflash_gdn_step (its inputs are the rollback capture) and the glue on the dflash_stack_*
kernels (SwiGLU is folded into the down projection's input prep).  The all-reduce runs
over peer memory: the row-sharded projection's qmm kernel stores its output into every
rank's exchange buffer over NVLink as epoch-tagged words (dflash_qmm_ex with push) and
the next RMSNorm sums the slots once every word carries the exchange's epoch
(dflash_stack_add_rmsnorm_reduce); NCCL through torch.distributed is the alternative
(`allreduce="nccl"`).  The whole forward is
captured once as a CUDA graph and replayed.

Weights are seeded synthetic MLX-packed 4-bit tensors (no checkpoint is available):
every rank draws the same global tensor from the same seed and keeps its shard, so a
TP=P run computes the same function as TP=1.

Run as a benchmark (one line of JSON per run):
    python dflash-swift_b200/verify_stack.py                      # TP=1
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        dflash-swift_b200/verify_stack.py
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
from dataclasses import dataclass, asdict, replace
from pathlib import Path
from typing import Callable, Optional

import torch

HERE = Path(__file__).resolve().parent


@dataclass(frozen=True)
class StackConfig:
    layers: int = 64
    hidden: int = 5120
    intermediate: int = 17408
    attn_interval: int = 4      # layer i is an attention layer when (i + 1) % attn_interval == 0
    gdn_heads: int = 32         # gated-delta heads (q, k and v alike)
    gdn_dk: int = 128
    gdn_dv: int = 128
    conv_kernel: int = 4
    attn_heads: int = 24
    kv_heads: int = 4
    head_dim: int = 256
    rotary_dim: int = 64        # partial rotary: the first 64 of 256 dims
    rope_theta: float = 1.0e7
    eps: float = 1.0e-6
    group: int = 64
    bits: int = 4
    context: int = 1024         # tokens already in each attention cache
    block: int = 8              # M: rows verified per forward
    vocab: int = 248320         # LM head rows (sharded by vocabulary over the ranks)
    gdn_key_heads: int = 0      # gated-delta q / k heads (0: gdn_heads); each shared by
                                # gdn_heads / gdn_key_heads value heads (linear_num_key_heads)

    @property
    def gdn_kheads(self) -> int:
        return self.gdn_key_heads or self.gdn_heads

    @property
    def max_len(self) -> int:
        return self.context + self.block

    def is_attention(self, layer: int) -> bool:
        return (layer + 1) % self.attn_interval == 0

    def layer_kinds(self):
        return ["attn" if self.is_attention(i) else "gdn" for i in range(self.layers)]


# 64-layer hybrid, hidden 5120, MLP 17408, 48 GDN + 16 GQA, 4-bit g64, M=8.
CONFIG4 = StackConfig()
# A small stack of the same structure for parity tests (3 GDN + 1 attention layers).
TINY = StackConfig(layers=4, hidden=256, intermediate=512, gdn_heads=4, gdn_dk=64, gdn_dv=64, attn_heads=4,
                   kv_heads=2, head_dim=64, rotary_dim=64, rope_theta=1.0e4, context=24, block=8, vocab=1024)
# The same with 2 gated-delta key heads for the 4 value heads (as the reference's fixture
# has, Tests/DFlashKitTests/TinyHybridTarget.swift:27-30).
TINY_GROUPED = replace(TINY, gdn_key_heads=2)
# A small stack that shards over 1, 2, 4 and 8 ranks (every row-sharded K a whole number
# of groups at 8 ranks; 2 kv heads, so at 4 and 8 ranks a kv head is replicated): the
# benchmark's check that TP = N computes TP = 1's function on the same GPUs.
TP_CHECK = StackConfig(layers=4, hidden=512, intermediate=1024, gdn_heads=8, gdn_dk=64, gdn_dv=64, attn_heads=8,
                       kv_heads=2, head_dim=64, rotary_dim=64, rope_theta=1.0e4, context=24, block=8, vocab=2048)


# ----------------------------------------------------------------------------- shard plan

@dataclass(frozen=True)
class ShardPlan:
    rank: int
    world: int
    gdn_heads: int          # gated-delta heads on this rank
    gdn_head0: int
    attn_heads: int         # q heads on this rank
    attn_head0: int
    kv_heads: int           # kv heads this rank computes (replicated when world > kv_heads)
    kv_head0: int
    inter: int              # MLP intermediate units on this rank
    inter0: int
    vocab: int = 0          # LM head rows on this rank
    vocab0: int = 0
    gdn_key_heads: int = 0  # gated-delta q / k heads on this rank (those its value heads read)
    gdn_key_head0: int = 0


def shard_plan(cfg: StackConfig, rank: int, world: int) -> ShardPlan:
    """Which heads / units of each layer rank `rank` of `world` owns.

    Gated-delta heads, q heads and intermediate units split evenly.  KV heads split
    evenly when world divides them; with more ranks than kv heads each rank computes the
    one kv head its q heads read (so that head is replicated on world / kv_heads ranks).
    Row-sharded K extents (heads * dv, heads * head_dim, intermediate / world) must be
    whole quantization groups."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    for name, total in (("gdn_heads", cfg.gdn_heads), ("attn_heads", cfg.attn_heads),
                        ("intermediate", cfg.intermediate)):
        if total % world:
            raise ValueError(f"{name}={total} does not split over {world} ranks")
    if cfg.attn_heads % cfg.kv_heads:
        raise ValueError("attn_heads must be a multiple of kv_heads")
    if cfg.gdn_dk != cfg.gdn_dv:
        raise ValueError("the gated-delta conv treats q, k and v as equal parts: gdn_dk must equal gdn_dv")
    if cfg.gdn_heads % cfg.gdn_kheads or cfg.gdn_kheads % world:
        raise ValueError(f"gdn_key_heads={cfg.gdn_kheads} must divide gdn_heads and split over {world} ranks")
    gh = cfg.gdn_heads // world
    gkh = cfg.gdn_kheads // world  # value heads [rank gh, ...) read key heads [rank gkh, ...)
    ah = cfg.attn_heads // world
    q_per_kv = cfg.attn_heads // cfg.kv_heads
    if cfg.kv_heads % world == 0:
        kvh, kv0 = cfg.kv_heads // world, rank * (cfg.kv_heads // world)
    elif q_per_kv % ah == 0:
        kvh, kv0 = 1, (rank * ah) // q_per_kv
    else:
        raise ValueError(f"{world} ranks split the {q_per_kv} q heads of a kv head unevenly")
    inter = cfg.intermediate // world
    for name, k in (("gdn out_proj", gh * cfg.gdn_dv), ("o_proj", ah * cfg.head_dim), ("down", inter)):
        if k % cfg.group:
            raise ValueError(f"{name} shard K={k} is not a multiple of group {cfg.group}")
    if cfg.vocab % world:
        raise ValueError(f"vocab={cfg.vocab} does not split over {world} ranks")
    vr = cfg.vocab // world
    return ShardPlan(rank, world, gh, rank * gh, ah, rank * ah, kvh, kv0, inter, rank * inter, vr, rank * vr,
                     gkh, rank * gkh)


def _ranges_gdn_in(cfg: StackConfig, p: ShardPlan):
    """Global row ranges of the in_proj [q | k | v | z | b | a] this rank keeps, in order
    (q and k have gdn_kheads heads, the rest one entry per value head)."""
    H, Hk, dk, dv = cfg.gdn_heads, cfg.gdn_kheads, cfg.gdn_dk, cfg.gdn_dv
    h0, h1 = p.gdn_head0, p.gdn_head0 + p.gdn_heads
    k0, k1 = p.gdn_key_head0, p.gdn_key_head0 + p.gdn_key_heads
    v_off = 2 * Hk * dk
    return [(k0 * dk, k1 * dk), (Hk * dk + k0 * dk, Hk * dk + k1 * dk), (v_off + h0 * dv, v_off + h1 * dv),
            (v_off + H * dv + h0 * dv, v_off + H * dv + h1 * dv), (v_off + 2 * H * dv + h0, v_off + 2 * H * dv + h1),
            (v_off + 2 * H * dv + H + h0, v_off + 2 * H * dv + H + h1)]


def gdn_conv_channels(cfg: StackConfig, p: ShardPlan):
    """Global channel ranges of the gated-delta conv [q | k | v] this rank keeps (its key
    heads' q and k channels, its value heads' v channels), in order."""
    Hk, dk = cfg.gdn_kheads, cfg.gdn_dk
    k0, k1 = p.gdn_key_head0 * dk, (p.gdn_key_head0 + p.gdn_key_heads) * dk
    h0, h1 = p.gdn_head0 * dk, (p.gdn_head0 + p.gdn_heads) * dk
    return [(k0, k1), (Hk * dk + k0, Hk * dk + k1), (2 * Hk * dk + h0, 2 * Hk * dk + h1)]


def _ranges_attn_qkv(cfg: StackConfig, p: ShardPlan):
    """Global row ranges of the qkv projection [q | gate | k | v] this rank keeps."""
    d, Hq, Hkv = cfg.head_dim, cfg.attn_heads, cfg.kv_heads
    q0, q1 = p.attn_head0 * d, (p.attn_head0 + p.attn_heads) * d
    k0, k1 = p.kv_head0 * d, (p.kv_head0 + p.kv_heads) * d
    return [(q0, q1), (Hq * d + q0, Hq * d + q1), (2 * Hq * d + k0, 2 * Hq * d + k1),
            (2 * Hq * d + Hkv * d + k0, 2 * Hq * d + Hkv * d + k1)]


def _ranges_gate_up(cfg: StackConfig, p: ShardPlan):
    I = cfg.intermediate
    return [(p.inter0, p.inter0 + p.inter), (I + p.inter0, I + p.inter0 + p.inter)]


# ----------------------------------------------------------------------------- weights

@dataclass
class Quant:
    """MLX affine-quantized matrix: packed u32 (stored as int32) [N, K*bits/32], bf16
    scales and biases [N, K/group]."""
    w: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    group: int
    bits: int

    @property
    def N(self) -> int:
        return self.w.shape[0]

    @property
    def K(self) -> int:
        return self.w.shape[1] * 32 // self.bits

    def rows(self, ranges) -> "Quant":
        idx = lambda t: torch.cat([t[a:b] for a, b in ranges]).contiguous()
        return Quant(idx(self.w), idx(self.scales), idx(self.biases), self.group, self.bits)

    def cols(self, k0: int, k1: int) -> "Quant":
        if k0 % self.group or k1 % self.group:
            raise ValueError("K shard must be group-aligned")
        wpk = 32 // self.bits
        return Quant(self.w[:, k0 // wpk:k1 // wpk].contiguous(), self.scales[:, k0 // self.group:k1 // self.group]
                     .contiguous(), self.biases[:, k0 // self.group:k1 // self.group].contiguous(), self.group,
                     self.bits)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.w, self.scales, self.biases))


def random_quant(gen: torch.Generator, N: int, K: int, group: int, bits: int, device, w_std: float = 0.02) -> Quant:
    """Uniform random codes with per-group scales around w_std / std(code) and biases
    centring the codes, so dequantised weights have roughly N(0, w_std) spread."""
    words = K * bits // 32
    w = torch.randint(-2 ** 31, 2 ** 31 - 1, (N, words), dtype=torch.int32, generator=gen, device=device)
    levels = 2 ** bits
    code_std = math.sqrt((levels * levels - 1) / 12.0)
    s = (w_std / code_std) * (0.5 + torch.rand((N, K // group), generator=gen, device=device))
    b = -(levels - 1) / 2.0 * s + 0.1 * w_std * torch.randn((N, K // group), generator=gen, device=device)
    return Quant(w, s.to(torch.bfloat16), b.to(torch.bfloat16), group, bits)


def _norm_weight(gen, n, device):
    return (1.0 + 0.1 * torch.randn(n, generator=gen, device=device)).to(torch.bfloat16)


def layer_seed(seed: int, layer: int, slot: int) -> int:
    return (seed * 1_000_003 + layer * 101 + slot) & 0x7FFFFFFF


def build_rank_weights(cfg: StackConfig, plan: ShardPlan, seed: int, device) -> dict:
    """This rank's shard of every layer.  Each global tensor is drawn from its own seed
    on `device` and sliced, so every rank (and an unsharded run) sees the same model."""
    dev = torch.device(device)

    def g(layer, slot):
        gen = torch.Generator(device=dev)
        gen.manual_seed(layer_seed(seed, layer, slot))
        return gen

    H, G, B = cfg.hidden, cfg.group, cfg.bits
    layers = []
    for li, kind in enumerate(cfg.layer_kinds()):
        L = {"kind": kind, "ln": _norm_weight(g(li, 0), H, dev), "post_ln": _norm_weight(g(li, 1), H, dev)}
        if kind == "gdn":
            Hg, Hk, dk, dv, kc = cfg.gdn_heads, cfg.gdn_kheads, cfg.gdn_dk, cfg.gdn_dv, cfg.conv_kernel
            n_in = 2 * Hk * dk + 2 * Hg * dv + 2 * Hg
            L["in_proj"] = random_quant(g(li, 2), n_in, H, G, B, dev).rows(_ranges_gdn_in(cfg, plan))
            L["out_proj"] = random_quant(g(li, 3), H, Hg * dv, G, B, dev).cols(plan.gdn_head0 * dv,
                                                                              (plan.gdn_head0 + plan.gdn_heads) * dv)
            gg = g(li, 4)
            conv = (0.5 * torch.randn((2 * Hk + Hg) * dk, kc, generator=gg, device=dev)).to(torch.bfloat16)
            a_log = torch.log(torch.empty(Hg, device=dev).uniform_(1.0, 16.0, generator=gg))
            dt_bias = 0.5 * torch.randn(Hg, generator=gg, device=dev)
            heads = slice(plan.gdn_head0, plan.gdn_head0 + plan.gdn_heads)
            conv3 = torch.cat([conv[a:b] for a, b in gdn_conv_channels(cfg, plan)]).contiguous()
            L.update(conv=conv3, a_log=a_log[heads].contiguous(), dt_bias=dt_bias[heads].contiguous(),
                     gdn_norm=_norm_weight(gg, dv, dev))
        else:
            Hq, Hkv, d = cfg.attn_heads, cfg.kv_heads, cfg.head_dim
            L["qkv"] = random_quant(g(li, 2), 2 * Hq * d + 2 * Hkv * d, H, G, B, dev).rows(_ranges_attn_qkv(cfg, plan))
            L["o_proj"] = random_quant(g(li, 3), H, Hq * d, G, B, dev).cols(plan.attn_head0 * d,
                                                                            (plan.attn_head0 + plan.attn_heads) * d)
            gg = g(li, 4)
            L.update(q_norm=_norm_weight(gg, d, dev), k_norm=_norm_weight(gg, d, dev))
        I = cfg.intermediate
        L["gate_up"] = random_quant(g(li, 5), 2 * I, H, G, B, dev).rows(_ranges_gate_up(cfg, plan))
        L["down"] = random_quant(g(li, 6), H, I, G, B, dev).cols(plan.inter0, plan.inter0 + plan.inter)
        layers.append(L)
    final_norm = _norm_weight(g(cfg.layers, 0), H, dev)
    lm_head = random_quant(g(cfg.layers, 1), cfg.vocab, H, G, B, dev).rows([(plan.vocab0, plan.vocab0 + plan.vocab)])
    return {"layers": layers, "final_norm": final_norm, "lm_head": lm_head}


def build_rank_state(cfg: StackConfig, plan: ShardPlan, seed: int, device) -> dict:
    """Pre-round state of this rank's shard: gated-delta snapshots (fp32 [h, dv, dk]) and
    conv windows (bf16 [kc-1, (2 hk + h) dk]); attention caches (bf16 [hkv, max_len, d])
    holding `context` random tokens."""
    dev = torch.device(device)
    out = []
    for li, kind in enumerate(cfg.layer_kinds()):
        gen = torch.Generator(device=dev)
        gen.manual_seed(layer_seed(seed + 7, li, 9))
        if kind == "gdn":
            Hg, Hk, dk, dv, kc = cfg.gdn_heads, cfg.gdn_kheads, cfg.gdn_dk, cfg.gdn_dv, cfg.conv_kernel
            heads = slice(plan.gdn_head0, plan.gdn_head0 + plan.gdn_heads)
            snap = 0.1 * torch.randn(Hg, dv, dk, generator=gen, device=dev)
            win = torch.randn(kc - 1, (2 * Hk + Hg) * dk, generator=gen, device=dev).to(torch.bfloat16)
            out.append({"snapshot": snap[heads].contiguous(),
                        "window": torch.cat([win[:, a:b] for a, b in gdn_conv_channels(cfg, plan)], 1).contiguous()})
        else:
            Hkv, d = cfg.kv_heads, cfg.head_dim
            kv = slice(plan.kv_head0, plan.kv_head0 + plan.kv_heads)
            ck = torch.zeros(Hkv, cfg.max_len, d, dtype=torch.bfloat16, device=dev)
            cv = torch.zeros_like(ck)
            ck[:, :cfg.context] = torch.randn(Hkv, cfg.context, d, generator=gen, device=dev).to(torch.bfloat16)
            cv[:, :cfg.context] = torch.randn(Hkv, cfg.context, d, generator=gen, device=dev).to(torch.bfloat16)
            out.append({"cache_k": ck[kv].contiguous(), "cache_v": cv[kv].contiguous()})
    return {"layers": out}


def make_block(cfg: StackConfig, seed: int, device) -> torch.Tensor:
    """The verify block's input hidden states, bf16 [M, hidden] ~ N(0, 1)."""
    gen = torch.Generator(device=torch.device(device))
    gen.manual_seed(layer_seed(seed + 3, 0, 0))
    return torch.randn(cfg.block, cfg.hidden, generator=gen, device=device).to(torch.bfloat16)


def weight_bytes(weights: dict) -> int:
    n = 0
    for L in weights["layers"]:
        for v in L.values():
            if isinstance(v, Quant):
                n += v.nbytes()
    return n


# ----------------------------------------------------------------------------- the CUDA stack

class VerifyStack:
    """One rank's shard of the hybrid target, run on libdflashcuda.

    forward(hidden) runs the verify forward of one block of `cfg.block` rows from the
    pre-round state (gated-delta snapshots and conv windows are only read; the new
    states go to `state_out`, the attention caches receive the block's k and v at
    positions context .. context + M - 1), and returns the final-norm hidden states
    bf16 [M, hidden] (identical on every rank)."""

    def __init__(self, cfg: StackConfig, rank: int = 0, world: int = 1, seed: int = 0, device=None,
                 group=None, weights: Optional[dict] = None, state: Optional[dict] = None, allreduce: str = "peer",
                 tree: bool = False, device_position: bool = False):
        import dflashcuda as dc
        self.dc = dc
        self.cfg = cfg
        self.tree = tree
        # tokens already in the attention caches: the block's rows go to cache rows
        # context .. context + block - 1.  advance() moves it.  A captured graph keeps the
        # value it was captured with, unless device_position: the attention kernels then
        # read it from `position` (device int32), which advance() rewrites, so one captured
        # round serves a whole decode loop.
        self.context = cfg.context
        self.device_position = device_position
        self.plan = shard_plan(cfg, rank, world)
        self.world = world
        self.pg = group
        self.device = torch.device(device if device is not None else f"cuda:{torch.cuda.current_device()}")
        if self.device.type != "cuda":
            raise RuntimeError("VerifyStack runs on libdflashcuda only (no CPU path)")
        self.w = weights if weights is not None else build_rank_weights(cfg, self.plan, seed, self.device)
        self.state = state if state is not None else build_rank_state(cfg, self.plan, seed, self.device)
        self._alloc()
        self.graph = None
        if allreduce not in ("peer", "nccl"):
            raise ValueError("allreduce is 'peer' (NVLink stores into the peers' exchange buffers) or 'nccl'")
        self.allreduce = allreduce if world > 1 else "none"
        self.exchange = None
        self._set = 0
        self.key_exchange = None
        if self.allreduce == "peer":
            self.exchange = self._connect_exchange(rank, self.cfg.hidden)
            self.key_exchange = self._connect_exchange(rank, 4)  # the LM head's argmax keys, 8 bytes a row

    def _connect_exchange(self, rank, H):
        """Allocate this rank's exchange buffer for [block, H], swap IPC handles with the
        other ranks and map theirs; the barrier ensures every buffer is zeroed before
        anyone pushes."""
        ex = self.dc.PeerExchange(self.world, self.cfg.block, H)
        handles = [None] * self.world
        torch.distributed.all_gather_object(handles, ex.handle(), group=self.pg)
        ex.connect(rank, handles)
        torch.cuda.synchronize(self.device)
        torch.distributed.barrier(group=self.pg)
        return ex

    def close(self):
        """Unmap the peers' exchange buffers and free this rank's (after a barrier, so no
        peer still pushes into it)."""
        if self.exchange is not None:
            torch.cuda.synchronize(self.device)
            torch.distributed.barrier(group=self.pg)
            self.exchange.close()
            self.key_exchange.close()
            self.exchange = self.key_exchange = None

    def _alloc(self):
        cfg, p, dev = self.cfg, self.plan, self.device
        M, H = cfg.block, cfg.hidden
        bf = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        self.resid = torch.zeros(M, H, **f32)
        self.normed = torch.empty(M, H, **bf)
        self.delta = torch.zeros(M, H, **bf)
        self.out = torch.empty(M, H, **bf)
        self.keys = torch.empty(M, dtype=torch.int64, device=dev)
        self.tokens = torch.empty(M, dtype=torch.int32, device=dev)
        self.accepted = torch.empty(1, dtype=torch.int32, device=dev)
        # the sign bit, for ordering unsigned keys as signed int64 in a max all-reduce (made
        # here: a host-to-device copy is not allowed while a CUDA graph is being captured)
        self._sign = torch.full((1,), -(2 ** 63), dtype=torch.int64, device=dev)
        # tree rounds: the block's parent list, read by the tree kernels in stream order so a
        # captured round replays with whatever tree set_tree last wrote (a chain until then)
        self.position = (torch.tensor([self.context], dtype=torch.int32, device=dev) if self.device_position
                         else None)
        self.parents = torch.tensor([-1] + list(range(M - 1)), dtype=torch.int32, device=dev) if self.tree else None
        self.tree_plan = None
        if self.tree:  # the drafted token of every row, and the device walk's accepted path
            self.tree_tokens = torch.zeros(M, dtype=torch.int32, device=dev)
            self.path = torch.zeros(M, dtype=torch.int32, device=dev)
            self.path_len = torch.zeros(1, dtype=torch.int32, device=dev)
            self.next_token = torch.zeros(1, dtype=torch.int32, device=dev)
        h, dk, dv = p.gdn_heads, cfg.gdn_dk, cfg.gdn_dv
        # per layer: the in-projection (its q | k | v channels are the conv inputs that
        # commit() rebuilds the conv window from) and the conv output q | k | v, which with
        # alpha and beta is the capture the recurrence replays
        n_gdn = sum(1 for k in cfg.layer_kinds() if k == "gdn")
        hk = p.gdn_key_heads or h
        self.gdn_proj = torch.empty(n_gdn, M, 2 * hk * dk + 2 * h * dv + 2 * h, **bf)
        # [3, M, h, dk] per layer; with shared key heads the q, k and v blocks are
        # [M, hk, dk], [M, hk, dk], [M, h, dk] back to back (gdn_qkv gives the views)
        self.capture_qkv = (torch.empty(n_gdn, 3, M, h, dk, **bf) if hk == h else
                            torch.empty(n_gdn, M * (2 * hk + h) * dk, **bf))
        self.capture_alpha = torch.empty(n_gdn, M, h, **f32)
        self.capture_beta = torch.empty(n_gdn, M, h, **f32)
        self.state_out = torch.empty(n_gdn, h, dv, dk, **f32)
        self.gdn_o = torch.empty(M, h, dv, **bf)
        self.gdn_normed = torch.empty(M, h * dv, **bf)
        d = cfg.head_dim
        self.qkv = torch.empty(M, (2 * p.attn_heads + 2 * p.kv_heads) * d, **bf)
        self.attn_out = torch.empty(M, p.attn_heads * d, **bf)
        self.gate_up = torch.empty(M, 2 * p.inter, **bf)
        need = 0
        for L in self.w["layers"]:
            for v in L.values():
                if isinstance(v, Quant):
                    need = max(need, self.dc.qmm_workspace_bytes(M, v.N, v.K, v.group, v.bits))
        self.ws = self.dc.Workspace(need, dev)

    # -- pieces
    def _qmm(self, x, q: Quant, out):
        self.dc.qmm(x, q.w, q.scales, q.biases, q.group, q.bits, out=out, workspace=self.ws)

    def _qmm_reduced(self, x, q: Quant, swiglu: bool = False):
        """A row-sharded projection whose output is all-reduced: with the peer exchange the
        qmm kernel pushes its result straight into every rank's slot; otherwise it writes
        self.delta, which NCCL (or nothing, at TP=1) reduces.  Returns the pending delta
        for the next norm."""
        if self.allreduce == "peer":
            self.dc.qmm_ex(x, q.w, q.scales, q.biases, q.group, q.bits, workspace=self.ws, swiglu=swiglu,
                           exchange=self.exchange, set_=self._set)
            pending = ("exchange", self._set)
            self._set ^= 1
            return pending
        self.dc.qmm_ex(x, q.w, q.scales, q.biases, q.group, q.bits, out=self.delta, workspace=self.ws, swiglu=swiglu)
        return self._reduce(self.delta)

    def _reduce(self, part):
        """All-reduce of a partial written to memory (NCCL, or nothing at TP=1); returns
        what the next norm adds."""
        if self.allreduce == "nccl":
            torch.distributed.all_reduce(part, group=self.pg)
        return part

    def _norm(self, pending, weight, out):
        """resid += the pending delta (a local tensor or the peer exchange); out = RMSNorm(resid)."""
        if isinstance(pending, tuple):
            self.dc.stack_add_rmsnorm_reduce(self.resid, self.exchange, pending[1], weight, out, self.cfg.eps)
        else:
            self.dc.stack_add_rmsnorm(self.resid, pending, weight, out, self.cfg.eps)

    def gdn_qkv(self, gi):
        """Layer gi's captured q, k ([M, hk, dk]) and v ([M, h, dv]) after the conv."""
        M, h, dk = self.cfg.block, self.plan.gdn_heads, self.cfg.gdn_dk
        hk = self.plan.gdn_key_heads or h
        qkv = self.capture_qkv[gi]
        if hk == h:
            return qkv[0], qkv[1], qkv[2]
        n = M * hk * dk
        return qkv[:n].view(M, hk, dk), qkv[n:2 * n].view(M, hk, dk), qkv[2 * n:].view(M, h, dk)

    def _gdn(self, L, S, gi):
        cfg, p, dc = self.cfg, self.plan, self.dc
        M, h, dk, dv = cfg.block, p.gdn_heads, cfg.gdn_dk, cfg.gdn_dv
        hk = p.gdn_key_heads or h
        proj = self.gdn_proj[gi]
        self._qmm(self.normed, L["in_proj"], proj)
        qkv = self.capture_qkv[gi]
        q, k, v = self.gdn_qkv(gi)
        ab = proj[:, 2 * hk * dk + 2 * h * dv:]
        alpha, beta = self.capture_alpha[gi], self.capture_beta[gi]
        dc.stack_gdn_conv_gates(proj, S["window"], L["conv"], qkv, ab, L["a_log"], L["dt_bias"], alpha, beta,
                                h, dk, parents=self.parents, k_heads=hk)
        if self.parents is None:
            dc.gdn_step(S["snapshot"], self.state_out[gi], q, k, v, alpha, beta, out=self.gdn_o,
                        q_scale=1.0 / math.sqrt(dk))
        else:  # no state after a tree round: commit() replays the accepted path
            dc.gdn_step_tree(S["snapshot"], q, k, v, alpha, beta, self.parents, self.gdn_o,
                             q_scale=1.0 / math.sqrt(dk))
        z = proj[:, 2 * hk * dk + h * dv:]
        dc.stack_gated_norm(self.gdn_o, z, L["gdn_norm"], self.gdn_normed, cfg.eps)
        return self._qmm_reduced(self.gdn_normed, L["out_proj"])

    def _attn(self, L, S):
        cfg, p, dc = self.cfg, self.plan, self.dc
        self._qmm(self.normed, L["qkv"], self.qkv)
        dc.stack_attn_prep(self.qkv, L["q_norm"], L["k_norm"], S["cache_k"], S["cache_v"], p.attn_heads, p.kv_heads,
                           cfg.rotary_dim, self.context, cfg.eps, cfg.rope_theta, parents=self.parents,
                           position=self.position)
        dc.stack_attn_decode(self.qkv, S["cache_k"], S["cache_v"], self.attn_out, p.attn_heads, p.kv_heads,
                             self.context, 1.0 / math.sqrt(cfg.head_dim), parents=self.parents,
                             position=self.position)
        return self._qmm_reduced(self.attn_out, L["o_proj"])

    def _mlp(self, L):
        self._qmm(self.normed, L["gate_up"], self.gate_up)
        return self._qmm_reduced(self.gate_up, L["down"], swiglu=True)  # SwiGLU inside the down qmm

    def _forward_body(self, hidden):
        cfg, dc = self.cfg, self.dc
        self.resid.zero_()
        pending = hidden
        gi = 0
        for L, S in zip(self.w["layers"], self.state["layers"]):
            self._norm(pending, L["ln"], self.normed)
            if L["kind"] == "gdn":
                pending = self._gdn(L, S, gi)
                gi += 1
            else:
                pending = self._attn(L, S)
            self._norm(pending, L["post_ln"], self.normed)
            pending = self._mlp(L)
        self._norm(pending, self.w["final_norm"], self.out)
        return self.out

    def forward(self, hidden):
        return self._forward_body(hidden)

    def _accept_body(self, proposals):
        """LM head of this rank's vocabulary shard reduced to argmax keys in its epilogue,
        the keys combined over the ranks, and the greedy accept (acceptedPrefix,
        DFlashSpeculativeGenerator.swift:555-571)."""
        q, p, dc = self.w["lm_head"], self.plan, self.dc
        dc.lm_head_argmax(self.out, q.w, q.scales, q.biases, q.group, q.bits, keys=self.keys, workspace=self.ws,
                          index_base=p.vocab0)
        if self.allreduce == "peer":
            # one key exchange per round; the layers' all-reduces in between keep the ranks
            # in step, so its slot set can stay fixed
            self.key_exchange.push(self.keys.view(torch.bfloat16).view(self.cfg.block, 4), 0)
            dc.accept_reduce(self.key_exchange, 0, proposals, self.tokens, self.accepted)
        else:
            if self.allreduce == "nccl":
                # unsigned keys as signed int64 with the sign bit flipped keep their order
                self.keys.bitwise_xor_(self._sign)
                torch.distributed.all_reduce(self.keys, op=torch.distributed.ReduceOp.MAX, group=self.pg)
                self.keys.bitwise_xor_(self._sign)
            dc.accept(self.keys, proposals, self.tokens, self.accepted)
        if self.tree:  # the accepted path over the tree, on the device
            dc.accept_tree(self.tokens, self.parents, self.tree_tokens, self.path, self.path_len, self.next_token)
        return self.tokens, self.accepted

    def verify(self, hidden, proposals):
        """One verify round: forward of the block, LM head, accept.  proposals: int32
        [block - 1] on the device.  Returns (target tokens int32 [block], accepted int32
        [1]), identical on every rank."""
        self._forward_body(hidden)
        return self._accept_body(proposals)

    def set_tree(self, parents):
        """The next rounds verify a speculative tree: parents[r] is row r's parent row (-1
        for the anchor row 0), cfg.block rows.  Call between rounds, never while a round is
        being captured."""
        from tree import SpeculativeTreePlan
        if not self.tree:
            raise RuntimeError("this stack was built without tree=True")
        plan = SpeculativeTreePlan(parents)
        if plan.rows != self.cfg.block:
            raise ValueError(f"a tree of {plan.rows} rows for a block of {self.cfg.block}")
        self.parents.copy_(torch.tensor(plan.parents, dtype=torch.int32))
        self.tree_plan = plan
        return plan

    def verify_tree(self, hidden, tokens):
        """One tree round: forward of the block under the current tree, LM head argmax
        combined over the ranks, and the accepted-path walk on the device
        (dflash_accept_tree, DFlashDraftTree.acceptedPath).  tokens: the drafted token of
        every row (host ints, row 0 the anchor's), written to the stack's device buffer
        like the parent list, so a captured round replays with new tokens.  Returns
        (accepted rows, the target's next token)."""
        if not self.tree:
            raise RuntimeError("this stack was built without tree=True")
        if self.tree_plan is None:
            self.set_tree([-1] + list(range(self.cfg.block - 1)))
        if len(tokens) != self.cfg.block:
            raise ValueError(f"{len(tokens)} drafted tokens for a block of {self.cfg.block}")
        self.tree_tokens.copy_(torch.tensor([int(t) for t in tokens], dtype=torch.int32))
        self.verify(hidden, self.tree_tokens[1:])  # the chain accept count is not used
        n = int(self.path_len.item())
        return self.path[:n].tolist(), int(self.next_token.item())

    def commit(self, rows):
        """After a round, make its accepted rows (anchor first: a chain's 0 .. keep-1, a
        tree's accepted path) the committed state, as rollbackGatedDeltaRound / Tree do
        (DFlashSpeculativeGenerator.swift:453-460): every gated-delta state is replayed
        from its snapshot over those rows' capture (dflash_gdn_replay) and its conv window
        rebuilt from their conv inputs (dflash_gdn_conv_rollback); after a tree round the
        rows' attention cache entries move to context .. context + keep - 1
        (dflash_stack_kv_compact).  The snapshots and windows are updated in place, so a
        captured round keeps its pointers; advancing the context by len(rows) is the
        caller's (advance)."""
        cfg, p, dc = self.cfg, self.plan, self.dc
        rows = [int(r) for r in rows]
        keep = len(rows)
        if not 1 <= keep <= cfg.block or rows[0] != 0:
            raise ValueError(f"accepted rows {rows}: 1..{cfg.block} rows starting at the anchor")
        if self.tree_plan is not None and not self.tree_plan.is_root_path(rows):
            raise ValueError(f"rows {rows} are not a root path of the current tree")
        if self.tree_plan is None and rows != list(range(keep)):
            raise ValueError(f"a chain round keeps rows 0 .. keep-1, not {rows}")
        C = (2 * (p.gdn_key_heads or p.gdn_heads) + p.gdn_heads) * cfg.gdn_dk
        gi = 0
        for L, S in zip(self.w["layers"], self.state["layers"]):
            if L["kind"] == "gdn":
                _, k, v = self.gdn_qkv(gi)
                dc.gdn_replay(S["snapshot"][None], self.state_out[gi][None], k[None], v[None],
                              self.capture_alpha[gi][None], self.capture_beta[gi][None], keep=keep, rows=rows)
                S["snapshot"].copy_(self.state_out[gi])
                conv_in = self.gdn_proj[gi][:, :C].contiguous()
                window = torch.empty_like(S["window"])
                dc.gdn_conv_rollback(S["window"][None], window[None], conv_in[None], keep=keep, rows=rows)
                S["window"].copy_(window)
                gi += 1
            elif rows != list(range(keep)):
                dc.stack_kv_compact(S["cache_k"], S["cache_v"], self.context, rows)

    def advance(self, n: int):
        """After commit(rows): the caches now hold n = len(rows) more tokens."""
        if n < 0 or any(S["cache_k"].shape[1] < self.context + n for S in self.state["layers"] if "cache_k" in S):
            raise ValueError(f"advancing the context by {n} runs past the attention caches")
        self.context += n
        if self.position is not None:  # stream-ordered after the round that was just read back
            self.position.fill_(self.context)

    def capture(self, hidden_buf, proposals=None):
        """Capture forward(hidden_buf) — or, with proposals, the whole verify round — as a
        CUDA graph (run eagerly once first)."""
        body = (lambda: self.verify(hidden_buf, proposals)) if proposals is not None else \
            (lambda: self._forward_body(hidden_buf))
        body()
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            body()
        self.graph = g
        return g

    def kernels_per_forward(self) -> int:
        """Library kernel launches per forward (dflash_qmm is two launches)."""
        n = 1  # final norm
        for k in self.cfg.layer_kinds():
            n += 2  # two add_rmsnorm
            if k == "gdn":
                n += 2 + 1 + 1 + 1 + 2  # in_proj, conv + gates, gdn_step, gated_norm, out_proj
            else:
                n += 2 + 1 + 1 + 2  # qkv, prep, decode, o_proj
            n += 2 + 2  # gate_up, down (SwiGLU inside its prep; pushes inside the qmm epilogues)
        return n


# ----------------------------------------------------------------------------- benchmark

# Roles of the library calls in a forward, for the per-role time split of phase_times().
PHASES = {
    "qmm": "quantized projections", "qmm_ex": "quantized projections",
    "stack_add_rmsnorm": "residual add + RMSNorm (+ all-reduce)",
    "stack_add_rmsnorm_reduce": "residual add + RMSNorm (+ all-reduce)",
    "stack_gdn_conv_gates": "gated-delta conv + gates", "gdn_step": "gated-delta step",
    "gdn_step_tree": "gated-delta step", "stack_gated_norm": "gated norm",
    "stack_attn_prep": "attention prep", "stack_attn_decode": "decode attention",
}


def phase_times(stack, hidden, rounds: int = 3, hold_ms: float = 60.0):
    """Device time of one eager forward split by the role of each library call: every call is
    bracketed by CUDA events on the current stream (which also serialises the calls, so the
    parts add up to more than a graph-replayed forward; read them as shares).  A sleep kernel
    of `hold_ms` at the head of the stream lets the host enqueue the whole forward before
    the device starts it, so no span includes time the device spent waiting for the host.
    The last of `rounds` forwards is kept; with several ranks each part is the max over the
    ranks."""
    dc = stack.dc
    saved = {name: getattr(dc, name) for name in PHASES}
    log = []

    def wrap(name, fn):
        def timed(*a, **k):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            r = fn(*a, **k)
            e1.record()
            log.append((PHASES[name], e0, e1))
            return r
        return timed

    try:
        for name, fn in saved.items():
            setattr(dc, name, wrap(name, fn))
        clock_khz = torch.cuda.get_device_properties(stack.device).clock_rate
        for _ in range(rounds):
            log.clear()
            if stack.world > 1:
                torch.distributed.barrier(group=stack.pg)
            torch.cuda._sleep(int(hold_ms * clock_khz))
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            stack.forward(hidden)
            t1.record()
            torch.cuda.synchronize(stack.device)
    finally:
        for name, fn in saved.items():
            setattr(dc, name, fn)
    parts = {}
    for role, e0, e1 in log:
        parts[role] = parts.get(role, 0.0) + e0.elapsed_time(e1) * 1000.0
    roles = sorted(set(PHASES.values()))
    vec = torch.tensor([parts.get(r, 0.0) for r in roles] + [t0.elapsed_time(t1) * 1000.0], device=stack.device)
    if stack.world > 1:
        torch.distributed.all_reduce(vec, op=torch.distributed.ReduceOp.MAX, group=stack.pg)
    vec = vec.tolist()
    total = vec[-1]
    return {"eager_forward_us": round(total, 1),
            "parts_us": {r: round(v, 1) for r, v in zip(roles, vec[:-1]) if v > 0},
            "parts_share": {r: round(v / total, 3) for r, v in zip(roles, vec[:-1]) if v > 0}}


def _dist_env():
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), \
        int(os.environ.get("LOCAL_RANK", "0"))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--tiny", action="store_true", help="the small parity-test stack instead of config 4")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--context", type=int, default=None)
    ap.add_argument("--allreduce", choices=["peer", "nccl"], default="peer",
                    help="peer: NVLink stores into the other ranks' exchange buffers, summed by the next "
                         "RMSNorm; nccl: torch.distributed.all_reduce")
    ap.add_argument("--gdn-key-heads", type=int, default=None,
                    help="gated-delta q / k heads, each shared by gdn_heads / this many value heads")
    ap.add_argument("--phase-times", action="store_true",
                    help="also report one eager forward's device time split by the role of each library call")
    ap.add_argument("--tree", default=None,
                    help="verify a speculative tree instead of a chain: comma-separated parent rows, one per "
                         "block row (-1 for the anchor), e.g. -1,0,0,1,1,2,3,5")
    args = ap.parse_args(argv)

    sys.path.insert(0, str(HERE))
    world, rank, local = _dist_env()
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    pg = None
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
        pg = torch.distributed.group.WORLD
    cfg = TINY if args.tiny else CONFIG4
    if args.layers is not None:
        cfg = replace(cfg, layers=args.layers)
    if args.context is not None:
        cfg = replace(cfg, context=args.context)
    if args.gdn_key_heads is not None:
        cfg = replace(cfg, gdn_key_heads=args.gdn_key_heads)

    stack = VerifyStack(cfg, rank, world, seed=args.seed, device=dev, group=pg, allreduce=args.allreduce,
                        tree=args.tree is not None)
    if args.tree is not None:
        stack.set_tree([int(v) for v in args.tree.split(",")])
    hidden = make_block(cfg, args.seed, dev)
    proposals = torch.zeros(cfg.block - 1, dtype=torch.int32, device=dev)

    def timed(g):
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            g.replay()
        stop.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([start.elapsed_time(stop) / args.steps], device=dev)
        if world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    g = stack.capture(hidden)
    ms = timed(g)
    del g
    g = stack.capture(hidden, proposals)  # forward + LM head (vocabulary-sharded) + accept
    ms_round = timed(g)
    wbytes = weight_bytes(stack.w)
    checksum = float(stack.out.float().abs().sum().item())
    if rank == 0:
        print(json.dumps({
            "metric": "verify forward µs (M-row block through the full stack)",
            "value": round(ms * 1000.0, 2), "unit": "us", "tokens_per_s": round(cfg.block / (ms / 1000.0), 1),
            "round_us": round(ms_round * 1000.0, 2),
            "tp": world, "steps": args.steps, "warmup": args.warmup,
            "weight_bytes_per_gpu": wbytes, "weight_gbs_per_gpu": round(wbytes / (ms / 1000.0) / 1e9, 1),
            "kernels_per_forward": stack.kernels_per_forward(), "all_reduces_per_forward": 2 * cfg.layers,
            "allreduce": stack.allreduce, "tree": None if args.tree is None else stack.tree_plan.parents,
            "config": {k: v for k, v in asdict(cfg).items()}, "out_abs_sum": checksum,
        }), flush=True)
    del g
    stack.graph = None
    if args.phase_times:
        split = phase_times(stack, hidden)
        if rank == 0:
            print(json.dumps({"phase_times": split, "tp": world}), flush=True)
    if world > 1:
        stack.close()
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

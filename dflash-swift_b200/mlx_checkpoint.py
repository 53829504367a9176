"""MLX quantized safetensors checkpoints for the verify stack.

The reference loads checkpoint directories of `config.json` plus `*.safetensors` shards
read in name order and merged (Sources/DFlashKit/DFlashLoader.swift:37-62, errors
`missingConfiguration` / `missingWeights` at :10-21); an MLX quantized linear layer is
three tensors under one prefix — `weight` (uint32 [N, K·bits/32]), `scales` and `biases`
(bf16 [N, K/group]) — shared as-is by the small-M kernel
(Sources/DFlashKit/SmallMQuantizedMatmul.swift:243-248), with the group size and bits in
`config.json` under "quantization" (per-layer overrides under the layer's prefix).

This module reads and writes that format with no dependency beyond numpy/torch (the
file is an 8-byte little-endian header length, a JSON header of name → dtype, shape and
byte range, then the raw bytes, read through a memory map), finds the quantized layers,
and maps a checkpoint onto the verify stack's layout (`verify_stack.StackConfig`),
sharding it for tensor parallelism with the same row/column cuts as the synthetic
weights.  The tensor names of the reference's external Qwen3.5 fork are not available
here; the names below are this stack's, and a real checkpoint whose projections are
stored as separate parts loads through the part names.

Stack tensor names (one prefix per projection; a fused projection may instead be given
as its parts, whose rows are concatenated in the order listed):
  model.layers.{i}.input_layernorm.weight, .post_attention_layernorm.weight
  gated-delta layer:  .linear_attn.in_proj       = [q | k | v | z | b | a] (q, k: key heads)
                        (or in_proj_q, in_proj_k, in_proj_v, in_proj_z, in_proj_b, in_proj_a)
                      .linear_attn.out_proj, .linear_attn.conv1d.weight [3·H·dk, kc],
                      .linear_attn.A_log, .linear_attn.dt_bias, .linear_attn.norm.weight
  attention layer:    .self_attn.qkv_proj        = [q | gate | k | v]
                        (or q_proj, gate_proj, k_proj, v_proj)
                      .self_attn.o_proj, .self_attn.q_norm.weight, .self_attn.k_norm.weight
  every layer:        .mlp.gate_up_proj          = [gate | up]  (or gate_proj, up_proj)
                      .mlp.down_proj
  model.norm.weight, lm_head (quantized, [vocab, hidden]; sharded by vocabulary rows)
"""
from __future__ import annotations

import json
import struct
from pathlib import Path
from typing import Dict, Optional

import numpy as np
import torch

# safetensors dtype -> (numpy storage dtype, torch dtype of the loaded tensor)
_DTYPES = {
    "U32": (np.uint32, torch.int32),      # packed MLX weights: bit pattern kept, held as int32
    "I32": (np.int32, torch.int32),
    "U8": (np.uint8, torch.uint8),
    "I64": (np.int64, torch.int64),
    "BF16": (np.uint16, torch.bfloat16),  # bit pattern, viewed as bf16
    "F16": (np.float16, torch.float16),
    "F32": (np.float32, torch.float32),
}
_TORCH_TO_ST = {torch.int32: "I32", torch.uint8: "U8", torch.int64: "I64", torch.bfloat16: "BF16",
                torch.float16: "F16", torch.float32: "F32"}


class CheckpointError(RuntimeError):
    """A checkpoint directory or file the loader cannot use."""


# ----------------------------------------------------------------------------- safetensors

def read_header(path) -> tuple[dict, int]:
    """(header without __metadata__, byte offset of the data region)."""
    path = Path(path)
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise CheckpointError(f"{path}: truncated safetensors header")
        (n,) = struct.unpack("<Q", raw)
        if n > 100 * 1024 * 1024:
            raise CheckpointError(f"{path}: header of {n} bytes")
        header = json.loads(f.read(n))
    header.pop("__metadata__", None)
    return header, 8 + n


def load_file(path, names=None) -> Dict[str, torch.Tensor]:
    """Tensors of one safetensors file (CPU).  `names` limits the load."""
    path = Path(path)
    header, start = read_header(path)
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, info in header.items():
        if names is not None and name not in names:
            continue
        dt = info["dtype"]
        if dt not in _DTYPES:
            raise CheckpointError(f"{path}: tensor {name} has unsupported dtype {dt}")
        np_dt, th_dt = _DTYPES[dt]
        a, b = info["data_offsets"]
        shape = tuple(info["shape"])
        count = int(np.prod(shape)) if shape else 1
        if b - a != count * np.dtype(np_dt).itemsize:
            raise CheckpointError(f"{path}: tensor {name}: {b - a} bytes for shape {shape} {dt}")
        arr = np.frombuffer(mm, dtype=np_dt, count=count, offset=start + a).reshape(shape)
        if np_dt == np.uint16:
            arr = arr.view(np.int16)
        elif np_dt == np.uint32:
            arr = arr.view(np.int32)
        t = torch.from_numpy(arr.copy())
        if dt == "BF16":
            t = t.view(torch.bfloat16)
        out[name] = t
    return out


def save_file(path, tensors: Dict[str, torch.Tensor], metadata: Optional[dict] = None,
              u32_names=()) -> None:
    """Write tensors as safetensors; names in `u32_names` (int32 tensors holding packed
    words) are stored with dtype U32, as MLX writes quantized weights."""
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        t = tensors[name].detach().to("cpu").contiguous()
        dt = "U32" if name in u32_names else _TORCH_TO_ST.get(t.dtype)
        if dt is None:
            raise CheckpointError(f"cannot store {name} of dtype {t.dtype}")
        if t.dtype == torch.bfloat16:
            data = t.view(torch.int16).numpy().tobytes()
        else:
            data = t.numpy().tobytes()
        header[name] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for d in blobs:
            f.write(d)


def load_directory(directory) -> tuple[dict, Dict[str, torch.Tensor]]:
    """(config.json, merged tensors of every *.safetensors shard in name order)."""
    directory = Path(directory)
    cfg_path = directory / "config.json"
    if not cfg_path.exists():
        raise CheckpointError(f"No config.json in {directory}")
    shards = sorted(p for p in directory.iterdir() if p.suffix == ".safetensors")
    if not shards:
        raise CheckpointError(f"No .safetensors weights in {directory}")
    config = json.loads(cfg_path.read_text())
    tensors: Dict[str, torch.Tensor] = {}
    for shard in shards:
        tensors.update(load_file(shard))
    return config, tensors


# ----------------------------------------------------------------------------- quantized layers

def quantization_of(config: dict, prefix: str) -> tuple[int, int]:
    """(group_size, bits) of the layer at `prefix`: its own entry under "quantization"
    if present, else the global one."""
    q = config.get("quantization") or config.get("quantization_config")
    if not q:
        raise CheckpointError("config.json has no quantization entry")
    own = q.get(prefix)
    if isinstance(own, dict):
        return int(own["group_size"]), int(own["bits"])
    return int(q["group_size"]), int(q["bits"])


def quantized_layer(tensors: Dict[str, torch.Tensor], config: dict, prefix: str):
    """The Quant at `prefix` (weight / scales / biases), its bits checked against the
    packed width: words per row × 32 must equal K × bits with K = groups × group_size."""
    from verify_stack import Quant
    try:
        w, s, b = (tensors[f"{prefix}.{k}"] for k in ("weight", "scales", "biases"))
    except KeyError as e:
        raise CheckpointError(f"quantized layer {prefix}: missing {e.args[0]}") from None
    group, bits = quantization_of(config, prefix)
    K = s.shape[1] * group
    if w.shape[1] * 32 != K * bits or w.shape[0] != s.shape[0] or b.shape != s.shape:
        raise CheckpointError(f"quantized layer {prefix}: weight {tuple(w.shape)}, scales {tuple(s.shape)} "
                              f"do not match group {group}, bits {bits}")
    return Quant(w.view(torch.int32), s.to(torch.bfloat16), b.to(torch.bfloat16), group, bits)


def quantized_layers(tensors: Dict[str, torch.Tensor], config: dict) -> dict:
    """Every quantized layer of a checkpoint, by prefix."""
    prefixes = sorted({n[:-len(".scales")] for n in tensors if n.endswith(".scales")})
    return {p: quantized_layer(tensors, config, p) for p in prefixes if f"{p}.weight" in tensors}


# ----------------------------------------------------------------------------- verify stack

_FUSED_PARTS = {
    "linear_attn.in_proj": ("in_proj_q", "in_proj_k", "in_proj_v", "in_proj_z", "in_proj_b", "in_proj_a"),
    "self_attn.qkv_proj": ("q_proj", "gate_proj", "k_proj", "v_proj"),
    "mlp.gate_up_proj": ("gate_proj", "up_proj"),
}


def _fused(tensors, config, layer_prefix, name):
    from verify_stack import Quant
    full = f"{layer_prefix}.{name}"
    if f"{full}.weight" in tensors:
        return quantized_layer(tensors, config, full)
    block = name.split(".")[0]
    parts = [quantized_layer(tensors, config, f"{layer_prefix}.{block}.{p}") for p in _FUSED_PARTS[name]]
    g, bits = parts[0].group, parts[0].bits
    if any(p.group != g or p.bits != bits or p.K != parts[0].K for p in parts):
        raise CheckpointError(f"{full}: parts differ in K, group or bits")
    return Quant(torch.cat([p.w for p in parts]), torch.cat([p.scales for p in parts]),
                 torch.cat([p.biases for p in parts]), g, bits)


def stack_config_from_json(config: dict, context: int, block: int = 8):
    """verify_stack.StackConfig of a checkpoint's config.json, in the keys of the target's
    Qwen3.5 configuration (the reference's fixture spells them out:
    Tests/DFlashKitTests/TinyHybridTarget.swift:20-44): hidden_size, num_hidden_layers,
    intermediate_size, full_attention_interval, linear_num_value_heads /
    linear_num_key_heads, linear_key_head_dim / linear_value_head_dim,
    linear_conv_kernel_dim, num_attention_heads, num_key_value_heads, head_dim,
    rope_parameters {rope_theta, partial_rotary_factor} (or the same keys at the top
    level), rms_norm_eps, vocab_size, and the global "quantization" entry.  `context` and
    `block` size the attention caches and the verify block.

    Fewer key heads than value heads (each key head shared by linear_num_value_heads /
    linear_num_key_heads value heads) becomes gdn_key_heads; a key-head count that does
    not divide the value heads, or a rotary width the attention prep cannot take, is
    rejected with CheckpointError."""
    import verify_stack as vs

    def need(key):
        if key not in config:
            raise CheckpointError(f"config.json has no {key!r}")
        return config[key]

    rope = config.get("rope_parameters") or {}
    theta = float(rope.get("rope_theta", config.get("rope_theta", 10000.0)))
    factor = float(rope.get("partial_rotary_factor", config.get("partial_rotary_factor", 1.0)))
    head_dim = int(need("head_dim"))
    rot = int(round(head_dim * factor))
    hv, hk = int(need("linear_num_value_heads")), int(need("linear_num_key_heads"))
    if hk < 1 or hv % hk:
        raise CheckpointError(f"{hk} gated-delta key heads do not divide {hv} value heads")
    if rot % 64 or rot > head_dim:
        raise CheckpointError(f"rotary width {rot} of head dim {head_dim}: a multiple of 64 up to the head dim needed")
    q = config.get("quantization") or config.get("quantization_config")
    if not q:
        raise CheckpointError("config.json has no quantization entry")
    return vs.StackConfig(
        layers=int(need("num_hidden_layers")), hidden=int(need("hidden_size")),
        intermediate=int(need("intermediate_size")), attn_interval=int(need("full_attention_interval")),
        gdn_heads=hv, gdn_dk=int(need("linear_key_head_dim")), gdn_dv=int(need("linear_value_head_dim")),
        conv_kernel=int(need("linear_conv_kernel_dim")), attn_heads=int(need("num_attention_heads")),
        kv_heads=int(need("num_key_value_heads")), head_dim=head_dim, rotary_dim=rot, rope_theta=theta,
        eps=float(config.get("rms_norm_eps", 1e-6)), group=int(q["group_size"]), bits=int(q["bits"]),
        context=int(context), block=int(block), vocab=int(need("vocab_size")), gdn_key_heads=hk if hk != hv else 0)


def stack_from_checkpoint(cfg, plan, config: dict, tensors: Dict[str, torch.Tensor], device) -> dict:
    """The rank's shard of a checkpoint in verify_stack's weight layout (the same
    structure build_rank_weights returns)."""
    import verify_stack as vs
    dev = torch.device(device)
    get = lambda n: tensors[n] if n in tensors else (_ for _ in ()).throw(CheckpointError(f"missing {n}"))
    layers = []
    for i, kind in enumerate(cfg.layer_kinds()):
        pre = f"model.layers.{i}"
        L = {"kind": kind, "ln": get(f"{pre}.input_layernorm.weight").to(torch.bfloat16),
             "post_ln": get(f"{pre}.post_attention_layernorm.weight").to(torch.bfloat16)}
        if kind == "gdn":
            Hg, Hk, dk, kc = cfg.gdn_heads, cfg.gdn_kheads, cfg.gdn_dk, cfg.conv_kernel
            L["in_proj"] = _fused(tensors, config, pre, "linear_attn.in_proj").rows(vs._ranges_gdn_in(cfg, plan))
            out = quantized_layer(tensors, config, f"{pre}.linear_attn.out_proj")
            L["out_proj"] = out.cols(plan.gdn_head0 * cfg.gdn_dv, (plan.gdn_head0 + plan.gdn_heads) * cfg.gdn_dv)
            conv = get(f"{pre}.linear_attn.conv1d.weight").to(torch.bfloat16).reshape((2 * Hk + Hg) * dk, kc)
            heads = slice(plan.gdn_head0, plan.gdn_head0 + plan.gdn_heads)
            L["conv"] = torch.cat([conv[a:b] for a, b in vs.gdn_conv_channels(cfg, plan)]).contiguous()
            L["a_log"] = get(f"{pre}.linear_attn.A_log").float()[heads].contiguous()
            L["dt_bias"] = get(f"{pre}.linear_attn.dt_bias").float()[heads].contiguous()
            L["gdn_norm"] = get(f"{pre}.linear_attn.norm.weight").to(torch.bfloat16)
        else:
            d = cfg.head_dim
            L["qkv"] = _fused(tensors, config, pre, "self_attn.qkv_proj").rows(vs._ranges_attn_qkv(cfg, plan))
            o = quantized_layer(tensors, config, f"{pre}.self_attn.o_proj")
            L["o_proj"] = o.cols(plan.attn_head0 * d, (plan.attn_head0 + plan.attn_heads) * d)
            L["q_norm"] = get(f"{pre}.self_attn.q_norm.weight").to(torch.bfloat16)
            L["k_norm"] = get(f"{pre}.self_attn.k_norm.weight").to(torch.bfloat16)
        L["gate_up"] = _fused(tensors, config, pre, "mlp.gate_up_proj").rows(vs._ranges_gate_up(cfg, plan))
        L["down"] = quantized_layer(tensors, config, f"{pre}.mlp.down_proj").cols(plan.inter0, plan.inter0 + plan.inter)
        for k, v in list(L.items()):
            if isinstance(v, torch.Tensor):
                L[k] = v.to(dev)
            elif isinstance(v, vs.Quant):
                L[k] = vs.Quant(v.w.to(dev), v.scales.to(dev), v.biases.to(dev), v.group, v.bits)
        layers.append(L)
    head = quantized_layer(tensors, config, "lm_head").rows([(plan.vocab0, plan.vocab0 + plan.vocab)])
    head = vs.Quant(head.w.to(dev), head.scales.to(dev), head.biases.to(dev), head.group, head.bits)
    return {"layers": layers, "final_norm": get("model.norm.weight").to(torch.bfloat16).to(dev), "lm_head": head}


def save_stack_checkpoint(directory, cfg, weights: dict, shard_bytes: int = 1 << 30) -> None:
    """Write unsharded (TP=1) stack weights as an MLX quantized checkpoint: config.json
    with the quantization entry, and shards of at most `shard_bytes`."""
    import verify_stack as vs
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    tensors, u32 = {}, set()

    def put_quant(prefix, q):
        tensors[f"{prefix}.weight"], tensors[f"{prefix}.scales"], tensors[f"{prefix}.biases"] = q.w, q.scales, q.biases
        u32.add(f"{prefix}.weight")

    names = {"in_proj": "linear_attn.in_proj", "out_proj": "linear_attn.out_proj", "qkv": "self_attn.qkv_proj",
             "o_proj": "self_attn.o_proj", "gate_up": "mlp.gate_up_proj", "down": "mlp.down_proj"}
    plain = {"ln": "input_layernorm.weight", "post_ln": "post_attention_layernorm.weight",
             "conv": "linear_attn.conv1d.weight", "a_log": "linear_attn.A_log", "dt_bias": "linear_attn.dt_bias",
             "gdn_norm": "linear_attn.norm.weight", "q_norm": "self_attn.q_norm.weight",
             "k_norm": "self_attn.k_norm.weight"}
    for i, L in enumerate(weights["layers"]):
        pre = f"model.layers.{i}"
        for k, v in L.items():
            if isinstance(v, vs.Quant):
                put_quant(f"{pre}.{names[k]}", v)
            elif k in plain:
                tensors[f"{pre}.{plain[k]}"] = v
    tensors["model.norm.weight"] = weights["final_norm"]
    put_quant("lm_head", weights["lm_head"])
    config = {"model_type": "dflash_verify_stack", "hidden_size": cfg.hidden, "num_hidden_layers": cfg.layers,
              "intermediate_size": cfg.intermediate, "full_attention_interval": cfg.attn_interval,
              "linear_num_value_heads": cfg.gdn_heads, "linear_num_key_heads": cfg.gdn_kheads,
              "linear_key_head_dim": cfg.gdn_dk, "linear_value_head_dim": cfg.gdn_dv,
              "linear_conv_kernel_dim": cfg.conv_kernel, "num_attention_heads": cfg.attn_heads,
              "num_key_value_heads": cfg.kv_heads, "head_dim": cfg.head_dim, "rms_norm_eps": cfg.eps,
              "vocab_size": cfg.vocab,
              "rope_parameters": {"rope_type": "default", "rope_theta": cfg.rope_theta,
                                  "partial_rotary_factor": cfg.rotary_dim / cfg.head_dim},
              "quantization": {"group_size": cfg.group, "bits": cfg.bits}}
    (directory / "config.json").write_text(json.dumps(config, indent=1))
    shard, size, n = {}, 0, 0
    for name in sorted(tensors):
        nb = tensors[name].numel() * tensors[name].element_size()
        if shard and size + nb > shard_bytes:
            save_file(directory / f"model-{n:05d}.safetensors", shard, u32_names=u32)
            shard, size, n = {}, 0, n + 1
        shard[name] = tensors[name]
        size += nb
    save_file(directory / f"model-{n:05d}.safetensors", shard, u32_names=u32)
